"""coda-wan-dit_b200: B200-native (sm_100a) fused GEMMs for the non-attention half of the
Wan2.1 DiT block, behind the reference's block / op interface.

Import name: ``coda_wan_dit_b200`` (the directory name has hyphens; load it with
``load_package()`` from the repository root helpers, or add the directory's parent to
``sys.path`` and register it under that name).
"""
from . import _lib, ops, sampler  # noqa: F401
from .block import Carry, CodaFullBlock, FusedWanBlock  # noqa: F401
from .model import WAN_14B, WAN_1_3B, FusedWanModel, WanParams, WanShape, build_wan  # noqa: F401
from .ulysses import SeqParallel  # noqa: F401

__all__ = [
    "ops",
    "FusedWanBlock",
    "CodaFullBlock",
    "Carry",
    "FusedWanModel",
    "WanParams",
    "WanShape",
    "WAN_1_3B",
    "WAN_14B",
    "build_wan",
    "SeqParallel",
    "sampler",
]
