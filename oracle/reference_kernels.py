"""Import the reference's own coda_wan/wan_coda_kernels.py on CPU (golden-vector source).

Test infrastructure only, and only where the reference tree is mounted (the build
container): tests/golden/make_golden.py uses it to run the reference's Triton kernels
(_layernorm_modulation_kernel, _qk_rms_rope_kernel, _rmsnorm_kernel) through Triton's CPU
interpreter (TRITON_INTERPRET=1) and its torch-only helpers (build_wan_rope_table,
prepack_*). The GEMM-epilogue parts need coda-kernels (`rapier`, `kernels`), which are not
installed; those modules are replaced by inert stubs that only satisfy the imports, and
nothing that calls them is executed.
"""
from __future__ import annotations

import os
import sys
import types
from pathlib import Path

# Root of a checkout of the reference (the directory holding coda_wan/), from the environment.
REFERENCE_DIR = Path(os.environ["WDIT_REFERENCE_DIR"]) if os.environ.get("WDIT_REFERENCE_DIR") else None

_STUB_MODULES = [
    "rapier",
    "rapier.epilogue",
    "rapier.gemm",
    "rapier.gemm.gemm_interface",
    "rapier.ops",
    "kernels",
    "kernels.gens",
    "kernels.gens.epilogue",
    "kernels.gens.epilogue.kernel_0",
    "kernels.gens.gpt",
]


class _InertEVT:
    class EpilogueTensorsLoop:  # noqa: D401 - attribute holder
        pass

    class EpilogueParams:
        pass

    class EpilogueArguments:
        pass


def available() -> bool:
    return REFERENCE_DIR is not None and (REFERENCE_DIR / "coda_wan" / "wan_coda_kernels.py").is_file()


def load():
    """Return the reference module `wan_coda_kernels` (Triton in interpreter mode)."""
    if not available():
        raise FileNotFoundError("reference sources not found: set WDIT_REFERENCE_DIR to a checkout of "
                                f"Owen718/CODA-Wan-DiT (now: {REFERENCE_DIR})")
    if "triton" in sys.modules and os.environ.get("TRITON_INTERPRET") != "1":
        raise RuntimeError("set TRITON_INTERPRET=1 before triton is imported")
    os.environ["TRITON_INTERPRET"] = "1"
    for name in _STUB_MODULES:
        sys.modules.setdefault(name, types.ModuleType(name))
    ep = sys.modules["rapier.epilogue"]
    for attr in ("EVTColBlockReductionStore", "EVTList", "EVTRowOrColBias", "EVTResidual", "EpilogueVisitorTree"):
        setattr(ep, attr, _InertEVT)
    gi = sys.modules["rapier.gemm.gemm_interface"]
    for attr in ("gemm_epilogue", "preprocess_tensor", "preprocess_vector"):
        setattr(gi, attr, None)
    sys.modules["rapier.ops"].misc_utils = None
    sys.modules["kernels.gens.epilogue.kernel_0"]._create_mean_sq_reduction_op = None
    sys.modules["kernels.gens.gpt"]._dispatch = None
    path = str(REFERENCE_DIR / "coda_wan")
    if path not in sys.path:
        sys.path.insert(0, path)
    import wan_coda_kernels  # noqa: E402  (the reference module)

    return wan_coda_kernels
