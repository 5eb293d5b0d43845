"""ctypes binding of libwdit.so (the C ABI declared in include/wdit.h).

Only plain pointers, integers, floats and a cudaStream_t cross the boundary. The library
is loaded once per process; if it is missing it is built in-tree with nvcc. There is no
fallback implementation: a missing toolchain or library raises.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import c_double, c_float, c_int, c_longlong, c_uint, c_ulonglong, c_void_p
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
_LIB_PATH = _PKG / "libwdit.so"
_lock = threading.Lock()
_lib: ctypes.CDLL | None = None
_dev_state = threading.local()

WDIT_ERR_NAMES = {
    1: "invalid argument",
    2: "unsupported shape",
    3: "misaligned pointer or stride",
    4: "partially overlapping in-place buffers",
    5: "workspace missing or too small",
    6: "tensor map rejected by the driver",
    7: "driver entry point unavailable",
    8: "problem exceeds the static scratch limit",
}

P = c_void_p
F = c_float
I = c_int

# name -> (restype, argtypes); must match include/wdit.h
_SIGNATURES = {
    "wdit_num_sms": (c_int, []),
    "wdit_set_cta_pair": (c_int, [I]),
    "wdit_ipc_handle": (c_int, [P, P, ctypes.POINTER(c_longlong)]),
    "wdit_ipc_open": (c_int, [P, ctypes.POINTER(c_void_p)]),
    "wdit_ipc_close": (c_int, [P]),
    "wdit_p2p_qkv_exchange": (c_int, [P, I, P, I, P, P, F, P, P, I, I, I, I, I, I, I, P, c_longlong, c_longlong,
                                      c_uint, P, P]),
    "wdit_p2p_out_exchange": (c_int, [P, c_longlong, c_longlong, I, I, I, I, I, I, P, c_longlong, I, c_longlong,
                                      c_uint, P, P]),
    "wdit_p2p_wait": (c_int, [P, I, c_uint, P]),
    "wdit_set_device": (c_int, [I]),
    "wdit_stats_tile_width": (c_int, []),
    "wdit_set_wait_limit_ns": (c_int, [c_ulonglong]),
    "wdit_read_error": (c_int, [P, I]),
    "wdit_wait_selftest": (c_int, [P, P]),
    "wdit_gemm_act": (c_int, [P, I, P, I, P, I, I, I, I, P, I, P, P, I, I, F, P, I, I, P, I]),
    "wdit_gemm_residual": (c_int, [P, I, P, I, P, I, P, I, I, I, I, P, P, P, I, I, P, I, P, P, I]),
    "wdit_gemm_norm_workspace_bytes": (c_longlong, [I, I, I, I]),
    "wdit_gemm_norm": (
        c_int,
        [P, I, P, I, P, I, I, I, I, P, P, P, I, I, F, I, I, P, P, F, I, P, P, I, I, I, P, c_longlong, P, I],
    ),
    "wdit_gemm_norm_fused": (
        c_int,
        [P, I, P, I, P, I, I, I, I, P, P, P, I, I, F, I, I, P, P, F, I, P, P, I, I, I, P, I],
    ),
    "wdit_gemm_norm_exchange": (
        c_int,
        [P, I, P, I, P, I, I, I, P, P, P, I, I, F, P, P, F, P, P, I, I, I, I, I, I, P, c_longlong, c_longlong,
         c_uint, P, P, I],
    ),
    "wdit_gemm_norm_static": (
        c_int,
        [P, I, P, I, P, I, I, I, I, P, P, P, I, I, F, I, I, P, P, F, I, P, P, I, I, I, P, I],
    ),
    "wdit_static_scratch_bytes": (c_longlong, []),
    "wdit_ln_stats": (c_int, [P, I, I, I, I, P, P, P, P]),
    "wdit_fold_weight": (c_int, [P, I, I, I, F, P, P, P, P, P, P, I, P, P, P]),
    "wdit_fold_weight_batch": (c_int, [P, I, P]),
    "wdit_layernorm_modulation": (c_int, [P, I, I, I, I, P, P, F, P, I, P]),
    "wdit_rmsnorm": (c_int, [P, I, I, I, P, F, P, I, P]),
    "wdit_qk_rms_rope_from_partials": (c_int, [P, I, P, I, I, P, P, P, P, F, P]),
    "wdit_rms_apply_layers": (c_int, [P, I, I, P, I, I, P, F, I, c_longlong, I, I, P]),
    "wdit_patch_rows": (c_int, [P, I, I, I, I, I, I, I, c_longlong, I, I, P, P]),
    "wdit_rope_table": (c_int, [P, I, I, I, I, I, P, P, P]),
    "wdit_ulysses_pack": (c_int, [P, I, I, I, I, I, I, I, P, P]),
    "wdit_seq_gather": (c_int, [P, I, I, I, I, I, P, P]),
    "wdit_seq_scatter": (c_int, [P, c_longlong, c_longlong, I, I, I, I, P, P]),
    "wdit_ulysses_unpack": (c_int, [P, I, I, I, I, I, P, I, P]),
}


class FoldJob(ctypes.Structure):
    """struct wdit_fold_job of include/wdit.h."""

    _fields_ = [
        ("W", c_void_p), ("ldw", c_int), ("N", c_int), ("K", c_int), ("mult_c", c_float),
        ("mult_a", c_void_p), ("mult_b", c_void_p), ("shift_a", c_void_p), ("shift_b", c_void_p),
        ("bias", c_void_p), ("W_out", c_void_p), ("ldw_out", c_int), ("csum_out", c_void_p), ("vec_out", c_void_p),
    ]


FOLD_JOBS_PER_LAUNCH = 64  # jobs per fold_batch_kernel launch (kMaxFoldJobs in csrc/aux.cu)


def library_path() -> Path:
    return _LIB_PATH


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load (building first if needed) and return the shared library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if build_if_missing:
            from . import build as _build

            if _build.needs_build():
                _build.build()
        if not _LIB_PATH.exists():
            raise RuntimeError(f"wdit CUDA library not found at {_LIB_PATH}")
        lib = ctypes.CDLL(str(_LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class WditError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != 0:
        if rc >= 1000:
            msg = f"CUDA error {rc - 1000}"
        else:
            msg = WDIT_ERR_NAMES.get(rc, f"code {rc}")
        raise WditError(f"{what}: {msg}")


# Entry points that launch device work (counted by launch_counter for the benchmark).
_LAUNCHING = {
    "wdit_gemm_act", "wdit_gemm_residual", "wdit_gemm_norm", "wdit_gemm_norm_fused", "wdit_gemm_norm_exchange",
    "wdit_ln_stats",
    "wdit_fold_weight",
    "wdit_fold_weight_batch", "wdit_rms_apply_layers", "wdit_patch_rows",
    "wdit_layernorm_modulation", "wdit_rmsnorm", "wdit_qk_rms_rope_from_partials", "wdit_rope_table",
    "wdit_ulysses_pack", "wdit_seq_gather", "wdit_seq_scatter", "wdit_ulysses_unpack",
    "wdit_p2p_qkv_exchange", "wdit_p2p_out_exchange", "wdit_p2p_wait",
}
launch_counter = {"n": 0}


def call(name: str, *args, kernels: int = 1) -> int:
    """Call a library entry point on the current torch device and raise on failure.
    `kernels`: device kernels the entry point launches (counted in launch_counter)."""
    lib = load()
    _sync_device(lib)
    if name in _LAUNCHING:
        launch_counter["n"] += kernels
    rc = getattr(lib, name)(*args)
    if isinstance(rc, int) and name not in ("wdit_gemm_norm_workspace_bytes", "wdit_static_scratch_bytes"):
        check(rc, name)
    return rc


def _sync_device(lib: ctypes.CDLL) -> None:
    # The library links its own CUDA runtime; keep its current device equal to torch's.
    dev = torch.cuda.current_device()
    if getattr(_dev_state, "dev", None) != dev:
        check(lib.wdit_set_device(dev), "wdit_set_device")
        _dev_state.dev = dev


def stream_ptr(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def read_error(clear: bool = True) -> tuple[int, int, int, int]:
    """Synchronize and return the device error record (all zeros when nothing failed)."""
    lib = load()
    _sync_device(lib)
    out = (c_uint * 4)()
    check(lib.wdit_read_error(ctypes.cast(out, c_void_p), 1 if clear else 0), "wdit_read_error")
    return tuple(int(v) for v in out)


def raise_on_device_error() -> None:
    err = read_error(clear=True)
    if err[0] != 0:
        raise WditError(
            f"device-side failure code=0x{err[0]:x} site={err[1]} block={err[2]} extra={err[3]} "
            "(a bounded wait ran out)"
        )


__all__ = [
    "load",
    "call",
    "check",
    "ptr",
    "stream_ptr",
    "read_error",
    "raise_on_device_error",
    "WditError",
    "library_path",
    "exported_symbols",
    "c_double",
]
