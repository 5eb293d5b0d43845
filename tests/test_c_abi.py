"""The C ABI library builds, loads and exports every symbol include/wdit.h declares; host-side
argument validation rejects bad calls before touching a device. CPU only (no compute)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "wdit.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(wdit_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib(pkg):
    return pkg._lib.load(build_if_missing=True)


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    for s in ("wdit_gemm_act", "wdit_gemm_residual", "wdit_gemm_norm", "wdit_ln_stats", "wdit_fold_weight",
              "wdit_layernorm_modulation", "wdit_rmsnorm", "wdit_qk_rms_rope_from_partials", "wdit_rope_table"):
        assert s in syms


def test_library_exports_every_declared_symbol(lib, pkg):
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} declared in include/wdit.h but not exported"
    # ...and the Python binding declares a signature for each of them.
    assert set(declared_symbols()) <= set(pkg._lib.exported_symbols())


def test_library_is_built_for_sm100a():
    so = (ROOT / "coda-wan-dit_b200" / "libwdit.so").read_bytes()
    assert b"sm_100a" in so or b"sm_100" in so


def test_argument_validation_without_device(lib):
    null = ctypes.c_void_p(None)
    # NULL operands -> WDIT_ERR_ARG; bad shapes -> WDIT_ERR_SHAPE; no CUDA call is reached.
    assert lib.wdit_gemm_act(null, 64, null, 64, null, 64, 128, 256, 64, null, 0, null, null, 0, 0, 0.0, null, 0, 0,
                             null, 0) == 1
    dummy = ctypes.c_void_p(0x1000)
    assert lib.wdit_gemm_act(dummy, 64, dummy, 64, dummy, 64, 128, 100, 64, null, 0, null, null, 0, 0, 0.0, null, 0, 0,
                             null, 0) == 2  # N % 64 != 0
    assert lib.wdit_gemm_act(dummy, 32, dummy, 64, dummy, 256, 128, 256, 64, null, 0, null, null, 0, 0, 0.0, null, 0,
                             0, null, 0) == 2  # lda < K
    assert lib.wdit_gemm_act(dummy, 64, dummy, 64, dummy, 256, 128, 256, 64, null, 0, null, null, 0, 0, 0.0, dummy, 2,
                             192, null, 0) == 2  # mean-square columns not a multiple of 128
    assert lib.wdit_gemm_residual(dummy, 64, dummy, 64, null, 256, dummy, 256, 128, 256, 64, null, null, null, 0, 0,
                                  null, 0, null, null, 0) == 1  # no residual
    assert lib.wdit_ln_stats(null, 0, 64, 4, 64, null, null, null, null) == 1
    assert lib.wdit_fold_weight(dummy, 60, 4, 60, 1.0, null, null, null, null, null, dummy, 60, dummy, dummy,
                                null) == 2  # K % 8 != 0


def test_norm_workspace_size(lib):
    # RMSNorm partials M x (groups * width/128) fp32, 256-byte rounded
    M, groups, width = 1000, 2, 1536
    part = ((M * groups * (width // 128) * 4 + 255) // 256) * 256
    assert lib.wdit_gemm_norm_workspace_bytes(M, 4608, groups, width) == part
    assert lib.wdit_stats_tile_width() == 256


def test_p2p_argument_validation_without_device(lib):
    null = ctypes.c_void_p(None)
    dummy = ctypes.c_void_p(0x1000)
    peers = (ctypes.c_void_p * 2)(0x100000, 0x200000)
    # NULL operands -> WDIT_ERR_ARG
    assert lib.wdit_p2p_qkv_exchange(null, 4608, dummy, 24, dummy, dummy, 1e-6, dummy, dummy, 64, 2, 96, 12, 128, 2, 0,
                                     peers, 0, 0, 1, dummy, null) == 1
    # head_dim other than 128, units that do not divide over the ranks -> WDIT_ERR_SHAPE
    assert lib.wdit_p2p_qkv_exchange(dummy, 4608, dummy, 24, dummy, dummy, 1e-6, dummy, dummy, 64, 2, 96, 12, 64, 2, 0,
                                     peers, 0, 0, 1, dummy, null) == 2
    assert lib.wdit_p2p_qkv_exchange(dummy, 4608, dummy, 24, dummy, dummy, 1e-6, dummy, dummy, 64, 1, 96, 12, 128, 8, 0,
                                     peers, 0, 0, 1, dummy, null) == 2
    # a rank outside [0, P) -> WDIT_ERR_SHAPE; misaligned region offsets -> WDIT_ERR_ALIGN
    assert lib.wdit_p2p_out_exchange(dummy, 128, 128, 2, 96, 12, 128, 2, 2, peers, 0, 1536, 0, 1, dummy, null) == 2
    assert lib.wdit_p2p_out_exchange(dummy, 128, 128, 2, 96, 12, 128, 2, 0, peers, 100, 1536, 0, 1, dummy, null) == 3
    assert lib.wdit_p2p_wait(null, 2, 1, null) == 1
    assert lib.wdit_p2p_wait(dummy, 0, 1, null) == 2
    assert lib.wdit_ipc_handle(null, null, None) == 1
    assert lib.wdit_ipc_open(null, None) == 1


def test_gemm_norm_exchange_validates_without_device(lib):
    null = ctypes.c_void_p(None)
    d = ctypes.c_void_p(0x1000)
    peers = (ctypes.c_void_p * 2)(0x100000, 0x200000)

    def call(*, A=d, scratch=d, ld=4608, M=192, batch=2, Lp=96, H=12, P=2, rank=0, bases=peers, full_off=0,
             flag_off=0, ctr=d):
        return lib.wdit_gemm_norm_exchange(A, 1536, d, 1536, scratch, ld, M, 1536, d, null, null, 0, 0, 0.0, d, d,
                                           1e-6, d, d, 64, batch, Lp, H, P, rank, bases, full_off, flag_off, 1, ctr,
                                           null, 0)

    assert call(M=0) == 0                           # no rows: nothing to do
    assert call(A=null) == 1                        # null operand
    assert call(scratch=null) == 1
    assert call(ctr=null) == 1
    assert call(bases=None) == 1
    assert call(M=190) == 2                         # batch * Lp != M
    assert call(H=5, ld=1920, P=4) == 2             # 10 (batch, head) units do not divide over 4 ranks
    assert call(rank=2) == 2                        # rank outside [0, P)
    assert call(P=9) == 2                           # more ranks than the kernel's peer table
    assert call(ld=3072) == 2                       # scratch narrower than 3 D
    assert call(full_off=100) == 3                  # region offsets not 256-byte aligned
    assert call(flag_off=4) == 3
    bad = (ctypes.c_void_p * 2)(0x100000, 0x200010)
    assert call(bases=bad) == 3                     # a peer region not 256-byte aligned


def test_batched_entry_points_validate_without_device(lib, pkg):
    null = ctypes.c_void_p(None)
    dummy = ctypes.c_void_p(0x1000)
    # rms_apply_layers: null operands, no layers, last layer past the row, misaligned layer stride
    assert lib.wdit_rms_apply_layers(null, 9216, 4, dummy, 72, 1536, dummy, 1e-6, 3, 3072, 24, 1536, null) == 1
    assert lib.wdit_rms_apply_layers(dummy, 9216, 4, dummy, 72, 1536, dummy, 1e-6, 0, 3072, 24, 1536, null) == 2
    assert lib.wdit_rms_apply_layers(dummy, 9216, 4, dummy, 72, 1536, dummy, 1e-6, 4, 3072, 24, 1536, null) == 2
    assert lib.wdit_rms_apply_layers(dummy, 9216, 4, dummy, 59, 1536, dummy, 1e-6, 3, 3072, 24, 1536, null) == 2
    assert lib.wdit_rms_apply_layers(dummy, 9216, 4, dummy, 72, 1536, dummy, 1e-6, 2, 3076, 24, 1536, null) == 3
    # fold batch: negative count, a job with K % 8 != 0, a null output
    jobs = (pkg._lib.FoldJob * 2)()
    for j in jobs:
        j.W, j.ldw, j.N, j.K, j.mult_c = 0x1000, 64, 4, 64, 1.0
        j.W_out, j.ldw_out, j.csum_out, j.vec_out = 0x2000, 64, 0x3000, 0x4000
    assert lib.wdit_fold_weight_batch(jobs, -1, null) == 1
    jobs[1].K = 60
    assert lib.wdit_fold_weight_batch(jobs, 2, null) == 2
    jobs[1].K, jobs[1].W_out = 64, None
    assert lib.wdit_fold_weight_batch(jobs, 2, null) == 1
    assert lib.wdit_fold_weight_batch(jobs, 0, null) == 0


def test_patch_rows_validates_without_device(lib):
    null = ctypes.c_void_p(None)
    dummy = ctypes.c_void_p(0x1000)
    assert lib.wdit_patch_rows(null, 16, 21, 60, 104, 1, 2, 2, 0, 32760, 64, dummy, null) == 1
    assert lib.wdit_patch_rows(dummy, 16, 21, 60, 104, 1, 2, 2, 0, 32760, 56, dummy, null) == 2  # Kp < K
    assert lib.wdit_patch_rows(null, 16, 21, 60, 104, 1, 2, 2, 0, 0, 64, null, null) == 0        # no rows
    assert lib.wdit_patch_rows(dummy, 16, 21, 60, 104, 1, 2, 2, 0, 32760, 64, ctypes.c_void_p(0x1008), null) == 3


def test_fold_job_struct_matches_header(pkg, tmp_path):
    """The ctypes mirror of struct wdit_fold_job has the C layout (size and every offset)."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    fields = [f for f, _ in pkg._lib.FoldJob._fields_]
    src = tmp_path / "layout.c"
    src.write_text(
        "#include <stddef.h>\n#include <stdio.h>\n#include \"wdit.h\"\nint main(void) {\n"
        "  printf(\"%zu\\n\", sizeof(wdit_fold_job));\n"
        + "".join(f"  printf(\"%zu\\n\", offsetof(wdit_fold_job, {f}));\n" for f in fields)
        + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    want = [ctypes.sizeof(pkg._lib.FoldJob)] + [getattr(pkg._lib.FoldJob, f).offset for f in fields]
    assert got == want


def _ctype_of(decl: str):
    """ctypes class expected for one C parameter / return type of include/wdit.h."""
    t = re.sub(r"\bconst\b", "", decl).strip()
    if "*" in t:
        return "pointer"
    t = re.sub(r"\s+[A-Za-z_][A-Za-z0-9_]*$", "", t).strip() if " " in t else t  # drop the name
    return {"int": ctypes.c_int, "float": ctypes.c_float, "long long": ctypes.c_longlong,
            "unsigned int": ctypes.c_uint, "unsigned long long": ctypes.c_ulonglong}[t]


def test_binding_signatures_match_the_header(pkg):
    """Every prototype's return and argument types agree with the ctypes table (count and kind)."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    protos = re.findall(r"\b(int|long long)\s+(wdit_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text)
    assert len(protos) == len(declared_symbols())
    sigs = pkg._lib._SIGNATURES
    for ret, name, params in protos:
        res, args = sigs[name]
        assert res == {"int": ctypes.c_int, "long long": ctypes.c_longlong}[ret], name
        params = [p.strip() for p in params.split(",")] if params.strip() not in ("", "void") else []
        assert len(params) == len(args), f"{name}: {len(params)} C parameters, {len(args)} in the binding"
        for i, (p, a) in enumerate(zip(params, args)):
            want = _ctype_of(p)
            if want == "pointer":
                assert a is ctypes.c_void_p or issubclass(a, ctypes._Pointer), f"{name} arg {i}: {p}"
            else:
                assert a is want, f"{name} arg {i}: {p} vs {a}"


def test_zero_rows_is_a_no_op_without_device(lib, pkg):
    """M = 0 returns OK before any pointer is looked at (null pointers, no device)."""
    null = ctypes.c_void_p(None)
    assert lib.wdit_gemm_act(null, 64, null, 64, null, 64, 0, 64, 64, null, 0, null, null, 0, 0, 0.0, null, 0, 0,
                             null, 0) == 0
    assert lib.wdit_gemm_residual(null, 64, null, 64, null, 64, null, 64, 0, 64, 64, null, null, null, 0, 0, null, 0,
                                  null, null, 0) == 0
    assert lib.wdit_gemm_norm(null, 64, null, 64, null, 256, 0, 256, 64, null, null, null, 0, 0, 0.0, 1, 128, null,
                              null, 1e-6, 0, null, null, 0, 0, 0, null, 0, null, 0) == 0
    assert lib.wdit_gemm_norm_static(null, 64, null, 64, null, 256, 0, 256, 64, null, null, null, 0, 0, 0.0, 1, 128,
                                     null, null, 1e-6, 0, null, null, 0, 0, 0, null, 0) == 0
    assert lib.wdit_ln_stats(null, 1, 1536, 0, 1536, null, null, null, null) == 0
    assert lib.wdit_layernorm_modulation(null, 1, 1536, 0, 1536, null, null, 1e-6, null, 1536, null) == 0
    assert lib.wdit_rmsnorm(null, 1536, 0, 1536, null, 1e-6, null, 1536, null) == 0
    assert lib.wdit_qk_rms_rope_from_partials(null, 3072, null, 0, 1536, null, null, null, null, 1e-6, null) == 0
    assert lib.wdit_rms_apply_layers(null, 9216, 0, null, 72, 1536, null, 1e-6, 3, 3072, 24, 1536, null) == 0
    assert lib.wdit_fold_weight(null, 64, 0, 64, 1.0, null, null, null, null, null, null, 64, null, null, null) == 0
    jobs = (pkg._lib.FoldJob * 3)()  # all empty: nothing launched
    assert lib.wdit_fold_weight_batch(jobs, 3, null) == 0


def test_fold_jobs_per_launch_matches_kernel(pkg):
    src = (ROOT / "coda-wan-dit_b200" / "csrc" / "aux.cu").read_text()
    m = re.search(r"constexpr int kMaxFoldJobs = (\d+);", src)
    assert m and int(m.group(1)) == pkg._lib.FOLD_JOBS_PER_LAUNCH
