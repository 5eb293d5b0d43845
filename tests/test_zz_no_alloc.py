"""The allocation-free norm GEMM entry point (wdit_gemm_norm_static), called through the C ABI.

It exists for callers that cannot allocate device memory where they issue the GEMM (code
running where allocation is not allowed, or whose allocator belongs to another runtime):
its scratch is a fixed 4 MiB device array inside the library instead of a caller-supplied
workspace. This file is collected last so that a failure here leaves every other test run.
It checks, on two calls in a row with different inputs, that the result is bit-identical to
the workspace-taking entry point's on the same inputs (both run the same kernels in the same
order; only where the partials live differs, so any scratch aliasing or stale partials from the
previous call would show), and that a problem larger than the static scratch is refused before
anything is launched.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rand(shape, scale=1.0, seed=0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return (scale * torch.randn(shape, generator=g)).to(dtype).to(DEV)


def rel_l2(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm()).item()


def test_static_scratch_matches_workspace_entry_point(pkg):
    lib = pkg._lib.load()
    torch.cuda.set_device(0)
    assert lib.wdit_set_device(torch.cuda.current_device()) == 0
    M, D, K = 1000, 1536, 1536
    N = 3 * D
    stream = torch.cuda.current_stream().cuda_stream
    P = ctypes.c_void_p
    need = lib.wdit_gemm_norm_workspace_bytes(M, N, 2, D)
    assert 0 < need <= lib.wdit_static_scratch_bytes() == 4 << 20

    for call in range(2):
        # different inputs on each call: partials left over from call 0 must not leak into call 1
        s0 = 10 * call
        a = rand((M, K), 1.0 + call, seed=s0 + 1)
        w = rand((N, K), 0.02, seed=s0 + 2)
        vec = rand((N,), 0.01, seed=s0 + 3, dtype=torch.float32)
        wq = 1.0 + rand((D,), 0.1, seed=s0 + 4, dtype=torch.float32)
        wk = 1.0 + rand((D,), 0.1, seed=s0 + 5, dtype=torch.float32)
        ang = rand((M, 64), 3.0, seed=s0 + 6, dtype=torch.float32)
        cos, sin = torch.cos(ang).contiguous(), torch.sin(ang).contiguous()  # token-major [M, 64]
        ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
        ref = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
        rc = lib.wdit_gemm_norm(P(a.data_ptr()), K, P(w.data_ptr()), K, P(ref.data_ptr()), N, M, N, K,
                                P(vec.data_ptr()), None, None, 0, 0, 0.0, 2, D, P(wq.data_ptr()), P(wk.data_ptr()),
                                1e-6, 2, P(cos.data_ptr()), P(sin.data_ptr()), 64, M, 0, P(ws.data_ptr()), need,
                                P(stream), 0)
        assert rc == 0, call
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
        rc = lib.wdit_gemm_norm_static(P(a.data_ptr()), K, P(w.data_ptr()), K, P(out.data_ptr()), N, M, N, K,
                                       P(vec.data_ptr()), None, None, 0, 0, 0.0, 2, D, P(wq.data_ptr()),
                                       P(wk.data_ptr()), 1e-6, 2, P(cos.data_ptr()), P(sin.data_ptr()), 64, M, 0,
                                       P(stream), 0)
        assert rc == 0, call
        torch.cuda.synchronize()
        assert torch.equal(out, ref), (call, rel_l2(out, ref))
    pkg._lib.raise_on_device_error()


def test_static_scratch_rejects_oversized_problem(pkg):
    lib = pkg._lib.load()
    assert lib.wdit_set_device(torch.cuda.current_device()) == 0
    M, D = 200_000, 1536  # needs about 19.2 MB of partials: above the 4 MiB array
    dummy = ctypes.c_void_p(0x10000)
    rc = lib.wdit_gemm_norm_static(dummy, D, dummy, D, dummy, 3 * D, M, 3 * D, D, None, None, None, 0, 0, 0.0, 2,
                                   D, dummy, dummy, 1e-6, 0, None, None, 0, M, 0, None, 0)
    assert rc == 8  # WDIT_ERR_SCRATCH_LIMIT, refused before any launch
