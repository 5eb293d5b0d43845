"""Failure detection without a GPU fault: a device-side wait on a flag that nothing sets runs
out after the (shortened) wait limit, the kernel records a timeout in the library's error
record and returns, the host reads the record, and the context stays usable."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(pkg):
    lib = pkg._lib
    lib.read_error(clear=True)
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")  # never set
    lib.call("wdit_set_wait_limit_ns", 50_000_000)  # 50 ms
    try:
        lib.call("wdit_wait_selftest", flag.data_ptr(), lib.stream_ptr())
        err = lib.read_error(clear=True)
    finally:
        lib.call("wdit_set_wait_limit_ns", 2_000_000_000)
    assert err[0] == 0x7117 and err[1] == 8, err
    # the context is still usable: a fused GEMM runs and is correct afterwards
    a = torch.randn(256, 512, device="cuda").to(torch.bfloat16)
    w = (0.02 * torch.randn(512, 512, device="cuda")).to(torch.bfloat16)
    out = pkg.ops.gemm_act(a, w)
    ref = a.float() @ w.float().t()
    assert ((out.float() - ref).norm() / ref.norm()).item() < 5e-3
    assert lib.read_error(clear=True) == (0, 0, 0, 0)


def test_wait_selftest_passes_when_flag_is_set(pkg):
    lib = pkg._lib
    flag = torch.ones(4, dtype=torch.int32, device="cuda")
    lib.call("wdit_wait_selftest", flag.data_ptr(), lib.stream_ptr())
    assert lib.read_error(clear=True) == (0, 0, 0, 0)


def test_p2p_arrival_wait_reports_the_missing_rank(pkg):
    """The NVLink exchange's arrival wait on one GPU: rank 1 never publishes epoch 3, so the
    bounded wait gives up, records {timeout, site 9, rank 1, epoch 3} and returns."""
    lib = pkg._lib
    lib.read_error(clear=True)
    flags = torch.tensor([3, 2, 3, 3], dtype=torch.int32, device="cuda")  # rank 1 is one epoch behind
    lib.call("wdit_set_wait_limit_ns", 50_000_000)
    try:
        lib.call("wdit_p2p_wait", flags.data_ptr(), 4, 3, lib.stream_ptr())
        err = lib.read_error(clear=True)
        flags[1] = 3
        lib.call("wdit_p2p_wait", flags.data_ptr(), 4, 3, lib.stream_ptr())  # everyone arrived: no error
        ok = lib.read_error(clear=True)
    finally:
        lib.call("wdit_set_wait_limit_ns", 2_000_000_000)
    assert err == (0x7117, 9, 1, 3), err
    assert ok == (0, 0, 0, 0)
