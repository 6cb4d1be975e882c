"""Failure handling of the bounded device-side waits, made to run out on purpose without faulting the GPU.

Every mbarrier wait of the library (the tensor-core GEMM's operand ring and accumulators, the scan's chunk copies)
polls for a bounded time, then sets a device flag, and the kernel returns through its common exit.  Here the limit
is shortened to 2 ms and a one-thread kernel waits, through that same bounded wait, on a barrier nothing arrives on
and no copy completes: the kernel must return, report that its wait gave up, sdm_device_status must answer
SDM_ERR_TIMEOUT once and SDM_OK after the flag is cleared, and the tensor-core GEMM must still compute correctly."""
import pytest
import torch

from sdmchat_b200 import _lib

pytestmark = pytest.mark.gpu

SDM_OK, SDM_ERR_TIMEOUT = 0, 4


def test_bounded_wait_gives_up_and_reports(cuda_ok):
    lib = _lib.lib()
    st = _lib.stream_ptr()
    torch.cuda.synchronize()
    assert lib.sdm_device_status(st) == SDM_OK  # nothing pending from earlier tests
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check(lib.sdm_set_wait_limit_ns(2_000_000), "sdm_set_wait_limit_ns")
    try:
        _lib.check(lib.sdm_wait_probe(_lib.ptr(done), st), "sdm_wait_probe")
        assert lib.sdm_device_status(st) == SDM_ERR_TIMEOUT  # synchronises: the probe has returned
        assert int(done.item()) == 2  # the wait gave up rather than completing
        assert lib.sdm_device_status(st) == SDM_OK  # the flag was cleared by the previous read
    finally:
        _lib.check(lib.sdm_set_wait_limit_ns(0), "sdm_set_wait_limit_ns")
    # the context is intact: a tensor-core GEMM after the timeout matches torch
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(300, 256, device="cuda", generator=g).to(torch.bfloat16)
    w = torch.randn(192, 256, device="cuda", generator=g).to(torch.bfloat16)
    y = torch.empty(300, 192, device="cuda")
    _lib.check(lib.sdm_gemm(_lib.ptr(x), _lib.ptr(w), 300, 256, 192, 1, _lib.ptr(y), st), "sdm_gemm")
    want = x.float() @ w.float().t()
    torch.testing.assert_close(y, want, atol=1e-3, rtol=1e-3)
    assert lib.sdm_device_status(st) == SDM_OK
