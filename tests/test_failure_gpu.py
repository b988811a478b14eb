"""Failure detection without a GPU fault: a bounded on-device wait that runs out.

The self-test kernel waits on an mbarrier nothing arrives at, with a 2 ms limit.  The wait
gives up, records the device error flag and returns; swa_check_device reports
SWA_ERR_DEVICE_TIMEOUT once, clears the flag, and the next attention call works normally.
"""
import pytest
import torch

from tests._pkg import pkg, submodule

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    L = submodule("_lib")
    lib = L.lib()
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream(dev).cuda_stream
    assert lib.swa_check_device(stream) == L.SWA_OK
    assert lib.swa_selftest_wait_timeout(2000, stream) == L.SWA_OK
    assert lib.swa_check_device(stream) == L.SWA_ERR_DEVICE_TIMEOUT
    assert lib.swa_check_device(stream) == L.SWA_OK          # flag was cleared
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 2, 64, 32, generator=g).to(torch.bfloat16).to(dev)
    o = pkg().flash_swda_with_sink(q, q, q, 16, 2)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all()
    assert lib.swa_check_device(stream) == L.SWA_OK


def test_selftest_rejects_bad_limits():
    L = submodule("_lib")
    assert L.lib().swa_selftest_wait_timeout(0, None) == L.SWA_ERR_INVALID_ARG
    assert L.lib().swa_selftest_wait_timeout(10**7, None) == L.SWA_ERR_INVALID_ARG


def _small(dev):
    g = torch.Generator().manual_seed(1)
    return torch.randn(1, 2, 64, 32, generator=g).to(torch.bfloat16).to(dev)


def test_timeout_raises_on_the_next_api_call_instead_of_returning_zeros():
    L = submodule("_lib")
    dev = torch.device("cuda:0")
    q = _small(dev)
    L.selftest_wait_timeout(2000, dev)      # a launch whose bounded wait gives up
    torch.cuda.synchronize()
    with pytest.raises(L.SwaDeviceTimeout):
        pkg().flash_swda_with_sink(q, q, q, 16, 2)
    # the flag was cleared by the raise: the next call computes normally
    o = pkg().flash_swda_with_sink(q, q, q, 16, 2)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all() and o.abs().sum() > 0
    assert L.lib().swa_check_device(torch.cuda.current_stream(dev).cuda_stream) == L.SWA_OK


def test_timeout_from_a_raw_launch_is_reported_one_call_later():
    # a timeout the Python layer did not poll (raw C-ABI call): the next API call's own
    # kernels skip their work, its poll sees the flag, and the call after it raises
    L = submodule("_lib")
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream(dev).cuda_stream
    q = _small(dev)
    assert L.lib().swa_selftest_wait_timeout(2000, stream) == L.SWA_OK
    pkg().flash_swda_with_sink(q, q, q, 16, 2)
    torch.cuda.synchronize()
    with pytest.raises(L.SwaDeviceTimeout):
        pkg().flash_swda_with_sink(q, q, q, 16, 2)
    o = pkg().flash_swda_with_sink(q, q, q, 16, 2)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all() and o.abs().sum() > 0
