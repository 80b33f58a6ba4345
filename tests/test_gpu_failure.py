"""Failure detection on the device without a GPU fault: every libnk kernel
waits on its barriers with a time limit, records NK_TIMEOUT in the device
error word when the limit runs out, and returns.  nk_selftest_wait_timeout
launches one such wait that nothing completes; the host then reads the
status through nk_device_status, and the context stays usable."""
import time

import pytest
import torch

import nk

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(cuda):
    nk.device_status()  # no error pending
    t0 = time.monotonic()
    nk.call("nk_selftest_wait_timeout", nk.stream_ptr())
    with pytest.raises(nk.NkError) as e:
        nk.device_status()
    elapsed = time.monotonic() - t0
    assert e.value.code == nk.TIMEOUT
    assert 1.0 < elapsed < 60.0
    nk.device_status()  # reading the status cleared it
    # the context still runs kernels: a projection after the timeout
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(40, 256, device="cuda", generator=g).bfloat16()
    w = (torch.randn(384, 256, device="cuda", generator=g) * 0.05).bfloat16()
    y = nk.gemm(x, w, out_dtype=torch.float32)
    ref = x.float() @ w.float().t()
    torch.cuda.synchronize()
    assert (y - ref).abs().max().item() <= 1e-3 * ref.abs().max().item()
    nk.device_status()
