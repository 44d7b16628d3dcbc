"""Failure detection on the GPU without a fault.

Every wait of the pipelined kernels is bounded (2 s): when what it waits for
never comes, the wait records SPK_DEV_PIPE_TIMEOUT and its site, the kernel
returns, and the host reads the status; the context stays usable.  The
self-test kernel waits on an mbarrier that nothing completes."""
import time

import pytest
import torch

from spikestack_lite_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_the_context_survives():
    torch.cuda.synchronize()
    _lib.device_error(clear=True)
    t0 = time.monotonic()
    _lib.check(_lib.load().spk_selftest_wait_timeout(_lib.stream_of(torch.zeros(1, device="cuda"))),
               "spk_selftest_wait_timeout")
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    site = _lib.timeout_site()
    bits = _lib.device_error(clear=True)
    assert bits & _lib.SPK_DEV_PIPE_TIMEOUT
    assert site is not None and site[0] == 0 and site[1] == 0  # block 0, warp 0
    assert 1.5 < elapsed < 60
    # the same context still computes, and the error word is clean again
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(256, 128, generator=g, device="cuda")
    w = torch.randn(256, 128, generator=g, device="cuda") / 128 ** 0.5
    y = ops.linear_act(x, w)
    ref = x.double() @ w.double().t()
    assert (y.double() - ref).abs().max().item() <= 1e-5 * ref.abs().max().item()
    assert _lib.device_error(clear=True) == 0
