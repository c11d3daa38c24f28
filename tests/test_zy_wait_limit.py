"""The bounded wait of the tensor-core kernels gives up with an error status instead of hanging:
a barrier that nothing completes is waited on for about a second, the status word records where
the wait gave up, and the context stays usable (the next launches run and check out).  The failure
is made by the wait itself (a phase that never completes); no fault, trap or endless loop.
Collected just before the allocation-free test, after the parity tests."""

import time

import pytest
import torch

import gpu_util as U
from fsctep_b200 import _native as N

pytestmark = [pytest.mark.gpu, U.needs_gpu]


def _probe(parity, where, err):
    t0 = time.monotonic()
    N.check(N.lib().fsc_bounded_wait_probe(parity, where, N.ptr(err), N.stream_ptr(err.device)), "fsc_bounded_wait_probe")
    torch.cuda.synchronize()
    return time.monotonic() - t0


def test_wait_on_a_phase_that_never_completes_ends_with_its_status():
    dev = torch.device("cuda")
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    assert _probe(1, 41, err) < 5.0 and int(err.item()) == 0  # the completed (previous) phase: at once
    dt = _probe(0, 42, err)                                      # nothing completes phase 0
    assert int(err.item()) == 42
    assert 0.2 < dt < 30.0
    # the context is usable: another launch of the library and a torch kernel run normally
    out = torch.empty(4 * 256, dtype=torch.float32, device=dev)
    flops = N.C.c_double(0.0)
    N.check(N.lib().fsc_fp32_fma_probe(1, 4, 8, N.ptr(out), N.C.byref(flops), N.stream_ptr(dev)), "fsc_fp32_fma_probe")
    x = torch.arange(1000, device=dev, dtype=torch.float32)
    torch.cuda.synchronize()
    assert float(x.sum().item()) == 499500.0 and flops.value > 0
