"""Bounded waits on a B200: a wait that runs out is reported, not hung on.

Every mbarrier wait in the tensor-core kernels gives up after the wait limit (1 s by default, set with
tattn_set_wait_limit_ns); the CTA then records TATTN_DEV_WAIT_TIMEOUT in the device status word,
drains its own work, frees its TMEM and exits. tattn_selftest_wait runs that path on purpose: its
first wait is on a barrier that nothing completes. These tests make that wait run out after a few
milliseconds, read the status bit, clear it, and check that the GPU and the context are still usable
by running attention right after. Nothing here faults or hangs the GPU: the wait itself gives up.
"""

from __future__ import annotations

import math
import time

import numpy as np
import pytest
import torch

from oracle import naive_attention, naive_gradients
from tattn import _lib, attention

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _restore_limit():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    lib = _lib.load()
    before = lib.tattn_get_wait_limit_ns()
    yield lib
    lib.tattn_set_wait_limit_ns(before)


def test_short_wait_limit_runs_out_and_is_reported(_restore_limit) -> None:
    lib = _restore_limit
    assert _lib.device_status() == 0
    lib.tattn_set_wait_limit_ns(2_000_000)  # 2 ms
    assert lib.tattn_get_wait_limit_ns() == 2_000_000
    t0 = time.perf_counter()
    _lib.check("tattn_selftest_wait", lib.tattn_selftest_wait(None))
    status = _lib.device_status(clear=False)  # synchronises: the kernel has returned
    elapsed = time.perf_counter() - t0
    assert status & _lib.DEV_WAIT_TIMEOUT, status
    assert elapsed < 5.0, elapsed  # gave up after ~2 ms, not the 1 s default
    assert _lib.device_status() == status  # read and clear
    assert _lib.device_status() == 0


def test_default_limit_is_restored_by_zero(_restore_limit) -> None:
    lib = _restore_limit
    lib.tattn_set_wait_limit_ns(12345)
    lib.tattn_set_wait_limit_ns(0)
    assert lib.tattn_get_wait_limit_ns() == 1_000_000_000


def test_context_stays_usable_after_a_wait_ran_out(_restore_limit) -> None:
    lib = _restore_limit
    lib.tattn_set_wait_limit_ns(1_000_000)
    _lib.check("tattn_selftest_wait", lib.tattn_selftest_wait(None))
    assert _lib.device_status() & _lib.DEV_WAIT_TIMEOUT
    lib.tattn_set_wait_limit_ns(0)
    # A normal forward + backward right after, on the same context, with the default limit.
    g = torch.Generator().manual_seed(5)
    shape = (1, 2, 300, 64)
    q, k, v, do = (torch.randn(shape, generator=g).half().cuda() for _ in range(4))
    qg, kg, vg = (t.clone().requires_grad_() for t in (q, k, v))
    out = attention(qg, kg, vg, causal=True)
    out.backward(do)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    qn, kn, vn, dn = (t.float().cpu().numpy() for t in (q, k, v, do))
    scale = 1.0 / math.sqrt(64)
    tol = {"atol": 2e-3, "rtol": 2e-3}
    torch.testing.assert_close(out.detach().float().cpu(), torch.as_tensor(naive_attention(qn, kn, vn, True, scale)), **tol)
    for t, w in zip((qg, kg, vg), naive_gradients(qn, kn, vn, dn, True, scale), strict=True):
        torch.testing.assert_close(t.grad.float().cpu(), torch.as_tensor(np.asarray(w)), **tol)
