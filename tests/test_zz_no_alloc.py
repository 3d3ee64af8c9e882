"""tattn_bwd_noalloc: the backward in one call with no device allocation, for callers that cannot
provide the fp32 row buffer (delta) the three-call backward needs -- runtimes that serve every device
byte from a fixed arena, or host bindings that can only pass the buffers they were given.

The entry point keeps delta in a fixed library-owned device array (TATTN_BWD_NOALLOC_MAX_ROWS rows)
shared by every call on a GPU. These tests call it through the C ABI twice in a row, on different
problems, and compare each result with the regular entry points' (tattn_bwd_preprocess +
tattn_bwd_dkdv + tattn_bwd_dq with a caller-allocated delta), within the parity tolerances of the
GPU test-suite, and with the numpy oracle's gradients of the definition; and check that problems beyond
the limit are refused before anything runs.
This file is named so pytest collects it last.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import naive_gradients
from tattn import _lib, api

pytestmark = pytest.mark.gpu

TOL = {torch.float16: {"atol": 2e-3, "rtol": 2e-3}, torch.float32: {"atol": 1e-4, "rtol": 1e-4}}


def _case(shape, dtype, causal, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v, do = (torch.randn(shape, generator=g).to(dtype).cuda() for _ in range(4))
    scale = 1.0 / math.sqrt(shape[-1])
    o, m = api._forward(q, k, v, causal, scale)
    return q, k, v, o, do, m, scale


def _noalloc(q, k, v, o, do, m, causal, scale):
    lib = _lib.load()
    z, h, n, d = q.shape
    dq, dk, dv = (torch.empty((z, h, n, d), device=q.device, dtype=q.dtype) for _ in range(3))
    strides = _lib.strides_array(q.stride(), k.stride(), v.stride(), o.stride(), do.stride())
    code = _lib.TATTN_F16 if q.dtype == torch.float16 else _lib.TATTN_F32
    rc = lib.tattn_bwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), m.data_ptr(), strides,
        z, h, n, d, code, int(causal), scale, torch.cuda.current_stream().cuda_stream,
    )  # fmt: skip
    _lib.check("tattn_bwd_noalloc", rc)
    return dq, dk, dv


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_noalloc_matches_regular_backward_twice(dtype: torch.dtype) -> None:
    # Problems back to back: a later call must not see an earlier call's leftovers in the shared array
    # (the larger problem runs first, so stale rows exist beyond the later ones'). Sequence lengths are
    # not multiples of the kernels' 128-row blocks; D = 128 takes the D = 128 kernels through the array.
    cases = [((2, 4, 700, 64), True, 1), ((3, 2, 129, 32), False, 2), ((1, 3, 333, 128), True, 3)]
    for shape, causal, seed in cases:
        q, k, v, o, do, m, scale = _case(shape, dtype, causal, seed)
        want = api._backward(q, k, v, o, m, do, causal, scale)
        got = _noalloc(q, k, v, o, do, m, causal, scale)
        torch.cuda.synchronize()
        for g, w, name in zip(got, want, ("dq", "dk", "dv"), strict=True):
            torch.testing.assert_close(g, w, **TOL[dtype], msg=lambda s, n=name: f"{n}: {s}")
        # The same gradients against the oracle's (numpy, fp32) gradients of the definition.
        qn, kn, vn, dn = (np.ascontiguousarray(t.float().cpu().numpy()) for t in (q, k, v, do))
        for g, w, name in zip(got, naive_gradients(qn, kn, vn, dn, causal, scale), ("dq", "dk", "dv"), strict=True):
            torch.testing.assert_close(g.float().cpu(), torch.as_tensor(w), **TOL[dtype],
                                       msg=lambda s, n=name: f"{n} vs oracle: {s}")  # fmt: skip
    assert _lib.device_status() == 0


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
def test_noalloc_refuses_problems_beyond_its_buffer() -> None:
    lib = _lib.load()
    n = _lib.BWD_NOALLOC_MAX_ROWS + 1
    st = _lib.strides_array(*([(n * 64, n * 64, 64, 1)] * 5))
    # Refused on the host before any pointer is touched or anything is launched.
    rc = lib.tattn_bwd_noalloc(16, 16, 16, 16, 16, 16, 16, 16, 16, st, 1, 1, n, 64, 0, 0, 0.125, None)
    assert rc == _lib.ERR_TOO_LARGE
    assert "no-allocation" in _lib.status_string(rc)
