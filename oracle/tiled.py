"""CPU oracle for the tattn attention hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference's own PyTorch implementation of the path
(amaanmithani/triton-attn, ``src/tattn/reference.py``). Only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it, and only as
the checker or the timed CPU baseline. The product path (``tattn``) never calls it: on a machine
without the CUDA library the product raises instead of falling back here.

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference's ``tiled_forward``,
``tiled_backward`` and ``naive_attention`` on seeded inputs and stored their outputs under
``tests/golden/``; ``tests/test_oracle.py`` checks this module against those fixtures.

Semantics restated here (all from ``src/tattn/reference.py``):
  * scores are scaled by ``sm_scale * log2(e)`` and exponentiated with ``exp2`` (base-2 softmax);
  * the forward returns ``M = rowmax + log2(rowsum)`` in those base-2 units, one fp32 per row;
  * the causal mask keeps ``row >= col`` (top-left aligned, equal query/key lengths);
  * the backward rebuilds ``P = exp2(S - M)`` from ``M`` and uses ``D = rowsum(dO * O)``
    computed from ``O`` as stored (fp16-rounded for fp16 inputs);
  * fp16 inputs are upcast to fp32, all arithmetic is fp32, results are cast back to the
    input dtype (``M`` stays fp32).
"""

from __future__ import annotations

import math

import numpy as np

LOG2E = 1.4426950408889634  # reference.py:15


def _scale(d: int, sm_scale: float | None) -> float:
    return sm_scale if sm_scale is not None else 1.0 / math.sqrt(d)


def naive_attention(q, k, v, causal: bool = False, sm_scale: float | None = None) -> np.ndarray:
    """fp32 materialised softmax(Q K^T * scale) V, cast to q's dtype (reference.py:18-26)."""
    scale = _scale(q.shape[-1], sm_scale)
    s = (q.astype(np.float32) @ np.swapaxes(k.astype(np.float32), -1, -2)) * np.float32(scale)
    if causal:
        n = q.shape[-2]
        s = np.where(np.triu(np.ones((n, n), dtype=bool), 1), np.float32(-np.inf), s)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(-1, keepdims=True)
    return (p @ v.astype(np.float32)).astype(q.dtype)


def naive_gradients(q, k, v, do, causal: bool = False, sm_scale: float | None = None):
    """Analytic gradients (dq, dk, dv) of ``naive_attention`` in fp32, cast to the input dtype.

    The reference's tests obtain these with torch autograd on ``naive_attention``
    (tests/test_attention.py:43-54); this is the same derivative written out:
    dV = P^T dO, dP = dO V^T, dS = P * (dP - rowsum(dP * P)), dQ = dS K * s, dK = dS^T Q * s.
    """
    scale = np.float32(_scale(q.shape[-1], sm_scale))
    qf, kf, vf, dof = (t.astype(np.float32) for t in (q, k, v, do))
    s = (qf @ np.swapaxes(kf, -1, -2)) * scale
    if causal:
        n = q.shape[-2]
        s = np.where(np.triu(np.ones((n, n), dtype=bool), 1), np.float32(-np.inf), s)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(-1, keepdims=True)
    dv = np.swapaxes(p, -1, -2) @ dof
    dp = dof @ np.swapaxes(vf, -1, -2)
    ds = p * (dp - (dp * p).sum(-1, keepdims=True))
    dq = (ds @ kf) * scale
    dk = (np.swapaxes(ds, -1, -2) @ qf) * scale
    return dq.astype(q.dtype), dk.astype(k.dtype), dv.astype(v.dtype)


def tiled_forward(
    q, k, v, causal: bool = False, sm_scale: float | None = None, block_m: int = 16, block_n: int = 16,
    row_blocks: int | None = None,
):
    """Block-by-block FlashAttention-2 forward with base-2 online softmax (reference.py:29-64).

    Returns ``(O, M)``: ``O`` in q's dtype, ``M = m_i + log2(l_i)`` fp32 of shape ``q.shape[:-1]``.
    ``row_blocks`` (bench sampling only) stops after that many query blocks; rows not reached
    are left at zero.
    """
    *batch, n, d = q.shape
    scale = np.float32(_scale(d, sm_scale) * LOG2E)
    qf, kf, vf = (t.astype(np.float32) for t in (q, k, v))
    out = np.zeros((*batch, n, d), dtype=np.float32)
    lse = np.zeros((*batch, n), dtype=np.float32)
    for bi, sm in enumerate(range(0, n, block_m)):
        if row_blocks is not None and bi >= row_blocks:
            break
        rows = np.arange(sm, min(sm + block_m, n))
        qb = qf[..., sm : sm + len(rows), :]
        m_i = np.full((*batch, len(rows)), -np.inf, dtype=np.float32)
        l_i = np.zeros((*batch, len(rows)), dtype=np.float32)
        acc = np.zeros((*batch, len(rows), d), dtype=np.float32)
        hi = min(sm + block_m, n) if causal else n  # reference.py:48: skip blocks above the diagonal
        for sn in range(0, hi, block_n):
            cols = np.arange(sn, min(sn + block_n, n))
            s = (qb @ np.swapaxes(kf[..., sn : sn + len(cols), :], -1, -2)) * scale
            if causal:
                s = np.where(rows[:, None] < cols[None, :], np.float32(-np.inf), s)
            m_new = np.maximum(m_i, s.max(-1))
            p = np.exp2(s - m_new[..., None])
            alpha = np.exp2(m_i - m_new)
            l_i = l_i * alpha + p.sum(-1)
            acc = acc * alpha[..., None] + p @ vf[..., sn : sn + len(cols), :]
            m_i = m_new
        out[..., sm : sm + len(rows), :] = acc / l_i[..., None]
        lse[..., sm : sm + len(rows)] = m_i + np.log2(l_i)
    return out.astype(q.dtype), lse


def preprocess_delta(o, do) -> np.ndarray:
    """``D = rowsum(dO * O)`` in fp32 from the stored O (reference.py:85; kernels.py:324-337)."""
    return (do.astype(np.float32) * o.astype(np.float32)).sum(-1)


def tiled_backward(
    q, k, v, o, lse, do, causal: bool = False, sm_scale: float | None = None,
    block_m: int = 16, block_n: int = 16, col_blocks: int | None = None,
):
    """FlashAttention-2 backward: P rebuilt from ``lse``, dK/dV per key block, dQ per query block
    (reference.py:67-102). Returns ``(dq, dk, dv)`` in the input dtypes.

    ``col_blocks`` (bench sampling only) stops after that many key blocks.
    """
    *_, n, d = q.shape
    sm = np.float32(_scale(d, sm_scale))
    scale = np.float32(_scale(d, sm_scale) * LOG2E)
    qf, kf, vf, dof = (t.astype(np.float32) for t in (q, k, v, do))
    delta = preprocess_delta(o, do)
    dq = np.zeros_like(qf)
    dk = np.zeros_like(kf)
    dv = np.zeros_like(vf)
    for bj, sn in enumerate(range(0, n, block_n)):
        if col_blocks is not None and bj >= col_blocks:
            break
        cols = np.arange(sn, min(sn + block_n, n))
        cs = slice(sn, sn + len(cols))
        lo = (sn // block_m) * block_m if causal else 0  # reference.py:90
        for sm_ in range(lo, n, block_m):
            rows = np.arange(sm_, min(sm_ + block_m, n))
            rs = slice(sm_, sm_ + len(rows))
            s = (qf[..., rs, :] @ np.swapaxes(kf[..., cs, :], -1, -2)) * scale
            p = np.exp2(s - lse[..., rs, None])
            if causal:
                p = np.where(rows[:, None] < cols[None, :], np.float32(0.0), p)
            dv[..., cs, :] += np.swapaxes(p, -1, -2) @ dof[..., rs, :]
            dp = dof[..., rs, :] @ np.swapaxes(vf[..., cs, :], -1, -2)
            ds = p * (dp - delta[..., rs, None])
            dk[..., cs, :] += (np.swapaxes(ds, -1, -2) @ qf[..., rs, :]) * sm
            dq[..., rs, :] += (ds @ kf[..., cs, :]) * sm
    return dq.astype(q.dtype), dk.astype(k.dtype), dv.astype(v.dtype)


def flops(b: int, h: int, n: int, d: int, causal: bool, mode: str) -> float:
    """Algorithmic FLOPs: 4*B*H*N^2*D, halved when causal, x3.5 for fwd+bwd (bench/bench.py:31-35)."""
    f = 4.0 * b * h * n * n * d
    if causal:
        f /= 2
    return f * (3.5 if mode == "fwd+bwd" else 1.0)
