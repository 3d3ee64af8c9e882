"""Public API: ``attention(q, k, v, causal=False, sm_scale=None)`` with autograd.

Drop-in for the reference's ``src/tattn/api.py``: same signature, the same input validation and
error messages (api.py:45-56), the same default scale (api.py:182), the same autograd contract
(api.py:149-173: saves q, k, v, O and the per-row base-2 log-sum-exp M; the backward is
once-differentiable and returns no gradient for ``causal``/``sm_scale``), and the same private
``_forward`` / ``_backward`` hooks with an explicit tile ``config`` (api.py:69-146) that tests use to
check every tile variant. What changes is underneath: each kernel launch goes through the C ABI of
``libtattn_b200.so`` (include/tattn.h) to hand-written sm_100a CUDA. There is no CPU path: a
non-CUDA tensor, or a missing library, raises.
"""

from __future__ import annotations

import math
from typing import Any

import torch
from torch.autograd.function import once_differentiable

from tattn import _lib

# Explicit tile variants per kernel family; TILE_CONFIGS[kind][i] is the library's tile_cfg i + 1
# (tile_cfg 0 = the library's default for the call's (D, causal, dtype)). They stand in for the
# reference's autotune spaces (kernels.py:21-41): "BLOCK_M" is the rows a CTA owns (the forward's two
# 128-row query tiles; the backward's 128-row key or query tile), "BLOCK_N" the rows of each inner block
# it loops over, "num_stages" the depth of the TMA ring. "bwd" covers the split backward (dK/dV and dQ
# kernels); the fused backward (the default for fp16) has one shape per head dim. This copy of the library's
# table (csrc/tiles.h) is checked against tattn_tile_config_info by the CPU tests.
TILE_CONFIGS: dict[str, list[dict[str, int]]] = {
    "fwd": [
        {"BLOCK_M": 256, "BLOCK_N": 128, "num_stages": 4},
        {"BLOCK_M": 256, "BLOCK_N": 64, "num_stages": 4},
        {"BLOCK_M": 256, "BLOCK_N": 128, "num_stages": 2},
    ],
    "bwd": [
        {"BLOCK_M": 128, "BLOCK_N": 128, "num_stages": 4},
        {"BLOCK_M": 128, "BLOCK_N": 64, "num_stages": 4},
    ],
}
_KIND = {"fwd": 0, "bwd": 1}


def _check(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    """Argument validation with the reference's messages (api.py:45-56)."""
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError(
            f"expected q, k, v of equal shape [batch, heads, seq, dim]; got {q.shape}, {k.shape}, {v.shape}"
        )
    if not (q.device == k.device == v.device):
        raise ValueError(f"q, k, v must be on one device, got {q.device}, {k.device}, {v.device}")
    d = q.shape[-1]
    if d not in (16, 32, 64, 128):
        raise ValueError(f"head dim must be 16, 32, 64 or 128, got {d}")
    if not (q.dtype == k.dtype == v.dtype) or q.dtype not in (torch.float16, torch.float32):
        raise ValueError(f"q, k, v must share dtype float16 or float32, got {q.dtype}, {k.dtype}, {v.dtype}")


def cuda_available(device: torch.device) -> bool:
    """True when ``device`` is a CUDA sm_100 device and the native library loads."""
    if device.type != "cuda" or not torch.cuda.is_available():
        return False
    if torch.cuda.get_device_capability(device)[0] != 10:
        return False
    try:
        _lib.load()
    except (RuntimeError, OSError):
        return False
    return True


def triton_available(device: torch.device) -> bool:
    """Kept for API compatibility with the reference (api.py:35-42): this build has no Triton, so it
    reports whether the native sm_100 path can run on ``device``."""
    return cuda_available(device)


def _require_cuda(t: torch.Tensor) -> None:
    if t.device.type != "cuda":
        raise RuntimeError(
            f"tattn_b200 runs only on CUDA sm_100 devices (got a tensor on {t.device}); there is no CPU path"
        )


def _tile_cfg(config: dict[str, int] | None, kind: str) -> int:
    """Map a reference-style tile ``config`` (its BLOCK_M / BLOCK_N / num_stages keys; others such as
    num_warps have no meaning here) or {"tile_cfg": i} to the library's tile_cfg (0 = default)."""
    if config is None:
        return 0
    if "tile_cfg" in config:
        idx = int(config["tile_cfg"])
        if not 0 <= idx <= len(TILE_CONFIGS[kind]):
            raise ValueError(f"tile_cfg {idx} out of range for {kind}")
        return idx
    want = {key: config[key] for key in ("BLOCK_M", "BLOCK_N", "num_stages") if key in config}
    for idx, cand in enumerate(TILE_CONFIGS[kind]):
        if all(cand.get(key) == val for key, val in want.items()):
            return idx + 1
    raise ValueError(f"no {kind} tile variant matches {config}; available: {TILE_CONFIGS[kind]}")


def tile_supported(config: dict[str, int] | None, kind: str, head_dim: int) -> bool:
    """Whether the fp16 kernels of family ``kind`` can run ``config`` at ``head_dim`` (the reference
    prunes configs that do not fit its shared memory, kernels.py:44-54; here TMEM and shared memory
    decide, and an explicit config that does not fit is an error)."""
    return bool(_lib.load().tattn_tile_supported(_KIND[kind], _tile_cfg(config, kind), head_dim))


def _strides(t: torch.Tensor) -> tuple[int, ...]:
    return tuple(t.stride())


def _tma_ready(t: torch.Tensor) -> torch.Tensor:
    """fp16 tensors are read through TMA: keep them in place when the library can address them,
    otherwise make a dense, aligned copy (the reference makes such copies too, api.py:111)."""
    lib = _lib.load()
    z, h, n, d = t.shape
    if lib.tattn_layout_ok(t.data_ptr(), _lib.strides_array(_strides(t)), z, h, n, d):
        return t
    c = t.contiguous()
    if c.data_ptr() % 16 != 0:
        c = torch.empty_like(c, memory_format=torch.contiguous_format).copy_(c)
    return c


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _dtype_code(t: torch.Tensor) -> int:
    return _lib.TATTN_F16 if t.dtype == torch.float16 else _lib.TATTN_F32


def _forward(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, scale: float,
    config: dict[str, int] | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:  # fmt: skip
    """Returns (O, M): O like q (``empty_like``, api.py:87), M fp32 [Z, H, N] (api.py:88)."""
    _require_cuda(q)
    lib = _lib.load()
    z, h, n, d = q.shape
    tile = _tile_cfg(config, "fwd")
    if q.dtype == torch.float16:
        q, k, v = (_tma_ready(t) for t in (q, k, v))
    o = torch.empty_like(q)
    if q.dtype == torch.float16 and not lib.tattn_layout_ok(o.data_ptr(), _lib.strides_array(_strides(o)), z, h, n, d):
        o = torch.empty((z, h, n, d), device=q.device, dtype=q.dtype)
    m = torch.empty((z, h, n), device=q.device, dtype=torch.float32)
    strides = _lib.strides_array(_strides(q), _strides(k), _strides(v), _strides(o))
    with torch.cuda.device(q.device):
        rc = lib.tattn_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), m.data_ptr(), strides,
            z, h, n, d, _dtype_code(q), int(bool(causal)), float(scale), tile, _stream(q),
        )  # fmt: skip
    _lib.check("tattn_fwd", rc)
    return o, m


# The fp16 backward runs as one fused kernel (tattn_bwd_fused) unless this is False; the two-kernel
# path (tattn_bwd_dkdv + tattn_bwd_dq, the reference's split) is used otherwise.
FUSED_BACKWARD = True


def _backward(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, m: torch.Tensor, do: torch.Tensor,
    causal: bool, scale: float, config: dict[str, int] | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:  # fmt: skip
    """Returns contiguous (dq, dk, dv): preprocess -> dK/dV -> dQ, as api.py:102-146 (for fp16 with no
    explicit tile config: the same results from the fused backward, tattn_bwd_fused)."""
    _require_cuda(q)
    lib = _lib.load()
    z, h, n, d = q.shape
    tile = _tile_cfg(config, "bwd")
    if q.dtype == torch.float16:
        q, k, v, do, o = (_tma_ready(t) for t in (q, k, v, do.to(q.dtype), o))
    else:
        q, k, v, do, o = (t.contiguous() for t in (q, k, v, do.to(q.dtype), o))
    m = m.contiguous()
    delta = torch.empty((z, h, n), device=q.device, dtype=torch.float32)
    dq = torch.empty((z, h, n, d), device=q.device, dtype=q.dtype)
    dk = torch.empty_like(dq)
    dv = torch.empty_like(dq)
    code, stream, causal_i, sc = _dtype_code(q), _stream(q), int(bool(causal)), float(scale)
    qkvdo = _lib.strides_array(_strides(q), _strides(k), _strides(v), _strides(do))
    with torch.cuda.device(q.device):
        if FUSED_BACKWARD and config is None and code == 0:
            # One call: delta, then one kernel for dQ, dK and dV (scores and exponentials computed once);
            # dQ is summed in an fp32 workspace. Other shapes, and explicit tile configs, take the
            # reference's three-kernel path below.
            ws = torch.empty(lib.tattn_bwd_fused_workspace_bytes(z, h, n, d), device=q.device, dtype=torch.uint8)
            strides = _lib.strides_array(_strides(q), _strides(k), _strides(v), _strides(o), _strides(do))
            rc = lib.tattn_bwd_fused(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), dq.data_ptr(),
                dk.data_ptr(), dv.data_ptr(), m.data_ptr(), delta.data_ptr(), ws.data_ptr(), strides,
                z, h, n, d, code, causal_i, sc, stream,
            )  # fmt: skip
            _lib.check("tattn_bwd_fused", rc)
            return dq, dk, dv
        rc = lib.tattn_bwd_preprocess(
            o.data_ptr(), do.data_ptr(), delta.data_ptr(), _lib.strides_array(_strides(o), _strides(do)),
            z, h, n, d, code, stream,
        )  # fmt: skip
        _lib.check("tattn_bwd_preprocess", rc)
        rc = lib.tattn_bwd_dkdv(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), dk.data_ptr(), dv.data_ptr(),
            m.data_ptr(), delta.data_ptr(), qkvdo, z, h, n, d, code, causal_i, sc, tile, stream,
        )  # fmt: skip
        _lib.check("tattn_bwd_dkdv", rc)
        rc = lib.tattn_bwd_dq(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), dq.data_ptr(),
            m.data_ptr(), delta.data_ptr(), qkvdo, z, h, n, d, code, causal_i, sc, tile, stream,
        )  # fmt: skip
        _lib.check("tattn_bwd_dq", rc)
    return dq, dk, dv


class _Attention(torch.autograd.Function):
    @staticmethod
    def forward(
        ctx: Any, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, scale: float
    ) -> torch.Tensor:
        o, m = _forward(q, k, v, causal, scale)
        ctx.save_for_backward(q, k, v, o, m)
        ctx.causal, ctx.scale = causal, scale
        return o

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, do: torch.Tensor) -> tuple[torch.Tensor | None, ...]:
        q, k, v, o, m = ctx.saved_tensors
        dq, dk, dv = _backward(q, k, v, o, m, do, ctx.causal, ctx.scale)
        return dq, dk, dv, None, None


def attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False, sm_scale: float | None = None
) -> torch.Tensor:
    """Fused attention over [batch, heads, seq, dim] tensors on an sm_100 GPU (api.py:176-184)."""
    _check(q, k, v)
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    out: torch.Tensor = _Attention.apply(q, k, v, causal, scale)
    return out
