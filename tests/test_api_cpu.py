"""Host-side behaviour that needs no GPU: argument validation (same messages as the reference,
tests/test_attention.py:67-77, 134-137), the tile-config hook, and the absence of any CPU path."""

from __future__ import annotations

import pytest
import torch

from tattn import api, attention


def test_rejects_bad_inputs() -> None:
    x = torch.zeros(1, 1, 8, 16)
    with pytest.raises(ValueError, match="equal shape"):
        attention(x, x[..., :4, :], x)
    with pytest.raises(ValueError, match="head dim"):
        y = torch.zeros(1, 1, 8, 24)
        attention(y, y, y)
    with pytest.raises(ValueError, match="dtype"):
        attention(x, x.double(), x)
    with pytest.raises(ValueError, match="equal shape"):
        attention(x[0], x[0], x[0])
    with pytest.raises(ValueError, match="dtype"):
        b = x.to(torch.bfloat16)
        attention(b, b, b)


def test_rejects_mixed_devices() -> None:
    x = torch.zeros(1, 1, 8, 16)
    with pytest.raises(ValueError, match="one device"):
        attention(x, x.to("meta"), x)


def test_no_cpu_fallback() -> None:
    """A valid CPU call must raise, not silently compute on the CPU (the reference falls back to its
    tiled PyTorch path here, api.py:154-160; this build has no CPU path by design)."""
    x = torch.zeros(1, 1, 8, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        attention(x, x, x)
    with pytest.raises(RuntimeError, match="CUDA"):
        api._forward(x, x, x, False, 0.25)


def test_backend_probe_on_cpu() -> None:
    assert not api.triton_available(torch.device("cpu"))
    assert not api.cuda_available(torch.device("cpu"))


def test_tile_config_hook() -> None:
    assert api._tile_cfg(None, "fwd") == 0
    for kind, table in api.TILE_CONFIGS.items():
        for i, cfg in enumerate(table):
            assert api._tile_cfg(cfg, kind) == i
            assert api._tile_cfg({"tile_cfg": i}, kind) == i
    with pytest.raises(ValueError):
        api._tile_cfg({"BLOCK_M": 3, "BLOCK_N": 5}, "fwd")
    with pytest.raises(ValueError):
        api._tile_cfg({"tile_cfg": 99}, "bwd")
