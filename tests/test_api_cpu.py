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
            assert api._tile_cfg(cfg, kind) == i + 1
            assert api._tile_cfg({"tile_cfg": i + 1}, kind) == i + 1
            # the reference's config dicts carry num_warps too; it has no meaning here and is ignored
            assert api._tile_cfg({**cfg, "num_warps": 4}, kind) == i + 1
    with pytest.raises(ValueError):
        api._tile_cfg({"BLOCK_M": 3, "BLOCK_N": 5}, "fwd")
    with pytest.raises(ValueError):
        api._tile_cfg({"tile_cfg": 99}, "bwd")


def test_tile_table_matches_the_library() -> None:
    """api.TILE_CONFIGS is the library's table (csrc/tiles.h), and each family has several variants;
    the default for every fp16 (D, causal) is one of them and can run that head dim."""
    import ctypes

    from tattn import _lib

    lib = _lib.load()
    for kind, table in api.TILE_CONFIGS.items():
        k = api._KIND[kind]
        assert lib.tattn_tile_configs(k) == len(table) >= 2
        for i, cfg in enumerate(table):
            bm, bn, st = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
            assert lib.tattn_tile_config_info(k, i + 1, bm, bn, st) == _lib.OK
            assert cfg == {"BLOCK_M": bm.value, "BLOCK_N": bn.value, "num_stages": st.value}
        assert lib.tattn_tile_config_info(k, 0, bm, bn, st) == _lib.ERR_INVALID_ARGUMENT
        assert lib.tattn_tile_config_info(k, len(table) + 1, bm, bn, st) == _lib.ERR_INVALID_ARGUMENT
        for d in (16, 32, 64, 128):
            for causal in (0, 1):
                t = lib.tattn_tile_default(k, d, causal, _lib.TATTN_F16)
                assert 1 <= t <= len(table)
                assert lib.tattn_tile_supported(k, t, d) == 1
                assert lib.tattn_tile_default(k, d, causal, _lib.TATTN_F32) == 0
        # 64-row inner blocks fit every head dim; 128-row ones at D = 128 only in the forward with a
        # 2-stage ring (P written over S in TMEM; 4 stages of 128 x 128 K and V exceed shared memory)
        for i, cfg in enumerate(table):
            fits = cfg["BLOCK_N"] == 64 or (kind == "fwd" and cfg["num_stages"] <= 2)
            assert lib.tattn_tile_supported(k, i + 1, 128) == fits
            assert lib.tattn_tile_supported(k, i + 1, 64) == 1
            assert api.tile_supported(cfg, kind, 128) == fits
    assert lib.tattn_tile_default(0, 48, 0, _lib.TATTN_F16) == -1
