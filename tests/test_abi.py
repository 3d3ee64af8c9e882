"""The C-ABI library: it loads, exports every entry point ``include/tattn.h`` declares, and its
host-side argument checks answer without touching a GPU (they run before any device call)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from tattn import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tattn.h")


def _declared() -> set[str]:
    text = open(HEADER).read()
    return set(re.findall(r"TATTN_API\s+[\w\s\*]+?\b(tattn_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def lib() -> ctypes.CDLL:
    if not os.path.exists(_lib.LIB_PATH):
        import importlib.util

        spec = importlib.util.spec_from_file_location("tattn_build", os.path.join(ROOT, "triton-attn_b200", "build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)  # type: ignore[union-attr]
        mod.build()
    return _lib.load()


def test_header_declares_the_binding(lib: ctypes.CDLL) -> None:
    declared = _declared()
    assert declared == set(_lib.SIGNATURES), declared ^ set(_lib.SIGNATURES)


def test_every_declared_symbol_is_exported(lib: ctypes.CDLL) -> None:
    for name in _declared():
        assert hasattr(lib, name), name


def test_only_the_abi_is_exported(lib: ctypes.CDLL) -> None:
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("nm unavailable")
    names = {line.split()[-1] for line in out.stdout.splitlines() if line.strip()}
    assert names == _declared()


def test_version_and_status_strings(lib: ctypes.CDLL) -> None:
    assert lib.tattn_abi_version() == _lib.ABI_VERSION
    for code in range(7):
        assert lib.tattn_status_string(code)
    assert lib.tattn_status_string(12345) == b"unknown status"
    assert lib.tattn_tile_configs(0) >= 1 and lib.tattn_tile_configs(1) >= 1
    assert lib.tattn_tile_configs(7) == 0


def _strides(*shape4: int) -> ctypes.Array:
    z, h, n, d = shape4
    st = (h * n * d, n * d, d, 1)
    return _lib.strides_array(st, st, st, st)


def test_argument_errors_need_no_device(lib: ctypes.CDLL) -> None:
    s = _strides(1, 1, 8, 24)
    bad_d = lib.tattn_fwd(16, 16, 16, 16, 16, s, 1, 1, 8, 24, 0, 0, 0.1, 0, None)
    assert bad_d == _lib.ERR_INVALID_ARGUMENT
    bad_dtype = lib.tattn_fwd(16, 16, 16, 16, 16, _strides(1, 1, 8, 16), 1, 1, 8, 16, 7, 0, 0.1, 0, None)
    assert bad_dtype == _lib.ERR_INVALID_ARGUMENT
    bad_tile = lib.tattn_bwd_dq(16, 16, 16, 16, 16, 16, 16, _strides(1, 1, 8, 16), 1, 1, 8, 16, 0, 0, 0.1, 99, None)
    assert bad_tile == _lib.ERR_INVALID_ARGUMENT
    # The self-tests validate their arguments before touching a device too.
    assert lib.tattn_selftest_exp2(None, None, None, None, -1, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.tattn_selftest_exp2_poly4(None, None, -1, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.tattn_selftest_exp2_poly4(None, None, 4, None) == _lib.ERR_INVALID_ARGUMENT
    # Empty problems are valid no-ops.
    assert lib.tattn_fwd(None, None, None, None, None, _strides(0, 1, 8, 16), 0, 1, 8, 16, 0, 0, 0.1, 0, None) == 0
    assert lib.tattn_bwd_preprocess(None, None, None, _lib.strides_array((0,) * 8), 2, 2, 0, 64, 0, None) == 0
    assert lib.tattn_selftest_exp2_poly4(None, None, 0, None) == 0


def test_layout_rules(lib: ctypes.CDLL) -> None:
    ok = lib.tattn_layout_ok
    dense = _lib.strides_array((2 * 17 * 64, 17 * 64, 64, 1))
    assert ok(256, dense, 1, 2, 17, 64) == 1
    assert ok(258, dense, 1, 2, 17, 64) == 0  # base not 16-byte aligned
    assert ok(256, _lib.strides_array((2 * 17 * 64, 17 * 64, 1, 17)), 1, 2, 17, 64) == 0  # D not unit stride
    # [B, N, H, D] transposed to [B, H, N, D]: n stride H*D, h stride D.
    assert ok(256, _lib.strides_array((5 * 70 * 16, 16, 5 * 16, 1)), 3, 5, 70, 16) == 1
    assert ok(256, _lib.strides_array((7 * 70 * 16, 20, 7 * 20, 1)), 3, 7, 70, 16) == 0  # n stride 20: not 8-aligned
    # Strides of extent-1 dims are ignored.
    assert ok(256, _lib.strides_array((3, 5, 64, 1)), 1, 1, 9, 64) == 1


def test_wait_limit_is_host_state(lib: ctypes.CDLL) -> None:
    """The bound of the kernels' waits is a host-side setting (no GPU needed to set or read it);
    0 restores the 1 s default."""
    before = lib.tattn_get_wait_limit_ns()
    try:
        assert lib.tattn_set_wait_limit_ns(2_500_000) == _lib.OK
        assert lib.tattn_get_wait_limit_ns() == 2_500_000
        assert lib.tattn_set_wait_limit_ns(0) == _lib.OK
        assert lib.tattn_get_wait_limit_ns() == 1_000_000_000
    finally:
        lib.tattn_set_wait_limit_ns(before)


def test_fused_workspace_size(lib: ctypes.CDLL) -> None:
    """tattn_bwd_fused's workspace: the fp32 dQ sums [Z, H, N, D] plus 16 bytes for its grid-barrier
    counter; -1 for dimensions the library refuses (a bad head dim, negative sizes, an overflowing
    product). Host arithmetic only."""
    for z, h, n, d in ((1, 2, 333, 64), (4, 16, 4096, 128), (3, 5, 1, 16), (0, 4, 7, 32)):
        assert lib.tattn_bwd_fused_workspace_bytes(z, h, n, d) == z * h * n * d * 4 + 16
    assert lib.tattn_bwd_fused_workspace_bytes(1, 1, 8, 48) == -1
    assert lib.tattn_bwd_fused_workspace_bytes(-1, 1, 8, 64) == -1
    assert lib.tattn_bwd_fused_workspace_bytes(1 << 30, 1 << 30, 1 << 30, 64) == -1
