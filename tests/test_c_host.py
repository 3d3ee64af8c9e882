"""The C ABI from a plain-C host (tests/c_host/attention_from_c.c): no Python or PyTorch between the caller
and the library, as for a cgo, JNI or C plugin binding (include/tattn.h is the whole interface).

Without a GPU: the program compiles as C99 with warnings as errors and links against the library and the
CUDA runtime. On a GPU: it runs the forward and the fused backward through the ABI on three cases and
checks them against its own double-precision attention (O and gradients within 2e-3 + 2e-3 |ref|, M
within 1e-3)."""

from __future__ import annotations

import os
import shutil
import subprocess

import pytest

from tattn import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c_host", "attention_from_c.c")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _library() -> str:
    if not os.path.exists(_lib.LIB_PATH):
        import importlib.util

        spec = importlib.util.spec_from_file_location("tattn_build", os.path.join(ROOT, "triton-attn_b200", "build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)  # type: ignore[union-attr]
        mod.build()
    return _lib.LIB_PATH


def _compile(out: str) -> None:
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    libdir = os.path.dirname(_library())
    cudalib = os.path.join(CUDA, "lib64")
    cmd = [cc, "-std=c99", "-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), SRC, "-o", out, "-L", libdir, "-ltattn_b200", "-L", cudalib,
           "-lcudart", "-lm", f"-Wl,-rpath,{libdir}:{cudalib}"]  # fmt: skip
    p = subprocess.run(cmd, capture_output=True, text=True)
    assert p.returncode == 0, p.stdout + p.stderr


def test_c_host_builds(tmp_path) -> None:
    _compile(str(tmp_path / "attention_from_c"))


@pytest.mark.gpu
def test_c_host_runs_against_its_own_reference(tmp_path) -> None:
    exe = str(tmp_path / "attention_from_c")
    _compile(exe)
    p = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(p.stdout)
    assert p.returncode == 0, p.stdout + p.stderr
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("case ")]
    assert len(lines) == 3 and all(ln.endswith(" ok") for ln in lines), p.stdout
