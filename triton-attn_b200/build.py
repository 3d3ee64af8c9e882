"""Build the tattn_b200 CUDA library in-tree: ``triton-attn_b200/tattn/libtattn_b200.so``.

Every ``csrc/*.cu`` is compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``) with
nvcc, then linked into one shared library with a static CUDA runtime. Only the ``tattn_*`` C entry
points of ``include/tattn.h`` are exported. Objects go to ``triton-attn_b200/_build/``; a file is
rebuilt when it or any header is newer than its object. ``-Xptxas -v`` output (registers, spills,
shared memory per kernel) is kept in ``_build/ptxas.log``.

    python triton-attn_b200/build.py [--force] [-j N]
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "tattn", "libtattn_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "--expt-relaxed-constexpr", "-Xptxas", "-v", "-I", os.path.join(ROOT, "include")]  # fmt: skip


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the tattn_b200 library needs the CUDA toolkit to build")


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + [
        os.path.join(ROOT, "include", "tattn.h")
    ]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, jobs: int = 0, verbose: bool = False) -> str:
    """Compile and link; returns the library path. Raises RuntimeError with nvcc's output on failure."""
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = _headers()
    cc = nvcc()

    def compile_one(src: str) -> tuple[str, str]:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        if not force and not _stale(obj, [src, *headers]):
            return obj, ""
        cmd = [cc, *ARCH, *CFLAGS, "-c", src, "-o", obj]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{' '.join(cmd)}\n{p.stdout}\n{p.stderr}")
        with open(obj[:-2] + ".ptxas.log", "w") as f:  # per source, so ptxas.log covers every object
            f.write(p.stdout + p.stderr)
        return obj, p.stdout + p.stderr

    workers = jobs or min(len(sources), os.cpu_count() or 1)
    with ThreadPoolExecutor(max_workers=max(1, workers)) as ex:
        results = list(ex.map(compile_one, sources))
    objs = [o for o, _ in results]
    logs = ""
    for o in objs:
        lp = o[:-2] + ".ptxas.log"
        if os.path.exists(lp):
            with open(lp) as f:
                logs += f.read()
    with open(os.path.join(BUILD, "ptxas.log"), "w") as f:
        f.write(logs)
    if verbose and logs:
        print(logs)
    if force or _stale(LIB, objs):
        exports = os.path.join(BUILD, "exports.map")
        with open(exports, "w") as f:
            f.write("{ global: tattn_*; local: *; };\n")
        cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs,
               "-Xlinker", f"--version-script={exports}"]  # fmt: skip
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{p.stdout}\n{p.stderr}")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=0)
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    try:
        print(build(args.force, args.jobs, args.verbose))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)


if __name__ == "__main__":
    main()
