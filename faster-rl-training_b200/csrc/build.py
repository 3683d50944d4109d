"""Build libkvs_b200.so (all kernels, sm_100a) next to the kvstreams package.

    python faster-rl-training_b200/csrc/build.py [--force] [--verbose]

Each .cu file is compiled by nvcc for sm_100a (`-gencode arch=compute_100a,code=sm_100a`),
objects go to faster-rl-training_b200/_build/, and the shared library is linked to
faster-rl-training_b200/kvstreams/libkvs_b200.so.  Up-to-date objects are reused.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG_ROOT = CSRC.parent
REPO = PKG_ROOT.parent
BUILD_DIR = PKG_ROOT / "_build"
LIB_PATH = PKG_ROOT / "kvstreams" / "libkvs_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{REPO / 'include'}",
    f"-I{CSRC}",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the kvstreams CUDA library cannot be built")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((REPO / "include").glob("*.h"))


def _compile(src: Path, force: bool, verbose: bool, extra: list[str]) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in headers()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout.strip() or r.stderr.strip()):
        print(r.stdout, r.stderr, sep="\n", flush=True)
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force or ptxas_verbose, verbose or ptxas_verbose, extra), srcs))
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args(argv)
    path = build(a.force, a.verbose, a.ptxas_verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
