"""Build libvqb200.so in-tree with nvcc for sm_100a (no torch extension).

    python -m vqlab_b200.build            # incremental
    python -m vqlab_b200.build --force

Each csrc/*.cu is compiled to an object under vqlab_b200/_build/ (in
parallel), then linked into vqlab_b200/libvqb200.so with the static CUDA
runtime, so the library carries no torch or libcudart version dependency.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libvqb200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                     "--expt-relaxed-constexpr", "-I", str(ROOT / "include")]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and pathlib.Path(c).exists():
            return c
    raise RuntimeError("nvcc not found: the B200 runtime needs the CUDA toolkit to build")


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((ROOT / "include").glob("*.h"))


def _stale(target: pathlib.Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> pathlib.Path:
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    hdrs = _headers()
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_v else []

    def compile_one(src: pathlib.Path):
        obj = BUILD / (src.stem + ".o")
        if force or _stale(obj, [src] + hdrs):
            cmd = [cc] + NVCC_FLAGS + extra + ["-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
            if ptxas_v or verbose:
                sys.stderr.write(r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(compile_one, srcs))
    if force or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [cc] + ARCH + ["-shared", "-cudart", "static", "-o", str(tmp)] + [str(o) for o in objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, ptxas_v=a.ptxas_v))
    return 0


if __name__ == "__main__":
    sys.exit(main())
