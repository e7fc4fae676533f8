"""Build the sm_100a C-ABI library `libw8a8_b200.so` in-tree with nvcc.

Every `csrc/*.cu` is compiled for `arch=compute_100a,code=sm_100a` (nvcc
cross-compiles without a GPU) into `_build/*.o`, and linked into
`libw8a8_b200.so` next to this file, where `_lib.py` loads it.  Objects are
rebuilt when their source or any header under `csrc/` or `include/` is newer.

usage: python gemma-npu_b200/build.py [--force] [--verbose-ptxas]
"""
import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libw8a8_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
              f"-I{INCLUDE}"]


def nvcc_path():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def build(force=False, verbose_ptxas=False, quiet=False):
    """Compile and link; returns the path of the shared library."""
    os.makedirs(BUILD, exist_ok=True)
    nvcc = nvcc_path()
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    hdr_time = _newest(headers)
    objs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_time):
            continue
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        if not quiet:
            print("[build]", os.path.basename(src), flush=True)
        subprocess.run(cmd, check=True)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        tmp = LIB + ".tmp"
        subprocess.run([nvcc, *ARCH, "-shared", "-o", tmp, *objs], check=True)
        os.replace(tmp, LIB)
        if not quiet:
            print("[build] linked", LIB, flush=True)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args(argv)
    build(force=a.force, verbose_ptxas=a.verbose_ptxas)


if __name__ == "__main__":
    sys.exit(main())
