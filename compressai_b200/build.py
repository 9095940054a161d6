"""Build recipe for the sm_100a C-ABI library ``compressai_b200/lib/libvq2_b200.so``.

Every ``csrc/*.cu`` is compiled by nvcc for ``sm_100a`` only (no PTX for other targets) and
linked into one shared library with a static CUDA runtime; the library exports only the
``vq2_*`` symbols declared in ``include/vq2_b200.h``. Object files are cached under
``compressai_b200/_build`` and rebuilt when a source or header is newer.

Usage: python -m compressai_b200.build [--force] [--jobs N]
"""
import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libvq2_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-Xptxas", "-v", "-DVQ2_BUILD"]


def nvcc():
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(p):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build compressai_b200")
    return p


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(obj, src):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(f) > t for f in [src] + _headers())


def _compile(src, force):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    log = obj + ".ptxas.txt"
    if not force and not _stale(obj, src):
        return obj, None
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    with open(log, "w") as f:
        f.write(r.stderr)
    return obj, log


def build(force=False, jobs=None):
    """Compile every csrc/*.cu for sm_100a and link lib/libvq2_b200.so. Returns the path."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = [o for o, _ in ex.map(lambda s: _compile(s, force), srcs)]
    if force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    a = ap.parse_args(argv)
    print(build(force=a.force, jobs=a.jobs))


if __name__ == "__main__":
    sys.exit(main())
