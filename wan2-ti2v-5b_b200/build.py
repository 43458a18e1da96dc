"""Build libwanb200.so in-tree with nvcc for sm_100a (no torch extension machinery).

    python wan2-ti2v-5b_b200/build.py [--force]

The shared library lands next to this file (wanb200/libwanb200.so) so it travels with the
repository snapshot.  Objects are cached under _build/ and rebuilt when a source or header is
newer.
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "wanb200", "libwanb200.so")
BUILD = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", os.path.join(ROOT, "include")]


def _newest(paths):
    return max(os.path.getmtime(p) for p in paths)


def build(force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    hdr_time = _newest(headers) if headers else 0
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_time):
            cmd = [NVCC] + ARCH + FLAGS + ["-c", s, "-o", o]
            if verbose:
                cmd += ["-Xptxas", "-v"]
            print(" ".join(cmd), flush=True)
            subprocess.check_call(cmd)
    if force or not os.path.exists(OUT) or os.path.getmtime(OUT) < _newest(objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", OUT] + objs
        print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
