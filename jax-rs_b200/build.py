"""Build libjaxrs_cuda.so (sm_100a) in-tree with nvcc.

Usage: python jax-rs_b200/build.py [--force] [--verbose]

Every .cu under csrc/ is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) and linked into one shared
library that exports the C ABI declared in include/jaxrs_cuda.h.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libjaxrs_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills",
    "-DJX_BUILD_LIB",
]
LINK_LIBS = ["-lcudart_static", "-ldl", "-lrt", "-lpthread"]
# Per-file flags.  layers.cu computes the reference's unfused f32 arithmetic
# and wants no contraction anywhere.
FILE_FLAGS = {"layers.cu": ["--fmad=false"]}


def _nccl_flags():
    """NCCL headers/libs: the system copy (same ABI as the wheel torch loads)."""
    inc, libdir = [], []
    for cand in ("/usr/lib/x86_64-linux-gnu/libnccl.so",):
        if os.path.exists(cand):
            libdir = ["-L" + os.path.dirname(cand)]
    return inc, libdir


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(HERE, "..", "include", "*.h")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _write_tape_prelude():
    """_build/tape_prelude.inc: the source every NVRTC-compiled op-tape kernel
    starts with -- the JX_UN_*/JX_BIN_* codes of the C ABI header followed by
    csrc/jx_math.cuh -- as a C++ string literal."""
    import re
    with open(os.path.join(HERE, "..", "include", "jaxrs_cuda.h")) as f:
        hdr = f.read()
    defines = re.findall(r"^#define (JX_(?:UN|BIN)_\w+) (\d+)", hdr, flags=re.M)
    with open(os.path.join(CSRC, "jx_math.cuh")) as f:
        math_src = f.read()
    body = "".join(f"#define {k} {v}\n" for k, v in defines) + math_src + "\n"
    out = os.path.join(BUILD, "tape_prelude.inc")
    text = 'R"JXPRELUDE(' + body + ')JXPRELUDE"\n'
    if not os.path.exists(out) or open(out).read() != text:
        with open(out, "w") as f:
            f.write(text)
    return out


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    inc, libdir = _nccl_flags()
    inc = inc + ["-I" + BUILD]
    _write_tape_prelude()
    hdrs = _headers() + [os.path.join(BUILD, "tape_prelude.inc")]
    objs = []
    jobs = []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, os.path.abspath(__file__)] + hdrs):
            cmd = [NVCC] + NVCC_FLAGS + FILE_FLAGS.get(os.path.basename(src), []) + inc + ["-c", src, "-o", obj]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            for cmd, r in ex.map(run, jobs):
                if r.returncode != 0:
                    sys.stderr.write(r.stdout + r.stderr)
                    raise RuntimeError("nvcc failed: " + cmd[-3])
                if verbose and (r.stdout or r.stderr):
                    sys.stderr.write(r.stdout + r.stderr)
    if force or jobs or _stale(LIB, objs):
        cuda_lib = os.path.join(os.path.dirname(os.path.dirname(NVCC)), "lib64")
        cmd = ([NVCC] + ARCH + ["-shared", "-o", LIB] + objs +
               ["-L" + cuda_lib, "-lnvrtc", "-Xlinker", "-rpath," + cuda_lib] + LINK_LIBS)
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
