"""Build the library (libgck.so, CUDA for sm_100a) and the host synthesis helper (libgcksynth.so) in-tree.

    python -m goethe_engine_b200.build

nvcc cross-compiles sm_100a without a GPU. Objects go to goethe_engine_b200/_build/; the shared libraries sit next to
this file so they travel with the source tree.
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libgck.so")
SYNTH = os.path.join(HERE, "libgcksynth.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
         "-I", CSRC, "-I", os.path.join(ROOT, "include")]
SOURCES = ["runtime.cu", "k_misc.cu", "k_gemm.cu", "k_gemm_tc.cu", "k_gemv.cu", "k_attn.cu"]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build failed: {os.path.basename(cmd[-1])}")
    return r.stdout + r.stderr


def build_synth():
    src = os.path.join(CSRC, "synth.c")
    if os.path.exists(SYNTH) and os.path.getmtime(SYNTH) >= os.path.getmtime(src):
        return SYNTH
    _run(["gcc", "-O3", "-shared", "-fPIC", "-o", SYNTH, src, "-lpthread", "-lm"])
    return SYNTH


def build(verbose=False, force=False):
    os.makedirs(OUT, exist_ok=True)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(ROOT, "include", "gc.h")]
    newest = max(os.path.getmtime(p) for p in deps)
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= newest:
        build_synth()
        return LIB

    def one(src):
        obj = os.path.join(OUT, src.replace(".cu", ".o"))
        cmd = [NVCC, *ARCH, *FLAGS, "-Xptxas", "-v" if verbose else "-O3", "-c", os.path.join(CSRC, src), "-o", obj]
        log = _run(cmd)
        if verbose:
            sys.stderr.write(log)
        return obj

    with ThreadPoolExecutor(len(SOURCES)) as ex:
        objs = list(ex.map(one, SOURCES))
    _run([NVCC, *ARCH, "-shared", "-o", LIB + ".tmp", *objs, "-cudart", "static", "-lpthread"])
    os.replace(LIB + ".tmp", LIB)
    build_synth()
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
