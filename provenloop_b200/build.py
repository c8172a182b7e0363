"""Build libtsgpu.so (the CUDA engine behind the C ABI in include/tsgpu.h).

Compiles every CUDA source for sm_100a only, in-tree, with plain nvcc:

    python -m provenloop_b200.build           # or __graft_entry__.build()

Host code is compiled with -ffp-contract=off so the f64 FFT tables built on
the host round exactly like the reference's (glibc cos/sin, no FMA).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libtsgpu.so")
SOURCES = ["kernels.cu", "k_ntt.cu", "k_encode.cu", "k_encrypt.cu", "k_decrypt.cu", "tsgpu.cu", "noalloc.cu"]
HEADERS = ["common.cuh", "ntt.cuh", "fft.cuh", "kernels.cuh", "launch.cuh"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def flags(verbose_ptxas: bool = False):
    f = [
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC,-ffp-contract=off,-fno-fast-math",
        "-I", os.path.join(ROOT, "include"),
    ]
    if verbose_ptxas:
        f += ["-Xptxas", "-v"]
    return f


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS] + [os.path.join(ROOT, "include", "tsgpu.h")]
    return any(os.path.getmtime(p) > t for p in deps if os.path.exists(p))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    nvcc = nvcc_path()
    objs = []
    procs = []
    # the sources compile in parallel, each kernel whole within its file (not
    # --split-compile: its partitioning of a kernel file measured 10-20 %
    # slower, run-to-run unstable code for the fused decrypt kernel)
    for s in SOURCES:
        obj = os.path.join(CSRC, s.replace(".cu", ".o"))
        cmd = [nvcc, "-c", os.path.join(CSRC, s), "-o", obj] + flags(verbose)
        procs.append((s, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
        objs.append(obj)
    for s, p in procs:
        out, err = p.communicate()
        if p.returncode != 0:
            raise RuntimeError(f"nvcc failed for {s}:\n{out}\n{err}")
        if verbose:
            sys.stdout.write(out + err)
    tmp = LIB + ".tmp"
    cmd = [nvcc, "-shared", "-o", tmp] + objs + ["-gencode", "arch=compute_100a,code=sm_100a", "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    for o in objs:
        os.remove(o)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
