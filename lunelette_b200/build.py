"""Build lunelette_b200/liblunelette_cuda.so in-tree.

    python -m lunelette_b200.build [--force] [--jobs N]

CUDA sources compile for sm_100a only (nvcc -gencode arch=compute_100a,code=sm_100a
-lineinfo); host C compiles with the system gcc as C11. Objects live in
lunelette_b200/_build/. Symbols are hidden except the public C-ABI.
"""
import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBRARY = os.path.join(HERE, "liblunelette_cuda.so")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
CC = "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"
CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"

C_SOURCES = ["st.c", "weights.c", "runtime.c", "synth.c", "batch.c"]
CU_SOURCES = ["device.cu", "kernels.cu", "kernel_api.cu", "noalloc.cu", "mega.cu", "prefill.cu"]
INCLUDES = ["-I" + os.path.join(REPO, "include"), "-I" + CSRC, "-I" + os.path.join(CUDA_HOME, "include")]
CFLAGS = ["-std=c11", "-O2", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wextra",
          "-Wno-unused-parameter"]
NVFLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
           "-ccbin", CXX, "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
           "-Xptxas", "-v"]


def _headers():
    out = []
    for d in (CSRC, os.path.join(REPO, "include")):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh")):
                out.append(os.path.join(d, f))
    return out


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, force, verbose):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    deps = [src] + _headers()
    if not force and not _stale(obj, deps):
        return obj, ""
    if src.endswith(".cu"):
        cmd = [NVCC] + NVFLAGS + INCLUDES + ["-c", src, "-o", obj]
    else:
        cmd = [CC] + CFLAGS + INCLUDES + ["-c", src, "-o", obj]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    log = proc.stdout + proc.stderr
    if proc.returncode != 0:
        raise RuntimeError("compile failed: %s\n%s" % (" ".join(cmd), log))
    return obj, log if verbose else ""


def build(force=False, jobs=None, verbose=False):
    """Compile and link the library; returns its path."""
    if not os.path.exists(NVCC):
        raise RuntimeError("nvcc not found at %s" % NVCC)
    os.makedirs(BUILD, exist_ok=True)
    sources = [os.path.join(CSRC, s) for s in C_SOURCES + CU_SOURCES]
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as pool:
        results = list(pool.map(lambda s: _compile(s, force, verbose), sources))
    objects = [r[0] for r in results]
    for _, log in results:
        if log:
            sys.stdout.write(log)
    if force or _stale(LIBRARY, objects):
        tmp = LIBRARY + ".tmp"
        cmd = [NVCC, "-shared", "-ccbin", CXX, "-gencode", "arch=compute_100a,code=sm_100a",
               "-o", tmp] + objects + ["-lpthread", "-lm"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError("link failed: %s\n%s" % (" ".join(cmd), proc.stdout + proc.stderr))
        os.replace(tmp, LIBRARY)
    return LIBRARY


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    args = ap.parse_args()
    print(build(args.force, args.jobs, args.verbose))


if __name__ == "__main__":
    main()
