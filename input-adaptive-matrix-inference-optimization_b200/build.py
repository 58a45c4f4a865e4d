#!/usr/bin/env python3
"""Build libiamb200.so in-tree for sm_100a with nvcc (no JIT cache, no torch extension).

  python input-adaptive-matrix-inference-optimization_b200/build.py [--force] [-j N]

Objects go to _build/ (git-ignored); the library to lib/libiamb200.so, which travels with
the source tree to the GPU box.  CUDA runtime is linked statically; NCCL (for the
tensor-parallel path) is the one bundled with the installed torch (nvidia-nccl wheel), or
the system libnccl when that wheel is absent.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libiamb200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nccl_paths():
    try:
        import nvidia.nccl  # noqa: F401  (wheel bundled with torch)
        base = os.path.dirname(nvidia.nccl.__file__) if nvidia.nccl.__file__ else list(nvidia.nccl.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.exists(os.path.join(lib, "libnccl.so.2")):
            return inc, lib
    except Exception:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def compile_one(src, inc_nccl, force):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in headers()])
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep:
        return obj, None
    cmd = [NVCC, *ARCH, *FLAGS, "-I", os.path.join(ROOT, "include"), "-I", inc_nccl, "-c", src, "-o", obj]
    p = subprocess.run(cmd, capture_output=True, text=True)
    if p.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{' '.join(cmd)}\n{p.stdout}\n{p.stderr}")
    return obj, (p.stdout + p.stderr).strip() or None


def build(force=False, jobs=8, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    inc_nccl, lib_nccl = nccl_paths()
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(lambda s: compile_one(s, inc_nccl, force), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for o, msg in results:
            if msg:
                print(os.path.basename(o), msg)
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs,
               "-L", lib_nccl, "-l:libnccl.so.2", "-Xlinker", f"-rpath,{lib_nccl}"]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{p.stdout}\n{p.stderr}")
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.v))


if __name__ == "__main__":
    sys.exit(main())
