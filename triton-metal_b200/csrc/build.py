"""Build libb2.so (all CUDA sources in this folder) for sm_100a with nvcc,
then the Python binding _b2fast (torch_bind.cpp) that calls into it.

Usage: python build.py [--force] [-j N]
Objects go to ../_build/, the libraries to ../b200kern/.
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), "b200kern")
BUILD = os.path.join(os.path.dirname(HERE), "_build")
LIB = os.path.join(PKG, "libb2.so")
BIND_SRC = os.path.join(HERE, "torch_bind.cpp")
BIND = os.path.join(PKG, "_b2fast.so")
INCLUDE = os.path.join(os.path.dirname(os.path.dirname(HERE)), "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17", "--use_fast_math",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", INCLUDE,
]


def sources():
    return sorted(f for f in os.listdir(HERE) if f.endswith(".cu"))


def _deps_mtime(src):
    paths = [os.path.join(HERE, src)]
    paths += [os.path.join(HERE, f) for f in os.listdir(HERE) if f.endswith(".cuh")]
    paths.append(os.path.join(INCLUDE, "b2.h"))
    return max(os.path.getmtime(p) for p in paths)


def compile_one(src, force, verbose):
    obj = os.path.join(BUILD, src[:-3] + ".o")
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= _deps_mtime(src):
        return obj
    cmd = [NVCC, *FLAGS, "-c", os.path.join(HERE, src), "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose:
        sys.stderr.write(r.stderr)
    return obj


def build(force=False, jobs=8, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force, verbose), sources()))
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs,
           "-o", LIB, "-lcuda", "-Xcompiler", "-fPIC"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def build_binding(force=False):
    """_b2fast.so: the C++ argument handling of the per-layer decode call,
    linked against libb2.so (found next to it at run time) and libtorch."""
    deps = [BIND_SRC, LIB, os.path.join(INCLUDE, "b2.h")]
    if not force and os.path.exists(BIND) and os.path.getmtime(BIND) >= max(os.path.getmtime(p) for p in deps):
        return BIND
    import sysconfig
    import torch
    from torch.utils import cpp_extension as ce
    incs = ce.include_paths() + [sysconfig.get_paths()["include"], "/usr/local/cuda/include", INCLUDE]
    libdirs = ce.library_paths()
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", BIND_SRC, "-o", BIND,
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           "-DTORCH_EXTENSION_NAME=_b2fast", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    cmd += [f"-I{d}" for d in incs] + [f"-L{d}" for d in libdirs]
    cmd += [f"-Wl,-rpath,{d}" for d in libdirs]
    cmd += ["-L" + PKG, "-lb2", "-Wl,-rpath,$ORIGIN",
            "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"binding build failed:\n{r.stdout}\n{r.stderr}")
    return BIND


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true", help="print -Xptxas -v resource usage")
    a = ap.parse_args()
    print(build(a.force, a.j, a.v))
    print(build_binding(a.force))
