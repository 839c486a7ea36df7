"""Builds the native parts of fast_b200 in-tree.

  fast_b200/libfast_b200.so       C ABI + sm_100a kernels   (nvcc)
  fast_b200/_ext/fastAgg.so       drop-in fastAgg module     (g++ + libtorch)
  fast_b200/_ext/sampler_core.so  drop-in sampler_core       (g++ + libtorch)

Every target is rebuilt only when one of its sources is newer.  nvcc
cross-compiles for sm_100a, so this runs on machines without a GPU.
"""
import glob
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
INC = os.path.join(ROOT, "include")
CSRC = os.path.join(PKG, "csrc")
SHIM = os.path.join(PKG, "shim")
EXT = os.path.join(PKG, "_ext")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libfast_b200.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I" + INC]


def _newer(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + " ".join(cmd[:3]) + " ...")
    return r


def build_lib(verbose=False):
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [os.path.join(INC, "fast_b200.h")]
    os.makedirs(BUILD, exist_ok=True)
    objs, todo = [], []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        if _newer(o, [s] + hdrs):
            todo.append((s, o))
        objs.append(o)
    if todo:
        from concurrent.futures import ThreadPoolExecutor
        if verbose:
            print("nvcc", " ".join(os.path.basename(s) for s, _ in todo), flush=True)
        with ThreadPoolExecutor(max_workers=max(1, min(len(todo), os.cpu_count() or 1))) as ex:
            list(ex.map(lambda so: _run([NVCC] + NVCC_FLAGS + ["-c", so[0], "-o", so[1]]), todo))
    if _newer(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcuda"])
    return LIB


def _torch_flags():
    import torch.utils.cpp_extension as ce
    incs = ce.include_paths(device_type="cuda") if "device_type" in ce.include_paths.__code__.co_varnames \
        else ce.include_paths(cuda=True)
    flags = ["-I" + p for p in incs]
    flags += ["-I" + sysconfig.get_paths()["include"], "-I" + INC]
    for fn in ("_get_pybind11_abi_build_flags", "_get_glibcxx_abi_build_flags"):
        f = getattr(ce, fn, None)
        if f is not None:
            flags += f()
    tlib = os.path.join(os.path.dirname(ce.__file__), "..", "lib")
    tlib = os.path.abspath(tlib)
    ldflags = ["-L" + tlib, "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
               "-Wl,-rpath," + tlib, "-L" + PKG, "-lfast_b200", "-Wl,-rpath,$ORIGIN/..",
               "-L/usr/local/cuda/lib64", "-lcudart"]
    return flags, ldflags


def build_shim(name, src, verbose=False):
    os.makedirs(EXT, exist_ok=True)
    out = os.path.join(EXT, name + ".so")
    deps = [src, os.path.join(INC, "fast_b200.h"), LIB]
    if not _newer(out, deps):
        return out
    if verbose:
        print("g++", os.path.basename(src), flush=True)
    flags, ldflags = _torch_flags()
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-DTORCH_API_INCLUDE_EXTENSION_H",
           "-DTORCH_EXTENSION_NAME=" + name, "-I/usr/local/cuda/include"] + flags + [src, "-o", out] + ldflags
    _run(cmd)
    return out


def build_all(verbose=False):
    build_lib(verbose)
    build_shim("fastAgg", os.path.join(SHIM, "fastagg.cpp"), verbose)
    build_shim("sampler_core", os.path.join(SHIM, "sampler_core.cpp"), verbose)


if __name__ == "__main__":
    build_all(verbose=True)
    print("built", LIB)
