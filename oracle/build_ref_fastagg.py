"""Test infrastructure: builds the reference's own CUDA operators (getFastAgg,
the `fastAgg` pybind module) for sm_100a, as a speed point beside this
repository's attention kernels.  Nothing in the product imports the result.

The sources are copied into a temporary build directory (the reference tree is
read-only and is never copied into this repository) with two patches for the
installed PyTorch, which no longer has `Tensor::type()`: the `tensor.type()`
arguments of AT_DISPATCH_FLOATING_TYPES / AT_DISPATCH_ALL_TYPES become
`tensor.scalar_type()`, and the
CHECK_CUDA macro's `x.type().is_cuda()` becomes `x.is_cuda()`.  They are compiled
with torch's extension builder (the reference's setup.py, getFastAgg/
cuda_operators/setup.py:4-21, lists the same six sources and links curand),
for sm_100a instead of its sm_80, and the module is written to
oracle/_ref/fastAgg_ref.so.

K7/K8 (forward/backward_tgat) aggregate only the first ceil8(dst_num) edges
and K10 scales its gradient by the in-degree, so the module is a speed point
only, never a parity reference.
"""
import glob
import os
import re
import shutil
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)
from paths import REF_ROOT  # noqa: E402

SOURCES = ["operators.cpp", "aggregate_acc_kernel.cu", "aggregate_shd_kernel.cu", "edge_softmax.cu",
           "fused_attention.cu", "utils.cu"]
OUT = os.path.join(HERE, "_ref", "fastAgg_ref.so")


def build(verbose=False):
    src_dir = os.path.join(REF_ROOT, "getFastAgg", "cuda_operators")
    if not all(os.path.exists(os.path.join(src_dir, s)) for s in SOURCES):
        raise FileNotFoundError("reference CUDA operators not found under %s" % src_dir)
    from torch.utils.cpp_extension import load
    work = tempfile.mkdtemp(prefix="fastagg_ref_")
    try:
        srcs = []
        for s in SOURCES:
            with open(os.path.join(src_dir, s)) as f:
                text = f.read()
            text = re.sub(r"(AT_DISPATCH_(?:FLOATING|ALL)_TYPES)\((\w+)\.type\(\)", r"\1(\2.scalar_type()", text)
            text = text.replace(".type().is_cuda()", ".is_cuda()")
            dst = os.path.join(work, s)
            with open(dst, "w") as f:
                f.write(text)
            srcs.append(dst)
        build_dir = os.path.join(work, "build")
        os.makedirs(build_dir)
        mod = load(name="fastAgg_ref", sources=srcs, build_directory=build_dir, verbose=verbose,
                   extra_cflags=["-O3"],
                   extra_cuda_cflags=["-O3", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a"],
                   extra_ldflags=["-lcurand"])
        os.makedirs(os.path.dirname(OUT), exist_ok=True)
        built = glob.glob(os.path.join(build_dir, "fastAgg_ref*.so"))
        shutil.copyfile(built[0], OUT)
        return mod
    finally:
        shutil.rmtree(work, ignore_errors=True)


def load_built():
    """The module built above, loaded from oracle/_ref (no sources needed)."""
    import importlib.machinery
    import importlib.util
    import torch  # noqa: F401  (the module links against torch's libraries)
    loader = importlib.machinery.ExtensionFileLoader("fastAgg_ref", OUT)
    spec = importlib.util.spec_from_file_location("fastAgg_ref", OUT, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    build(verbose=True)
    print("built", OUT)
