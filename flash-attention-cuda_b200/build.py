"""In-tree build of the B200 attention library and its PyTorch binding.

    python flash-attention-cuda_b200/build.py [--force]

Produces, next to the Python package so they travel with the source tree:
  flashattn_cuda/libfa_b200.so   C ABI (include/fa_b200.h), sm_100a kernels
  flashattn_cuda/_C.<abi>.so     pybind operator layer linked to the above

Both are rebuilt only when a source is newer than the output (or --force).
nvcc cross-compiles for sm_100a, so this runs on machines without a GPU.
"""

import argparse
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
PKG = os.path.join(HERE, "flashattn_cuda")
INCLUDE = os.path.join(REPO, "include")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
LIB_NAME = "libfa_b200.so"
LIB_SOURCES = ["fa_all.cu", "capi.cu", "prefill_sm100.cu", "decode_sm100.cu",
               "prefill_d128_sm100.cu", "decode_d128_sm100.cu",
               "decode_gqa_sm100.cu",
               "noalloc.cu", "legacy_sm100.cu", "host_stage.cu", "fa_sm100.cuh", "fa_kernels.h"]


def _nvcc():
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda_home, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def _stale(output, inputs):
    if not os.path.exists(output):
        return True
    out_time = os.path.getmtime(output)
    return any(os.path.getmtime(p) > out_time for p in inputs)


def _run(cmd):
    print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)


def lib_path():
    return os.path.join(PKG, LIB_NAME)


def ext_path():
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return os.path.join(PKG, "_C" + suffix)


def build_lib(force=False):
    """nvcc -> flashattn_cuda/libfa_b200.so (one translation unit)."""
    inputs = [os.path.join(CSRC, s) for s in LIB_SOURCES]
    inputs.append(os.path.join(INCLUDE, "fa_b200.h"))
    out = lib_path()
    if not force and not _stale(out, inputs):
        return out
    cmd = [_nvcc(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17",
           "-Xptxas", "-v", "-I", INCLUDE, "-Xcompiler", "-fPIC", "-shared",
           os.path.join(CSRC, "fa_all.cu"), "-o", out + ".tmp"]
    _run(cmd)
    os.replace(out + ".tmp", out)
    return out


def build_ext(force=False):
    """g++ -> flashattn_cuda/_C.<abi>.so, linked against libfa_b200.so."""
    import torch
    from torch.utils import cpp_extension

    src = os.path.join(CSRC, "bindings.cpp")
    out = ext_path()
    inputs = [src, os.path.join(INCLUDE, "fa_b200.h"), lib_path()]
    if not force and not _stale(out, inputs):
        return out
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    includes = cpp_extension.include_paths("cuda") + [
        sysconfig.get_paths()["include"], INCLUDE,
        os.path.join(cuda_home, "include")]
    libdirs = cpp_extension.library_paths("cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{p}" for p in includes], src, "-o", out + ".tmp",
           *[f"-L{p}" for p in libdirs], f"-L{PKG}", "-lfa_b200",
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
           "-ltorch_python", f"-L{os.path.join(cuda_home, 'lib64')}",
           "-lcudart", "-Wl,-rpath,$ORIGIN"]
    _run(cmd)
    os.replace(out + ".tmp", out)
    return out


def build_all(force=False):
    build_lib(force)
    build_ext(force)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    build_all(args.force)
    sys.exit(0)
