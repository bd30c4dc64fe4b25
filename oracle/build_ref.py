"""Builds the reference's own CUDA extension into oracle/_ref (checker only).

    python oracle/build_ref.py [--force]

Test and measurement infrastructure: it compiles the reference's unmodified
source files where they lie (REFERENCE below; nothing is copied into this
repository) with the flags its setup.py gives them, for sm_100, into
oracle/_ref/ref_flashattn_C.<abi>.so. The product never loads it; the GPU
parity test and bench.py load it to run the reference kernels beside ours on
the same B200. The reference's own build system is not run: this is a
direct nvcc/g++ recipe over its few source files.

When the reference checkout is absent (as on the GPU machines) the script
does nothing; the built library travels with the source tree instead.
"""

import argparse
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
# The reference checkout: $FA_REFERENCE, else a "reference" folder beside
# this repository.
REFERENCE = os.environ.get(
    "FA_REFERENCE",
    os.path.normpath(os.path.join(HERE, os.pardir, os.pardir, "reference")))
MODULE = "ref_flashattn_C"
# setup.py:14-20 of the reference lists these sources.
SOURCES = [
    "csrc/bindings.cpp",
    "csrc/prefill.cu",
    "csrc/decode.cu",
    "csrc/legacy/legacy_ops.cu",
    "src/legacy/naive_attention.cu",
    "src/legacy/tiled_attention.cu",
    "src/legacy/fused_attention.cu",
]


def out_path():
    return os.path.join(OUT_DIR, MODULE + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def build(force=False):
    if not os.path.isdir(os.path.join(REFERENCE, "csrc")):
        print(f"build_ref: no reference checkout at {REFERENCE}; skipped")
        return None
    srcs = [os.path.join(REFERENCE, s) for s in SOURCES]
    out = out_path()
    if not force and os.path.exists(out) and all(
            os.path.getmtime(s) <= os.path.getmtime(out) for s in srcs):
        return out
    import torch
    from torch.utils import cpp_extension

    os.makedirs(OUT_DIR, exist_ok=True)
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    inc = cpp_extension.include_paths("cuda") + [sysconfig.get_paths()["include"]]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DTORCH_EXTENSION_NAME={MODULE}",
            "-DTORCH_API_INCLUDE_EXTENSION_H"]
    objs, procs = [], []
    for src in srcs:
        obj = os.path.join(OUT_DIR, os.path.basename(src) + ".o")
        objs.append(obj)
        if src.endswith(".cu"):
            cmd = [os.path.join(cuda_home, "bin", "nvcc"), "-c", src, "-o", obj,
                   "-gencode", "arch=compute_100,code=sm_100",
                   "-O3", "--use_fast_math", "-std=c++17", "-lineinfo",
                   "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
                   *cpp_extension.COMMON_NVCC_FLAGS, *defs,
                   *[f"-I{p}" for p in inc]]
        else:
            cmd = ["g++", "-c", src, "-o", obj, "-O3", "-std=c++17", "-fPIC",
                   *defs, *[f"-I{p}" for p in inc]]
        procs.append(subprocess.Popen(cmd))
    if any(p.wait() != 0 for p in procs):
        raise SystemExit("build_ref: compilation failed")
    link = ["g++", "-shared", *objs, "-o", out + ".tmp",
            *[f"-L{p}" for p in cpp_extension.library_paths("cuda")],
            "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
            "-ltorch_python", f"-L{os.path.join(cuda_home, 'lib64')}", "-lcudart"]
    subprocess.check_call(link)
    os.replace(out + ".tmp", out)
    for o in objs:
        os.remove(o)
    return out


def load():
    """Imports the built reference module (raises if it was never built)."""
    import importlib.util

    import torch  # noqa: F401  (loads libc10/libtorch first)
    spec = importlib.util.spec_from_file_location(MODULE, out_path())
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    build(ap.parse_args().force)
    sys.exit(0)
