"""Builds the native parts in place, for sm_100a only.

1. lib/libdecode_rope.so -- the C ABI library (include/decode_rope.h): kernels and host layer,
   compiled with nvcc -gencode arch=compute_100a,code=sm_100a, linked against the shared CUDA
   runtime so it shares one runtime with PyTorch in a process.
2. cuda/_ext*.so -- the PyTorch binding that mirrors the reference's decode_kernels.cuda._ext
   (csrc/bindings.cpp of the reference). It links libdecode_rope.so through an $ORIGIN rpath.

Objects are rebuilt only when a source or header is newer. No fast-math: the rotation must
round every multiply and add (the reference's setup.py:12-15 keeps the same policy).
"""
import glob
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB_DIR = os.path.join(PKG, "lib")
OBJ_DIR = os.path.join(ROOT, "_build", "obj")
LIB_PATH = os.path.join(LIB_DIR, "libdecode_rope.so")

CUDA_ARCH = "10.0a"
GENCODE = "-gencode=arch=compute_100a,code=sm_100a"
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", GENCODE, "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]
EXTRA_NVCC_FLAGS = os.environ.get("DECODE_NVCC_EXTRA_FLAGS", "").split()
LIB_SOURCES = ["abi.cu", "rope_kv_launch.cu", "rope_kv_attention.cu", "rope_kv_attention_tc.cu",
               "smoke.cu", "noalloc.cu", "positions.cu"]
BINDING_SOURCE = "bindings.cpp"
EXT_NAME = "_ext"


def cuda_home():
    home = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if home and os.path.exists(os.path.join(home, "bin", "nvcc")):
        return home
    return "/usr/local/cuda"


def _nvcc():
    return os.path.join(cuda_home(), "bin", "nvcc")


def _headers():
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n"
                           f"{proc.stdout}\n{proc.stderr}")
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout + proc.stderr, file=sys.stderr)
    return proc


def build_library(force=False, verbose=False, ptxas_verbose=False):
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    headers = _headers()
    flags = NVCC_FLAGS + EXTRA_NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else [])

    def compile_one(src):
        path = os.path.join(CSRC, src)
        obj = os.path.join(OBJ_DIR, os.path.splitext(src)[0] + ".o")
        if force or ptxas_verbose or _stale(obj, [path] + headers):
            _run([_nvcc()] + flags + ["-I", INCLUDE, "-I", CSRC, "-c", path, "-o", obj],
                 verbose or ptxas_verbose)
        return obj

    with ThreadPoolExecutor(max_workers=len(LIB_SOURCES)) as pool:
        objs = list(pool.map(compile_one, LIB_SOURCES))
    if force or _stale(LIB_PATH, objs):
        _run([_nvcc(), GENCODE, "-shared", "--cudart", "shared", "-o", LIB_PATH] + objs,
             verbose)
    return LIB_PATH


def extension_path():
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return os.path.join(PKG, "cuda", EXT_NAME + suffix)


def build_extension(force=False, verbose=False):
    """Compiles cuda/bindings.cpp against PyTorch's headers with the host compiler."""
    import torch
    from torch.utils import cpp_extension

    out = extension_path()
    src = os.path.join(CSRC, BINDING_SOURCE)
    if not force and not _stale(out, [src, LIB_PATH] + _headers()):
        return out
    os.makedirs(OBJ_DIR, exist_ok=True)
    includes = cpp_extension.include_paths(device_type="cuda") + [
        sysconfig.get_paths()["include"], INCLUDE, CSRC, os.path.join(cuda_home(), "include")]
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cxx = "g++"
    obj = os.path.join(OBJ_DIR, "bindings.o")
    _run([cxx, "-O2", "-fPIC", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
          "-DTORCH_EXTENSION_NAME=" + EXT_NAME, "-DTORCH_API_INCLUDE_EXTENSION_H",
          "-fvisibility=hidden", "-c", src, "-o", obj] + [f"-I{p}" for p in includes], verbose)
    rel = os.path.relpath(LIB_DIR, os.path.dirname(out))
    _run([cxx, "-shared", "-o", out, obj, f"-L{LIB_DIR}", "-ldecode_rope",
          f"-Wl,-rpath,$ORIGIN/{rel}", f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch",
          "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
          f"-L{os.path.join(cuda_home(), 'lib64')}", "-lcudart"], verbose)
    return out


def build(force=False, verbose=False):
    lib = build_library(force=force, verbose=verbose)
    ext = build_extension(force=force, verbose=verbose)
    return lib, ext


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
