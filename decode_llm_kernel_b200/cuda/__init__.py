"""Drop-in for the reference's `decode_kernels.cuda` (decode_kernels/cuda/__init__.py:1-55).

Same surface: BUILD_COMMAND, is_available(), unavailable_reason(), require(),
extension_path(), build_info(), smoke_fill(). The compiled module `_ext` is the PyTorch binding
over libdecode_rope.so (include/decode_rope.h); it is built in place by BUILD_COMMAND.
There is no fallback: every op raises if the extension cannot be loaded.
"""
import glob
import os

import torch  # noqa: F401  -- loads libc10/libtorch, without which _ext's symbols do not resolve

# The reference's build command, run in this project's checkout (setup.py there builds the
# library and the binding in place; `python -m decode_llm_kernel_b200._build` does the same).
BUILD_COMMAND = "python setup.py build_ext --inplace"

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
_IMPORT_ERROR = None
try:
    from . import _ext
except (ImportError, OSError) as e:      # not built, or built against a different torch
    _ext = None
    if glob.glob(os.path.join(_PKG_DIR, "_ext*.so")):
        _IMPORT_ERROR = f"a compiled _ext exists but will not load -- {type(e).__name__}: {e}"
    else:
        _IMPORT_ERROR = f"no compiled _ext*.so in {_PKG_DIR}"


def is_available():
    return _ext is not None


def unavailable_reason():
    return _IMPORT_ERROR


def require():
    """The extension module, or a RuntimeError that says how to get one."""
    if _ext is None:
        raise RuntimeError(f"the CUDA extension is not importable -- build it with "
                           f"'{BUILD_COMMAND}' in {os.path.dirname(os.path.dirname(_PKG_DIR))}. "
                           f"Underlying error: {_IMPORT_ERROR}")
    return _ext


def extension_path():
    return getattr(_ext, "__file__", None) if _ext is not None else None


def library_path():
    """The C ABI library the extension links (lib/libdecode_rope.so)."""
    return os.path.join(os.path.dirname(_PKG_DIR), "lib", "libdecode_rope.so")


def build_info():
    """Compile-time facts from the binary, plus which binary they came from."""
    info = dict(require().build_info())
    path = extension_path()
    info["extension_path"] = path
    info["extension_mtime"] = os.path.getmtime(path) if path else None
    info["library_path"] = library_path()
    return info


def smoke_fill(tensor, value):
    return require().smoke_fill(tensor, value)


def read_status(device=None, clear=True):
    """The kernels' bounds-report word for `device` (bits DRK_STATUS_*), cleared by default.
    Synchronises the current stream, so keep it out of timed regions."""
    if device is None:
        device = torch.cuda.current_device()
    return int(require().read_status(int(device), bool(clear)))


def check_status(device=None):
    """Raises RuntimeError if any kernel on `device` saw an out-of-range index since the last
    check. This replaces the reference's device-side assert, which ends the CUDA context."""
    word = read_status(device, clear=True)
    if word:
        raise RuntimeError(f"out-of-range addressing in a RoPE/KV-append call: "
                           f"{require().status_string(word)} (status 0x{word:x})")


__all__ = ["BUILD_COMMAND", "build_info", "check_status", "extension_path", "is_available",
           "library_path", "read_status", "require", "smoke_fill", "unavailable_reason"]
