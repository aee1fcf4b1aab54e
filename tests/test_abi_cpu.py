"""The C ABI library on a machine without a GPU: it loads, exports every symbol the public
header declares, and its host-side checks reject bad arguments with the reference's messages
before any CUDA call."""
import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "decode_rope.h")
LIB = os.path.join(ROOT, "decode_llm_kernel_b200", "lib", "libdecode_rope.so")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"DRK_API\s+[\w\s\*]+?\b(drk_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    assert os.path.exists(LIB), "build the library first (python -m decode_llm_kernel_b200._build)"
    return ctypes.CDLL(LIB)


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    for needed in ("drk_fused_rope_kv_append", "drk_rope_forward", "drk_kv_append",
                   "drk_smoke_fill", "drk_build_info", "drk_last_error"):
        assert needed in syms


def test_every_declared_symbol_is_exported(lib):
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert missing == []


class DrkTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("device", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("sizes", ctypes.c_int64 * 4), ("strides", ctypes.c_int64 * 4)]


CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3,
         torch.int32: 4, torch.int64: 5}


def desc(t, device=0):
    d = DrkTensor()
    d.data = t.data_ptr()
    d.dtype = CODES[t.dtype]
    d.ndim = t.dim()
    d.device = device
    for i in range(t.dim()):
        d.sizes[i] = t.size(i)
        d.strides[i] = t.stride(i)
    return d


def call_fused(lib, q, k, v, pos, cos, sin, kc, vc, ri, q_out, devices=None):
    devices = devices or {}
    ds = [desc(t, devices.get(name, 0)) for name, t in
          (("q", q), ("k", k), ("v", v), ("positions", pos), ("cos", cos), ("sin", sin),
           ("k_cache", kc), ("v_cache", vc), ("request_indices", ri), ("q_out", q_out))]
    fn = lib.drk_fused_rope_kv_append
    fn.restype = ctypes.c_int
    rc = fn(*[ctypes.byref(d) for d in ds], None, None)
    lib.drk_last_error.restype = ctypes.c_char_p
    return rc, lib.drk_last_error().decode()


def args(T=2, Hq=4, Hkv=2, D=8, B=2, S=4, dtype=torch.bfloat16):
    q = torch.zeros(T, Hq, D, dtype=dtype)
    k = torch.zeros(T, Hkv, D, dtype=dtype)
    v = torch.zeros(T, Hkv, D, dtype=dtype)
    pos = torch.zeros(T, dtype=torch.int64)
    cos = torch.zeros(S, D)
    sin = torch.zeros(S, D)
    kc = torch.zeros(B, S, Hkv, D, dtype=dtype)
    vc = torch.zeros(B, S, Hkv, D, dtype=dtype)
    ri = torch.zeros(T, dtype=torch.int64)
    q_out = torch.zeros(T, Hq, D, dtype=dtype)
    return [q, k, v, pos, cos, sin, kc, vc, ri, q_out]


@pytest.mark.parametrize("mutate,devices,expect", [
    (lambda a: a, {"cos": -1}, "cos must be a CUDA tensor, got cpu"),
    (lambda a: a, {"k": 1}, "k is on cuda:1 but the operation runs on cuda:0"),
    (lambda a: a.__setitem__(4, a[4].half()) or a, {}, "must be FP32"),
    (lambda a: a.__setitem__(6, a[6].float()) or a, {}, "must match its source dtype"),
    (lambda a: a.__setitem__(7, a[6]) or a, {}, "distinct buffers"),
    (lambda a: a.__setitem__(8, a[8].int()) or a, {}, "must share a dtype"),
    (lambda a: a.__setitem__(3, a[3].float()) or a, {}, "must be int32 or int64"),
    (lambda a: a.__setitem__(0, torch.zeros(2, 4, 7, dtype=torch.bfloat16)) or a, {},
     "head_dim must be even"),
    (lambda a: a.__setitem__(4, torch.zeros(4, 6)) or a.__setitem__(5, torch.zeros(4, 6)) or a,
     {}, "does not match q/k head_dim"),
    (lambda a: a.__setitem__(6, a[6].transpose(1, 2).contiguous().transpose(1, 2)) or
     a.__setitem__(7, a[7].transpose(1, 2).contiguous().transpose(1, 2)) or a, {},
     "must be contiguous, token-major"),
    (lambda a: a.__setitem__(0, torch.zeros(2, 4, 16, dtype=torch.bfloat16)[..., ::2]) or a, {},
     "needs a contiguous head_dim"),
])
def test_host_checks_reject_with_the_reference_messages(lib, mutate, devices, expect):
    a = mutate(args())
    rc, msg = call_fused(lib, *a, devices=devices)
    assert rc == -1
    assert expect in msg, msg


def test_integer_tensors_are_not_implemented(lib):
    a = args()
    for i in (0, 1, 2, 6, 7, 9):
        a[i] = a[i].to(torch.int32)
    rc, msg = call_fused(lib, *a)
    assert rc == -1 and "not implemented for 'Int'" in msg


def test_zero_tokens_returns_ok_without_touching_the_gpu(lib):
    rc, msg = call_fused(lib, *args(T=0))
    assert rc == 0, msg


def test_status_strings_and_version(lib):
    lib.drk_status_string.restype = ctypes.c_char_p
    lib.drk_version.restype = ctypes.c_char_p
    assert lib.drk_status_string(0) == b"ok"
    text = lib.drk_status_string(1 | 2 | 4 | 8).decode()
    for part in ("cache_alloc_len", "request index", "table", "block"):
        assert part in text
    assert lib.drk_version().decode().count(".") == 2


def test_torch_binding_raises_runtime_errors_on_cpu_tensors():
    from decode_llm_kernel_b200 import cuda
    from decode_llm_kernel_b200.cuda import ops
    assert cuda.is_available(), cuda.unavailable_reason()
    a = args()[:9]
    with pytest.raises(RuntimeError, match="q must be a CUDA tensor"):
        ops.fused_rope_kv_append(*a)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        ops.rope_forward(a[0], a[1], a[3], a[4], a[5])
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        ops.kv_append(a[1], a[2], a[3], a[8], a[6], a[7])
    with pytest.raises(RuntimeError, match="q must be"):
        ops.fused_rope_kv_append(torch.zeros(2, 2), *a[1:])
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        cuda.smoke_fill(torch.zeros(4), 1.0)


def test_copy_probe_checks_its_arguments_before_any_launch(lib):
    fn = lib.drk_launch_copy_probe
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    lib.drk_last_error.restype = ctypes.c_char_p
    for call, msg in (((16, 32, 32, 1, 128, 1, 1), "multiple of 32"),
                      ((64, 32, 32, 1, 128, 1, 1), "stride_bytes must be >= bytes"),
                      ((64, 64, 32, 1, 100, 1, 1), "threads_per_cta"),
                      ((64, 64, -1, 1, 128, 1, 1), "count must be >= 0")):
        bytes_, stride, count, _, threads, pdl, prefetch = call
        rc = fn(None, None, bytes_, stride, count, threads, pdl, prefetch, None)
        assert rc == -1 and msg in lib.drk_last_error().decode(), call
    assert fn(None, None, 64, 64, 1, 128, 1, 1, None) == -1
    assert "16-byte aligned" in lib.drk_last_error().decode()


def test_noalloc_rejects_a_malformed_call_with_the_regular_message_first(lib):
    """Argument checks run before the size check: a CPU positions tensor is named even when
    the intermediate would not fit the 8 MiB array."""
    a = args(T=4200, Hq=1, Hkv=8, D=128)
    fn = lib.drk_separate_rope_kv_append_noalloc
    fn.restype = ctypes.c_int
    lib.drk_last_error.restype = ctypes.c_char_p
    ds = [desc(t, -1 if i == 3 else 0) for i, t in enumerate(a)]
    rc = fn(*[ctypes.byref(d) for d in ds], None, None)
    assert rc == -1 and "positions must be a CUDA tensor" in lib.drk_last_error().decode()
    # a well-formed but over-size call names the limit
    ds = [desc(t, 0) for t in a]
    rc = fn(*[ctypes.byref(d) for d in ds], None, None)
    assert rc == -1 and "8 MiB" in lib.drk_last_error().decode()
