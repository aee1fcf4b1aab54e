"""Python face of the CPU oracle (test infrastructure: the checker, never the product path).

Wraps oracle/liboracle_rope_kv.so (built from rope_kv_oracle.c by oracle/build.py) behind the
reference's own call signature:

    fused_rope_kv_append_ref(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices)
        (decode_kernels/reference/rope_cache.py:26-36)

on CPU torch tensors. Q/K/V may be strided views (last dim contiguous); caches are any 4-D
[batch, position, kv_head, head_dim] view with a contiguous last dim, so a head-major cache is
passed as `cache_hm.transpose(1, 2)`. The rotary width is the table width: `cos.shape[1] ==
head_dim` is the reference's semantics, a narrower table rotates only the leading dims.

Only tests, the smoke check and the CPU-baseline leg of the benchmark import this module.
"""
import ctypes
import os

import torch

from . import build as _build

_DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3}
_ERRORS = {
    -1: "position out of the cache range",
    -2: "request index out of range",
    -3: "position out of the rope table range",
}

_lib = None


def _load():
    global _lib
    if _lib is None:
        path = _build.build()
        lib = ctypes.CDLL(path)
        i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
        lib.orc_fused_rope_kv_append.restype = i32
        lib.orc_fused_rope_kv_append.argtypes = (
            [i32, vp, vp, vp, i64, i32, i32, i32, i32] + [i64] * 6
            + [vp, vp, i64, i64, vp, vp, vp, vp, vp] + [i64] * 5 + [i32])
        lib.orc_rope_forward.restype = i32
        lib.orc_rope_forward.argtypes = (
            [i32, vp, vp, i64, i32, i32, i32, i32] + [i64] * 4
            + [vp, vp, i64, i64, vp, vp, vp, i32])
        lib.orc_kv_append.restype = i32
        lib.orc_kv_append.argtypes = (
            [i32, vp, vp, i64, i32, i32] + [i64] * 4 + [vp, vp, vp, vp] + [i64] * 5)
        lib.orc_decode_attention.restype = i32
        lib.orc_decode_attention.argtypes = (
            [i32, vp, i64, i32, i32, i32, vp, vp] + [i64] * 5
            + [vp, vp, ctypes.c_double, vp, i32])
        lib.orc_max_threads.restype = i32
        lib.orc_f32_to_bf16.restype = ctypes.c_uint16
        lib.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        lib.orc_f32_to_f16.restype = ctypes.c_uint16
        lib.orc_f32_to_f16.argtypes = [ctypes.c_float]
        lib.orc_f16_to_f32.restype = ctypes.c_float
        lib.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        lib.orc_bf16_to_f32.restype = ctypes.c_float
        lib.orc_bf16_to_f32.argtypes = [ctypes.c_uint16]
        _lib = lib
    return _lib


def library():
    return _load()


def max_threads():
    return int(_load().orc_max_threads())


def _check_cpu(*tensors):
    for t in tensors:
        if t.device.type != "cpu":
            raise ValueError("the oracle runs on CPU tensors only")


def _raise(rc):
    if rc:
        raise IndexError(_ERRORS.get(rc, f"oracle error {rc}"))


def _i64(t):
    return t.to(torch.int64).contiguous()


def _geometry(q, k, v, cos):
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    R = cos.shape[1]
    for name, x in (("q", q), ("k", k), ("v", v)):
        if x.dim() != 3 or x.stride(2) != 1 or x.shape[0] != T or x.shape[2] != D:
            raise ValueError(f"{name} must be [T, H, D] with a contiguous last dim")
    if R % 2 or R > D or D % 2:
        raise ValueError("rotary width must be even and at most head_dim")
    return T, Hq, Hkv, D, R


def fused_rope_kv_append(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices,
                         nthreads=1):
    """The reference oracle's semantics on CPU tensors; returns q_rot, mutates the caches."""
    _check_cpu(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices)
    T, Hq, Hkv, D, R = _geometry(q, k, v, cos)
    dt = _DTYPE_CODES[q.dtype]
    if not (q.dtype == k.dtype == v.dtype == k_cache.dtype == v_cache.dtype):
        raise ValueError("q, k, v and the caches must share a dtype")
    if k_cache.stride(3) != 1 or v_cache.stride() != k_cache.stride():
        raise ValueError("caches need a contiguous last dim and identical strides")
    cos_c, sin_c = cos.contiguous(), sin.contiguous()
    pos, ri = _i64(positions), _i64(request_indices)
    q_out = torch.empty((T, Hq, D), dtype=q.dtype)
    if T == 0:
        return q_out
    B, S = k_cache.shape[0], k_cache.shape[1]
    rc = _load().orc_fused_rope_kv_append(
        dt, q.data_ptr(), k.data_ptr(), v.data_ptr(), T, Hq, Hkv, D, R,
        q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
        cos_c.data_ptr(), sin_c.data_ptr(), cos_c.shape[0], cos_c.stride(0),
        pos.data_ptr(), ri.data_ptr(), q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        B, S, k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), int(nthreads))
    _raise(rc)
    return q_out


def rope_forward(q, k, positions, cos, sin, nthreads=1):
    """(q_rot, k_rot), both fresh contiguous tensors (csrc/rope.cu semantics)."""
    _check_cpu(q, k, positions, cos, sin)
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    R = cos.shape[1]
    cos_c, sin_c = cos.contiguous(), sin.contiguous()
    pos = _i64(positions)
    q_out = torch.empty((T, Hq, D), dtype=q.dtype)
    k_out = torch.empty((T, Hkv, D), dtype=k.dtype)
    if T == 0:
        return q_out, k_out
    rc = _load().orc_rope_forward(
        _DTYPE_CODES[q.dtype], q.data_ptr(), k.data_ptr(), T, Hq, Hkv, D, R,
        q.stride(0), q.stride(1), k.stride(0), k.stride(1),
        cos_c.data_ptr(), sin_c.data_ptr(), cos_c.shape[0], cos_c.stride(0), pos.data_ptr(),
        q_out.data_ptr(), k_out.data_ptr(), int(nthreads))
    _raise(rc)
    return q_out, k_out


def kv_append(k_rot, v, positions, request_indices, k_cache, v_cache):
    """Raw scatter of k_rot and v into their slots (csrc/kv_append.cu semantics)."""
    _check_cpu(k_rot, v, positions, request_indices, k_cache, v_cache)
    T, Hkv, D = k_rot.shape
    if T == 0:
        return
    pos, ri = _i64(positions), _i64(request_indices)
    rc = _load().orc_kv_append(
        _DTYPE_CODES[k_rot.dtype], k_rot.data_ptr(), v.data_ptr(), T, Hkv, D,
        k_rot.stride(0), k_rot.stride(1), v.stride(0), v.stride(1), pos.data_ptr(),
        ri.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0],
        k_cache.shape[1], k_cache.stride(0), k_cache.stride(1), k_cache.stride(2))
    _raise(rc)


def decode_attention(q_rot, k_cache, v_cache, positions, request_indices, scale=None,
                     nthreads=1):
    """Grouped-query decode attention of each token's rotated query over its request's cache
    positions [0, pos], evaluated in double and rounded once to the storage dtype. D <= 1024."""
    _check_cpu(q_rot, k_cache, v_cache, positions, request_indices)
    T, Hq, D = q_rot.shape
    Hkv = k_cache.shape[2]
    if scale is None:
        scale = D ** -0.5
    q_c = q_rot.contiguous()
    out = torch.empty((T, Hq, D), dtype=q_rot.dtype)
    if T == 0:
        return out
    if k_cache.stride(3) != 1 or v_cache.stride() != k_cache.stride() or D > 1024:
        raise ValueError("caches need a contiguous last dim, identical strides, head_dim <= 1024")
    pos, ri = _i64(positions), _i64(request_indices)
    rc = _load().orc_decode_attention(
        _DTYPE_CODES[q_rot.dtype], q_c.data_ptr(), T, Hq, Hkv, D, k_cache.data_ptr(),
        v_cache.data_ptr(), k_cache.shape[0], k_cache.shape[1], k_cache.stride(0),
        k_cache.stride(1), k_cache.stride(2), pos.data_ptr(), ri.data_ptr(), float(scale),
        out.data_ptr(), int(nthreads))
    if rc == -4:
        raise ValueError("num_q_heads must be a multiple of num_kv_heads")
    _raise(rc)
    return out


def f32_to_bf16_bits(x):
    return int(_load().orc_f32_to_bf16(float(x)))


def f32_to_f16_bits(x):
    return int(_load().orc_f32_to_f16(float(x)))
