"""The allocation-free entry point, drk_separate_rope_kv_append_noalloc, through the C ABI.

It is for callers that cannot allocate device memory when they launch the op (global-mode
stream capture, runtimes that gave all free HBM to their cache pool, hosts without a device
allocator): its k_rot intermediate lives in an 8 MiB static device array inside the library.
The test compares it with the existing separate op (ops.separate_rope_kv_append, which
allocates k_rot through PyTorch) on two calls in a row -- bit for bit, the tolerance every
kernel test here uses -- and checks that an over-size call is refused before any launch.

The file name sorts last so a run that stops at the first failure has run every other test.
"""
import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "decode_llm_kernel_b200", "lib", "libdecode_rope.so")
CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3,
         torch.int32: 4, torch.int64: 5}


class DrkTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("device", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("sizes", ctypes.c_int64 * 4), ("strides", ctypes.c_int64 * 4)]


def desc(t):
    d = DrkTensor()
    d.data = t.data_ptr()
    d.dtype = CODES[t.dtype]
    d.ndim = t.dim()
    d.device = t.device.index if t.is_cuda else -1
    for i in range(t.dim()):
        d.sizes[i] = t.size(i)
        d.strides[i] = t.stride(i)
    return d


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    from decode_llm_kernel_b200 import cuda
    cuda.require()
    handle = ctypes.CDLL(LIB)
    handle.drk_separate_rope_kv_append_noalloc.restype = ctypes.c_int
    handle.drk_last_error.restype = ctypes.c_char_p
    return handle


def noalloc(lib, q, k, v, positions, cos, sin, k_cache, v_cache, request_indices):
    q_out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    ds = [desc(t) for t in (q, k, v, positions, cos, sin, k_cache, v_cache, request_indices,
                            q_out)]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.drk_separate_rope_kv_append_noalloc(*[ctypes.byref(d) for d in ds], None, stream)
    return rc, q_out


def _args(seed, T=64, Hq=32, Hkv=8, D=128, S=256, dtype=torch.bfloat16, layout="packed"):
    from decode_llm_kernel_b200.rope_tables import build_rope_tables
    g = torch.Generator(device="cuda").manual_seed(seed)
    if layout == "packed":
        q = torch.randn(T, Hq, D, generator=g, device="cuda").to(dtype)
        k = torch.randn(T, Hkv, D, generator=g, device="cuda").to(dtype)
        v = torch.randn(T, Hkv, D, generator=g, device="cuda").to(dtype)
    else:
        fused = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g, device="cuda").to(dtype)
        q, k, v = (p.view(T, -1, D) for p in fused.split([Hq * D, Hkv * D, Hkv * D], dim=-1))
    positions = torch.randint(0, S, (T,), generator=g, device="cuda", dtype=torch.int64)
    request_indices = torch.randperm(T, generator=g, device="cuda")
    cos, sin = build_rope_tables(S, D, 500000.0, device="cuda")
    k_cache = torch.randn(T, S, Hkv, D, generator=g, device="cuda").to(dtype)
    v_cache = torch.randn(T, S, Hkv, D, generator=g, device="cuda").to(dtype)
    return [q, k, v, positions, cos, sin, k_cache, v_cache, request_indices]


def _bits(t):
    return t.contiguous().view({2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()])


def test_noalloc_matches_the_allocating_separate_op_on_two_calls_in_a_row(lib):
    from decode_llm_kernel_b200.cuda import ops
    cases = [_args(1234), _args(4321, T=48, layout="strided", dtype=torch.float16)]
    for args in cases:
        mine = list(args)
        mine[6], mine[7] = args[6].clone(), args[7].clone()
        rc, q_out = noalloc(lib, *mine)
        assert rc == 0, lib.drk_last_error().decode()
        q_ref = ops.separate_rope_kv_append(*args)
        torch.cuda.synchronize()
        assert torch.equal(_bits(q_out), _bits(q_ref))
        assert torch.equal(_bits(mine[6]), _bits(args[6]))
        assert torch.equal(_bits(mine[7]), _bits(args[7]))


def test_an_oversize_intermediate_is_refused_before_any_launch(lib):
    # k_rot = 4097 x 8 x 128 x 2 bytes > 8 MiB
    args = _args(7, T=4097, Hq=1, Hkv=8, D=128, S=2)
    before = [a.clone() for a in args[6:8]]
    rc, _ = noalloc(lib, *args)
    assert rc == -1
    assert "8 MiB" in lib.drk_last_error().decode()
    torch.cuda.synchronize()
    assert torch.equal(_bits(args[6]), _bits(before[0]))
    assert torch.equal(_bits(args[7]), _bits(before[1]))
