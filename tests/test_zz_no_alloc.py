"""The allocation-free entry point, drk_separate_rope_kv_append_noalloc, through the C ABI.

It is for callers that cannot allocate device memory when they launch the op (global-mode
stream capture, runtimes that gave all free HBM to their cache pool, hosts without a device
allocator): its k_rot intermediate lives in an 8 MiB static device array inside the library.
The tests compare it with the existing separate op (ops.separate_rope_kv_append, which
allocates k_rot through PyTorch) on two calls in a row -- bit for bit, the tolerance every
kernel test here uses -- and check that an over-size call is refused before any launch, that
argument errors are reported before the size check, and that a token past a short cos/sin table
keeps its K slot although the shared array holds an earlier call's rows.

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


def noalloc(lib, q, k, v, positions, cos, sin, k_cache, v_cache, request_indices, status=None):
    q_out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    ds = [desc(t) for t in (q, k, v, positions, cos, sin, k_cache, v_cache, request_indices,
                            q_out)]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    word = None if status is None else ctypes.c_void_p(status.data_ptr())
    rc = lib.drk_separate_rope_kv_append_noalloc(*[ctypes.byref(d) for d in ds], word, stream)
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


def test_a_position_past_a_short_table_keeps_its_k_slot(lib):
    """The scratch array keeps the previous call's k_rot rows. A token inside the cache but past
    a short cos/sin table gets no k_rot row from the rope step, and the append step must not
    copy the stale one: its K slot keeps its old contents, the out-of-table status bit is set,
    its V slot is written, and every other token matches the allocating separate op."""
    from decode_llm_kernel_b200 import cuda
    from decode_llm_kernel_b200.cuda import ops
    args = _args(99, T=8, S=64)
    noalloc(lib, *_args(98, T=8, S=64))   # leave other values in the shared array first
    args[3] = torch.tensor([0, 5, 40, 7, 1, 2, 3, 4], device="cuda")
    args[4], args[5] = args[4][:32].contiguous(), args[5][:32].contiguous()
    ref = list(args)
    ref[6], ref[7] = args[6].clone(), args[7].clone()
    before = args[6].clone()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc, q_out = noalloc(lib, *args, status=status)
    assert rc == 0, lib.drk_last_error().decode()
    cuda.read_status(clear=True)
    q_ref = ops.separate_rope_kv_append(*ref)
    torch.cuda.synchronize()
    assert int(status.item()) & 4            # DRK_STATUS_POSITION_OUT_OF_TABLE
    r2 = int(args[8][2])
    assert torch.equal(_bits(args[6][r2, 40]), _bits(before[r2, 40]))
    assert torch.equal(_bits(args[7][r2, 40]), _bits(args[2][2]))
    assert torch.equal(_bits(args[6]), _bits(ref[6]))
    assert torch.equal(_bits(args[7]), _bits(ref[7]))
    keep = torch.tensor([0, 1, 3, 4, 5, 6, 7], device="cuda")
    assert torch.equal(_bits(q_out[keep]), _bits(q_ref[keep]))


def test_argument_errors_come_before_the_size_check(lib):
    """A malformed call is refused with the regular message even when its k_rot would not fit
    the scratch array."""
    args = _args(7, T=4097, Hq=1, Hkv=8, D=128, S=2)
    args[3] = args[3].cpu()
    rc, _ = noalloc(lib, *args)
    assert rc == -1
    assert "must be a CUDA tensor" in lib.drk_last_error().decode()
