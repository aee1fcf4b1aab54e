"""The timeout path of the bulk-copy kernel's bounded waits, exercised without a GPU fault.

drk_testing_staged_timeout runs the fused op on the bulk-copy (TMA) kernel with the loads of one
token not issued and a 20 ms wait limit. Only that token's CTA waits, for copies that were never
issued (nothing is in flight toward it); when the limit passes it sets DRK_STATUS_TIMEOUT,
waits for its other copies and returns. The test checks that the call returns, the bit is set,
every other token landed bit-exact, the skipped token's slots are untouched, and the context
still runs a normal call bit-exactly afterwards.
"""
import ctypes
import os
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "decode_llm_kernel_b200", "lib", "libdecode_rope.so")
CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3,
         torch.int32: 4, torch.int64: 5}
TIMEOUT_BIT = 1 << 4
SENTINEL = 7.5


class DrkTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("device", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("sizes", ctypes.c_int64 * 4), ("strides", ctypes.c_int64 * 4)]


def desc(t):
    d = DrkTensor()
    d.data = t.data_ptr()
    d.dtype = CODES[t.dtype]
    d.ndim = t.dim()
    d.device = t.device.index
    for i in range(t.dim()):
        d.sizes[i] = t.size(i)
        d.strides[i] = t.stride(i)
    return d


def test_a_wait_that_runs_out_sets_the_timeout_bit_and_the_context_stays_usable():
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    from decode_llm_kernel_b200 import cuda
    from decode_llm_kernel_b200.cuda import ops
    from decode_llm_kernel_b200.rope_tables import build_rope_tables
    from oracle import oracle
    cuda.require()
    lib = ctypes.CDLL(LIB)
    lib.drk_testing_staged_timeout.restype = ctypes.c_int
    lib.drk_last_error.restype = ctypes.c_char_p

    T, Hq, Hkv, D, S, skip = 8, 32, 8, 128, 16, 3
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(T, Hq, D, generator=g, device="cuda").half()
    k = torch.randn(T, Hkv, D, generator=g, device="cuda").half()
    v = torch.randn(T, Hkv, D, generator=g, device="cuda").half()
    pos = torch.tensor([0, 3, 15, 7, 1, 2, 9, 4], device="cuda", dtype=torch.int32)
    ri = torch.arange(T, device="cuda", dtype=torch.int32)
    cos, sin = build_rope_tables(S, D, 10000.0, device="cuda")
    kc = torch.full((T, S, Hkv, D), SENTINEL, device="cuda", dtype=torch.float16)
    vc = torch.full_like(kc, SENTINEL)
    q_out = torch.full_like(q, SENTINEL)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ref = [t.cpu() for t in (q, k, v, pos, cos, sin)]
    kr, vr = kc.cpu().clone(), vc.cpu().clone()
    q_ref = oracle.fused_rope_kv_append(*ref, kr, vr, ri.cpu())

    args = [desc(t) for t in (q, k, v, pos, cos, sin, kc, vc, ri, q_out)]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    t0 = time.perf_counter()
    rc = lib.drk_testing_staged_timeout(*[ctypes.byref(a) for a in args], ctypes.c_int64(skip),
                                        ctypes.c_int64(20_000_000),
                                        ctypes.c_void_p(status.data_ptr()), stream)
    assert rc == 0, lib.drk_last_error().decode()
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 10.0
    assert int(status.item()) & TIMEOUT_BIT
    keep = [t for t in range(T) if t != skip]
    assert torch.equal(q_out[keep].cpu().view(torch.int16), q_ref[keep].view(torch.int16))
    assert bool((q_out[skip] == SENTINEL).all())
    for t in range(T):
        p_t = int(pos[t])
        if t == skip:
            assert bool((kc[t, p_t] == SENTINEL).all()) and bool((vc[t, p_t] == SENTINEL).all())
        else:
            assert torch.equal(kc[t, p_t].cpu().view(torch.int16), kr[t, p_t].view(torch.int16))
            assert torch.equal(vc[t, p_t].cpu().view(torch.int16), vr[t, p_t].view(torch.int16))

    # the context is usable: the normal op, forced onto the same kernel, lands bit-exact
    cuda.read_status(clear=True)
    out = ops.fused_rope_kv_append_ex(q, k, v, pos, cos, sin, kc, vc, ri, path="staged")
    torch.cuda.synchronize()
    cuda.check_status()
    assert torch.equal(out.cpu().view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(kc.cpu().view(torch.int16), kr.view(torch.int16))
    assert torch.equal(vc.cpu().view(torch.int16), vr.view(torch.int16))


def test_the_testing_entry_point_refuses_a_wait_limit_beyond_two_seconds():
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    lib = ctypes.CDLL(LIB)
    lib.drk_testing_staged_timeout.restype = ctypes.c_int
    lib.drk_last_error.restype = ctypes.c_char_p
    empty = DrkTensor()
    rc = lib.drk_testing_staged_timeout(*([ctypes.byref(empty)] * 10), ctypes.c_int64(0),
                                        ctypes.c_int64(3_000_000_000), None, None)
    assert rc == -1 and "wait_limit_ns" in lib.drk_last_error().decode()
