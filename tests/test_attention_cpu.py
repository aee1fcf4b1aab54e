"""Host side of the fused append + decode attention entry points, without a GPU: the workspace
size both kernels need, the kernel choice, and the rejected shapes."""
import ctypes
import os

import pytest
import torch

from test_abi_cpu import CODES, desc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "decode_llm_kernel_b200", "lib", "libdecode_rope.so")

AUTO, CUDA_CORES, TENSOR_CORES = 0, 1, 2
ERR_INVALID, ERR_UNSUPPORTED = -1, -3


class AttnOptions(ctypes.Structure):
    _fields_ = [("scale", ctypes.c_double), ("chunk", ctypes.c_int32),
                ("heads_per_cta", ctypes.c_int32), ("path", ctypes.c_int32),
                ("flags", ctypes.c_int32), ("reserved", ctypes.c_int64)]


@pytest.fixture(scope="module")
def lib():
    lib = ctypes.CDLL(LIB)
    lib.drk_attention_workspace_bytes.restype = ctypes.c_int64
    lib.drk_attention_workspace_bytes.argtypes = [
        ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
        ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32]
    lib.drk_last_error.restype = ctypes.c_char_p
    return lib


def ws_bytes(lib, T, Hq, Hkv, D, S, dtype=torch.bfloat16, chunk=0, hpb=0, path=AUTO):
    o = AttnOptions(0.0, chunk, hpb, path, 0, 0)
    return lib.drk_attention_workspace_bytes(T, Hq, Hkv, D, S, CODES[dtype], ctypes.byref(o), 0)


def expected(T, Hq, Hkv, D, S, chunk, nhb, tensor_cores=False):
    """Arrival counters (plus the tensor-core grid's unit counter), then fp32 partials."""
    max_chunks = -(-S // chunk)
    counters = -(-((T * Hkv * nhb + (1 if tensor_cores else 0)) * 4) // 256) * 256
    return counters + T * Hq * max_chunks * (D + 2) * 4


def test_tensor_core_workspace_rounds_chunk_to_tiles(lib):
    assert ws_bytes(lib, 4, 32, 8, 128, 1000, chunk=256, path=TENSOR_CORES) == \
        expected(4, 32, 8, 128, 1000, 256, 1, True)
    # a chunk that is not a multiple of the 128-position tile is rounded up
    assert ws_bytes(lib, 4, 32, 8, 128, 1000, chunk=200, path=TENSOR_CORES) == \
        expected(4, 32, 8, 128, 1000, 256, 1, True)
    # auto takes the tensor-core kernel for bf16 / head_dim 128, and for head_dim 64
    assert ws_bytes(lib, 4, 32, 8, 128, 1000, chunk=256) == \
        expected(4, 32, 8, 128, 1000, 256, 1, True)
    assert ws_bytes(lib, 4, 32, 8, 64, 1000, chunk=256) == \
        expected(4, 32, 8, 64, 1000, 256, 1, True)
    # with 64 dims a tile is 256 positions: chunks round up to a multiple of 256
    assert ws_bytes(lib, 4, 32, 8, 64, 1000, chunk=200) == \
        expected(4, 32, 8, 64, 1000, 256, 1, True)
    assert ws_bytes(lib, 4, 32, 8, 64, 1000, chunk=384) == \
        expected(4, 32, 8, 64, 1000, 512, 1, True)


def test_tensor_core_splits_large_groups_into_blocks_of_16(lib):
    assert ws_bytes(lib, 3, 71, 1, 128, 512, chunk=128, path=TENSOR_CORES) == \
        expected(3, 71, 1, 128, 512, 128, 5, True)


def test_cuda_core_workspace(lib):
    assert ws_bytes(lib, 4, 32, 8, 128, 1000, chunk=64, hpb=4, path=CUDA_CORES) == \
        expected(4, 32, 8, 128, 1000, 64, 1)
    assert ws_bytes(lib, 4, 32, 8, 128, 1000, chunk=64, hpb=1, path=CUDA_CORES) == \
        expected(4, 32, 8, 128, 1000, 64, 4)
    # fp32 and head_dim 96 go to the CUDA-core kernel under auto
    assert ws_bytes(lib, 2, 12, 12, 96, 300, dtype=torch.float32, chunk=100, hpb=1) == \
        expected(2, 12, 12, 96, 300, 100, 1)


@pytest.mark.parametrize("args, code, message", [
    (dict(Hq=6, Hkv=4, D=64), ERR_INVALID, "multiple of num_kv_heads"),
    (dict(Hq=4, Hkv=2, D=64, dtype=torch.float64), ERR_UNSUPPORTED, "fp32, fp16 and bf16"),
    (dict(Hq=4, Hkv=2, D=96, path=TENSOR_CORES), ERR_UNSUPPORTED, "head_dim 64 or 128"),
    (dict(Hq=4, Hkv=2, D=130), ERR_UNSUPPORTED, "multiple of 16 bytes"),
    (dict(Hq=4, Hkv=2, D=512), ERR_UNSUPPORTED, "head_dim <= 256"),
    (dict(Hq=4, Hkv=2, D=256, dtype=torch.float32), ERR_UNSUPPORTED, "head_dim <= 128"),
    (dict(Hq=4, Hkv=2, D=64, path=7), ERR_INVALID, "path must be"),
    (dict(Hq=4, Hkv=2, D=64, hpb=3, path=CUDA_CORES), ERR_INVALID, "heads_per_cta"),
])
def test_rejected_shapes(lib, args, code, message):
    a = dict(T=2, S=64, dtype=torch.bfloat16, chunk=0, hpb=0, path=AUTO)
    a.update(args)
    rc = ws_bytes(lib, a["T"], a["Hq"], a["Hkv"], a["D"], a["S"], dtype=a["dtype"],
                  chunk=a["chunk"], hpb=a["hpb"], path=a["path"])
    assert rc == code
    assert message in lib.drk_last_error().decode()


def test_zero_tokens_is_a_no_op(lib):
    """T = 0 passes every check and returns before touching the device or the workspace."""
    T, Hq, Hkv, D, S = 0, 8, 2, 128, 16
    q = torch.zeros(T, Hq, D, dtype=torch.bfloat16)
    k = torch.zeros(T, Hkv, D, dtype=torch.bfloat16)
    pos = torch.zeros(T, dtype=torch.int32)
    cos = torch.zeros(S, D)
    kc = torch.zeros(2, S, Hkv, D, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    out = torch.zeros(T, Hq, D, dtype=torch.bfloat16)
    ds = [desc(t) for t in (q, k, k, pos, cos, cos, kc, vc, pos)]
    do = desc(out)
    rc = lib.drk_fused_rope_kv_append_attention(
        *[ctypes.byref(d) for d in ds], None, ctypes.byref(do), None, None, ctypes.c_size_t(0),
        None, None, None)
    assert rc == 0, lib.drk_last_error()


def test_cuda_core_auto_chunk_fills_one_wave(lib):
    """Auto chunk of the CUDA-core kernel: the power of two nearest units * S / (SMs x CTAs
    per SM), within [128, 1024]. Without a GPU the plan sees one SM; one head per CTA of 16-bit
    data leaves 8 CTAs on it."""
    # 4 units x 600 positions / 8 slots = 300 -> 256 (3 chunks)
    assert ws_bytes(lib, 1, 4, 4, 96, 600) == expected(1, 4, 4, 96, 600, 256, 1)
    # 4 x 100 / 8 = 50 -> the 128 floor (one chunk)
    assert ws_bytes(lib, 1, 4, 4, 96, 100) == expected(1, 4, 4, 96, 100, 128, 1)
    # 4 x 3000 / 8 = 1500 -> the 1024 ceiling (3 chunks)
    assert ws_bytes(lib, 1, 4, 4, 96, 3000) == expected(1, 4, 4, 96, 3000, 1024, 1)


def test_tensor_core_auto_chunk_prefers_fewer_merges(lib):
    """On one SM every unit is its own round, so the cost model takes the whole cache as one
    chunk (no merge) rather than 512-position chunks."""
    assert ws_bytes(lib, 2, 32, 8, 128, 1000) == expected(2, 32, 8, 128, 1000, 1024, 1, True)
