"""Parity at the shapes of the five benchmark workloads, through the launch shapes bench.py times.

Each case runs the fused op as the bench runs it (the same kernel choice, programmatic
dependent launch where the bench uses it) and then checks, against the CPU oracle:
  * q_out, bit for bit;
  * the K slot and the V slot every token addresses, bit for bit (rotated K, raw V);
  * every other byte of both caches unchanged -- checked on the device against a copy taken
    before the call, with the addressed slots patched in, so the check does not depend on the
    cache size.
Caches are full size except where a note says otherwise.

  llama3_8b_b8        batch 8, 32:8:128 bf16, theta 5e5, cache [8, 4096, 8, 128], int32
                      positions with rows at 0 and 4095
  llama3_8b_decode32  one layer of the step: batch 64, cache [64, 8192, 8, 128], rows at 0 and
                      8191, with programmatic dependent launch
  llama3_70b_tp       64:8 heads, batch 256, cache [256, 8192, 8, 128] (the register kernel),
                      and every KV-head shard for 2, 4 and 8 GPUs (first and last rank)
  mistral_b4096       fp16, theta 1e4, 4096 tokens through the bulk-copy (TMA) kernel, and the
                      batch shards of 2048, 1024 and 512 tokens; the 4096 positions of the table
                      are all exercised by giving each of 64 cache rows 64 tokens at distinct
                      positions in [0, 4096) (a [64, 4096, 8, 128] cache instead of
                      [4096, 4096, 8, 128]: per-token work is the same)
  phi2_partial        32:32 heads, head_dim 80, rotary_dim 32, fp16, batch 128, cache
                      [128, 2048, 32, 80], positions shared by neighbouring sequences
"""
import pytest
import torch

from decode_llm_kernel_b200.harness import sharding
from decode_llm_kernel_b200.harness.configs import WORKLOADS, make_positions
from decode_llm_kernel_b200.harness.inputs import OpInputs, make_cache, make_qkv
from decode_llm_kernel_b200.rope_tables import build_rope_tables
from golden_io import bits_equal
from oracle import oracle

pytestmark = pytest.mark.gpu

SEED = 4242


@pytest.fixture(scope="module", autouse=True)
def _require_cuda():
    if not torch.cuda.is_available():
        pytest.fail("the gpu tests need a CUDA device")
    from decode_llm_kernel_b200 import cuda
    cuda.require()


def ops():
    from decode_llm_kernel_b200.cuda import ops as _ops
    return _ops


def workload_inputs(w, seed, positions=None, rows=None):
    """Inputs of one call of workload w on the GPU, caches N(0, 1)."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = make_qkv(w, gen, "cuda")
    cos, sin = build_rope_tables(w.cache_alloc_len, w.rotary, w.theta, device="cuda")
    if positions is None:
        positions = make_positions(w, seed, "cuda")
    if rows is None:
        rows = torch.arange(w.batch, device="cuda", dtype=positions.dtype)
    kc = make_cache(w, "cuda", "normal", gen)
    vc = make_cache(w, "cuda", "normal", gen)
    return OpInputs(q, k, v, positions.cuda(), cos, sin, kc, vc, rows.cuda())


def call_and_check(a, **kw):
    """Run the fused op on `a` (kwargs as for fused_rope_kv_append_ex), check it against the
    oracle as the module docstring describes, return the kernel path's q_out."""
    kc_before, vc_before = a.k_cache.clone(), a.v_cache.clone()
    q_out = ops().fused_rope_kv_append_ex(*a, **kw)
    torch.cuda.synchronize()
    from decode_llm_kernel_b200 import cuda
    cuda.check_status()
    q_ref, k_ref = oracle.rope_forward(a.q.cpu(), a.k.cpu(), a.positions.cpu(), a.cos.cpu(),
                                       a.sin.cpu())
    r, p = a.request_indices.long(), a.positions.long()
    assert bits_equal(q_out.cpu(), q_ref), "q_out"
    assert bits_equal(a.k_cache[r, p].cpu(), k_ref), "K slots"
    assert bits_equal(a.v_cache[r, p].cpu(), a.v.cpu().contiguous()), "V slots"
    kc_before[r, p] = a.k_cache[r, p]
    vc_before[r, p] = a.v_cache[r, p]
    as_bits = {2: torch.int16, 4: torch.int32, 8: torch.int64}[a.k_cache.element_size()]
    assert torch.equal(kc_before.view(as_bits), a.k_cache.view(as_bits)), "other K bytes moved"
    assert torch.equal(vc_before.view(as_bits), a.v_cache.view(as_bits)), "other V bytes moved"
    return q_out


def test_llama3_8b_b8_full_size():
    w = WORKLOADS["llama3_8b_b8"]
    p = make_positions(w, SEED, "cuda")
    p[0], p[-1] = 0, w.cache_alloc_len - 1
    a = workload_inputs(w, SEED, p)
    assert a.positions.dtype == torch.int32
    call_and_check(a)
    call_and_check(a, pdl=True, path="register")


def test_llama3_8b_decode32_layer_full_size():
    w = WORKLOADS["llama3_8b_decode32"]
    a = workload_inputs(w, SEED)
    assert int(a.positions.min()) == 0 and int(a.positions.max()) == w.cache_alloc_len - 1
    call_and_check(a, pdl=True)


def test_llama3_70b_tp_full_size_and_every_kv_head_shard():
    w = WORKLOADS["llama3_70b_tp"]
    a = workload_inputs(w, SEED)
    assert a.q.shape == (256, 64, 128) and a.k_cache.shape == (256, 8192, 8, 128)
    call_and_check(a, pdl=True)          # 256 tokens: the register kernel, as in the bench
    for n in (2, 4, 8):
        for rank in (0, n - 1):
            local = sharding.shard_kv_heads(a, rank, n)
            assert local.q.shape[1] == 64 // n and local.k.shape[1] == 8 // n
            call_and_check(local, pdl=True)
            del local
            torch.cuda.empty_cache()


def _mistral_inputs(tokens, seed):
    """4096-position rows, 64 tokens per row at distinct positions (see module docstring)."""
    from dataclasses import replace
    w = replace(WORKLOADS["mistral_b4096"], batch=tokens)
    rows_n = max(1, tokens // 64)
    g = torch.Generator().manual_seed(seed)
    rows = torch.arange(tokens) // 64
    positions = torch.empty(tokens, dtype=torch.int64)
    for r in range(rows_n):
        positions[r * 64:(r + 1) * 64] = torch.randperm(w.cache_alloc_len, generator=g)[:64]
    positions[0], positions[-1] = 0, w.cache_alloc_len - 1
    positions = positions.to(torch.int32)
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = make_qkv(w, gen, "cuda")
    cos, sin = build_rope_tables(w.cache_alloc_len, w.rotary, w.theta, device="cuda")
    cache_w = replace(w, batch=rows_n)
    kc = make_cache(cache_w, "cuda", "normal", gen)
    vc = make_cache(cache_w, "cuda", "normal", gen)
    return OpInputs(q, k, v, positions.cuda(), cos, sin, kc, vc, rows.to(torch.int32).cuda())


@pytest.mark.parametrize("tokens", [4096, 2048, 1024, 512])
def test_mistral_b4096_and_its_batch_shards_through_the_bulk_copy_kernel(tokens):
    a = _mistral_inputs(tokens, SEED + tokens)
    assert a.q.dtype == torch.float16
    q_auto = call_and_check(a, pdl=True)        # the default kernel: register at 512 tokens
    q_staged = call_and_check(a, path="staged")
    assert bits_equal(q_auto.cpu(), q_staged.cpu())


def test_phi2_partial_full_size_with_shared_positions():
    w = WORKLOADS["phi2_partial"]
    a = workload_inputs(w, SEED)
    p = a.positions.cpu()
    assert bool((p[1::4] == p[0::4]).all()), "neighbouring sequences share positions"
    assert a.cos.shape == (w.cache_alloc_len, 32)
    call_and_check(a, pdl=True, rotary_dim=32)
    call_and_check(a, rotary_dim=32, path="register")
