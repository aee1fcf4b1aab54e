"""The fused RoPE + KV append + decode attention kernel against the CPU oracle.

The append half must be bit-identical to the fused op's (the oracle's fused_rope_kv_append on
the same inputs); attn_out must match the oracle's double-precision decode attention over the
updated cache within a per-dtype tolerance (fp32 accumulation, one rounding of the output).
"""
import math

import pytest
import torch

from decode_llm_kernel_b200.rope_tables import build_rope_tables
from oracle import oracle

pytestmark = pytest.mark.gpu

# (atol, rtol) of attn_out against the double-precision oracle: one rounding of the output to
# the storage type plus fp32 accumulation error.
ATTN_TOL = {torch.bfloat16: (4e-3, 1.6e-2), torch.float16: (5e-4, 2e-3),
            torch.float32: (2e-5, 1e-4)}


@pytest.fixture(scope="module", autouse=True)
def _require_cuda():
    if not torch.cuda.is_available():
        pytest.fail("the gpu tests need a CUDA device")
    from decode_llm_kernel_b200 import cuda
    cuda.require()


def ops():
    from decode_llm_kernel_b200.cuda import ops as _ops
    return _ops


def make_case(seed, T, Hq, Hkv, D, S, dtype, R=None, B=None, index_dtype=torch.int32,
              positions=None, theta=10000.0):
    g = torch.Generator().manual_seed(seed)
    B = B or T
    q = torch.randn(T, Hq, D, generator=g).to(dtype)
    k = torch.randn(T, Hkv, D, generator=g).to(dtype)
    v = torch.randn(T, Hkv, D, generator=g).to(dtype)
    if positions is None:
        positions = torch.randint(0, S, (T,), generator=g)
        if T >= 2:
            positions[0], positions[1] = 0, S - 1
    positions = torch.as_tensor(positions).to(index_dtype)
    ri = torch.randperm(B, generator=g)[:T].to(index_dtype)
    cos, sin = build_rope_tables(S, R or D, theta)
    kc = torch.randn(B, S, Hkv, D, generator=g).to(dtype)
    vc = torch.randn(B, S, Hkv, D, generator=g).to(dtype)
    return q, k, v, positions, cos, sin, kc, vc, ri


def oracle_result(case, scale=None):
    q, k, v, p, cos, sin, kc, vc, ri = case
    kc_ref, vc_ref = kc.clone(), vc.clone()
    q_rot = oracle.fused_rope_kv_append(q, k, v, p, cos, sin, kc_ref, vc_ref, ri, nthreads=8)
    attn = oracle.decode_attention(q_rot, kc_ref, vc_ref, p, ri, scale=scale, nthreads=8)
    return q_rot, kc_ref, vc_ref, attn


def run_gpu(case, strided=False, **kw):
    from decode_llm_kernel_b200 import cuda
    q, k, v, p, cos, sin, kc, vc, ri = [t.cuda() for t in case]
    cuda.read_status()      # start from a clear status word
    if strided:
        # head-major [B, Hkv, S, D] storage, passed as its token-major view
        kc = kc.transpose(1, 2).contiguous().transpose(1, 2)
        vc = vc.transpose(1, 2).contiguous().transpose(1, 2)
        kw["strided_cache"] = True
    q_out = torch.empty_like(q)
    R = cos.shape[1]
    if R != q.shape[2]:
        kw["rotary_dim"] = R
    attn = ops().fused_rope_kv_append_attention(q, k, v, p, cos, sin, kc, vc, ri, q_out=q_out,
                                                **kw)
    torch.cuda.synchronize()
    return q_out.cpu(), kc.cpu(), vc.cpu(), attn.cpu()


def check(case, got, scale=None):
    q_rot, kc_ref, vc_ref, attn_ref = oracle_result(case, scale)
    q_out, kc, vc, attn = got
    assert torch.equal(q_out, q_rot), "q_out differs from the oracle's q_rot"
    assert torch.equal(kc, kc_ref), "k_cache differs from the oracle's append"
    assert torch.equal(vc, vc_ref), "v_cache differs from the oracle's append"
    atol, rtol = ATTN_TOL[case[0].dtype]
    torch.testing.assert_close(attn.double(), attn_ref.double(), atol=atol, rtol=rtol)
    from decode_llm_kernel_b200 import cuda
    assert cuda.read_status() == 0


HEADS = [  # (label, Hq, Hkv, D, R)
    ("gqa_llama3", 32, 8, 128, None),
    ("mha_llama2", 8, 8, 128, None),
    ("mqa_falcon", 71, 1, 64, None),
    ("mha96_phi3", 12, 12, 96, None),
    ("partial_phi2", 8, 8, 80, 32),
    ("gqa8_70b", 16, 2, 128, None),
    ("d256", 8, 2, 256, None),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("head", HEADS, ids=[h[0] for h in HEADS])
def test_matches_oracle(head, dtype):
    _, Hq, Hkv, D, R = head
    if dtype == torch.float32 and D > 128:
        pytest.skip("fp32 rows cover head_dim <= 128")
    case = make_case(11, 6, Hq, Hkv, D, 300, dtype, R=R)
    check(case, run_gpu(case))


TC_HEADS = [  # query / KV head shapes the tensor-core kernel takes (head_dim 64 or 128)
    ("gqa_llama3", 32, 8),
    ("mha_llama2", 8, 8),
    ("gqa8_70b", 16, 2),
    ("mqa_71", 71, 1),      # five blocks of up to 16 query heads per KV head
    ("gqa_20", 40, 2),      # a 16 + 4 split
]
TC_DIMS = [128, 64]


@pytest.mark.parametrize("D", TC_DIMS)
@pytest.mark.parametrize("path", ["tensor_cores", "cuda_cores"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("head", TC_HEADS, ids=[h[0] for h in TC_HEADS])
def test_both_kernels_match_oracle(head, dtype, path, D):
    _, Hq, Hkv = head
    case = make_case(31, 5, Hq, Hkv, D, 700, dtype)
    check(case, run_gpu(case, path=path))


@pytest.mark.parametrize("D", TC_DIMS)
@pytest.mark.parametrize("chunk", [0, 128, 256, 1000, 4096])
def test_tensor_core_chunks_and_tile_edges(chunk, D):
    """Positions on both sides of tile (128) and chunk edges, and the last slot."""
    positions = [0, 1, 126, 127, 128, 129, 255, 256, 511, 999]
    case = make_case(32, len(positions), 32, 8, D, 1000, torch.bfloat16,
                     positions=positions)
    check(case, run_gpu(case, chunk=chunk, path="tensor_cores"))


@pytest.mark.parametrize("D", TC_DIMS)
def test_tensor_core_head_major_cache_int64_partial_rotary(D):
    case = make_case(33, 6, 16, 4, D, 600, torch.float16, R=D // 2, index_dtype=torch.int64)
    check(case, run_gpu(case, strided=True, path="tensor_cores"))


def test_tensor_core_head_dim_64_long_cache():
    """Falcon / Llama-3.2-1B-shaped heads over an 8192-position cache, many chunks per token."""
    case = make_case(43, 12, 32, 8, 64, 8192, torch.bfloat16, theta=500000.0)
    check(case, run_gpu(case, path="tensor_cores"))


@pytest.mark.parametrize("chunk", [1, 7, 64, 4096])
@pytest.mark.parametrize("heads_per_cta", [1, 2, 4, 8])
def test_chunks_and_head_blocks(chunk, heads_per_cta):
    case = make_case(12, 5, 24, 4, 128, 500, torch.bfloat16)
    check(case, run_gpu(case, chunk=chunk, heads_per_cta=heads_per_cta))


@pytest.mark.parametrize("D", TC_DIMS)
@pytest.mark.parametrize("T", [300, 2100])
def test_tensor_core_many_ragged_tokens(T, D):
    """The grid hands out tokens longest first up to 2048 tokens (300: many equal positions,
    so the order's ties matter) and in index order beyond (2100)."""
    case = make_case(41, T, 4, 1, D, 200, torch.bfloat16)
    check(case, run_gpu(case, path="tensor_cores"))


def test_head_major_cache_and_int64_indices():
    case = make_case(13, 7, 32, 8, 128, 257, torch.float16, index_dtype=torch.int64)
    check(case, run_gpu(case, strided=True, chunk=32))


def test_scale_and_pdl():
    case = make_case(14, 4, 16, 4, 64, 200, torch.bfloat16)
    check(case, run_gpu(case, scale=0.05, pdl=True, chunk=16), scale=0.05)


def test_first_position_returns_v():
    """At position 0 the softmax has one term: attn_out is v itself, bit for bit."""
    case = make_case(15, 3, 8, 2, 128, 64, torch.bfloat16, positions=[0, 0, 0])
    _, _, vc, attn = run_gpu(case)
    v = case[2]
    for h in range(8):
        assert torch.equal(attn[:, h], v[:, h // 4])


def test_large_cache_matches_oracle():
    """A decode batch over a long cache, many chunks per token."""
    case = make_case(16, 16, 32, 8, 128, 8192, torch.bfloat16, theta=500000.0)
    check(case, run_gpu(case))


def test_repeated_calls_and_graph_replay():
    o = ops()
    case = make_case(17, 8, 32, 8, 128, 1024, torch.bfloat16)
    q, k, v, p, cos, sin, kc, vc, ri = [t.cuda() for t in case]
    ws_bytes = o.attention_workspace_bytes(8, 32, 8, 128, 1024, torch.bfloat16, chunk=64)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty_like(q)
    kc0, vc0 = kc.clone(), vc.clone()
    for _ in range(3):   # counters must be back at zero for the next call
        kc.copy_(kc0)
        vc.copy_(vc0)
        o.fused_rope_kv_append_attention(q, k, v, p, cos, sin, kc, vc, ri, attn_out=out,
                                         workspace=ws, chunk=64)
    torch.cuda.synchronize()
    _, _, _, attn_ref = oracle_result(case)
    atol, rtol = ATTN_TOL[torch.bfloat16]
    torch.testing.assert_close(out.cpu().double(), attn_ref.double(), atol=atol, rtol=rtol)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        o.fused_rope_kv_append_attention(q, k, v, p, cos, sin, kc, vc, ri, attn_out=out,
                                         workspace=ws, chunk=64)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        o.fused_rope_kv_append_attention(q, k, v, p, cos, sin, kc, vc, ri, attn_out=out,
                                         workspace=ws, chunk=64)
    out.zero_()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu().double(), attn_ref.double(), atol=atol, rtol=rtol)
    del graph


def test_out_of_range_position_sets_status_and_writes_nothing():
    from decode_llm_kernel_b200 import cuda
    o = ops()
    cuda.read_status()
    case = make_case(18, 3, 8, 2, 64, 32, torch.float16, positions=[3, 32, 5])
    q, k, v, p, cos, sin, kc, vc, ri = [t.cuda() for t in case]
    kc0 = kc.clone()
    attn = torch.full_like(q, 7.0)
    o.fused_rope_kv_append_attention(q, k, v, p, cos, sin, kc, vc, ri, attn_out=attn)
    status = cuda.read_status()
    assert status & 1, cuda.require().status_string(status)
    bad_row = int(case[8][1])
    assert torch.equal(kc[bad_row].cpu(), kc0[bad_row].cpu())
    assert torch.all(attn[1] == 7.0)


def test_rejected_shapes():
    o = ops()
    case = make_case(19, 2, 6, 4, 64, 16, torch.bfloat16)
    args = [t.cuda() for t in case]
    with pytest.raises(RuntimeError, match="multiple of num_kv_heads"):
        o.fused_rope_kv_append_attention(*args)
    case = make_case(19, 2, 4, 2, 64, 16, torch.float64)
    with pytest.raises(RuntimeError, match="fp32, fp16 and bf16"):
        o.fused_rope_kv_append_attention(*[t.cuda() for t in case])


def test_empty_batch():
    o = ops()
    case = make_case(20, 0, 8, 2, 64, 16, torch.bfloat16, positions=[], B=2)
    out = o.fused_rope_kv_append_attention(*[t.cuda() for t in case])
    assert out.shape == (0, 8, 64)


def test_default_scale_is_inverse_sqrt_head_dim():
    case = make_case(21, 4, 8, 8, 64, 128, torch.float32)
    got = run_gpu(case)
    check(case, got, scale=1.0 / math.sqrt(64))


def test_tensor_core_out_of_range_position_sets_status_and_writes_nothing():
    from decode_llm_kernel_b200 import cuda
    o = ops()
    cuda.read_status()
    case = make_case(34, 3, 32, 8, 128, 300, torch.bfloat16, positions=[5, 300, 299])
    q, k, v, p, cos, sin, kc, vc, ri = [t.cuda() for t in case]
    kc0 = kc.clone()
    attn = torch.full_like(q, 7.0)
    o.fused_rope_kv_append_attention(q, k, v, p, cos, sin, kc, vc, ri, attn_out=attn,
                                     path="tensor_cores")
    status = cuda.read_status()
    assert status & 1, cuda.require().status_string(status)
    bad_row = int(case[8][1])
    assert torch.equal(kc[bad_row].cpu(), kc0[bad_row].cpu())
    assert torch.all(attn[1] == 7.0)
    assert not torch.any(attn[0] == 7.0) and not torch.any(attn[2] == 7.0)


def paged_from(case, block_size, seed, spare=3):
    """A page pool holding the case's contiguous caches through a shuffled block table."""
    q, k, v, p, cos, sin, kc, vc, ri = case
    B, S, Hkv, D = kc.shape
    nblk = S // block_size
    g = torch.Generator().manual_seed(seed)
    num_blocks = B * nblk + spare
    table = torch.randperm(num_blocks, generator=g)[:B * nblk].view(B, nblk)
    kp = torch.randn(num_blocks, block_size, Hkv, D, generator=g).to(kc.dtype)
    vp = torch.randn(num_blocks, block_size, Hkv, D, generator=g).to(kc.dtype)
    for b in range(B):
        for j in range(nblk):
            kp[table[b, j]] = kc[b, j * block_size:(j + 1) * block_size]
            vp[table[b, j]] = vc[b, j * block_size:(j + 1) * block_size]
    return kp, vp, table.to(p.dtype)


def gather(pages, table):
    B, nblk = table.shape
    return pages[table.long().flatten()].view(B, nblk * pages.shape[1], *pages.shape[2:])


@pytest.mark.parametrize("D", TC_DIMS)
@pytest.mark.parametrize("block_size", [8, 16, 32, 64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_paged_cache_matches_oracle(block_size, dtype, D):
    from decode_llm_kernel_b200 import cuda
    case = make_case(35, 5, 32, 8, D, 512, dtype, B=7)
    kp, vp, table = paged_from(case, block_size, 36)
    q, k, v, p, cos, sin, _, _, ri = [t.cuda() for t in case]
    kpd, vpd, tbl = kp.cuda(), vp.cuda(), table.cuda()
    used = set(table.flatten().tolist())
    spare = [b for b in range(kp.shape[0]) if b not in used]
    cuda.read_status()
    q_out = torch.empty_like(q)
    attn = ops().paged_rope_kv_append_attention(q, k, v, p, cos, sin, kpd, vpd, tbl, ri,
                                                q_out=q_out)
    torch.cuda.synchronize()
    q_rot, kc_ref, vc_ref, attn_ref = oracle_result(case)
    assert torch.equal(q_out.cpu(), q_rot)
    assert torch.equal(gather(kpd.cpu(), table), kc_ref)
    assert torch.equal(gather(vpd.cpu(), table), vc_ref)
    assert torch.equal(kpd.cpu()[spare], kp[spare]) and torch.equal(vpd.cpu()[spare], vp[spare])
    atol, rtol = ATTN_TOL[dtype]
    torch.testing.assert_close(attn.cpu().double(), attn_ref.double(), atol=atol, rtol=rtol)
    assert cuda.read_status() == 0


@pytest.mark.parametrize("D", TC_DIMS)
def test_paged_cache_block_out_of_pool_sets_status(D):
    from decode_llm_kernel_b200 import cuda
    case = make_case(37, 3, 16, 4, D, 256, torch.bfloat16, positions=[10, 200, 255])
    kp, vp, table = paged_from(case, 64, 38)
    table[int(case[8][1]), 3] = kp.shape[0] + 5        # the page holding token 1's position 200
    q, k, v, p, cos, sin, _, _, ri = [t.cuda() for t in case]
    cuda.read_status()
    ops().paged_rope_kv_append_attention(q, k, v, p, cos, sin, kp.cuda(), vp.cuda(),
                                         table.cuda(), ri)
    status = cuda.read_status()
    assert status & 8, cuda.require().status_string(status)


def test_paged_cache_rejects_unsupported_shapes():
    case = make_case(39, 2, 8, 2, 96, 128, torch.bfloat16)
    kp, vp, table = paged_from(case, 16, 40)
    with pytest.raises(RuntimeError, match="head_dim 64 or 128"):
        ops().paged_rope_kv_append_attention(*[t.cuda() for t in case[:6]], kp.cuda(), vp.cuda(),
                                             table.cuda(), case[8].cuda())
    case = make_case(41, 2, 8, 2, 128, 120, torch.bfloat16)
    kp, vp, table = paged_from(case, 24, 42)
    with pytest.raises(RuntimeError, match="block sizes"):
        ops().paged_rope_kv_append_attention(*[t.cuda() for t in case[:6]], kp.cuda(), vp.cuda(),
                                             table.cuda(), case[8].cuda())


@pytest.mark.parametrize("path,chunk", [("tensor_cores", 256), ("tensor_cores", 0),
                                        ("cuda_cores", 128)])
def test_a_zeroed_workspace_stays_zeroed_and_can_skip_the_per_call_zeroing(path, chunk):
    """Every call leaves the workspace's counters (arrival counters and the persistent grid's
    unit counter) at zero, so a workspace zeroed once can be passed with workspace_zeroed=True
    call after call: three such calls give the same bits as the default path (which zeroes the
    counters itself), and the counters read zero after each."""
    case = make_case(31, 40, 16, 4, 128, 1024, torch.bfloat16)
    q, k, v, p, cos, sin, kc, vc, ri = [t.cuda() for t in case]
    hpc = 4      # CUDA-core kernel: all 4 query heads of a KV head in one CTA (one head block)
    nbytes = ops().attention_workspace_bytes(40, 16, 4, 128, 1024, torch.bfloat16, chunk=chunk,
                                             heads_per_cta=hpc, path=path)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    # the counter region comes first: 40 tokens x 4 KV heads x 1 head block arrival counters
    # (+ the unit counter of the tensor-core kernel), rounded up to 768 bytes
    counters = ws[:768].view(torch.int32)
    for step in range(3):
        pos = (p + step).clamp(max=1023)
        kc_a, vc_a, kc_b, vc_b = kc.clone(), vc.clone(), kc.clone(), vc.clone()
        want = ops().fused_rope_kv_append_attention(q, k, v, pos, cos, sin, kc_a, vc_a, ri,
                                                    chunk=chunk, heads_per_cta=hpc, path=path)
        got = ops().fused_rope_kv_append_attention(q, k, v, pos, cos, sin, kc_b, vc_b, ri,
                                                   chunk=chunk, heads_per_cta=hpc, path=path,
                                                   workspace=ws, workspace_zeroed=True)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), step
        assert torch.equal(kc_b.view(torch.int16), kc_a.view(torch.int16))
        assert torch.equal(vc_b.view(torch.int16), vc_a.view(torch.int16))
        assert int(counters.abs().sum()) == 0, step


@pytest.mark.parametrize("T,chunk", [(1, 512), (3, 0)])
def test_tensor_core_counter_is_reset_when_every_cta_has_one_unit(T, chunk):
    """With no more units than CTAs, no take past a CTA's first unit succeeds: the unit
    counter is still back at zero after each call (its last take resets it)."""
    case = make_case(45, T, 16, 4, 128, 1024, torch.bfloat16)
    q, k, v, p, cos, sin, kc, vc, ri = [t.cuda() for t in case]
    nbytes = ops().attention_workspace_bytes(T, 16, 4, 128, 1024, torch.bfloat16, chunk=chunk,
                                             path="tensor_cores")
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    counters = ws[:256].view(torch.int32)
    for step in range(2):
        kc_a, vc_a, kc_b, vc_b = kc.clone(), vc.clone(), kc.clone(), vc.clone()
        want = ops().fused_rope_kv_append_attention(q, k, v, p, cos, sin, kc_a, vc_a, ri,
                                                    chunk=chunk, path="tensor_cores")
        got = ops().fused_rope_kv_append_attention(q, k, v, p, cos, sin, kc_b, vc_b, ri,
                                                   chunk=chunk, path="tensor_cores",
                                                   workspace=ws, workspace_zeroed=True)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), step
        assert int(counters.abs().sum()) == 0, step


def test_workspace_zeroed_needs_a_workspace():
    case = make_case(3, 2, 8, 2, 128, 64, torch.bfloat16)
    args = [t.cuda() for t in case]
    with pytest.raises(RuntimeError, match="needs a workspace"):
        ops().fused_rope_kv_append_attention(*args, workspace_zeroed=True)
