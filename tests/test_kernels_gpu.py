"""The sm_100a kernels against the reference's golden fixtures and the CPU oracle, through the
drop-in ops (and hence the C ABI). Mirrors the reference's tests/test_rope_kv_kernels.py, with
bit-exactness required where the reference allowed a tolerance."""
import pytest
import torch

from decode_llm_kernel_b200.harness import positions as pos
from decode_llm_kernel_b200.harness.configs import HEAD_SHAPES
from decode_llm_kernel_b200.harness.inputs import SENTINEL, case, make_inputs
from gate import TOLERANCES, validate_candidate
from golden_io import Golden, bits_equal, names
from oracle import oracle

pytestmark = pytest.mark.gpu

SEED = 1234
NAMES = ("separate", "fused")


@pytest.fixture(scope="module", autouse=True)
def _require_cuda():
    if not torch.cuda.is_available():
        pytest.fail("the gpu tests need a CUDA device")
    from decode_llm_kernel_b200 import cuda
    cuda.require()          # fail loudly, never skip, when the extension is missing


def ops():
    from decode_llm_kernel_b200.cuda import ops as _ops
    return _ops


def kernel(name):
    o = ops()
    return {"separate": o.separate_rope_kv_append, "fused": o.fused_rope_kv_append}[name]


def cfg_for(head_cfg, dtype_label, batch=8, alloc=128, mode=pos.RAGGED, **kw):
    label, hq, hkv, d = head_cfg
    return case(label, hq, hkv, d, batch, alloc, dtype_label, mode, **kw)


def _oracle_args(args):
    return [t.cpu().clone() if i in (6, 7) else t.cpu() for i, t in enumerate(args)]


# ---------------------------------------------------------------- golden fixtures

@pytest.mark.parametrize("name", names())
@pytest.mark.parametrize("impl", ["fused", "separate", "fused_pdl", "register", "staged"])
def test_golden_fixture_bit_exact(name, impl):
    g = Golden(name, device="cuda")
    m = g.meta
    if impl == "separate" and (m["R"] != m["D"]):
        pytest.skip("the separate rungs follow the reference contract (full rotary)")
    _, _, kv, vv = g.fresh_caches()
    o = ops()
    extra = {}
    if m["R"] != m["D"]:
        extra["rotary_dim"] = m["R"]
    if m["cache_layout"] != "token_major":
        extra["strided_cache"] = True
    if impl == "fused" and not extra:
        q_out = o.fused_rope_kv_append(g.q, g.k, g.v, g.positions, g.cos, g.sin, kv, vv,
                                       g.request_indices)
    elif impl == "separate" and not extra:
        q_out = o.separate_rope_kv_append(g.q, g.k, g.v, g.positions, g.cos, g.sin, kv, vv,
                                          g.request_indices)
    elif impl == "separate":
        q_out, k_rot = o.rope_forward_ex(g.q, g.k, g.positions, g.cos, g.sin)
        o.kv_append_ex(k_rot, g.v, g.positions, g.request_indices, kv, vv,
                       strided_cache=extra.get("strided_cache", False))
    elif impl in ("register", "staged"):
        if impl == "staged" and m["cache_layout"] != "token_major":
            with pytest.raises(RuntimeError, match="bulk-copy kernel cannot take this call"):
                o.fused_rope_kv_append_ex(g.q, g.k, g.v, g.positions, g.cos, g.sin, kv, vv,
                                          g.request_indices, path="staged", **extra)
            return
        q_out = o.fused_rope_kv_append_ex(g.q, g.k, g.v, g.positions, g.cos, g.sin, kv, vv,
                                          g.request_indices, path=impl, **extra)
    else:
        q_out = o.fused_rope_kv_append_ex(g.q, g.k, g.v, g.positions, g.cos, g.sin, kv, vv,
                                          g.request_indices, pdl=(impl == "fused_pdl"), **extra)
    torch.cuda.synchronize()
    assert g.check(q_out, kv, vv) == []


# ---------------------------------------------------------------- the gate over the registry

@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("head_cfg", HEAD_SHAPES, ids=[h[0] for h in HEAD_SHAPES])
@pytest.mark.parametrize("dtype_label", ["fp32", "bf16", "fp16", "fp64"])
def test_the_gate_clears_every_registry_shape_bit_exactly(name, head_cfg, dtype_label):
    report = validate_candidate(kernel(name), cfg_for(head_cfg, dtype_label), "cuda", SEED)
    assert report["ok"], "; ".join(report["failures"])
    assert report["num_cases"] == 5
    assert report["q_bit_exact"] and report["k_bit_exact"]
    assert report["v_byte_exact"] and report["unaddressed_slots_intact"]


@pytest.mark.parametrize("name", NAMES)
def test_head_dim_96_non_power_of_two_half(name):
    head_cfg = next(h for h in HEAD_SHAPES if h[3] == 96)
    report = validate_candidate(kernel(name), cfg_for(head_cfg, "bf16", batch=33), "cuda", SEED)
    assert report["ok"] and report["q_bit_exact"] and report["k_bit_exact"]


@pytest.mark.parametrize("index_dtype", ["int32", "int64"])
@pytest.mark.parametrize("theta", [10000.0, 500000.0])
def test_llama3_shape_int32_and_theta(index_dtype, theta):
    cfg = cfg_for(("gqa", 32, 8, 128), "bf16", batch=64, alloc=512, theta=theta,
                  index_dtype=index_dtype)
    report = validate_candidate(kernel("fused"), cfg, "cuda", SEED)
    assert report["ok"] and report["q_bit_exact"] and report["k_bit_exact"]


def test_the_two_rungs_agree_with_each_other():
    cfg = cfg_for(("mha", 32, 32, 128), "bf16")
    p = pos.build_position_sets(cfg.batch, cfg.cache_alloc_len, cfg.positions, SEED,
                                1, "cuda")[0]
    outs, caches = [], []
    for impl in NAMES:
        args = make_inputs(cfg, "cuda", SEED, p)
        outs.append(kernel(impl)(*args))
        caches.append((args.k_cache, args.v_cache))
    assert bits_equal(outs[0], outs[1])
    assert bits_equal(caches[0][0], caches[1][0])
    assert bits_equal(caches[0][1], caches[1][1])


@pytest.mark.parametrize("name", NAMES)
def test_int32_positions_match_int64(name):
    cfg = cfg_for(("gqa", 32, 8, 128), "bf16")
    p = pos.build_position_sets(cfg.batch, cfg.cache_alloc_len, cfg.positions, SEED,
                                1, "cuda")[0]
    wide = make_inputs(cfg, "cuda", SEED, p)
    narrow = make_inputs(cfg, "cuda", SEED, p.to(torch.int32))
    narrow = narrow._replace(positions=narrow.positions.to(torch.int32),
                             request_indices=narrow.request_indices.to(torch.int32))
    assert bits_equal(kernel(name)(*wide), kernel(name)(*narrow))
    assert bits_equal(wide.k_cache, narrow.k_cache)


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("batch", [1, 2, 3])
def test_small_token_counts(name, batch):
    cfg = cfg_for(("mqa", 71, 1, 64), "bf16", batch=batch)
    report = validate_candidate(kernel(name), cfg, "cuda", SEED)
    assert report["ok"] and report["q_bit_exact"]


@pytest.mark.parametrize("name", NAMES)
def test_zero_tokens_is_a_no_op_not_a_crash(name):
    cfg = cfg_for(("mha", 32, 32, 128), "bf16", batch=0)
    args = make_inputs(cfg, "cuda", SEED, torch.zeros(0, dtype=torch.long, device="cuda"))
    q_rot = kernel(name)(*args)
    torch.cuda.synchronize()
    assert q_rot.shape == (0, 32, 128)


@pytest.mark.parametrize("name", NAMES)
def test_zero_token_caches_are_not_mistaken_for_aliases(name):
    cfg = cfg_for(("mha", 32, 32, 128), "bf16", batch=0)
    args = make_inputs(cfg, "cuda", SEED, torch.zeros(0, dtype=torch.long, device="cuda"))
    assert args.k_cache.data_ptr() == args.v_cache.data_ptr() == 0
    kernel(name)(*args)
    torch.cuda.synchronize()


# ---------------------------------------------------------------- vector widths and layouts

def _misaligned(t, shift):
    """Same values as t, stored `shift` elements past an aligned allocation."""
    flat = torch.empty(t.numel() + 16, dtype=t.dtype, device=t.device)
    view = flat[shift:shift + t.numel()].view(t.shape)
    view.copy_(t)
    return view


@pytest.mark.parametrize("dtype_label,shift", [("bf16", 1), ("bf16", 2), ("bf16", 4),
                                               ("fp32", 1), ("fp32", 2), ("fp16", 3),
                                               ("fp64", 1)])
def test_narrow_vector_paths_stay_bit_exact(dtype_label, shift):
    cfg = cfg_for(("gqa", 8, 2, 64), dtype_label, batch=5, alloc=32)
    p = pos.build_position_sets(5, 32, pos.RAGGED, SEED, 1, "cuda")[0]
    a = make_inputs(cfg, "cuda", SEED, p, cache_fill=SENTINEL)
    a = a._replace(q=_misaligned(a.q, shift), k=_misaligned(a.k, shift), v=_misaligned(a.v, shift))
    ref = _oracle_args(a)
    q_ref = oracle.fused_rope_kv_append(*ref)
    q = ops().fused_rope_kv_append(*a)
    assert bits_equal(q.cpu(), q_ref)
    assert bits_equal(a.k_cache.cpu(), ref[6])
    assert bits_equal(a.v_cache.cpu(), ref[7])


@pytest.mark.parametrize("name", NAMES)
def test_a_strided_qkv_view_is_not_copied_first(name):
    cfg = cfg_for(("mha96", 32, 32, 96), "bf16")
    p = pos.build_position_sets(cfg.batch, cfg.cache_alloc_len, cfg.positions, SEED,
                                1, "cuda")[0]
    strided = make_inputs(cfg, "cuda", SEED, p, qkv_layout="fused")
    assert not strided.q.is_contiguous()
    ref = _oracle_args(strided)
    expected = oracle.fused_rope_kv_append(*ref)
    assert bits_equal(kernel(name)(*strided).cpu(), expected)
    packed = make_inputs(cfg, "cuda", SEED, p, qkv_layout="packed")
    assert packed.q.is_contiguous()


@pytest.mark.parametrize("dtype_label", ["bf16", "fp16", "fp32"])
def test_partial_rotary_phi2_shape(dtype_label):
    cfg = case("phi2", 32, 32, 80, 16, 64, dtype_label, pos.RAGGED, rotary_dim=32)
    p = pos.build_position_sets(16, 64, pos.RAGGED, SEED, 1, "cuda")[0]
    a = make_inputs(cfg, "cuda", SEED, p, cache_fill=SENTINEL)
    assert a.cos.shape == (64, 32)
    ref = _oracle_args(a)
    q_ref = oracle.fused_rope_kv_append(*ref)
    q = ops().fused_rope_kv_append_ex(*a, rotary_dim=32)
    assert bits_equal(q.cpu(), q_ref)
    assert bits_equal(a.k_cache.cpu(), ref[6])
    assert bits_equal(a.v_cache.cpu(), ref[7])
    # pass-through dims are raw copies
    assert bits_equal(q[..., 32:].cpu(), a.q[..., 32:].cpu())


@pytest.mark.parametrize("dtype_label", ["bf16", "fp16"])
def test_head_major_cache(dtype_label):
    cfg = case("gqa", 32, 8, 128, 8, 64, dtype_label, pos.RAGGED, cache_layout="head_major")
    p = pos.build_position_sets(8, 64, pos.RAGGED, SEED, 1, "cuda")[0]
    a = make_inputs(cfg, "cuda", SEED, p, cache_fill=SENTINEL)
    assert not a.k_cache.is_contiguous()
    ref = _oracle_args(a)
    q_ref = oracle.fused_rope_kv_append(*ref)
    q = ops().fused_rope_kv_append_ex(*a, strided_cache=True)
    assert bits_equal(q.cpu(), q_ref)
    assert bits_equal(a.k_cache.cpu(), ref[6])
    assert bits_equal(a.v_cache.cpu(), ref[7])
    with pytest.raises(RuntimeError, match="must be contiguous, token-major"):
        ops().fused_rope_kv_append(*a)


@pytest.mark.parametrize("block_size", [16, 64])
@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
def test_paged_cache_matches_the_contiguous_oracle(block_size, index_dtype):
    T, Hq, Hkv, D, S = 12, 32, 8, 128, 256
    cfg = case("gqa", Hq, Hkv, D, T, S, "bf16", pos.RAGGED)
    p = pos.build_position_sets(T, S, pos.RAGGED, SEED, 1, "cuda")[0]
    a = make_inputs(cfg, "cuda", SEED, p, cache_fill=SENTINEL)
    max_blocks = S // block_size
    num_blocks = T * max_blocks + 3
    g = torch.Generator().manual_seed(SEED)
    perm = torch.randperm(num_blocks, generator=g)[: T * max_blocks].view(T, max_blocks)
    block_table = perm.to(device="cuda", dtype=index_dtype)
    k_pages = torch.full((num_blocks, block_size, Hkv, D), 7.5, dtype=torch.bfloat16,
                         device="cuda")
    v_pages = torch.full_like(k_pages, 7.5)
    q = ops().paged_rope_kv_append(a.q, a.k, a.v, a.positions.to(index_dtype), a.cos, a.sin,
                                   k_pages, v_pages, block_table,
                                   a.request_indices.to(index_dtype))
    ref = _oracle_args(a)
    q_ref = oracle.fused_rope_kv_append(*ref)
    assert bits_equal(q.cpu(), q_ref)
    ri, pp = a.request_indices.long().cpu(), a.positions.long().cpu()
    blk = perm[ri, pp // block_size]
    row = pp % block_size
    assert bits_equal(k_pages.cpu()[blk, row], ref[6][ri, pp])
    assert bits_equal(v_pages.cpu()[blk, row], ref[7][ri, pp])
    touched = torch.zeros(num_blocks, block_size, dtype=torch.bool)
    touched[blk, row] = True
    assert bool((k_pages.cpu()[~touched] == 7.5).all())


def test_in_register_trig_within_the_reference_tolerance():
    from decode_llm_kernel_b200.rope_tables import inverse_frequencies
    cfg = cfg_for(("gqa", 32, 8, 128), "bf16", batch=64, alloc=4096, theta=500000.0)
    p = pos.build_position_sets(64, 4096, pos.RAGGED, SEED, 1, "cuda")[0]
    a = make_inputs(cfg, "cuda", SEED, p, cache_fill=SENTINEL)
    ref = _oracle_args(a)
    q_ref = oracle.fused_rope_kv_append(*ref)
    inv = inverse_frequencies(128, 500000.0).cuda()
    q = ops().fused_rope_kv_append_ex(*a, inv_freq=inv).cpu()
    _assert_inreg_close(q, q_ref)
    assert bits_equal(a.v_cache.cpu(), ref[7])


def _assert_inreg_close(q, q_ref):
    """sincosf in registers differs from the table by an fp32 ulp now and then; after
    cancellation in x1*c - x2*s that can be many bf16 ulps of a near-zero output. Held to the
    reference's bf16 tolerance (atol = rtol = 8e-3) with at least 99.9% of elements within one
    bf16 ulp."""
    torch.testing.assert_close(q.float(), q_ref.float(), atol=8e-3, rtol=8e-3)
    ulp = (q.view(torch.int16).int() - q_ref.view(torch.int16).int()).abs()
    assert float((ulp <= 1).float().mean()) >= 0.999


# ---------------------------------------------------------------- graphs, streams, PDL

@pytest.mark.parametrize("name", NAMES)
def test_capturable_into_a_cuda_graph(name):
    cfg = cfg_for(("mha", 32, 32, 128), "bf16")
    sets = pos.build_position_sets(cfg.batch, cfg.cache_alloc_len, cfg.positions,
                                   SEED, 2, "cuda")
    args = make_inputs(cfg, "cuda", SEED, sets[0])
    static_positions = args.positions.clone()
    bound = args._replace(positions=static_positions)
    fn = kernel(name)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn(*bound)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = fn(*bound)
    static_positions.copy_(sets[1])
    graph.replay()
    torch.cuda.synchronize()
    expected_args = _oracle_args(make_inputs(cfg, "cuda", SEED, sets[1]))
    expected = oracle.fused_rope_kv_append(*expected_args)
    assert bits_equal(captured.cpu(), expected)
    ri, p1 = bound.request_indices.cpu(), sets[1].cpu()
    assert bits_equal(bound.k_cache.cpu()[ri, p1], expected_args[6][ri, p1])
    assert bits_equal(bound.v_cache.cpu()[ri, p1], bound.v.cpu())


def test_pdl_chain_inside_a_graph_matches_eager():
    """Eight layers chained with programmatic dependent launch inside one graph."""
    from decode_llm_kernel_b200.harness.decode_loop import DecodeStep, StepInputs
    from decode_llm_kernel_b200.rope_tables import build_rope_tables
    L, T, Hq, Hkv, D, S = 8, 16, 32, 8, 128, 64
    g = torch.Generator(device="cuda").manual_seed(SEED)
    mk = lambda *s: torch.randn(*s, generator=g, device="cuda").to(torch.bfloat16)  # noqa: E731
    kcs = [torch.zeros(T, S, Hkv, D, dtype=torch.bfloat16, device="cuda") for _ in range(L)]
    vcs = [torch.zeros_like(kcs[0]) for _ in range(L)]
    cos, sin = build_rope_tables(S, D, 500000.0, device="cuda")
    positions = torch.randint(0, S, (T,), device="cuda", dtype=torch.int32)
    ri = torch.arange(T, device="cuda", dtype=torch.int32)
    inputs = StepInputs(mk(L, T, Hq, D), mk(L, T, Hkv, D), mk(L, T, Hkv, D), positions, ri)
    step = DecodeStep(kcs, vcs, cos, sin, pdl=True)
    cap = step.capture(inputs)
    for c in kcs + vcs:
        c.zero_()
    cap.replay()
    torch.cuda.synchronize()
    for layer in range(L):
        kc, vc = torch.zeros(T, S, Hkv, D, dtype=torch.bfloat16), torch.zeros(T, S, Hkv, D,
                                                                             dtype=torch.bfloat16)
        q_ref = oracle.fused_rope_kv_append(inputs.q[layer].cpu(), inputs.k[layer].cpu(),
                                            inputs.v[layer].cpu(), positions.cpu(), cos.cpu(),
                                            sin.cpu(), kc, vc, ri.cpu())
        assert bits_equal(cap.q_out[layer].cpu(), q_ref)
        assert bits_equal(kcs[layer].cpu(), kc)
        assert bits_equal(vcs[layer].cpu(), vc)


def test_end_to_end_graph_copies_host_buffers():
    from decode_llm_kernel_b200.harness.decode_loop import DecodeStep, StepInputs, pinned_like
    from decode_llm_kernel_b200.rope_tables import build_rope_tables
    L, T, Hq, Hkv, D, S = 4, 8, 32, 8, 128, 32
    kcs = [torch.zeros(T, S, Hkv, D, dtype=torch.bfloat16, device="cuda") for _ in range(L)]
    vcs = [torch.zeros_like(kcs[0]) for _ in range(L)]
    cos, sin = build_rope_tables(S, D, 500000.0, device="cuda")
    dev = StepInputs(torch.zeros(L, T, Hq, D, dtype=torch.bfloat16, device="cuda"),
                     torch.zeros(L, T, Hkv, D, dtype=torch.bfloat16, device="cuda"),
                     torch.zeros(L, T, Hkv, D, dtype=torch.bfloat16, device="cuda"),
                     torch.zeros(T, dtype=torch.int32, device="cuda"),
                     torch.arange(T, dtype=torch.int32, device="cuda"))
    host = pinned_like(dev)
    cap = DecodeStep(kcs, vcs, cos, sin).capture(dev, host=host)
    host.q.copy_(torch.randn(L, T, Hq, D).to(torch.bfloat16))
    host.k.copy_(torch.randn(L, T, Hkv, D).to(torch.bfloat16))
    host.v.copy_(torch.randn(L, T, Hkv, D).to(torch.bfloat16))
    host.positions.copy_(torch.randint(0, S, (T,), dtype=torch.int32))
    cap.replay()
    torch.cuda.synchronize()
    for layer in range(L):
        kc, vc = torch.zeros(T, S, Hkv, D, dtype=torch.bfloat16), torch.zeros(T, S, Hkv, D,
                                                                             dtype=torch.bfloat16)
        q_ref = oracle.fused_rope_kv_append(host.q[layer], host.k[layer], host.v[layer],
                                            host.positions, cos.cpu(), sin.cpu(), kc, vc,
                                            host.request_indices)
        assert bits_equal(cap.host_q_out[layer].clone(), q_ref)


def test_runs_on_a_non_default_stream():
    cfg = cfg_for(("gqa", 32, 8, 128), "bf16")
    p = pos.build_position_sets(8, 128, pos.RAGGED, SEED, 1, "cuda")[0]
    a = make_inputs(cfg, "cuda", SEED, p)
    ref = _oracle_args(a)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        q = ops().fused_rope_kv_append(*a)
    torch.cuda.synchronize()
    assert bits_equal(q.cpu(), oracle.fused_rope_kv_append(*ref))


# ---------------------------------------------------------------- bounds: status word, no trap

def test_out_of_range_positions_set_status_and_skip_writes():
    from decode_llm_kernel_b200 import cuda
    cuda.read_status(clear=True)
    cfg = cfg_for(("gqa", 32, 8, 128), "bf16", batch=4, alloc=16)
    a = make_inputs(cfg, "cuda", SEED, torch.tensor([0, 3, 16, 5], device="cuda"),
                      cache_fill=SENTINEL)
    ops().fused_rope_kv_append(*a)
    word = cuda.read_status(clear=False)
    assert word & 1 and word & 4          # outside the cache and outside the table
    with pytest.raises(RuntimeError, match="out-of-range"):
        cuda.check_status()
    assert cuda.read_status() == 0        # check_status cleared it
    # the valid tokens were written, the invalid one was not; the context is still usable
    kc = a.k_cache.cpu()
    assert bool((kc[2] == 7.5).all())
    assert not bool((kc[0, 0] == 7.5).all())
    a2 = make_inputs(cfg, "cuda", SEED, torch.tensor([0, 3, 15, 5], device="cuda"),
                       cache_fill=SENTINEL)
    ops().fused_rope_kv_append(*a2)
    a2r = a2._replace(request_indices=torch.tensor([0, 1, 9, 3], device="cuda"))
    ops().fused_rope_kv_append(*a2r)
    assert cuda.read_status() & 2


@pytest.mark.parametrize("name", NAMES)
def test_a_position_past_a_short_table_keeps_its_k_slot_in_both_ops(name):
    """A cos/sin table shorter than the cache: the token whose position is inside the cache but
    past the table sets the out-of-table bit and keeps its K slot (the separate op's append is
    told the table length, so it never copies the k_rot row the rope step left unwritten); its
    V slot is written, as in the fused op; every other token lands bit-exact."""
    from decode_llm_kernel_b200 import cuda
    cuda.read_status(clear=True)
    cfg = cfg_for(("gqa", 32, 8, 128), "bf16", batch=4, alloc=32)
    a = make_inputs(cfg, "cuda", SEED, torch.tensor([0, 3, 20, 5], device="cuda"),
                    cache_fill=SENTINEL)
    a = a._replace(cos=a.cos[:16].contiguous(), sin=a.sin[:16].contiguous())
    for _ in range(2):                    # twice: a stale k_rot row from call 1 stays unused
        kernel(name)(*a)
        torch.cuda.synchronize()
        assert cuda.read_status() & 4     # DRK_STATUS_POSITION_OUT_OF_TABLE
        kc, vc = a.k_cache.cpu(), a.v_cache.cpu()
        assert bool((kc[2, 20] == SENTINEL).all()), "K slot past the table was written"
        assert bits_equal(vc[2, 20], a.v[2].cpu())
        ok = torch.tensor([0, 1, 3])
        sub = a._replace(q=a.q[ok], k=a.k[ok], v=a.v[ok], positions=a.positions[ok],
                         request_indices=a.request_indices[ok])
        ref = _oracle_args(sub)
        q_ref, k_ref = oracle.rope_forward(ref[0], ref[1], ref[3], ref[4], ref[5])
        r, p = ref[8].long(), ref[3].long()
        assert bits_equal(kc[r, p], k_ref)


# ---------------------------------------------------------------- errors (reference messages)

def _small():
    cfg = cfg_for(("mha", 32, 32, 128), "bf16", batch=2)
    p = pos.build_position_sets(2, 128, pos.RAGGED, SEED, 1, "cuda")[0]
    return make_inputs(cfg, "cuda", SEED, p)


def test_a_cache_dtype_mismatch_is_refused_rather_than_silently_cast():
    a = _small()
    with pytest.raises(RuntimeError, match="must match its source dtype"):
        ops().fused_rope_kv_append(a.q, a.k, a.v, a.positions, a.cos, a.sin, a.k_cache.float(),
                                   a.v_cache, a.request_indices)


def test_fp16_tables_are_refused():
    a = _small()
    with pytest.raises(RuntimeError, match="must be FP32"):
        ops().fused_rope_kv_append(a.q, a.k, a.v, a.positions, a.cos.half(), a.sin.half(),
                                   a.k_cache, a.v_cache, a.request_indices)


@pytest.mark.parametrize("name", NAMES)
def test_a_host_tensor_is_refused_rather_than_dereferenced_on_device(name):
    a = _small()
    fn = kernel(name)
    for args in ((a.q, a.k, a.v, a.positions, a.cos.cpu(), a.sin, a.k_cache, a.v_cache,
                  a.request_indices),
                 (a.q, a.k, a.v, a.positions.cpu(), a.cos, a.sin, a.k_cache, a.v_cache,
                  a.request_indices),
                 (a.q, a.k, a.v, a.positions, a.cos, a.sin, a.k_cache, a.v_cache,
                  a.request_indices.cpu())):
        with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
            fn(*args)


@pytest.mark.parametrize("name", NAMES)
def test_one_buffer_used_as_both_caches_is_refused(name):
    a = _small()
    with pytest.raises(RuntimeError, match="distinct buffers"):
        kernel(name)(a.q, a.k, a.v, a.positions, a.cos, a.sin, a.k_cache, a.k_cache,
                     a.request_indices)


def test_rope_forward_returns_a_contiguous_tuple():
    cfg = cfg_for(("gqa", 32, 8, 128), "fp32", batch=2)
    p = pos.build_position_sets(2, 128, pos.RAGGED, SEED, 1, "cuda")[0]
    a = make_inputs(cfg, "cuda", SEED, p)
    from decode_llm_kernel_b200 import cuda
    out = cuda.require().rope_forward(a.q, a.k, a.positions, a.cos, a.sin)
    assert isinstance(out, tuple)
    q_rot, k_rot = out
    assert q_rot.shape == (2, 32, 128) and k_rot.shape == (2, 8, 128)
    assert q_rot.is_contiguous() and k_rot.is_contiguous()


def test_fp32_margin_is_zero():
    """The reference reports its fp32 margin against atol 1e-6; this build is bit-exact."""
    cfg = cfg_for(("mha", 32, 32, 128), "fp32")
    report = validate_candidate(kernel("fused"), cfg, "cuda", SEED)
    assert report["ok"]
    assert report["max_abs_diff_q"] == 0.0 < TOLERANCES[torch.float32]["atol"]
    assert report["max_abs_diff_k_cache"] == 0.0


# ---------------------------------------------------------------- the bulk-copy (staged) kernel

@pytest.mark.parametrize("dtype_label", ["bf16", "fp16", "fp32", "fp64"])
@pytest.mark.parametrize("head_cfg", HEAD_SHAPES, ids=[h[0] for h in HEAD_SHAPES])
@pytest.mark.parametrize("layout", ["packed", "fused"])
def test_staged_kernel_bit_exact(dtype_label, head_cfg, layout):
    """Large token counts take the staged kernel by default; force it and compare."""
    cfg = cfg_for(head_cfg, dtype_label, batch=1100, alloc=64, qkv_layout=layout,
                  request_order="shuffled")
    p = pos.build_position_sets(1100, 64, pos.RAGGED, SEED, 1, "cuda")[0]
    a = make_inputs(cfg, "cuda", SEED, p, cache_fill=SENTINEL)
    ref = _oracle_args(a)
    q_ref = oracle.fused_rope_kv_append(*ref)
    for path in ("staged", "auto"):
        b = a._replace(k_cache=a.k_cache.clone(), v_cache=a.v_cache.clone())
        q = ops().fused_rope_kv_append_ex(*b, path=path)
        assert bits_equal(q.cpu(), q_ref), path
        assert bits_equal(b.k_cache.cpu(), ref[6]), path
        assert bits_equal(b.v_cache.cpu(), ref[7]), path


@pytest.mark.parametrize("T", [1, 7, 148, 1000])
def test_staged_kernel_token_counts_and_partial_rotary(T):
    cfg = case("phi2", 32, 32, 80, T, 128, "fp16", pos.RAGGED, rotary_dim=32)
    p = pos.build_position_sets(T, 128, pos.RAGGED, SEED, 1, "cuda")[0]
    a = make_inputs(cfg, "cuda", SEED, p, cache_fill=SENTINEL)
    ref = _oracle_args(a)
    q_ref = oracle.fused_rope_kv_append(*ref)
    q = ops().fused_rope_kv_append_ex(*a, rotary_dim=32, path="staged")
    assert bits_equal(q.cpu(), q_ref)
    assert bits_equal(a.k_cache.cpu(), ref[6])
    assert bits_equal(a.v_cache.cpu(), ref[7])


@pytest.mark.parametrize("rotary_dim", [8, 4])
def test_staged_kernel_walks_many_metadata_blocks(rotary_dim):
    """One head of 8 fp16 dims per token: small rows give a grid of thousands of CTAs, and
    160,000 tokens make each CTA walk ~60-70 of them, so the shared metadata array (two blocks
    of 32 tokens) is refilled during the walk. rotary_dim 8: the cos/sin rows (16 bytes)
    travel in the stage with the token's rows; rotary_dim 4 (8-byte rows): the lanes load
    them a token ahead."""
    T, S = 160_000, 4
    cfg = case("tiny", 1, 1, 8, T, S, "fp16", pos.RAGGED, rotary_dim=rotary_dim,
               request_order="shuffled")
    p = pos.build_position_sets(T, S, pos.RAGGED, SEED, 1, "cuda")[0]
    a = make_inputs(cfg, "cuda", SEED, p, cache_fill=SENTINEL)
    ref = _oracle_args(a)
    q_ref = oracle.fused_rope_kv_append(*ref)
    extra = {} if rotary_dim == 8 else {"rotary_dim": rotary_dim}
    q = ops().fused_rope_kv_append_ex(*a, path="staged", **extra)
    assert bits_equal(q.cpu(), q_ref)
    assert bits_equal(a.k_cache.cpu(), ref[6])
    assert bits_equal(a.v_cache.cpu(), ref[7])


def test_staged_kernel_paged_cache_many_metadata_blocks():
    """The block-table lookups of later metadata blocks (160,000 tokens, pages of 2 rows)."""
    T, S, bs = 160_000, 4, 2
    cfg = case("tiny", 1, 1, 8, T, S, "fp16", pos.RAGGED, request_order="shuffled")
    p = pos.build_position_sets(T, S, pos.RAGGED, SEED, 1, "cuda")[0]
    a = make_inputs(cfg, "cuda", SEED, p, cache_fill=SENTINEL)
    max_blocks = S // bs
    num_blocks = T * max_blocks + 5
    perm = torch.randperm(num_blocks, generator=torch.Generator().manual_seed(4))[
        : T * max_blocks].view(T, max_blocks).to(a.positions.dtype)
    k_pages = torch.full((num_blocks, bs, 1, 8), 7.5, dtype=torch.float16, device="cuda")
    v_pages = torch.full_like(k_pages, 7.5)
    q = ops().paged_rope_kv_append(a.q, a.k, a.v, a.positions, a.cos, a.sin, k_pages, v_pages,
                                   perm.cuda(), a.request_indices, path="staged")
    ref = _oracle_args(a)
    q_ref = oracle.fused_rope_kv_append(*ref)
    assert bits_equal(q.cpu(), q_ref)
    ri, pp = a.request_indices.long().cpu(), a.positions.long().cpu()
    blk, row = perm.long()[ri, pp // bs], pp % bs
    assert bits_equal(k_pages.cpu()[blk, row], ref[6][ri, pp])
    assert bits_equal(v_pages.cpu()[blk, row], ref[7][ri, pp])


def test_staged_kernel_paged_cache():
    T, Hq, Hkv, D, S, bs = 400, 32, 8, 128, 256, 16
    cfg = case("gqa", Hq, Hkv, D, T, S, "bf16", pos.RAGGED, request_order="shuffled")
    p = pos.build_position_sets(T, S, pos.RAGGED, SEED, 1, "cuda")[0]
    a = make_inputs(cfg, "cuda", SEED, p, cache_fill=SENTINEL)
    max_blocks = S // bs
    num_blocks = T * max_blocks + 5
    perm = torch.randperm(num_blocks, generator=torch.Generator().manual_seed(3))[
        : T * max_blocks].view(T, max_blocks)
    k_pages = torch.full((num_blocks, bs, Hkv, D), 7.5, dtype=torch.bfloat16, device="cuda")
    v_pages = torch.full_like(k_pages, 7.5)
    q = ops().paged_rope_kv_append(a.q, a.k, a.v, a.positions, a.cos, a.sin, k_pages, v_pages,
                                   perm.cuda(), a.request_indices, path="staged")
    ref = _oracle_args(a)
    q_ref = oracle.fused_rope_kv_append(*ref)
    assert bits_equal(q.cpu(), q_ref)
    ri, pp = a.request_indices.long().cpu(), a.positions.long().cpu()
    blk, row = perm[ri, pp // bs], pp % bs
    assert bits_equal(k_pages.cpu()[blk, row], ref[6][ri, pp])
    assert bits_equal(v_pages.cpu()[blk, row], ref[7][ri, pp])


def test_staged_kernel_out_of_range_and_pdl():
    from decode_llm_kernel_b200 import cuda
    cuda.read_status(clear=True)
    cfg = cfg_for(("gqa", 32, 8, 128), "bf16", batch=300, alloc=32)
    p = torch.randint(0, 32, (300,), generator=torch.Generator().manual_seed(1))
    p[5] = 32        # outside the cache and the table
    a = make_inputs(cfg, "cuda", SEED, p.cuda(), cache_fill=SENTINEL)
    q = ops().fused_rope_kv_append_ex(*a, path="staged", pdl=True)
    assert cuda.read_status() & 5
    kc = a.k_cache.cpu()
    assert bool((kc[5] == 7.5).all())
    good = torch.ones(300, dtype=torch.bool)
    good[5] = False
    pv = p.clone()
    pv[5] = 0
    a2 = make_inputs(cfg, "cuda", SEED, pv.cuda(), cache_fill=SENTINEL)
    ref = _oracle_args(a2)
    q_ref = oracle.fused_rope_kv_append(*ref)
    assert bits_equal(q.cpu()[good], q_ref[good])


def test_host_pipeline_runs_steps_in_order_with_copies_overlapped():
    """capture_host_pipeline: several end-to-end steps in one graph; each step's q_out comes
    back to its pinned buffer and the caches end as if the steps ran one after another."""
    from decode_llm_kernel_b200.harness.decode_loop import DecodeStep, StepInputs, pinned_like
    from decode_llm_kernel_b200.rope_tables import build_rope_tables
    L, T, Hq, Hkv, D, S, depth = 4, 8, 32, 8, 128, 16, 3
    kcs = [torch.zeros(T, S, Hkv, D, dtype=torch.bfloat16, device="cuda") for _ in range(L)]
    vcs = [torch.zeros_like(kcs[0]) for _ in range(L)]
    cos, sin = build_rope_tables(S, D, 500000.0, device="cuda")
    g = torch.Generator().manual_seed(11)
    hosts, devs = [], []
    for _ in range(depth):
        h = StepInputs(torch.randn(L, T, Hq, D, generator=g).to(torch.bfloat16),
                       torch.randn(L, T, Hkv, D, generator=g).to(torch.bfloat16),
                       torch.randn(L, T, Hkv, D, generator=g).to(torch.bfloat16),
                       torch.randint(0, S, (T,), generator=g, dtype=torch.int64).to(torch.int32),
                       torch.randperm(T, generator=g).to(torch.int32))
        hp = pinned_like(h)
        hosts.append(hp)
        devs.append(StepInputs(*(torch.zeros_like(x, device="cuda") for x in
                                 (h.q, h.k, h.v, h.positions, h.request_indices))))
    pipe = DecodeStep(kcs, vcs, cos, sin).capture_host_pipeline(devs, hosts)
    for c in kcs + vcs:
        c.zero_()
    pipe.replay()
    torch.cuda.synchronize()
    ref_k = [torch.zeros(T, S, Hkv, D, dtype=torch.bfloat16) for _ in range(L)]
    ref_v = [torch.zeros(T, S, Hkv, D, dtype=torch.bfloat16) for _ in range(L)]
    for i, h in enumerate(hosts):
        for layer in range(L):
            q_ref = oracle.fused_rope_kv_append(h.q[layer], h.k[layer], h.v[layer], h.positions,
                                                cos.cpu(), sin.cpu(), ref_k[layer], ref_v[layer],
                                                h.request_indices)
            assert bits_equal(pipe.host_q_outs[i][layer].clone(), q_ref)
    for layer in range(L):
        assert bits_equal(kcs[layer].cpu(), ref_k[layer])
        assert bits_equal(vcs[layer].cpu(), ref_v[layer])


def test_staged_kernel_in_register_trig_within_the_reference_tolerance():
    from decode_llm_kernel_b200.rope_tables import inverse_frequencies
    cfg = cfg_for(("gqa", 32, 8, 128), "bf16", batch=700, alloc=4096, theta=500000.0)
    p = pos.build_position_sets(700, 4096, pos.RAGGED, SEED, 1, "cuda")[0]
    a = make_inputs(cfg, "cuda", SEED, p, cache_fill=SENTINEL)
    ref = _oracle_args(a)
    q_ref = oracle.fused_rope_kv_append(*ref)
    inv = inverse_frequencies(128, 500000.0).cuda()
    q = ops().fused_rope_kv_append_ex(*a, inv_freq=inv, path="staged").cpu()
    _assert_inreg_close(q, q_ref)
    assert bits_equal(a.v_cache.cpu(), ref[7])


def test_decode_loop_advances_positions_on_the_device():
    """A captured step ending with advance_positions replays three decode steps with no
    host-side position copy: each replay appends at the next position."""
    from decode_llm_kernel_b200.harness.decode_loop import DecodeStep, StepInputs
    from decode_llm_kernel_b200.rope_tables import build_rope_tables
    L, T, Hq, Hkv, D, S = 3, 8, 32, 8, 128, 32
    kcs = [torch.zeros(T, S, Hkv, D, dtype=torch.bfloat16, device="cuda") for _ in range(L)]
    vcs = [torch.zeros_like(kcs[0]) for _ in range(L)]
    cos, sin = build_rope_tables(S, D, 500000.0, device="cuda")
    g = torch.Generator().manual_seed(5)
    start = torch.randint(0, S - 4, (T,), generator=g, dtype=torch.int64).to(torch.int32)
    inp = StepInputs(torch.randn(L, T, Hq, D, generator=g).to(torch.bfloat16).cuda(),
                     torch.randn(L, T, Hkv, D, generator=g).to(torch.bfloat16).cuda(),
                     torch.randn(L, T, Hkv, D, generator=g).to(torch.bfloat16).cuda(),
                     start.clone().cuda(), torch.arange(T, dtype=torch.int32).cuda())
    step = DecodeStep(kcs, vcs, cos, sin, pdl=True, advance_positions=True)
    cap = step.capture(inp)
    for c in kcs + vcs:
        c.zero_()
    assert torch.equal(inp.positions.cpu(), start)      # warm-up did not move the loop
    ref_k = [torch.zeros(T, S, Hkv, D, dtype=torch.bfloat16) for _ in range(L)]
    ref_v = [torch.zeros(T, S, Hkv, D, dtype=torch.bfloat16) for _ in range(L)]
    for s in range(3):
        cap.replay()
        torch.cuda.synchronize()
        for layer in range(L):
            q_ref = oracle.fused_rope_kv_append(
                inp.q[layer].cpu(), inp.k[layer].cpu(), inp.v[layer].cpu(), start + s,
                cos.cpu(), sin.cpu(), ref_k[layer], ref_v[layer], inp.request_indices.cpu())
            assert bits_equal(cap.q_out[layer].cpu(), q_ref)
    assert torch.equal(inp.positions.cpu(), start + 3)
    for layer in range(L):
        assert bits_equal(kcs[layer].cpu(), ref_k[layer])
        assert bits_equal(vcs[layer].cpu(), ref_v[layer])


@pytest.mark.parametrize("label", ["graph_cuda_fused", "graph_cuda_separate", "cuda_fused",
                                   "cuda_separate"])
def test_ladder_runners_drive_the_ops(label):
    """The operator ladder's drivers (harness/runners.py) over this build's ops: the eager
    runner calls through the binding, the graph runner replays one graph per device position
    set; every call in a rotation over three sets lands bit-exact, twice round."""
    from decode_llm_kernel_b200.harness import runners
    _, op_name, kind = next(r for r in runners.RUNGS if r[0] == label)
    op = kernel(op_name)
    cfg = cfg_for(("gqa", 32, 8, 128), "bf16", batch=8, alloc=64)
    sets = pos.build_position_sets(8, 64, pos.RAGGED, SEED, 3, "cuda")
    args = make_inputs(cfg, "cuda", SEED, sets[0])
    runner = kind(op, args, sets)
    for i in range(6):
        p = sets[i % 3]
        expect_in = _oracle_args(args._replace(positions=p))
        out = runner()
        torch.cuda.synchronize()
        # the oracle sees the caches as they were before this call
        q_ref = oracle.fused_rope_kv_append(*expect_in)
        assert bits_equal(out.cpu(), q_ref), (label, i)
        assert bits_equal(args.k_cache.cpu(), expect_in[6]), (label, i)
        assert bits_equal(args.v_cache.cpu(), expect_in[7]), (label, i)
    runner.release()
