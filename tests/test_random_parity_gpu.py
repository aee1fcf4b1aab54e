"""Seeded random configurations through the fused op, bit for bit against the CPU oracle:
head shapes, head_dim (even, 8..256), partial rotary, dtypes, index dtypes, packed / fused-QKV
strided / misaligned inputs, token-major / head-major / paged caches, permuted requests, and
token counts that land on both kernels (register below 512 tokens, staged from 512)."""
import random

import pytest
import torch

from decode_llm_kernel_b200.rope_tables import build_rope_tables
from golden_io import bits_equal
from oracle import oracle

pytestmark = pytest.mark.gpu

DTYPES = [torch.bfloat16, torch.float16, torch.float32, torch.float64]
CASES = 48


def _case(seed):
    rng = random.Random(seed)
    dt = rng.choice(DTYPES)
    D = rng.choice([8, 16, 32, 64, 80, 96, 128, 160, 256])
    R = D if rng.random() < 0.7 else rng.choice([r for r in range(2, D + 1, 2) if r <= D])
    Hkv = rng.choice([1, 2, 4, 8])
    Hq = Hkv * rng.choice([1, 2, 4, 8]) + (rng.choice([0, 3]) if Hkv == 1 else 0)
    T = rng.choice([0, 1, 2, 5, 33, 130, 520, 777])
    S = rng.choice([4, 16, 64])
    layout = rng.choice(["packed", "strided", "misaligned"])
    cache = rng.choice(["token_major", "head_major", "paged"])
    index = rng.choice([torch.int32, torch.int64])
    permuted = rng.random() < 0.5
    return dict(dt=dt, D=D, R=R, Hq=Hq, Hkv=Hkv, T=T, S=S, layout=layout, cache=cache,
                index=index, permuted=permuted, seed=seed)


def _inputs(c):
    g = torch.Generator().manual_seed(c["seed"])
    T, Hq, Hkv, D, dt = c["T"], c["Hq"], c["Hkv"], c["D"], c["dt"]
    if c["layout"] == "strided":
        fused = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(dt)
        q, k, v = (p.view(T, h, D) for p, h in zip(fused.split([Hq * D, Hkv * D, Hkv * D], dim=-1),
                                                  (Hq, Hkv, Hkv)))
    else:
        q = torch.randn(T, Hq, D, generator=g).to(dt)
        k = torch.randn(T, Hkv, D, generator=g).to(dt)
        v = torch.randn(T, Hkv, D, generator=g).to(dt)
    pos = torch.randint(0, c["S"], (T,), generator=g)
    ri = torch.randperm(T, generator=g) if c["permuted"] else torch.arange(T)
    return q, k, v, pos.to(c["index"]), ri.to(c["index"])


def _to_device(t, misaligned):
    if not misaligned or t.numel() == 0:
        return t.cuda()
    buf = torch.empty(t.numel() + 1, dtype=t.dtype, device="cuda")
    view = buf[1:].view(t.shape)
    view.copy_(t)
    return view


@pytest.mark.parametrize("seed", range(CASES))
def test_random_configuration_bit_exact(seed):
    from decode_llm_kernel_b200.cuda import ops
    c = _case(seed)
    q, k, v, pos, ri = _inputs(c)
    T, Hkv, D, R, S, dt = c["T"], c["Hkv"], c["D"], c["R"], c["S"], c["dt"]
    cos, sin = build_rope_tables(S, R, 10000.0 if seed % 2 else 500000.0)
    mis = c["layout"] == "misaligned"
    qd, kd, vd = (_to_device(x, mis) for x in (q, k, v))
    if c["layout"] == "strided" and T > 0:
        fused = torch.cat([q.reshape(T, -1), k.reshape(T, -1), v.reshape(T, -1)], dim=1).cuda()
        Hq = q.shape[1]
        qd, kd, vd = (p.view(T, h, D) for p, h in zip(
            fused.split([Hq * D, Hkv * D, Hkv * D], dim=-1), (Hq, Hkv, Hkv)))
    kw = {"rotary_dim": R} if R != D else {}
    # reference result on the CPU: a token-major cache of T requests
    kc_ref = torch.full((T, S, Hkv, D), 7.5, dtype=dt)
    vc_ref = kc_ref.clone()
    q_ref = oracle.fused_rope_kv_append(q, k, v, pos, cos, sin, kc_ref, vc_ref, ri)
    if c["cache"] == "paged":
        bs = 4
        nblk = T * (S // bs) + 2
        perm = torch.randperm(nblk, generator=torch.Generator().manual_seed(seed))[
            : T * (S // bs)].view(T, S // bs).to(c["index"])
        kp = torch.full((nblk, bs, Hkv, D), 7.5, dtype=dt, device="cuda")
        vp = torch.full_like(kp, 7.5)
        out = ops.paged_rope_kv_append(qd, kd, vd, pos.cuda(), cos.cuda(), sin.cuda(), kp, vp,
                                       perm.cuda(), ri.cuda(), **kw)
        blk = perm.long()[ri.long(), pos.long() // bs]
        row = pos.long() % bs
        assert bits_equal(kp.cpu()[blk, row], kc_ref[ri.long(), pos.long()])
        assert bits_equal(vp.cpu()[blk, row], vc_ref[ri.long(), pos.long()])
    else:
        if c["cache"] == "token_major":
            kc = torch.full((T, S, Hkv, D), 7.5, dtype=dt, device="cuda")
            vc = torch.full_like(kc, 7.5)
            kview, vview = kc, vc
            extra = {}
        else:
            kc = torch.full((T, Hkv, S, D), 7.5, dtype=dt, device="cuda")
            vc = torch.full_like(kc, 7.5)
            kview, vview = kc.transpose(1, 2), vc.transpose(1, 2)
            extra = {"strided_cache": True}
        out = ops.fused_rope_kv_append_ex(qd, kd, vd, pos.cuda(), cos.cuda(), sin.cuda(),
                                          kview, vview, ri.cuda(), **kw, **extra)
        assert bits_equal(kview.cpu().contiguous(), kc_ref)
        assert bits_equal(vview.cpu().contiguous(), vc_ref)
    assert bits_equal(out.cpu(), q_ref)
