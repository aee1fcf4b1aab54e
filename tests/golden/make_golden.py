"""Generates the golden fixtures in this directory from the reference project's own oracle.

Run where the reference checkout is present, naming it in $DECODE_REFERENCE_ROOT:

    DECODE_REFERENCE_ROOT=/path/to/reference python tests/golden/make_golden.py

It imports `decode_kernels.reference` from the reference checkout (rope_cache.py:3-36),
builds seeded inputs, runs `fused_rope_kv_append_ref` on CPU and stores inputs and outputs
as .npz files. The fixtures are what pin the CPU oracle (oracle/) and the CUDA kernels to the
reference; the GPU machines never see the reference itself.

Two cases go beyond the reference's own surface and are generated with the reference's
`apply_rope` on a slice, as the extension defines them:
  * partial rotary (Phi-2 style, rotary_dim < head_dim): apply_rope on x[..., :R] with a
    [P, R] table from build_rope_tables(P, R), dims [R, D) copied unchanged;
  * head-major caches [B, Hkv, S, D]: the reference oracle writes through the transposed view
    cache.transpose(1, 2), which is how its HF seam addresses such a cache.
"""
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.environ.get("DECODE_REFERENCE_ROOT")
SENTINEL = 7.5
SEED = 1234

DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16,
          "fp64": torch.float64}

# name, dtype, T, Hq, Hkv, D, R (None = D), B, S, theta, layout, mapping, index dtype,
# cache layout, position recipe
CASES = [
    ("llama3_8b_bf16_int32", "bf16", 8, 32, 8, 128, None, 8, 64, 500000.0, "packed",
     "identity", "int32", "token_major", "edges"),
    ("mistral_fp16_permuted", "fp16", 6, 32, 8, 128, None, 6, 32, 10000.0, "packed",
     "permuted", "int64", "token_major", "ragged"),
    ("mha_fp32_strided", "fp32", 4, 8, 8, 64, None, 4, 16, 10000.0, "strided",
     "identity", "int64", "token_major", "ragged"),
    ("falcon_mqa_bf16", "bf16", 3, 71, 1, 64, None, 3, 8, 10000.0, "packed",
     "identity", "int64", "token_major", "edges"),
    ("phi3_d96_bf16_strided", "bf16", 2, 32, 32, 96, None, 2, 16, 10000.0, "strided",
     "permuted", "int32", "token_major", "ragged"),
    ("gqa_fp64", "fp64", 3, 4, 2, 32, None, 3, 8, 10000.0, "packed",
     "identity", "int64", "token_major", "ragged"),
    ("phi2_partial_fp16", "fp16", 4, 32, 32, 80, 32, 4, 16, 10000.0, "packed",
     "identity", "int32", "token_major", "same"),
    ("gqa_bf16_head_major", "bf16", 4, 8, 2, 64, None, 4, 16, 500000.0, "packed",
     "permuted", "int64", "head_major", "edges"),
    ("gqa_bf16_single_token", "bf16", 1, 8, 2, 128, None, 1, 4, 10000.0, "packed",
     "identity", "int64", "token_major", "last"),
    ("empty_bf16", "bf16", 0, 32, 8, 128, None, 0, 4, 10000.0, "packed",
     "identity", "int64", "token_major", "ragged"),
]


def _reference():
    if not REF_ROOT or not os.path.isdir(os.path.join(REF_ROOT, "decode_kernels")):
        raise SystemExit("set DECODE_REFERENCE_ROOT to the reference checkout")
    sys.path.insert(0, REF_ROOT)
    from decode_kernels.reference import rope_cache  # noqa: E402
    return rope_cache


def _positions(recipe, T, S, g):
    if T == 0:
        return torch.zeros(0, dtype=torch.int64)
    if recipe == "edges":
        p = torch.randint(0, S, (T,), generator=g)
        p[0] = 0
        p[-1] = S - 1
        return p
    if recipe == "same":
        # duplicate positions across sequences: slots stay unique because the rows differ
        return torch.full((T,), S // 2, dtype=torch.int64)
    if recipe == "last":
        return torch.full((T,), S - 1, dtype=torch.int64)
    return torch.randint(0, S, (T,), generator=g)


def _raw(t):
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def make_case(rc, spec):
    (name, dtl, T, Hq, Hkv, D, R, B, S, theta, layout, mapping, idx, cache_layout,
     recipe) = spec
    R = D if R is None else R
    dt = DTYPES[dtl]
    g = torch.Generator().manual_seed(SEED)
    if layout == "packed":
        q = torch.randn(T, Hq, D, generator=g).to(dt)
        k = torch.randn(T, Hkv, D, generator=g).to(dt)
        v = torch.randn(T, Hkv, D, generator=g).to(dt)
        fused = None
    else:
        fused = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(dt)
        parts = fused.split([Hq * D, Hkv * D, Hkv * D], dim=-1)
        q, k, v = (p.view(T, -1, D) for p in parts)
    positions = _positions(recipe, T, S, g)
    if mapping == "permuted":
        request_indices = torch.randperm(T, generator=g)
    else:
        request_indices = torch.arange(T)
    index_dtype = torch.int32 if idx == "int32" else torch.int64
    positions = positions.to(index_dtype)
    request_indices = request_indices.to(index_dtype)

    cos, sin = rc.build_rope_tables(S, R, theta)
    if cache_layout == "token_major":
        k_cache = torch.full((B, S, Hkv, D), SENTINEL, dtype=dt)
        v_cache = torch.full((B, S, Hkv, D), SENTINEL, dtype=dt)
        k_view, v_view = k_cache, v_cache
    else:
        k_cache = torch.full((B, Hkv, S, D), SENTINEL, dtype=dt)
        v_cache = torch.full((B, Hkv, S, D), SENTINEL, dtype=dt)
        k_view, v_view = k_cache.transpose(1, 2), v_cache.transpose(1, 2)

    # The reference indexes with int64 tensors; int32 is the kernel-side variant of the same.
    pos64, ri64 = positions.to(torch.int64), request_indices.to(torch.int64)
    if R == D:
        q_out = rc.fused_rope_kv_append_ref(q, k, v, pos64, cos, sin, k_view, v_view, ri64)
    else:
        cos_p, sin_p = cos[pos64].float(), sin[pos64].float()
        q_rot = rc.apply_rope(q[..., :R].float(), cos_p, sin_p).to(dt)
        k_rot = rc.apply_rope(k[..., :R].float(), cos_p, sin_p).to(dt)
        q_out = torch.cat((q_rot, q[..., R:]), dim=-1)
        k_view[ri64, pos64] = torch.cat((k_rot, k[..., R:]), dim=-1)
        v_view[ri64, pos64] = v

    k_slots = k_view[ri64, pos64].clone()
    v_slots = v_view[ri64, pos64].clone()
    # Everything outside the addressed slots must still be the sentinel.
    mask = torch.zeros(B, S, dtype=torch.bool)
    mask[ri64, pos64] = True
    assert bool((k_view[~mask] == SENTINEL).all()) and bool((v_view[~mask] == SENTINEL).all())

    meta = dict(name=name, dtype=dtl, T=T, Hq=Hq, Hkv=Hkv, D=D, R=R, B=B, S=S, theta=theta,
                layout=layout, mapping=mapping, index_dtype=idx, cache_layout=cache_layout,
                sentinel=SENTINEL, seed=SEED,
                generator="reference decode_kernels.reference.rope_cache on CPU, torch "
                          + torch.__version__)
    arrays = dict(meta=np.array(json.dumps(meta)), positions=positions.numpy(),
                  request_indices=request_indices.numpy(), cos=cos.numpy(), sin=sin.numpy(),
                  q_out=_raw(q_out), k_slots=_raw(k_slots), v_slots=_raw(v_slots))
    if fused is None:
        arrays.update(q=_raw(q), k=_raw(k), v=_raw(v))
    else:
        arrays.update(fused=_raw(fused))
    np.savez(os.path.join(HERE, f"{name}.npz"), **arrays)
    return meta


def main():
    rc = _reference()
    for spec in CASES:
        meta = make_case(rc, spec)
        print(f"wrote {meta['name']}.npz")


if __name__ == "__main__":
    main()
