"""The tensors of one call of the op, built from a Workload (harness/configs.py).

`make_inputs(w, device, seed, positions)` returns an `OpInputs` -- the nine arguments of
fused_rope_kv_append in their order -- for workload `w`:

  q, k, v          seeded N(0, 1) draws in w.dtype. qkv_layout "packed": three contiguous
                   tensors; "fused": [T, H, D] views into one [T, (Hq + 2 Hkv) D] projection,
                   so the token stride is the fused width and only head_dim is contiguous.
  positions        the caller's tensor, moved to the device in w's index dtype.
  cos, sin         fp32 [S, rotary] tables (rope_tables.build_rope_tables, theta = w.theta).
  request_indices  request_order "identity": token t writes row t; "shuffled": a seeded
                   permutation, so each row is still written once but the token index is no
                   longer the row.
  k_cache, v_cache [B, S, Hkv, D] views in w.cache_layout, filled with a constant (a
                   sentinel that shows untouched slots) or with N(0, 1) draws ("normal").

`case(...)` makes the small Workloads the tests and the validation gate use.
"""
from dataclasses import replace
from typing import NamedTuple

import torch

from ..rope_tables import build_rope_tables
from .configs import Workload

# The value a test prefills caches with, so a slot the op must not touch can be recognised.
SENTINEL = 7.5


class OpInputs(NamedTuple):
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    positions: torch.Tensor
    cos: torch.Tensor
    sin: torch.Tensor
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    request_indices: torch.Tensor


def case(name, num_q_heads, num_kv_heads, head_dim, batch, cache_alloc_len, dtype_label,
         positions="ragged", **fields):
    """A small Workload for tests: theta 1e4 and int64 indices unless given (the reference's
    harness defaults), one layer, no sharding."""
    fields.setdefault("theta", 10000.0)
    fields.setdefault("index_dtype", "int64")
    return Workload(name, num_q_heads, num_kv_heads, head_dim, batch, cache_alloc_len,
                    dtype_label, positions=positions, **fields)


def _normal(shape, gen, dtype, device):
    # drawn in fp32 and rounded once, so every dtype sees the same distribution
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dtype)


def make_qkv(w, gen, device, layout=None):
    layout = layout or w.qkv_layout
    T, D = w.batch, w.head_dim
    heads = (w.num_q_heads, w.num_kv_heads, w.num_kv_heads)
    if layout == "packed":
        return tuple(_normal((T, h, D), gen, w.dtype, device) for h in heads)
    if layout == "fused":
        projection = _normal((T, sum(heads) * D), gen, w.dtype, device)
        return tuple(part.view(T, h, D)
                     for part, h in zip(projection.split([h * D for h in heads], dim=1), heads))
    raise ValueError(f"unknown qkv_layout {layout!r}")


def request_rows(w, seed, device, order=None):
    order = order or w.request_order
    if order == "identity":
        rows = torch.arange(w.batch)
    elif order == "shuffled":
        rows = torch.randperm(w.batch, generator=torch.Generator().manual_seed(seed ^ 0x5EED))
    else:
        raise ValueError(f"unknown request_order {order!r}")
    return rows.to(device=device, dtype=w.index_torch_dtype)


def make_cache(w, device, fill, gen=None):
    """A [B, S, Hkv, D] view of one cache in w.cache_layout. fill: a number, or "normal"."""
    B, S, H, D = w.batch, w.cache_alloc_len, w.num_kv_heads, w.head_dim
    token_major = w.cache_layout == "token_major"
    storage = torch.empty((B, S, H, D) if token_major else (B, H, S, D), dtype=w.dtype,
                          device=device)
    if fill == "normal":
        flat = storage.view(-1)
        slab = 1 << 28           # fill in slabs: a large cache never needs an fp32 copy
        for lo in range(0, flat.numel(), slab):
            hi = min(flat.numel(), lo + slab)
            flat[lo:hi] = _normal((hi - lo,), gen, w.dtype, device)
    else:
        storage.fill_(float(fill))
    return storage if token_major else storage.transpose(1, 2)


def make_inputs(w, device, seed, positions, *, cache_fill=0.0, qkv_layout=None,
                request_order=None):
    """One call's OpInputs for workload w (see the module docstring)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    q, k, v = make_qkv(w, gen, device, qkv_layout)
    cos, sin = build_rope_tables(w.cache_alloc_len, w.rotary, w.theta, device=device)
    rows = request_rows(w, seed, device, request_order)
    k_cache = make_cache(w, device, cache_fill, gen)
    v_cache = make_cache(w, device, cache_fill, gen)
    positions = positions.to(device=device, dtype=w.index_torch_dtype)
    return OpInputs(q, k, v, positions, cos, sin, k_cache, v_cache, rows)


def with_layout(w, **fields):
    """w with other layout fields (qkv_layout, request_order, cache_layout, ...)."""
    return replace(w, **fields)
