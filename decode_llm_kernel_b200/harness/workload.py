"""One invocation's tensors, and the registry of head shapes (benchmarks/workload.py:31-126 of
the reference).

A `Config` fixes the head shape, batch, cache length, dtype and position mode, plus the serving
variants the reference's gate exercises: strided Q/K/V views of one fused QKV projection, and a
permuted token -> request mapping. The extensions used by the B200 workloads are here too:
RoPE theta, int32 indices, partial rotary, head-major caches and N(0, 1)-filled caches.
"""
import itertools
from dataclasses import asdict, dataclass
from typing import NamedTuple

import torch

from ..rope_tables import build_rope_tables
from . import positions as pos

DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16,
          "fp64": torch.float64}
INDEX_DTYPES = {"int32": torch.int32, "int64": torch.int64}

# Attention shapes of released models (label, Hq, Hkv, head_dim): Llama-2-7B (MHA),
# Mistral-7B / Llama-3-8B (GQA 32:8), Falcon-7B (MQA 71:1, head_dim 64), Phi-3-mini
# (head_dim 96, the non-power-of-two half).
HEAD_CONFIGS = [("mha", 32, 32, 128), ("gqa", 32, 8, 128), ("mqa", 71, 1, 64),
                ("mha96", 32, 32, 96)]

CACHE_SENTINEL = 7.5
NUM_POSITION_SETS = 8

PACKED = "packed"
STRIDED = "strided"
LAYOUTS = (PACKED, STRIDED)

IDENTITY = "identity"
PERMUTED = "permuted"
REQUEST_MAPPINGS = (IDENTITY, PERMUTED)

TOKEN_MAJOR = "token_major"
HEAD_MAJOR = "head_major"
CACHE_LAYOUTS = (TOKEN_MAJOR, HEAD_MAJOR)

SERVING_VARIANT_BATCHES = (1, 32)


@dataclass(frozen=True)
class Config:
    head_label: str
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    num_requests: int
    cache_alloc_len: int
    dtype_label: str
    position_mode: str
    layout: str = PACKED
    request_mapping: str = IDENTITY
    theta: float = 10000.0
    rotary_dim: int = 0             # 0: full head_dim (the reference's semantics)
    index_dtype: str = "int64"
    cache_layout: str = TOKEN_MAJOR

    @property
    def dtype(self):
        return DTYPES[self.dtype_label]

    @property
    def rotary(self):
        return self.rotary_dim or self.head_dim

    def as_row(self):
        return asdict(self)

    def label(self):
        label = (f"{self.head_label}_b{self.num_requests}_alloc{self.cache_alloc_len}"
                 f"_{self.dtype_label}_{self.position_mode}")
        if (self.layout, self.request_mapping) != (PACKED, IDENTITY):
            label += f"_{self.layout}_{self.request_mapping}"
        if self.rotary_dim:
            label += f"_rot{self.rotary_dim}"
        if self.cache_layout != TOKEN_MAJOR:
            label += f"_{self.cache_layout}"
        return label


class OpArgs(NamedTuple):
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    positions: torch.Tensor
    cos: torch.Tensor
    sin: torch.Tensor
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    request_indices: torch.Tensor


def build_position_sets(cfg, seed, device, num_sets=NUM_POSITION_SETS):
    return pos.build_position_sets(cfg.num_requests, cfg.cache_alloc_len, cfg.position_mode,
                                   seed, num_sets, device, INDEX_DTYPES[cfg.index_dtype])


def build_request_mapping(num_requests, kind, seed, device, dtype=torch.long):
    """Which cache row each token targets. A permuted mapping is a bijection, so slots stay
    unique while `token index == request index` stops holding."""
    if kind == IDENTITY:
        return torch.arange(num_requests, device=device, dtype=dtype)
    if kind == PERMUTED:
        g = torch.Generator().manual_seed(seed + 9973)
        return torch.randperm(num_requests, generator=g).to(device=device, dtype=dtype)
    raise ValueError(f"unknown request mapping {kind!r}, expected one of {REQUEST_MAPPINGS}")


def _randn(shape, g, dt, device):
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(dt)


def build_qkv(t, hq, hkv, d, dt, device, g, layout):
    if layout == PACKED:
        return tuple(_randn((t, h, d), g, dt, device) for h in (hq, hkv, hkv))
    if layout == STRIDED:
        # views of one fused QKV projection: head_dim contiguous, token stride = fused width
        fused = _randn((t, (hq + 2 * hkv) * d), g, dt, device)
        parts = fused.split([hq * d, hkv * d, hkv * d], dim=-1)
        return tuple(p.view(t, -1, d) for p in parts)
    raise ValueError(f"unknown layout {layout!r}, expected one of {LAYOUTS}")


def make_cache(cfg, device, fill, g=None):
    """A [B, S, Hkv, D] view of a cache in cfg.cache_layout, filled with a constant or with
    N(0, 1) draws (fill == "normal")."""
    B, S, H, D = cfg.num_requests, cfg.cache_alloc_len, cfg.num_kv_heads, cfg.head_dim
    shape = (B, S, H, D) if cfg.cache_layout == TOKEN_MAJOR else (B, H, S, D)
    if fill == "normal":
        storage = torch.empty(shape, dtype=cfg.dtype, device=device)
        # Fill in slabs so a large cache never needs an fp32 copy of itself.
        flat = storage.view(-1)
        step = 1 << 28
        for start in range(0, flat.numel(), step):
            n = min(step, flat.numel() - start)
            flat[start:start + n] = torch.randn(n, generator=g, device=device,
                                                dtype=torch.float32).to(cfg.dtype)
    else:
        storage = torch.full(shape, float(fill), dtype=cfg.dtype, device=device)
    return storage if cfg.cache_layout == TOKEN_MAJOR else storage.transpose(1, 2)


def build_op_args(cfg, device, seed, positions, *, sentinel_cache=False, request_mapping=None,
                  layout=None, cache_fill=None):
    """Allocate one invocation's tensors. RoPE tables stay fp32 [S, rotary]."""
    t, hq, hkv, d = cfg.num_requests, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
    request_mapping = cfg.request_mapping if request_mapping is None else request_mapping
    layout = cfg.layout if layout is None else layout
    g = torch.Generator(device=device).manual_seed(seed)
    q, k, v = build_qkv(t, hq, hkv, d, cfg.dtype, device, g, layout)
    cos, sin = build_rope_tables(cfg.cache_alloc_len, cfg.rotary, cfg.theta, device=device)
    index_dtype = INDEX_DTYPES[cfg.index_dtype]
    request_indices = build_request_mapping(t, request_mapping, seed, device, index_dtype)
    if cache_fill is None:
        cache_fill = CACHE_SENTINEL if sentinel_cache else 0.0
    k_cache = make_cache(cfg, device, cache_fill, g)
    v_cache = make_cache(cfg, device, cache_fill, g)
    positions = positions.to(device=device, dtype=index_dtype)
    return OpArgs(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices)


def make_thunk(fn, args, position_sets):
    """Timed callable. Cycles pre-built device position tensors; no host generation or sync."""
    cyc = itertools.cycle(position_sets)
    q, k, v = args.q, args.k, args.v
    cos, sin = args.cos, args.sin
    kc, vc, ri = args.k_cache, args.v_cache, args.request_indices

    def run():
        fn(q, k, v, next(cyc), cos, sin, kc, vc, ri)
    return run


def build_matrix(quick=False, position_modes=(pos.RAGGED,), head_labels=None, batches=None,
                 allocs=None, dtypes=None, include_serving_variants=True):
    """The sweep's configurations: head shapes x batches x cache lengths x dtypes."""
    if quick:
        batches = batches or [1, 32]
        allocs = allocs or [2048]
        dtypes = dtypes or ["bf16"]
    else:
        batches = batches or [1, 8, 32, 128]
        allocs = allocs or [128, 2048]
        dtypes = dtypes or ["bf16", "fp16", "fp32"]
    heads = HEAD_CONFIGS
    if head_labels:
        heads = [h for h in heads if h[0] in head_labels]
    variants = [pair for pair in itertools.product(LAYOUTS, REQUEST_MAPPINGS)
                if pair != (PACKED, IDENTITY)]
    for (hl, hq, hkv, hd), b, alloc, dl, pm in itertools.product(
            heads, batches, allocs, dtypes, position_modes):
        yield Config(hl, hq, hkv, hd, b, alloc, dl, pm)
        if include_serving_variants and b in SERVING_VARIANT_BATCHES:
            for layout, request_mapping in variants:
                yield Config(hl, hq, hkv, hd, b, alloc, dl, pm, layout, request_mapping)
