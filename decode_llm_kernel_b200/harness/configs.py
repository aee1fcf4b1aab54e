"""Workloads of this path: the shape of one call (or one multi-layer step) and how it shards.

The five B200 workloads, at full size:

  llama3_8b_b8        one layer, batch 8, 32 Q / 8 KV heads, head_dim 128, theta 5e5, bf16,
                      cache [8, 4096, 8, 128], int32 positions uniform in [0, 4095]
  llama3_8b_decode32  a 32-layer decode step under a CUDA graph, batch 64, same heads,
                      per-layer caches [64, 8192, 8, 128], positions include 0 and 8191
  llama3_70b_tp       batch 256, 64 Q / 8 KV heads, theta 5e5, bf16, cache [256, 8192, 8, 128],
                      sharded by KV head over 1/2/4/8 GPUs (8 Q heads per KV head)
  mistral_b4096       batch 4096 sharded by batch, 32 / 8 heads, theta 1e4, fp16, per-GPU cache
                      [4096/n, 4096, 8, 128]: the bandwidth-bound one
  phi2_partial        batch 128, 32 / 32 heads, head_dim 80 with rotary_dim 32, theta 1e4, fp16,
                      cache [128, 2048, 32, 80], positions with duplicates across sequences

The same dataclass describes the small cases the tests build (harness/inputs.py): three layout
fields select the serving variants a kernel must handle -- Q/K/V as separate tensors or as
views of one fused projection, identity or shuffled token -> request rows, token-major or
head-major cache storage.

Caches are token-major [B, S, Hkv, D] (the reference's layout); the same bytes as the
[B, Hkv, S, D] notation. Inputs and caches are seeded N(0, 1) draws: no dataset is involved.
"""
from dataclasses import dataclass, replace

import torch

from .timing import bytes_per_token

DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16,
          "fp64": torch.float64}
INDEX_DTYPES = {"int32": torch.int32, "int64": torch.int64}

# Attention head shapes of released models (name, Hq, Hkv, head_dim): Llama-2-7B (MHA),
# Mistral-7B / Llama-3-8B (GQA 32:8), Falcon-7B (MQA 71:1, head_dim 64), Phi-3-mini (head_dim
# 96, whose rotate_half half is 48, not a power of two).
HEAD_SHAPES = (("mha", 32, 32, 128), ("gqa", 32, 8, 128), ("mqa", 71, 1, 64),
               ("mha96", 32, 32, 96))

QKV_LAYOUTS = ("packed", "fused")               # separate tensors | views of one projection
REQUEST_ORDERS = ("identity", "shuffled")       # token t -> row t | a seeded permutation
CACHE_LAYOUTS = ("token_major", "head_major")


@dataclass(frozen=True)
class Workload:
    name: str
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    batch: int
    cache_alloc_len: int
    dtype_label: str
    theta: float = 10000.0
    rotary_dim: int = 0
    layers: int = 1
    index_dtype: str = "int32"
    positions: str = "uniform_random"   # uniform_random | edges | duplicates | ragged | last
    shard: str = "none"                 # none | kv_head | batch
    qkv_layout: str = "packed"
    request_order: str = "identity"
    cache_layout: str = "token_major"

    def __post_init__(self):
        if self.qkv_layout not in QKV_LAYOUTS:
            raise ValueError(f"qkv_layout {self.qkv_layout!r} not in {QKV_LAYOUTS}")
        if self.request_order not in REQUEST_ORDERS:
            raise ValueError(f"request_order {self.request_order!r} not in {REQUEST_ORDERS}")
        if self.cache_layout not in CACHE_LAYOUTS:
            raise ValueError(f"cache_layout {self.cache_layout!r} not in {CACHE_LAYOUTS}")

    @property
    def dtype(self):
        return DTYPES[self.dtype_label]

    @property
    def index_torch_dtype(self):
        return INDEX_DTYPES[self.index_dtype]

    @property
    def rotary(self):
        return self.rotary_dim or self.head_dim

    @property
    def elem_bytes(self):
        return torch.empty(0, dtype=self.dtype).element_size()

    def label(self):
        parts = [self.name, f"b{self.batch}", f"s{self.cache_alloc_len}", self.dtype_label,
                 self.positions]
        parts += [x for x, default in ((self.qkv_layout, "packed"),
                                       (self.request_order, "identity"),
                                       (self.cache_layout, "token_major")) if x != default]
        if self.rotary_dim and self.rotary_dim != self.head_dim:
            parts.append(f"rot{self.rotary_dim}")
        return "_".join(parts)

    def bytes_per_token(self):
        return bytes_per_token(self.num_q_heads, self.num_kv_heads, self.head_dim,
                               self.elem_bytes, self.rotary_dim or None)

    def bytes_per_call(self):
        return self.batch * self.bytes_per_token()

    def bytes_per_step(self):
        return self.layers * self.bytes_per_call()

    def cache_bytes(self):
        return (2 * self.layers * self.batch * self.cache_alloc_len * self.num_kv_heads
                * self.head_dim * self.elem_bytes)

    def shard_for(self, rank, world):
        """This rank's slice: KV heads (and their Q heads) or batch rows. No exchange step."""
        if world == 1 or self.shard == "none":
            return self
        if self.shard == "kv_head":
            if self.num_kv_heads % world:
                raise ValueError(f"{self.num_kv_heads} KV heads do not split over {world}")
            return replace(self, num_q_heads=self.num_q_heads // world,
                           num_kv_heads=self.num_kv_heads // world)
        if self.shard == "batch":
            if self.batch % world:
                raise ValueError(f"batch {self.batch} does not split over {world}")
            return replace(self, batch=self.batch // world)
        raise ValueError(f"unknown shard kind {self.shard!r}")

    def describe(self):
        return {"workload": self.name, "batch": self.batch, "num_q_heads": self.num_q_heads,
                "num_kv_heads": self.num_kv_heads, "head_dim": self.head_dim,
                "rotary_dim": self.rotary, "theta": self.theta,
                "cache_alloc_len": self.cache_alloc_len, "layers": self.layers,
                "dtype": self.dtype_label, "index_dtype": self.index_dtype,
                "cache_layout": ("token_major [B, S, Hkv, D]" if self.cache_layout == "token_major"
                                 else "head_major [B, Hkv, S, D]")}


WORKLOADS = {
    "llama3_8b_b8": Workload("llama3_8b_b8", 32, 8, 128, 8, 4096, "bf16", 500000.0),
    "llama3_8b_decode32": Workload("llama3_8b_decode32", 32, 8, 128, 64, 8192, "bf16",
                                   500000.0, layers=32, positions="edges"),
    "llama3_70b_tp": Workload("llama3_70b_tp", 64, 8, 128, 256, 8192, "bf16", 500000.0,
                              shard="kv_head"),
    "mistral_b4096": Workload("mistral_b4096", 32, 8, 128, 4096, 4096, "fp16", 10000.0,
                              shard="batch"),
    "phi2_partial": Workload("phi2_partial", 32, 32, 80, 128, 2048, "fp16", 10000.0,
                             rotary_dim=32, positions="duplicates"),
}


def make_positions(w, seed, device, batch=None):
    """int positions for one step of workload w (seeded): uniform in [0, S), with position 0
    and S - 1 present ("edges"), or with neighbouring sequences sharing positions
    ("duplicates"; each request still gets one slot)."""
    b = w.batch if batch is None else batch
    g = torch.Generator().manual_seed(seed)
    p = torch.randint(0, w.cache_alloc_len, (b,), generator=g)
    if w.positions == "edges" and b >= 2:
        p[0] = 0
        p[-1] = w.cache_alloc_len - 1
    elif w.positions == "duplicates" and b >= 4:
        p[1::4] = p[0::4][: p[1::4].numel()]      # same position in neighbouring sequences
    return p.to(device=device, dtype=INDEX_DTYPES[w.index_dtype])
