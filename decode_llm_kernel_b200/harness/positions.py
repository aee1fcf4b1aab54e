"""Device-resident position sets for timed loops (benchmarks/positions.py:8-37 of the reference).

uniform: every request decodes at the last valid slot (a controlled comparison).
ragged:  seeded positions stratified over the early, middle and late thirds of the cache, so
         successive timed calls touch varied slots.
edges:   ragged, with the first token at position 0 and the last at cache_alloc_len - 1.
"""
import torch

UNIFORM = "uniform"
RAGGED = "ragged"
EDGES = "edges"
MODES = (UNIFORM, RAGGED, EDGES)


def build_position_sets(num_tokens, cache_alloc_len, mode, seed, num_sets, device,
                        dtype=torch.long):
    if mode == UNIFORM:
        p = torch.full((num_tokens,), cache_alloc_len - 1, dtype=dtype, device=device)
        return [p] * num_sets
    if mode not in (RAGGED, EDGES):
        raise ValueError(f"unknown position mode {mode!r}, expected one of {MODES}")
    sets = _stratified(num_tokens, cache_alloc_len, seed, num_sets)
    if mode == EDGES and num_tokens > 0:
        for s in sets:
            s[0] = 0
            s[-1] = cache_alloc_len - 1
    return [s.to(device=device, dtype=dtype) for s in sets]


def _stratified(num_tokens, m, seed, num_sets):
    g = torch.Generator().manual_seed(seed)
    total = num_sets * num_tokens
    u = torch.rand(total, generator=g, dtype=torch.float64)
    if m < 3:
        vals = (u * m).long().clamp_(0, m - 1)
    else:
        third = m // 3
        lo = torch.tensor([0, third, 2 * third])[torch.arange(total) % 3]
        hi = torch.tensor([third, 2 * third, m])[torch.arange(total) % 3]
        vals = (lo + (u * (hi - lo).to(torch.float64)).long()).clamp_(0, m - 1)
    return [vals[i * num_tokens:(i + 1) * num_tokens].clone() for i in range(num_sets)]


def position_span(position_sets, cache_alloc_len):
    """Coverage of a list of position sets over the early/middle/late thirds."""
    allp = torch.cat([p.reshape(-1).cpu() for p in position_sets])
    third = cache_alloc_len // 3
    return {
        "min": int(allp.min()),
        "max": int(allp.max()),
        "distinct": int(torch.unique(allp).numel()),
        "in_bounds": bool((allp >= 0).all() and (allp < cache_alloc_len).all()),
        "early": int((allp < third).sum()),
        "middle": int(((allp >= third) & (allp < 2 * third)).sum()),
        "late": int((allp >= 2 * third).sum()),
    }
