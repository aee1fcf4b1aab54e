"""The validation gate: a candidate implementation against the CPU oracle on identical inputs.

Follows the reference's gate (benchmarks/validation.py:16-177): five cases per configuration
(two timed position sets, a uniform set, a permuted token -> request mapping, and strided Q/K/V
views of one fused projection); checks rotated Q, rotated K at the addressed slots, byte-exact
V at the addressed slots, and that every unaddressed slot still holds the sentinel. The
reference compares against its PyTorch oracle; here the oracle is the CPU restatement in
oracle/ (pinned to the reference by the golden fixtures), and the report also says whether Q
and K are bit-exact, which this build's kernels are held to.
"""
from typing import NamedTuple

import torch

from decode_llm_kernel_b200.harness import positions as pos
from decode_llm_kernel_b200.harness.inputs import SENTINEL, make_inputs
from golden_io import bits_equal
from oracle import oracle

# The reference's tolerances (benchmarks/validation.py:16-20). Candidates in this build are
# additionally required to be bit-exact (report["q_bit_exact"], report["k_bit_exact"]).
TOLERANCES = {
    torch.float64: {"atol": 1e-6, "rtol": 1e-6},
    torch.float32: {"atol": 1e-6, "rtol": 1e-6},
    torch.float16: {"atol": 1e-3, "rtol": 1e-3},
    torch.bfloat16: {"atol": 8e-3, "rtol": 8e-3},
}


class ValidationError(AssertionError):
    pass


class AddressingError(ValueError):
    pass


class ValidationCase(NamedTuple):
    label: str
    positions: torch.Tensor
    request_order: str      # "identity" | "shuffled" token -> request rows
    qkv_layout: str         # "packed" | "fused" (views of one QKV projection)


def assert_valid_addressing(positions, request_indices, cache_alloc_len, batch_size):
    """In-bounds, non-negative, no two tokens per slot (benchmarks/validation.py:38-53)."""
    if positions.numel() == 0:
        return
    if int(positions.min()) < 0 or int(positions.max()) >= cache_alloc_len:
        raise AddressingError(f"positions out of [0, {cache_alloc_len}): "
                              f"min={int(positions.min())} max={int(positions.max())}")
    if int(request_indices.min()) < 0 or int(request_indices.max()) >= batch_size:
        raise AddressingError(f"request_indices out of [0, {batch_size}): "
                              f"min={int(request_indices.min())} "
                              f"max={int(request_indices.max())}")
    flat = request_indices.to(torch.int64) * cache_alloc_len + positions.to(torch.int64)
    duplicates = flat.numel() - int(torch.unique(flat).numel())
    if duplicates:
        raise AddressingError(f"{duplicates} duplicate (request, position) slot(s); the "
                              f"reference has no defined result for them")


def _max_abs_diff(a, b):
    if a.numel() == 0:
        return 0.0
    return float((a.double() - b.double()).abs().max())


def _host(t):
    return t.detach().to("cpu")


def validate_once(candidate, cfg, device, seed, case):
    tol = TOLERANCES[cfg.dtype]
    a = make_inputs(cfg, device, seed, case.positions, cache_fill=SENTINEL,
                    request_order=case.request_order, qkv_layout=case.qkv_layout)
    assert_valid_addressing(a.positions, a.request_indices, cfg.cache_alloc_len,
                            cfg.batch)
    ref = [_host(t).clone() if i in (6, 7) else _host(t) for i, t in enumerate(a)]
    q_ref = oracle.fused_rope_kv_append(*ref)
    q_cand = _host(candidate(*a))
    ri, p = _host(a.request_indices).long(), _host(a.positions).long()
    kc, vc = _host(a.k_cache), _host(a.v_cache)
    k_ref_slots, k_cand_slots = ref[6][ri, p], kc[ri, p]
    v_cand_slots = vc[ri, p]
    v_in = _host(a.v)
    mask = torch.zeros(cfg.batch, cfg.cache_alloc_len, dtype=torch.bool)
    mask[ri, p] = True

    atol, rtol = tol["atol"], tol["rtol"]
    failures = []
    if q_cand.shape != q_ref.shape or not torch.allclose(q_cand.double(), q_ref.double(),
                                                         atol=atol, rtol=rtol):
        failures.append(f"q_rot mismatch vs oracle (max_abs={_max_abs_diff(q_cand, q_ref):.3e})")
    if not torch.allclose(k_cand_slots.double(), k_ref_slots.double(), atol=atol, rtol=rtol):
        failures.append("k_cache written slots mismatch vs oracle "
                        f"(max_abs={_max_abs_diff(k_cand_slots, k_ref_slots):.3e})")
    v_exact = bits_equal(v_cand_slots, v_in.contiguous())
    if not v_exact:
        failures.append("v_cache written slots are not byte-exact raw v "
                        f"(max_abs={_max_abs_diff(v_cand_slots, v_in):.3e})")
    intact = bool((kc[~mask] == SENTINEL).all() and (vc[~mask] == SENTINEL).all())
    if not intact:
        n_k = int((kc[~mask] != SENTINEL).sum())
        n_v = int((vc[~mask] != SENTINEL).sum())
        failures.append(f"unaddressed cache slots modified (k:{n_k} v:{n_v} elements)")
    return {
        "ok": not failures,
        "failures": [f"[{case.label}] {f}" for f in failures],
        "max_abs_diff_q": _max_abs_diff(q_cand, q_ref) if q_cand.shape == q_ref.shape else 1e9,
        "max_abs_diff_k_cache": _max_abs_diff(k_cand_slots, k_ref_slots),
        "q_bit_exact": bits_equal(q_cand, q_ref),
        "k_bit_exact": bits_equal(k_cand_slots.contiguous(), k_ref_slots.contiguous()),
        "v_byte_exact": v_exact,
        "unaddressed_slots_intact": intact,
        "num_addressed_slots": int(mask.sum()),
        "tolerance": tol,
    }


def validation_cases(cfg, device, seed):
    timed = pos.build_position_sets(cfg.batch, cfg.cache_alloc_len, cfg.positions,
                                    seed, 2, device)
    cases = [ValidationCase(f"{cfg.positions}[{i}]", p, cfg.request_order, cfg.qkv_layout)
             for i, p in enumerate(timed)]
    if cfg.positions != pos.UNIFORM:
        uniform = pos.build_position_sets(cfg.batch, cfg.cache_alloc_len, pos.UNIFORM,
                                          seed, 1, device)[0]
        cases.append(ValidationCase("uniform", uniform, cfg.request_order, cfg.qkv_layout))
    cases.append(ValidationCase("permuted-requests", timed[0], "shuffled", "packed"))
    cases.append(ValidationCase("strided-qkv", timed[0], "identity", "fused"))
    return cases


def validate_candidate(candidate, cfg, device, seed):
    """Aggregate validation over every case. Returns a report; never raises."""
    cases = validation_cases(cfg, device, seed)
    with torch.inference_mode():
        reports = [validate_once(candidate, cfg, device, seed, c) for c in cases]
    failures = [f for r in reports for f in r["failures"]]
    return {
        "ok": not failures,
        "failures": failures,
        "num_cases": len(reports),
        "cases": [c.label for c in cases],
        "max_abs_diff_q": max(r["max_abs_diff_q"] for r in reports),
        "max_abs_diff_k_cache": max(r["max_abs_diff_k_cache"] for r in reports),
        "q_bit_exact": all(r["q_bit_exact"] for r in reports),
        "k_bit_exact": all(r["k_bit_exact"] for r in reports),
        "v_byte_exact": all(r["v_byte_exact"] for r in reports),
        "unaddressed_slots_intact": all(r["unaddressed_slots_intact"] for r in reports),
        "tolerance": reports[0]["tolerance"],
    }


def validate_or_raise(candidate, cfg, device, seed):
    report = validate_candidate(candidate, cfg, device, seed)
    if not report["ok"]:
        raise ValidationError(f"{cfg.label()}: " + "; ".join(report["failures"]))
    return report
