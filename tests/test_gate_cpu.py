"""The gate itself, on CPU: an independent correct implementation passes, and each planted bug
is caught by the check named for it (the reference's tests/test_benchmark_validation.py:41-151,
re-pointed at this build's gate and oracle). The candidates here are CPU test doubles."""
import pytest
import torch

from decode_llm_kernel_b200.harness import positions as pos
from decode_llm_kernel_b200.harness.inputs import case
from gate import (AddressingError, ValidationCase, ValidationError, assert_valid_addressing,
                  validate_candidate, validate_once, validate_or_raise, validation_cases)

DEVICE = "cpu"
SEED = 1234
MHA_BF16 = case("mha", 8, 8, 64, 4, 128, "bf16", pos.RAGGED)
GQA_BF16 = case("gqa", 8, 2, 64, 4, 128, "bf16", pos.RAGGED)


def _rope(x, cos, sin, positions):
    c = cos[positions].float().unsqueeze(-2)
    s = sin[positions].float().unsqueeze(-2)
    xf = x.float()
    half = xf.shape[-1] // 2
    rotated = torch.cat((-xf[..., half:], xf[..., :half]), dim=-1)
    return (xf * c + rotated * s).to(x.dtype)


def correct_alternate(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices):
    q_rot = _rope(q, cos, sin, positions)
    k_rot = _rope(k, cos, sin, positions)
    for i in range(q.shape[0]):
        k_cache[request_indices[i], positions[i]] = k_rot[i]
        v_cache[request_indices[i], positions[i]] = v[i]
    return q_rot


def unrotated_q(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices):
    k_cache[request_indices, positions] = _rope(k, cos, sin, positions)
    v_cache[request_indices, positions] = v
    return q.clone()


def unrotated_k_in_cache(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices):
    k_cache[request_indices, positions] = k
    v_cache[request_indices, positions] = v
    return _rope(q, cos, sin, positions)


def rotated_v_in_cache(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices):
    k_cache[request_indices, positions] = _rope(k, cos, sin, positions)
    v_cache[request_indices, positions] = _rope(v, cos, sin, positions)
    return _rope(q, cos, sin, positions)


def wrong_slot(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices):
    shifted = torch.clamp(positions - 1, min=0)
    k_cache[request_indices, shifted] = _rope(k, cos, sin, positions)
    v_cache[request_indices, shifted] = v
    return _rope(q, cos, sin, positions)


def ignores_request_indices(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices):
    rows = torch.arange(q.shape[0])
    k_cache[rows, positions] = _rope(k, cos, sin, positions)
    v_cache[rows, positions] = v
    return _rope(q, cos, sin, positions)


def assumes_packed_qkv(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices):
    def packed(x):
        t, h, d = x.shape
        return x.as_strided((t, h, d), (h * d, d, 1))
    k_cache[request_indices, positions] = _rope(packed(k), cos, sin, positions)
    v_cache[request_indices, positions] = packed(v)
    return _rope(packed(q), cos, sin, positions)


def clobbers_unrelated_slot(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices):
    k_cache[request_indices, positions] = _rope(k, cos, sin, positions)
    v_cache[request_indices, positions] = v
    k_cache[0, 0] = 0.0
    return _rope(q, cos, sin, positions)


@pytest.mark.parametrize("dtype_label", ["fp32", "fp16", "bf16"])
@pytest.mark.parametrize("mode", [pos.UNIFORM, pos.RAGGED])
def test_independent_correct_implementation_passes_bit_exactly(dtype_label, mode):
    for cfg in (case("mha", 8, 8, 64, 4, 128, dtype_label, mode),
                case("gqa", 8, 2, 64, 4, 128, dtype_label, mode)):
        report = validate_candidate(correct_alternate, cfg, DEVICE, SEED)
        assert report["ok"], report["failures"]
        assert report["q_bit_exact"] and report["k_bit_exact"]
        assert report["v_byte_exact"] and report["unaddressed_slots_intact"]


@pytest.mark.parametrize("broken,expect", [
    (unrotated_q, "q_rot"),
    (unrotated_k_in_cache, "k_cache"),
    (rotated_v_in_cache, "v_cache"),
    (wrong_slot, "cache"),
    (clobbers_unrelated_slot, "unaddressed"),
    (ignores_request_indices, "cache"),
    (assumes_packed_qkv, "q_rot"),
])
def test_broken_implementations_are_caught(broken, expect):
    report = validate_candidate(broken, MHA_BF16, DEVICE, SEED)
    assert not report["ok"]
    assert any(expect in f for f in report["failures"]), report["failures"]


def _identity_packed_case(cfg):
    p = pos.build_position_sets(cfg.batch, cfg.cache_alloc_len, cfg.positions,
                                SEED, 1, DEVICE)[0]
    return ValidationCase("identity-packed", p, "identity", "packed")


@pytest.mark.parametrize("broken,case_label", [
    (ignores_request_indices, "permuted-requests"),
    (assumes_packed_qkv, "strided-qkv"),
])
def test_contract_case_is_what_catches_the_bug(broken, case_label):
    lenient = validate_once(broken, MHA_BF16, DEVICE, SEED, _identity_packed_case(MHA_BF16))
    assert lenient["ok"], lenient["failures"]
    report = validate_candidate(broken, MHA_BF16, DEVICE, SEED)
    assert not report["ok"]
    assert all(f.startswith(f"[{case_label}]") for f in report["failures"]), report["failures"]


def test_flags_on_the_report():
    assert validate_candidate(clobbers_unrelated_slot, MHA_BF16, DEVICE,
                              SEED)["unaddressed_slots_intact"] is False
    assert validate_candidate(rotated_v_in_cache, MHA_BF16, DEVICE, SEED)["v_byte_exact"] is False
    assert not validate_candidate(unrotated_k_in_cache, GQA_BF16, DEVICE, SEED)["ok"]


def test_case_lists():
    ragged = validate_candidate(correct_alternate, MHA_BF16, DEVICE, SEED)
    uniform_cfg = case("mha", 8, 8, 64, 4, 128, "bf16", pos.UNIFORM)
    uniform = validate_candidate(correct_alternate, uniform_cfg, DEVICE, SEED)
    assert ragged["cases"] == ["ragged[0]", "ragged[1]", "uniform", "permuted-requests",
                               "strided-qkv"]
    assert uniform["cases"] == ["uniform[0]", "uniform[1]", "permuted-requests", "strided-qkv"]
    cfg = case("mha", 8, 8, 64, 4, 128, "bf16", pos.RAGGED, qkv_layout="fused",
               request_order="shuffled")
    cases = validation_cases(cfg, DEVICE, SEED)
    assert cases[0].qkv_layout == "fused" and cases[0].request_order == "shuffled"


def test_addressing_contract():
    assert_valid_addressing(torch.tensor([0, 5, 5, 127]), torch.tensor([0, 1, 2, 3]), 128, 4)
    for p, ri, expect in (([0, 1, 2, 128], [0, 1, 2, 3], "positions out of"),
                          ([0, 1, 2, -1], [0, 1, 2, 3], "positions out of"),
                          ([0, 1, 2, 3], [0, 1, 2, 4], "request_indices out of"),
                          ([0, 1, 2, 3], [0, 1, 2, -1], "request_indices out of"),
                          ([7, 7, 2, 3], [1, 1, 2, 3], "duplicate")):
        with pytest.raises(AddressingError, match=expect):
            assert_valid_addressing(torch.tensor(p), torch.tensor(ri), 128, 4)


def test_validate_or_raise():
    with pytest.raises(ValidationError):
        validate_or_raise(unrotated_q, MHA_BF16, DEVICE, SEED)
    assert validate_or_raise(correct_alternate, MHA_BF16, DEVICE, SEED)["ok"]


def test_candidate_is_validated_under_inference_mode():
    seen = []

    def recording(*op_args):
        seen.append(torch.is_inference_mode_enabled())
        return correct_alternate(*op_args)

    assert validate_candidate(recording, MHA_BF16, DEVICE, SEED)["ok"]
    assert seen and all(seen)
