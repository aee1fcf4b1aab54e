"""bench.py on a machine without a GPU: the reference arm (the reference's PyTorch CPU path on
the host cores, or the C port of it when the reference is not installed) runs and prints the
contract's JSON line with the same config dict as this build's arm; the workload byte
accounting matches the roofline numerator; the parity restatement bench.py checks timed runs
with agrees with the CPU oracle bit for bit."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "3",
                           "--warmup", "1"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr
    line = json.loads(proc.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "dtype", "config", "cpu_baseline", "e2e"):
        assert key in line
    assert line["unit"] == "GB/s" and line["value"] > 0
    ref_installed = os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "decode_kernels"))
    assert line["cpu_baseline"]["kind"] == ("reference" if ref_installed else "port")
    assert line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    # the same config dict this build's arm prints (bench.workload_config), key for key
    sys.path.insert(0, ROOT)
    import bench
    from decode_llm_kernel_b200.harness.configs import WORKLOADS
    assert line["config"] == bench.workload_config(WORKLOADS["llama3_8b_decode32"], 1)


def test_reference_arm_non_zero_ranks_exit_quietly():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                           "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=300,
                          env=env)
    assert proc.returncode == 0, proc.stderr
    assert proc.stdout.strip() == ""


def test_bytes_per_token_matches_the_reference_formula():
    from decode_llm_kernel_b200.harness.configs import WORKLOADS
    from decode_llm_kernel_b200.harness.timing import logical_bytes
    import torch
    w = WORKLOADS["llama3_8b_b8"]
    T, Hq, Hkv, D = 8, 32, 8, 128
    q = torch.empty(T, Hq, D, dtype=torch.bfloat16)
    k = torch.empty(T, Hkv, D, dtype=torch.bfloat16)
    cos = torch.empty(16, D)
    lb = logical_bytes(q, k, k, cos, cos, k, k)
    assert lb["total_bytes"] == w.bytes_per_call() == 200704
    assert WORKLOADS["phi2_partial"].bytes_per_token() == 30848
    assert WORKLOADS["llama3_70b_tp"].bytes_per_token() == 41472


def test_the_bench_parity_restatement_matches_the_oracle():
    """bench.rope_torch (run on the GPU after each timed region) is bit-identical to the CPU
    oracle on every dtype, full and partial rotary."""
    import torch
    sys.path.insert(0, ROOT)
    import bench
    from decode_llm_kernel_b200.rope_tables import build_rope_tables
    from oracle import oracle
    g = torch.Generator().manual_seed(5)
    for dt in (torch.bfloat16, torch.float16, torch.float32, torch.float64):
        for D, R in ((128, 128), (80, 32), (96, 96)):
            T, S = 37, 300
            q = torch.randn(T, 6, D, generator=g).to(dt)
            k = torch.randn(T, 2, D, generator=g).to(dt)
            pos = torch.randint(0, S, (T,), generator=g)
            cos, sin = build_rope_tables(S, R, 500000.0)
            q_ref, k_ref = oracle.rope_forward(q, k, pos, cos, sin)
            assert bench.differing(bench.rope_torch(q, pos, cos, sin, R), q_ref) == 0, (dt, D, R)
            assert bench.differing(bench.rope_torch(k, pos, cos, sin, R), k_ref) == 0, (dt, D, R)


def test_ulp_distance_of_the_parity_report():
    import torch
    sys.path.insert(0, ROOT)
    import bench
    one = torch.tensor([1.0], dtype=torch.bfloat16)
    up = torch.nextafter(torch.tensor([1.0]), torch.tensor([2.0])).to(torch.bfloat16)
    nxt = (one.view(torch.int16) + 1).view(torch.bfloat16)
    assert bench.max_ulp(one, nxt) == 1 and bench.max_ulp(nxt, one) == 1
    assert bench.max_ulp(torch.tensor([0.0]), torch.tensor([-0.0])) == 0
    neg = -one
    assert bench.max_ulp(neg, (neg.view(torch.int16) + 1).view(torch.bfloat16)) == 1
    assert bench.max_ulp(torch.tensor([-1e-45]), torch.tensor([1e-45])) == 2   # across zero
    assert bench.max_ulp(one, up) == 0                    # 1 + fp32 ulp rounds back to 1
    counts = {"q": 3, "k_slots": 1, "v_slots": 0, "max_ulp": 1, "elements": 100}
    assert bench.parity_label(counts).startswith("within 1 ulp")
    assert bench.parity_label(dict(counts, max_ulp=3)).startswith("within 3 ulp")
    assert bench.parity_label(dict(counts, v_slots=1)).startswith("MISMATCH")
    assert bench.parity_label(dict(counts, q=0, k_slots=0, max_ulp=0)) == "bit-exact"
