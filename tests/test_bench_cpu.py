"""bench.py on a machine without a GPU: the reference arm (the CPU oracle on host cores) runs
and prints the contract's JSON line; the workload byte accounting matches the roofline
numerator."""
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
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"] == "llama3_8b_decode32"


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
