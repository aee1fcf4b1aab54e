"""Benchmark of the decode-step RoPE + KV-cache append path on B200.

Default workload (N=1 and per GPU for N>1): `llama3_8b_decode32` -- a 32-layer Llama-3-8B-shaped
decode step (batch 64 per GPU, 32 Q / 8 KV heads, head_dim 128, theta 5e5, bf16, per-layer
caches [64, 8192, 8, 128] prefilled N(0, 1), int32 ragged positions including 0 and 8191),
captured as one CUDA graph of 32 fused launches chained with programmatic dependent launch.
A step is one replay. Inputs rotate over enough distinct input sets (q/k/v/positions/q_out)
that their total exceeds 3x L2, so no step is served from L2.

metric: achieved HBM GB/s per decode step = algorithmic bytes (reads of q, k, v and the rotary
half-rows of cos/sin, writes of q_out and the K and V cache slots) / device time; value is the
whole job's total over all ranks. us_per_step and us_per_call (per layer launch) are reported
beside it.

Every timed configuration is checked after its timed region: one sampled input set's call is
issued again and its q_out and K/V slots are compared bit for bit with a PyTorch fp32
restatement on the GPU ("parity" keys).

Beside this build's numbers the line carries, at N=1: the reference's own kernels rebuilt for
sm_100a on the same workloads (`reference_gpu`, from baseline/_ref, installed by
baseline/build_ref.py), the reference's PyTorch CPU path on the host cores
(`cpu_baseline_torch`) and the C port of it (`cpu_baseline`); at every N the strong-scaling
records of the two sharded workloads (`strong_scaling`).

Launch: python bench.py [--gpus N --steps K --warmup W]; for N > 1 under torchrun, one rank per
GPU, each owning its own batch shard and caches (weak scaling, no collective on the data path;
NCCL only for the barrier and the max-over-ranks time).
`--impl reference` times the reference's CPU implementation (its PyTorch oracle, all host
threads; the C port when the reference is not installed) on the same workload and prints the
same JSON line with impl=reference.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
import types
from dataclasses import replace

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from decode_llm_kernel_b200.harness.configs import WORKLOADS, make_positions  # noqa: E402

FALLBACK_HBM_GBS = 6650.0
# ncu captures (profiles/): DRAM bytes read + written per launch
DECODE32_NCU_DRAM_BYTES = 878848 + 0
MISTRAL_NCU_DRAM_BYTES = 51549696 + 4873728
E2E_STEPS_PER_GRAPH = 32
L2_BYTES = 126 * 1024 * 1024
METRIC = "achieved HBM GB/s per decode step (algorithmic bytes / device time), with us/call"


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=50)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", default="llama3_8b_decode32", choices=sorted(WORKLOADS))
    p.add_argument("--no-pdl", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-bw-probe", action="store_true")
    p.add_argument("--no-floor", action="store_true", help="skip the empty-kernel launch floor")
    p.add_argument("--no-ladder", action="store_true",
                   help="skip the per-call operator ladder at batch 8")
    p.add_argument("--no-attention", action="store_true",
                   help="skip the fused append + decode attention measurement")
    p.add_argument("--no-reference-gpu", action="store_true",
                   help="skip the reference's own kernels (baseline/_ref) on the GPU")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--mode", choices=["full", "bw", "single", "attention"], default="full",
                   help="bw: only the bandwidth-bound launch loop (for profiling small cases); "
                        "single: only the single-layer loop of --probe; "
                        "attention: only the fused append + decode attention measurement")
    p.add_argument("--probe", default="mistral_b4096", choices=sorted(WORKLOADS),
                   help="single mode: the workload of the single-layer loop")
    p.add_argument("--cache-len", type=int, default=0,
                   help="override cache_alloc_len (profiling runs only: keeps a case small)")
    p.add_argument("--launches", type=int, default=400, help="bw mode: timed launches")
    p.add_argument("--attention-case", choices=ATTENTION_CASES, default=None,
                   help="attention mode: run this case alone")
    return p.parse_args()


# ------------------------------------------------------------------------- distributed setup

class stdout_to_stderr:
    """Sends file descriptor 1 to stderr for a block, so library banners printed while the
    process group starts never mix with the one JSON line this script prints."""

    def __enter__(self):
        sys.stdout.flush()
        self._saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self._saved, 1)
        os.close(self._saved)
        return False


def init_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        if args.impl == "ours":
            torch.cuda.set_device(local)
            with stdout_to_stderr():
                dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                        device_id=torch.device("cuda", local))
                dist.barrier()
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(value, world):
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------- peaks and clocks

def measured_hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback (6.65 TB/s, earlier measurement on this pool)"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms while running."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        try:
            self.device_id = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
        except Exception:  # noqa: BLE001 -- fall back to the ordinal
            self.device_id = str(device_index)
        self.samples = []
        self._proc = None
        self._thread = None

    def start(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_id}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None
            return self
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()
        return self

    def _read(self):
        for line in self._proc.stdout:
            self.samples.append((time.perf_counter(), line.strip()))

    def stop(self):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self, t0, t1):
        rows = [s for t, s in self.samples if t0 <= t <= t1] or [s for _, s in self.samples]
        sm, sm_max, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for row in rows:
            parts = [x.strip() for x in row.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": sm_max,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------- GPU state

def build_tables(w, device):
    from decode_llm_kernel_b200.rope_tables import build_rope_tables
    return build_rope_tables(w.cache_alloc_len, w.rotary_dim or w.head_dim, w.theta,
                             device=device)


def normal_(t, g):
    flat = t.view(-1)
    step = 1 << 28
    for start in range(0, flat.numel(), step):
        n = min(step, flat.numel() - start)
        flat[start:start + n] = torch.randn(n, generator=g, device=t.device).to(t.dtype)
    return t


def build_step_state(w, device, seed, num_sets):
    """Caches for every layer and `num_sets` distinct device input sets of one step."""
    from decode_llm_kernel_b200.harness.decode_loop import StepInputs
    g = torch.Generator(device=device).manual_seed(seed)
    shape = (w.batch, w.cache_alloc_len, w.num_kv_heads, w.head_dim)
    k_caches = [normal_(torch.empty(shape, dtype=w.dtype, device=device), g)
                for _ in range(w.layers)]
    v_caches = [normal_(torch.empty(shape, dtype=w.dtype, device=device), g)
                for _ in range(w.layers)]
    idx = torch.int32 if w.index_dtype == "int32" else torch.int64
    sets = []
    for i in range(num_sets):
        L, T = w.layers, w.batch
        sets.append(StepInputs(
            normal_(torch.empty(L, T, w.num_q_heads, w.head_dim, dtype=w.dtype, device=device), g),
            normal_(torch.empty(L, T, w.num_kv_heads, w.head_dim, dtype=w.dtype, device=device), g),
            normal_(torch.empty(L, T, w.num_kv_heads, w.head_dim, dtype=w.dtype, device=device), g),
            make_positions(w, seed + i, device),
            torch.arange(T, device=device, dtype=idx)))
    return k_caches, v_caches, sets


def input_set_bytes(w):
    return (w.layers * w.batch * (2 * w.num_q_heads + 2 * w.num_kv_heads) * w.head_dim
            * w.elem_bytes)


def sets_needed(w):
    return max(4, min(64, -(-3 * L2_BYTES // max(1, input_set_bytes(w)))))


def time_graph_steps(captured, steps, stream):
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for i in range(steps):
        captured[i % len(captured)].replay()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end)


# ------------------------------------------------------------------------- parity of timed runs

def rope_torch(x, pos, cos, sin, rotary):
    """RoPE of x [T, H, D] at positions pos [T], computed with PyTorch on x's device: fp32, each
    multiply and each add a separate elementwise op (each rounded once, never a fused
    multiply-add), one rounding to x's dtype; dims past `rotary` are copied. This is the
    arithmetic the reference specifies, evaluated independently of the kernels."""
    half = rotary // 2
    xf = x[..., :rotary].float()
    idx = pos.long()
    c = cos[idx, :rotary].unsqueeze(1)
    s = sin[idx, :rotary].unsqueeze(1)
    turned = torch.cat((-xf[..., half:], xf[..., :half]), dim=-1)
    y = (xf * c + turned * s).to(x.dtype)
    return torch.cat((y, x[..., rotary:]), dim=-1) if rotary < x.shape[-1] else y


def _bits(t):
    return t.contiguous().view({1: torch.uint8, 2: torch.int16, 4: torch.int32,
                                8: torch.int64}[t.element_size()])


def differing(a, b):
    """Elements whose bits differ (0 means bit-exact)."""
    return int((_bits(a) != _bits(b)).sum().item())


def _ordered(t):
    """Integer keys of a float tensor whose differences count ulps (+0 and -0 coincide)."""
    b = _bits(t).to(torch.int64)
    magnitude = b & ((1 << (8 * t.element_size() - 1)) - 1)
    return torch.where(b < 0, -magnitude, b)


def max_ulp(a, b):
    if a.numel() == 0:
        return 0
    return int((_ordered(a) - _ordered(b)).abs().max().item())


def check_call(q, k, v, pos, ri, cos, sin, q_out, k_cache, v_cache, rotary):
    """One call's outputs against rope_torch: q_out, and the K and V slots [ri, pos] of the
    caches (which must hold this call's writes). Returns mismatching element counts and the
    largest distance in ulps of the storage type."""
    idx_r, idx_p = ri.long(), pos.long()
    q_ref, k_ref = rope_torch(q, pos, cos, sin, rotary), rope_torch(k, pos, cos, sin, rotary)
    k_got = k_cache[idx_r, idx_p]
    return {"q": differing(q_out, q_ref), "k_slots": differing(k_got, k_ref),
            "v_slots": differing(v_cache[idx_r, idx_p], v),
            "max_ulp": max(max_ulp(q_out, q_ref), max_ulp(k_got, k_ref)),
            "elements": q_ref.numel() + k_ref.numel()}


def parity_label(counts):
    """'bit-exact'; or, when only rotated elements differ, how many and by how many ulps of the
    storage type at most; 'MISMATCH' when a V slot (a byte copy) differs."""
    bad = counts["q"] + counts["k_slots"] + counts["v_slots"]
    if bad == 0:
        return "bit-exact"
    if counts["v_slots"] == 0:
        ulp = counts["max_ulp"]
        return (f"within {ulp} ulp: {counts['q'] + counts['k_slots']} of {counts['elements']} "
                f"rotated elements differ (by at most {ulp} ulp), V bit-exact")
    return f"MISMATCH {counts}"


PARITY_NOTE = ("after the timed region one sampled input set's call is issued again; its q_out "
               "and its K/V cache slots are compared bit for bit with a PyTorch fp32 "
               "restatement on the GPU (separately rounded multiplies and adds)")


# ------------------------------------------------------------------------- the reference

REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def load_reference():
    """The reference project installed by baseline/build_ref.py: its ops over its own CUDA
    extension rebuilt for sm_100a, and its PyTorch oracle. Raises RuntimeError(reason) when it
    is not installed or does not load."""
    if not os.path.isdir(os.path.join(REF_DIR, "decode_kernels")):
        raise RuntimeError("the reference is not installed (python baseline/build_ref.py)")
    if REF_DIR not in sys.path:
        sys.path.append(REF_DIR)
    from decode_kernels import cuda as ref_cuda
    from decode_kernels.cuda import ops as ref_ops
    from decode_kernels.reference import fused_rope_kv_append_ref
    return types.SimpleNamespace(ops=ref_ops, oracle=fused_rope_kv_append_ref,
                                 gpu_ok=ref_cuda.is_available(),
                                 gpu_reason=ref_cuda.unavailable_reason(),
                                 ext_path=ref_cuda.extension_path())


def reference_or_reason():
    try:
        return load_reference(), None
    except Exception as e:  # noqa: BLE001 -- reported in the line, never fatal
        return None, f"{type(e).__name__}: {e}"


# ------------------------------------------------------------------------- single-layer probes

def single_layer_probe(name, world, rank, device, seed, peak, cache_len=0, iters=400,
                       impl="ours", rung="fused", ref=None):
    """One launch per call of a single-layer workload (sharded for this rank), input sets
    rotated so they exceed 3x L2, calls replayed from a CUDA graph, device time per call from
    CUDA events, max over ranks. impl "ours": the fused op with programmatic dependent launch
    between calls (no call writes another's positions, indices or tables); impl "reference":
    the reference's own fused (or separate) op over its sm_100a build, same inputs, same graph
    replay. cache_len > 0 shrinks the caches (same per-token work) for profiling runs."""
    from decode_llm_kernel_b200.cuda import ops
    w = WORKLOADS[name].shard_for(rank, world)
    if cache_len:
        w = replace(w, cache_alloc_len=cache_len)
    rot = w.rotary_dim if w.rotary_dim and w.rotary_dim != w.head_dim else 0
    if impl == "reference" and rot:
        return {"workload": name, "unsupported": "the reference has no partial rotary: its "
                "tables must be [max_position, head_dim] (csrc/kernel_common.cuh:70-72)"}
    g = torch.Generator(device=device).manual_seed(seed + 17)
    shape = (w.batch, w.cache_alloc_len, w.num_kv_heads, w.head_dim)
    kc = normal_(torch.empty(shape, dtype=w.dtype, device=device), g)
    vc = normal_(torch.empty(shape, dtype=w.dtype, device=device), g)
    cos, sin = build_tables(w, device)
    nsets = max(4, -(-3 * L2_BYTES // (w.bytes_per_call())))
    idx = torch.int32
    sets = []
    for i in range(nsets):
        sets.append((normal_(torch.empty(w.batch, w.num_q_heads, w.head_dim, dtype=w.dtype,
                                         device=device), g),
                     normal_(torch.empty(w.batch, w.num_kv_heads, w.head_dim, dtype=w.dtype,
                                         device=device), g),
                     normal_(torch.empty(w.batch, w.num_kv_heads, w.head_dim, dtype=w.dtype,
                                         device=device), g),
                     make_positions(w, seed + 100 + i, device),
                     torch.arange(w.batch, device=device, dtype=idx),
                     torch.empty(w.batch, w.num_q_heads, w.head_dim, dtype=w.dtype,
                                 device=device)))

    if impl == "ours":
        def call(i):
            q, k, v, p, ri, qo = sets[i % nsets]
            ops.fused_rope_kv_append_ex(q, k, v, p, cos, sin, kc, vc, ri, q_out=qo, pdl=True,
                                        rotary_dim=rot)
            return qo
    else:
        fn = ref.ops.fused_rope_kv_append if rung == "fused" else ref.ops.separate_rope_kv_append

        def call(i):
            q, k, v, p, ri, _ = sets[i % nsets]
            return fn(q, k, v, p, cos, sin, kc, vc, ri)

    # Calls are replayed from a CUDA graph so host call overhead cannot pace the GPU.
    for i in range(nsets):
        call(i)
    torch.cuda.synchronize()
    per_graph = 2 * nsets
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(per_graph):
            call(i)
    for _ in range(3):
        graph.replay()
    reps = max(2, iters // per_graph)
    stream = torch.cuda.current_stream()
    barrier(world)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(reps):
        graph.replay()
    end.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end), world)
    iters = reps * per_graph
    per_launch_s = ms / 1e3 / iters
    del graph
    # parity of the timed configuration: set 0 once more, then its outputs and slots
    q0, k0, v0, p0, r0, _ = sets[0]
    out0 = call(0)
    torch.cuda.synchronize()
    counts = check_call(q0, k0, v0, p0, r0, cos, sin, out0, kc, vc, w.rotary)
    gbs_rank = w.bytes_per_call() / per_launch_s / 1e9
    if impl == "ours":
        kernel = ("drk::rope_kv_staged_kernel (TMA bulk copies, 3-stage mbarrier pipeline)"
                  if w.batch >= 512 else "drk::rope_kv_kernel (register kernel)")
    else:
        kernel = f"reference cuda_{rung} (its csrc kernels rebuilt for sm_100a)"
    out = {"workload": name, "impl": impl, "shard": w.shard, "batch_per_gpu": w.batch,
           "q_heads_per_gpu": w.num_q_heads, "kv_heads_per_gpu": w.num_kv_heads,
           "head_dim": w.head_dim, "rotary_dim": w.rotary, "dtype": w.dtype_label,
           "cache_alloc_len": w.cache_alloc_len, "launches": iters,
           "pdl": impl == "ours", "kernel": kernel,
           "bytes_per_launch": w.bytes_per_call(), "us_per_launch": per_launch_s * 1e6,
           "achieved_gbs_per_gpu": gbs_rank, "frac_of_peak": gbs_rank / peak,
           "aggregate_gbs": gbs_rank * world, "input_sets": nsets,
           "parity": parity_label(counts)}
    if name == "mistral_b4096" and world == 1 and impl == "ours":
        out["traffic"] = MISTRAL_NCU_DRAM_BYTES
        out["traffic_note"] = ("dram__bytes_read.sum + dram__bytes_write.sum of one launch, "
                               "profiles/rope_kv_staged_kernel_mistral_b4096_fp16.md (caches cut "
                               "to 128 positions): reads 51.5 MB = the algorithmic reads; 4.9 MB "
                               "of the 51.4 MB of writes reach DRAM within the launch, the rest "
                               "drains from L2 afterwards")
    del kc, vc, sets
    torch.cuda.empty_cache()
    return out


def bandwidth_probe(world, rank, device, seed, peak, cache_len=0, iters=400):
    """The bandwidth-bound workload (mistral_b4096, sharded by batch)."""
    return single_layer_probe("mistral_b4096", world, rank, device, seed, peak, cache_len, iters)


def reference_gpu(device, seed, peak, ours):
    """The reference's own kernels (cuda_fused and cuda_separate, its csrc rebuilt for sm_100a
    by baseline/build_ref.py) on the single-layer workloads, with the inputs, graph replay and
    timing of this build's arm; `ours` maps each workload to this build's probe result."""
    ref, why = reference_or_reason()
    if ref is None or not ref.gpu_ok:
        return {"unavailable": why or ref.gpu_reason}
    out = {"extension": os.path.relpath(ref.ext_path, ROOT)}
    for name in ("llama3_8b_b8", "llama3_70b_tp", "mistral_b4096", "phi2_partial"):
        row = {}
        for rung in ("fused", "separate"):
            r = single_layer_probe(name, 1, 0, device, seed, peak, impl="reference", rung=rung,
                                   ref=ref)
            if "unsupported" in r:
                row = r
                break
            row[f"cuda_{rung}"] = {k: r[k] for k in ("us_per_launch", "achieved_gbs_per_gpu",
                                                      "frac_of_peak", "parity")}
        mine = ours.get(name)
        if mine and "cuda_fused" in row:
            row["ours_us"] = mine["us_per_launch"]
            row["speedup_vs_reference_fused"] = (row["cuda_fused"]["us_per_launch"]
                                                 / mine["us_per_launch"])
            row["speedup_vs_reference_separate"] = (row["cuda_separate"]["us_per_launch"]
                                                    / mine["us_per_launch"])
        out[name] = row
    return out


def reference_decode_step(ref, k_caches, v_caches, sets, cos, sin, steps, warmup, w):
    """The reference's fused op as the 32-layer decode step (one graph of 32 launches per
    input set, no programmatic dependent launch: the reference's kernel has none), over the
    same caches and input sets as this build's step."""
    fn = ref.ops.fused_rope_kv_append
    graphs, outs = [], []
    for s in sets:
        for layer in range(w.layers):
            fn(s.q[layer], s.k[layer], s.v[layer], s.positions, cos, sin, k_caches[layer],
               v_caches[layer], s.request_indices)
    torch.cuda.synchronize()
    for s in sets:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            o = [fn(s.q[layer], s.k[layer], s.v[layer], s.positions, cos, sin, k_caches[layer],
                    v_caches[layer], s.request_indices) for layer in range(w.layers)]
        graphs.append(g)
        outs.append(o)
    for i in range(warmup):
        graphs[i % len(graphs)].replay()
    stream = torch.cuda.current_stream()
    ms = time_graph_steps(graphs, steps, stream)
    graphs[0].replay()
    torch.cuda.synchronize()
    s0 = sets[0]
    bad = {"q": 0, "k_slots": 0, "v_slots": 0, "max_ulp": 0, "elements": 0}
    for layer in range(w.layers):
        counts = check_call(s0.q[layer], s0.k[layer], s0.v[layer], s0.positions,
                            s0.request_indices, cos, sin, outs[0][layer], k_caches[layer],
                            v_caches[layer], w.rotary)
        for key in bad:
            bad[key] = max(bad[key], counts[key]) if key == "max_ulp" else bad[key] + counts[key]
    del graphs, outs
    per_step_us = ms * 1e3 / steps
    return {"us_per_step": per_step_us, "us_per_layer": per_step_us / w.layers,
            "achieved_gbs": w.bytes_per_step() / (per_step_us * 1e-6) / 1e9,
            "parity": parity_label(bad),
            "kernel": "reference cuda_fused (its csrc kernel rebuilt for sm_100a), 32 launches "
                      "per graph"}


def run_ours(args, world, rank, local):
    from decode_llm_kernel_b200 import cuda
    from decode_llm_kernel_b200.harness.decode_loop import DecodeStep, StepInputs, pinned_like
    cuda.require()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    w = WORKLOADS[args.workload].shard_for(rank, world)
    if args.cache_len:
        # profiling runs only: smaller caches, same per-token work (one slot per token)
        w = replace(w, cache_alloc_len=args.cache_len)
    peak, peak_src = measured_hbm_peak()
    cos, sin = build_tables(w, device)
    nsets = sets_needed(w)
    k_caches, v_caches, sets = build_step_state(w, device, args.seed + 7919 * rank, nsets)
    step = DecodeStep(k_caches, v_caches, cos, sin, pdl=not args.no_pdl)
    captured = [step.capture(s) for s in sets]
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()

    sampler = ClockSampler(local).start()
    time.sleep(0.3)
    t_load0 = time.perf_counter()
    for i in range(args.warmup):
        captured[i % nsets].replay()
    torch.cuda.synchronize()
    barrier(world)
    t_timed0 = time.perf_counter()
    ms = time_graph_steps(captured, args.steps, stream)
    t_timed1 = time.perf_counter()
    barrier(world)
    ms_max = max_over_ranks(ms, world)
    sampler.stop()
    clocks = sampler.summary(t_load0, t_timed1)
    cuda.check_status(local)

    # parity of the timed step: input set 0 replayed once more, every layer checked
    captured[0].replay()
    torch.cuda.synchronize()
    s0 = sets[0]
    bad = {"q": 0, "k_slots": 0, "v_slots": 0, "max_ulp": 0, "elements": 0}
    for layer in range(w.layers):
        counts = check_call(s0.q[layer], s0.k[layer], s0.v[layer], s0.positions,
                            s0.request_indices, cos, sin, captured[0].q_out[layer],
                            k_caches[layer], v_caches[layer], w.rotary)
        for key in bad:
            bad[key] = max(bad[key], counts[key]) if key == "max_ulp" else bad[key] + counts[key]
    parity = {"result": parity_label(bad), "layers_checked": w.layers, "how": PARITY_NOTE}

    per_step_s = ms_max / 1e3 / args.steps
    bytes_step = w.bytes_per_step()
    value = world * bytes_step / per_step_s / 1e9
    per_launch_s = per_step_s / w.layers
    achieved = w.bytes_per_call() / per_launch_s / 1e9
    # DRAM traffic of one launch from an ncu capture of this kernel on the same workload with
    # caches cut to 256 positions (per-launch traffic does not depend on the cache size: one
    # slot per token); profiles/rope_kv_kernel_decode32_bf16.md
    traffic = DECODE32_NCU_DRAM_BYTES if args.workload == "llama3_8b_decode32" else None
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": traffic, "peak_source": peak_src,
                "traffic_note": "dram__bytes_read.sum + dram__bytes_write.sum per launch "
                                "(878,848 + 0) from profiles/rope_kv_kernel_decode32_bf16.md: "
                                "the reads of q/k/v plus table and slot lines; the launch's "
                                "0.8 MB of writes stay in L2 until later",
                "kernel": "drk::rope_kv_kernel<BF16, int, 16, kFused, kStrided, 1 row/thread>",
                "per_launch_bytes": w.bytes_per_call(), "us_per_launch": per_launch_s * 1e6,
                "note": "average launch = graph step time / layers, so it includes the gaps "
                        "between the chained launches"}

    # end to end: the public API's pipelined host path -- one graph holding `depth` decode
    # steps, each copying its q/k/v/positions in from pinned host memory and its q_out back.
    # Graph replays on one stream do not overlap, so each replay starts with a host-to-device
    # copy alone and ends with a device-to-host copy alone; 32 steps per graph spread that
    # over more steps (8 steps per graph: 587 us/step against 514 us of copies alone).
    e2e = None
    if not args.no_e2e:
        depth = E2E_STEPS_PER_GRAPH
        hosts = [pinned_like(sets[i % nsets]) for i in range(depth)]
        # device buffers beyond the bench's own sets: copies of them (the capture's warm-up
        # runs on the device contents before any host copy)
        def clone(x):
            return StepInputs(x.q.clone(), x.k.clone(), x.v.clone(), x.positions.clone(),
                              x.request_indices.clone())
        dev_sets = [sets[i] if i < nsets else clone(sets[i % nsets]) for i in range(depth)]
        pipe = step.capture_host_pipeline(dev_sets, hosts)
        h2d = sum(t.numel() * t.element_size() for t in (hosts[0].q, hosts[0].k, hosts[0].v,
                                                          hosts[0].positions,
                                                          hosts[0].request_indices))
        d2h = pipe.host_q_outs[0].numel() * pipe.host_q_outs[0].element_size()
        for _ in range(3):
            pipe.replay()
        torch.cuda.synchronize()
        replays = max(3, min(args.steps, 400) // depth)
        barrier(world)
        t0 = time.perf_counter()
        for _ in range(replays):
            pipe.replay()
        torch.cuda.synchronize()
        e2e_s = max_over_ranks(time.perf_counter() - t0, world)
        barrier(world)
        e2e_steps = replays * depth
        # the end-to-end results on the host: step 0's q_out against the PyTorch restatement
        h0 = hosts[0]
        e2e_q_bad = differing(pipe.host_q_outs[0][0],
                              rope_torch(h0.q[0], h0.positions, cos.cpu(), sin.cpu(), w.rotary))
        # the same copies without the decode work: the step's PCIe bound on this box
        cin, cout = torch.cuda.Stream(device), torch.cuda.Stream(device)
        hq, dq = pipe.host_q_outs[0], pipe.q_outs[0]
        src, dst = hosts[0], dev_sets[0]

        def copies(n):
            for _ in range(n):
                with torch.cuda.stream(cin):
                    for a, b in ((dst.q, src.q), (dst.k, src.k), (dst.v, src.v),
                                 (dst.positions, src.positions),
                                 (dst.request_indices, src.request_indices)):
                        a.copy_(b, non_blocking=True)
                with torch.cuda.stream(cout):
                    hq.copy_(dq, non_blocking=True)
            torch.cuda.synchronize()
        copies(3)
        t0 = time.perf_counter()
        copies(32)
        copy_us = (time.perf_counter() - t0) / 32 * 1e6
        e2e = {"value": world * bytes_step * e2e_steps / e2e_s / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "us_per_step": e2e_s / e2e_steps * 1e6, "steps": e2e_steps,
               "copies_alone_us_per_step": copy_us,
               "parity_layer0_q": "bit-exact" if e2e_q_bad == 0 else f"MISMATCH {e2e_q_bad}",
               "path": f"DecodeStep.capture_host_pipeline: {depth} steps per graph, each "
                       "copying q/k/v/positions in from pinned host memory, running the 32 "
                       "fused launches and copying q_out back; copies on their own streams; "
                       "wall clock with a sync on both sides"}
        pipe.release()
        del hosts, dev_sets

    floor = None
    if not args.no_floor:
        # one layer reads (and writes) half its algorithmic bytes; the fused kernel's 1-row
        # launch shape for this batch is 192-thread CTAs
        floor = launch_floor(stream, w.layers, copy_bytes=w.bytes_per_call() // 2 // 32 * 32)
        # The layer launch against the floors: the graph node without PDL (an empty kernel per
        # node, the floor the reference measures, with no PDL in its graphs), with PDL (the
        # chain this step runs), and the dependent copy with the layer's memory pattern.
        us_launch = per_launch_s * 1e6
        floor["layer_us"] = us_launch
        floor["layer_vs_graph_node"] = us_launch / floor["graph_us_per_node"]
        floor["layer_vs_graph_node_pdl"] = us_launch / floor["graph_us_per_node_pdl"]
        floor["layer_vs_dependent_copy"] = us_launch / floor["dependent_copy_us_per_node"]

    ref, ref_why = (None, "skipped")
    if world == 1 and not args.no_reference_gpu:
        ref, ref_why = reference_or_reason()
    ref_step = None
    if ref is not None and ref.gpu_ok:
        ref_step = reference_decode_step(ref, k_caches, v_caches, sets, cos, sin, args.steps,
                                         args.warmup, w)
        ref_step["speedup_of_ours"] = ref_step["us_per_step"] / (per_step_s * 1e6)
    ladder = None if (args.no_ladder or rank != 0) else operator_ladder(device, args.seed, ref)
    del captured, sets, k_caches, v_caches, step
    torch.cuda.empty_cache()
    bw = None if args.no_bw_probe else bandwidth_probe(world, rank, device, args.seed, peak)
    tp = None if args.no_bw_probe else single_layer_probe("llama3_70b_tp", world, rank, device,
                                                          args.seed, peak)
    partial, cfg1 = None, None
    if not args.no_bw_probe and world == 1:
        partial = single_layer_probe("phi2_partial", world, rank, device, args.seed, peak)
        cfg1 = single_layer_probe("llama3_8b_b8", world, rank, device, args.seed, peak)
    ref_gpu = None
    if world == 1 and rank == 0 and not args.no_reference_gpu and not args.no_bw_probe:
        ref_gpu = reference_gpu(device, args.seed, peak,
                                {"llama3_8b_b8": cfg1, "llama3_70b_tp": tp,
                                 "mistral_b4096": bw, "phi2_partial": partial})
        ref_gpu["llama3_8b_decode32"] = ref_step if ref_step is not None else {
            "unavailable": ref_why}
    attention = None
    if not args.no_attention and rank == 0:
        torch.cuda.empty_cache()
        attention = attention_probe(device, args.seed, peak)

    cpu, cpu_torch = None, None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, args.seed, args.cpu_seconds)
        if ref is not None:
            cpu_torch = cpu_baseline_torch(w, args.seed, args.cpu_seconds, ref)
        else:
            cpu_torch = {"unavailable": ref_why}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step_s * 1e3,
            "us_per_step": per_step_s * 1e6, "us_per_call": per_launch_s * 1e6,
            "tokens_per_s": world * w.batch / per_step_s,
            "frac_of_hbm_peak": value / world / peak,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": w.dtype_label,
            "data": "synthetic (seeded N(0,1) q/k/v and caches, int32 positions)",
            "config": workload_config(w, world),
            "timing": {"l2": f"inputs rotate over {nsets} distinct sets "
                             f"({nsets * input_set_bytes(w) / 2**20:.0f} MiB > 3x L2)",
                       "pdl": not args.no_pdl, "clock": "CUDA events on the launching stream, "
                       "max over ranks"},
            "parity": parity,
            "roofline": roofline, "e2e": e2e, "cpu_baseline": cpu,
            "cpu_baseline_torch": cpu_torch, "clocks": clocks,
            "gpu_launches": args.steps * w.layers, "launch_floor": floor,
            "strong_scaling": strong_scaling_record(bw, tp, world),
            "reference_gpu": ref_gpu, "operator_ladder": ladder,
            "bandwidth_config": bw, "tp_config": tp, "partial_rotary_config": partial,
            "single_layer_config": cfg1, "fused_attention": attention,
        }
        print(json.dumps(line), flush=True)


ATTENTION_CASES = ("full_cache_b32", "ragged_b64", "full_cache_b32_d64", "ragged_b64_d64",
                   "ragged_b64_paged16", "ragged_b64_paged256")


def attention_probe(device, seed, peak, sets=2, reps=12, only=None):
    """Fused RoPE + append + decode attention (one launch, the tensor-core kernel) against the
    append followed by a separate attention read of the same cache, graph-timed.

    Two shapes (Llama-3-8B heads, 32:8:128 bf16, 8192-position token-major caches):
      full_cache_b32:  every token at the last position, the read-side probe's configuration
                       (the baseline is our fused append, then SDPA over the cache viewed
                       head-major with enable_gqa);
      ragged_b64:      the decode loop's layer, positions U[0, 8192) (the baseline is our fused
                       append, then flash_attn's kv-cache decode with per-sequence lengths, when
                       flash_attn runs on this GPU);
      full_cache_b32_d64, ragged_b64_d64: the same two with head_dim 64 (Llama-3.2-1B heads,
                       32:8:64);
      ragged_b64_paged{16,256}: the same over a paged cache (pages shuffled through the block
                       table; the baseline is our paged append, then flash_attn's kv-cache
                       decode with the block table, which takes pages of 256 positions).
    Bytes per call: the K and V rows each token attends over (positions 0..pos), plus q, k, v,
    the appended slots and attn_out. Caches rotate over `sets` sets of 1-2 GiB (> L2).
    `only` names one case to run alone (for a profiler capture)."""
    from decode_llm_kernel_b200.cuda import ops
    from decode_llm_kernel_b200.rope_tables import build_rope_tables
    Hq, Hkv, D, S, dt = 32, 8, 128, 8192, torch.bfloat16
    tables = {d: build_rope_tables(S, d, 500000.0, device=device) for d in (64, 128)}
    cos, sin = tables[D]
    out = {}

    def graph_us(fns):
        for f in fns:
            f()
        torch.cuda.synchronize()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for f in fns:
                f()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for f in fns:
                f()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(reps):
            g.replay()
        s1.record()
        torch.cuda.synchronize()
        del g
        return s0.elapsed_time(s1) * 1e3 / (reps * len(fns))

    for label, T, full, D in (("full_cache_b32", 32, True, 128), ("ragged_b64", 64, False, 128),
                              ("full_cache_b32_d64", 32, True, 64),
                              ("ragged_b64_d64", 64, False, 64)):
        if only is not None and label != only:
            continue
        cos, sin = tables[D]
        gen = torch.Generator(device=device).manual_seed(seed)
        st = []
        for _ in range(sets):
            kc = torch.randn(T, S, Hkv, D, device=device, dtype=dt, generator=gen)
            vc = torch.randn(T, S, Hkv, D, device=device, dtype=dt, generator=gen)
            q = torch.randn(T, Hq, D, device=device, dtype=dt, generator=gen)
            k = torch.randn(T, Hkv, D, device=device, dtype=dt, generator=gen)
            v = torch.randn(T, Hkv, D, device=device, dtype=dt, generator=gen)
            if full:
                pos = torch.full((T,), S - 1, device=device, dtype=torch.int32)
            else:
                pos = torch.randint(0, S, (T,), device=device, dtype=torch.int32, generator=gen)
            ri = torch.arange(T, device=device, dtype=torch.int32)
            st.append(dict(q=q, k=k, v=v, p=pos, ri=ri, kc=kc, vc=vc,
                           out=torch.empty_like(q), qo=torch.empty_like(q)))
        attended = sum(int(x["p"].sum().item()) + T for x in st) / sets
        bytes_call = (2 * Hkv * D * 2 * attended + 2 * T * Hq * D * 2 + 4 * T * Hkv * D * 2)

        nbytes = ops.attention_workspace_bytes(T, Hq, Hkv, D, S, dt, device=device.index or 0)
        for x in st:
            x["ws"] = torch.zeros(nbytes, dtype=torch.uint8, device=device)

        def fused(x):
            # a persistent workspace, zeroed once: every call leaves its counters at zero
            return lambda: ops.fused_rope_kv_append_attention(
                x["q"], x["k"], x["v"], x["p"], cos, sin, x["kc"], x["vc"], x["ri"],
                attn_out=x["out"], workspace=x["ws"], workspace_zeroed=True)

        def append(x):
            return lambda: ops.fused_rope_kv_append_ex(x["q"], x["k"], x["v"], x["p"], cos, sin,
                                                       x["kc"], x["vc"], x["ri"], q_out=x["qo"])
        us = graph_us([fused(x) for x in st])
        res = {"T": T, "Hq": Hq, "Hkv": Hkv, "D": D, "cache_alloc_len": S, "dtype": "bf16",
               "positions": "all at S-1" if full else "U[0, S)",
               "bytes_per_call": bytes_call, "fused_us": us,
               "fused_gbs": bytes_call / us / 1e3, "frac_of_hbm_peak": bytes_call / us / 1e3 / peak,
               "kernel": "drk::rope_kv_attention_tc_kernel (tcgen05 + TMA, warp-specialized)",
               "workspace": "persistent per input set, zeroed once (workspace_zeroed=True)"}
        try:
            if full:
                import torch.nn.functional as F

                def read(x):
                    qh = x["qo"].view(T, Hq, 1, D)
                    kt, vt = x["kc"].transpose(1, 2), x["vc"].transpose(1, 2)
                    return lambda: F.scaled_dot_product_attention(qh, kt, vt, enable_gqa=True)
                base = "fused append, then torch SDPA over the token-major cache viewed head-major"
            else:
                from flash_attn import flash_attn_with_kvcache

                def read(x):
                    qh = x["qo"].view(T, 1, Hq, D)
                    lens = x["p"] + 1
                    return lambda: flash_attn_with_kvcache(qh, x["kc"], x["vc"],
                                                           cache_seqlens=lens)
                base = "fused append, then flash_attn_with_kvcache (per-sequence lengths)"

            def both(x):
                f1, f2 = append(x), read(x)
                return lambda: (f1(), f2())
            res["separate_us"] = graph_us([both(x) for x in st])
            res["separate"] = base
            res["speedup_vs_separate"] = res["separate_us"] / us
        except Exception as e:  # noqa: BLE001 -- an unavailable baseline is reported, not fatal
            res["separate"] = f"unavailable: {type(e).__name__}: {str(e)[:160]}"
        out[label] = res
        del st
        torch.cuda.empty_cache()

    # the decode layer over a paged cache: pages shuffled through the block table
    D = 128
    cos, sin = tables[D]
    for bs in (16, 256):
        if only is not None and only != f"ragged_b64_paged{bs}":
            continue
        T = 64
        gen = torch.Generator(device=device).manual_seed(seed + bs)
        nblk = S // bs
        st = []
        for _ in range(sets):
            kp = torch.randn(T * nblk, bs, Hkv, D, device=device, dtype=dt, generator=gen)
            vp = torch.randn(T * nblk, bs, Hkv, D, device=device, dtype=dt, generator=gen)
            table = torch.randperm(T * nblk, device=device, generator=gen).view(T, nblk)
            st.append(dict(q=torch.randn(T, Hq, D, device=device, dtype=dt, generator=gen),
                           k=torch.randn(T, Hkv, D, device=device, dtype=dt, generator=gen),
                           v=torch.randn(T, Hkv, D, device=device, dtype=dt, generator=gen),
                           p=torch.randint(0, S, (T,), device=device, dtype=torch.int32,
                                           generator=gen),
                           ri=torch.arange(T, device=device, dtype=torch.int32),
                           kp=kp, vp=vp, table=table.to(torch.int32),
                           out=torch.empty(T, Hq, D, device=device, dtype=dt),
                           qo=torch.empty(T, Hq, D, device=device, dtype=dt)))
        attended = sum(int(x["p"].sum().item()) + T for x in st) / sets
        bytes_call = (2 * Hkv * D * 2 * attended + 2 * T * Hq * D * 2 + 4 * T * Hkv * D * 2)

        nbytes = ops.attention_workspace_bytes(T, Hq, Hkv, D, nblk * bs, dt,
                                               device=device.index or 0, path="tensor_cores")
        for x in st:
            x["ws"] = torch.zeros(nbytes, dtype=torch.uint8, device=device)

        def fused_paged(x):
            return lambda: ops.paged_rope_kv_append_attention(
                x["q"], x["k"], x["v"], x["p"], cos, sin, x["kp"], x["vp"], x["table"], x["ri"],
                attn_out=x["out"], workspace=x["ws"], workspace_zeroed=True)
        us = graph_us([fused_paged(x) for x in st])
        res = {"T": T, "block_size": bs, "positions": "U[0, S)", "bytes_per_call": bytes_call,
               "fused_us": us, "fused_gbs": bytes_call / us / 1e3,
               "frac_of_hbm_peak": bytes_call / us / 1e3 / peak}
        try:
            from flash_attn import flash_attn_with_kvcache
            if bs % 256:
                raise ValueError(f"flash_attn takes pages of 256 positions and up, not {bs}")

            def both(x):
                def run():
                    q_rot = ops.paged_rope_kv_append(x["q"], x["k"], x["v"], x["p"], cos, sin,
                                                     x["kp"], x["vp"], x["table"], x["ri"])
                    flash_attn_with_kvcache(q_rot.view(T, 1, Hq, D), x["kp"], x["vp"],
                                            cache_seqlens=x["p"] + 1, block_table=x["table"])
                return run
            res["separate_us"] = graph_us([both(x) for x in st])
            res["separate"] = "paged append, then flash_attn_with_kvcache with the block table"
            res["speedup_vs_separate"] = res["separate_us"] / us
        except Exception as e:  # noqa: BLE001 -- an unavailable baseline is reported, not fatal
            why = f"{type(e).__name__}: {str(e)[:120]}"
            try:
                res.update(flashinfer_separate(st, T, Hq, Hkv, D, bs, cos, sin, device, graph_us))
                res["speedup_vs_separate"] = res["separate_us"] / us
            except Exception as e2:  # noqa: BLE001
                res["separate"] = (f"unavailable: flash_attn {why}; flashinfer "
                                   f"{type(e2).__name__}: {str(e2)[:120]}")
        out[f"ragged_b64_paged{bs}"] = res
        del st
        torch.cuda.empty_cache()
    return out


def flashinfer_separate(st, T, Hq, Hkv, D, bs, cos, sin, device, graph_us):
    """The separate baseline over a paged cache with any page size: this build's paged append,
    then flashinfer's batch decode over the same pages (its [num_pages, page_size, Hkv, D]
    "NHD" layout is this build's page layout), each input set planned once outside the graph;
    the faster of its CUDA-core and tensor-core decode kernels is reported."""
    import flashinfer
    from decode_llm_kernel_b200.cuda import ops
    best = None
    for tensor_cores in (False, True):
        runs = []
        for x in st:
            lens = x["p"].to(torch.int64) + 1
            npages = (lens + bs - 1) // bs
            indptr = torch.zeros(T + 1, dtype=torch.int32, device=device)
            indptr[1:] = torch.cumsum(npages, 0)
            used = torch.arange(x["table"].shape[1], device=device)[None, :] < npages[:, None]
            indices = x["table"][used].to(torch.int32)
            last = ((lens - 1) % bs + 1).to(torch.int32)
            work = torch.empty(128 << 20, dtype=torch.uint8, device=device)
            w = flashinfer.BatchDecodeWithPagedKVCacheWrapper(
                work, "NHD", use_cuda_graph=True, use_tensor_cores=tensor_cores,
                paged_kv_indptr_buffer=indptr, paged_kv_indices_buffer=indices,
                paged_kv_last_page_len_buffer=last)
            w.plan(indptr, indices, last, Hq, Hkv, D, bs, q_data_type=x["q"].dtype,
                   kv_data_type=x["kp"].dtype)

            def run(x=x, w=w, keep=(work, indptr, indices, last)):
                q_rot = ops.paged_rope_kv_append(x["q"], x["k"], x["v"], x["p"], cos, sin,
                                                 x["kp"], x["vp"], x["table"], x["ri"])
                w.run(q_rot, (x["kp"], x["vp"]))
            runs.append(run)
        t = graph_us(runs)
        if best is None or t < best[0]:
            best = (t, tensor_cores)
    return {"separate_us": best[0],
            "separate": (f"paged append, then flashinfer BatchDecodeWithPagedKVCacheWrapper "
                         f"(pages of {bs}, use_tensor_cores={best[1]}, the faster of the two)")}


def operator_ladder(device, seed, ref):
    """The reference's operator benchmark at its headline shape, for this build and for the
    reference's own kernels: Llama-3-8B heads (32 Q / 8 KV, head_dim 128), batch 8, bf16,
    theta 5e5, cache [8, 4096, 8, 128], eight rotating device position sets; each rung is
    driven eagerly through the op's Python binding or by replaying one graph per position set
    (harness/runners.py), and timed three ways (harness/timing.time_call). Then the fused op's
    amortised per-call cost at batch 1, 8, 32 and 128. The inputs are 200 KB, so like the
    reference's own rows these are launch-latency numbers."""
    from decode_llm_kernel_b200.cuda import ops
    from decode_llm_kernel_b200.harness import positions as pos
    from decode_llm_kernel_b200.harness.inputs import make_inputs
    from decode_llm_kernel_b200.harness.runners import RUNGS
    from decode_llm_kernel_b200.harness.timing import logical_bytes, time_call
    impls = {"ours": ops}
    if ref is not None and ref.gpu_ok:
        impls["reference"] = ref.ops
    names = {"fused": "fused_rope_kv_append", "separate": "separate_rope_kv_append"}
    base = WORKLOADS["llama3_8b_b8"]
    out = {"workload": "llama3_8b_b8 (batch 8, 32/8 heads, head_dim 128, bf16, theta 5e5)",
           "rungs": {}, "fused_amortized_us_by_batch": {}}
    for batch in (8, 1, 32, 128):
        w = replace(base, batch=batch, positions="ragged")
        sets = pos.build_position_sets(batch, w.cache_alloc_len, pos.RAGGED, seed, 8, device,
                                       torch.int32)
        inputs = make_inputs(w, device, seed, sets[0], cache_fill="normal")
        if batch == 8:
            out["logical_bytes_per_call"] = logical_bytes(
                inputs.q, inputs.k, inputs.v, inputs.cos, inputs.sin, inputs.k_cache,
                inputs.v_cache)["total_bytes"]
            for impl, mod in impls.items():
                for label, op_name, kind in RUNGS:
                    runner = kind(getattr(mod, names[op_name]), inputs, sets)
                    out["rungs"][f"{impl}:{label}"] = time_call(runner, warmup=200, iters=1000)
                    runner.release()
        for impl, mod in impls.items():
            runner = RUNGS[1][2](mod.fused_rope_kv_append, inputs, sets)
            out["fused_amortized_us_by_batch"].setdefault(impl, {})[batch] = time_call(
                runner, warmup=200, iters=1000)["amortized_us"]
        del inputs
    if "reference" not in impls:
        out["reference"] = "unavailable: " + (ref.gpu_reason if ref else "not installed")
    return out


def cpu_inputs(w, seed, cache_len):
    """Host tensors for whole steps of workload w with caches cut to cache_len positions per
    request (the op touches one slot per token, so per-token work is unchanged)."""
    g = torch.Generator().manual_seed(seed)
    L, T = w.layers, w.batch
    q = torch.randn(L, T, w.num_q_heads, w.head_dim, generator=g).to(w.dtype)
    k = torch.randn(L, T, w.num_kv_heads, w.head_dim, generator=g).to(w.dtype)
    v = torch.randn(L, T, w.num_kv_heads, w.head_dim, generator=g).to(w.dtype)
    kcs = [torch.randn(T, cache_len, w.num_kv_heads, w.head_dim, generator=g).to(w.dtype)
           for _ in range(L)]
    vcs = [torch.randn(T, cache_len, w.num_kv_heads, w.head_dim, generator=g).to(w.dtype)
           for _ in range(L)]
    from decode_llm_kernel_b200.rope_tables import build_rope_tables
    cos, sin = build_rope_tables(cache_len, w.rotary, w.theta)
    pos = torch.randint(0, cache_len, (T,), generator=g)
    ri = torch.arange(T)
    return q, k, v, kcs, vcs, cos, sin, pos, ri


CPU_CACHE_LEN = 64


def time_cpu_steps(one_step, seconds, max_steps=100000):
    one_step()
    steps, t0 = 0, time.perf_counter()
    while True:
        one_step()
        steps += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= seconds or steps >= max_steps:
            return elapsed / steps, steps


def cpu_baseline(w, seed, seconds):
    """The CPU oracle (a C port of the reference's PyTorch algorithm, OpenMP) on a bounded
    sample of the workload: whole steps (every layer, every token), caches cut to 64 positions
    per request, all host threads."""
    from oracle import oracle
    threads = os.cpu_count() or 1
    q, k, v, kcs, vcs, cos, sin, pos, ri = cpu_inputs(w, seed, CPU_CACHE_LEN)

    def one_step():
        for layer in range(w.layers):
            oracle.fused_rope_kv_append(q[layer], k[layer], v[layer], pos, cos, sin, kcs[layer],
                                        vcs[layer], ri, nthreads=threads)

    per_step, steps = time_cpu_steps(one_step, seconds)
    return {"value": w.bytes_per_step() / per_step / 1e9, "unit": "GB/s", "cores": threads,
            "kind": "port", "ms_per_step": per_step * 1e3, "steps": steps,
            "sample": f"{steps} whole {w.layers}-layer steps of {w.batch} tokens through the CPU "
                      f"oracle (C, OpenMP, {threads} threads); caches cut to {CPU_CACHE_LEN} "
                      f"positions per request and positions drawn in [0, {CPU_CACHE_LEN}), "
                      "which leaves per-token work unchanged"}


def cpu_baseline_torch(w, seed, seconds, ref, max_steps=100000):
    """The reference's own PyTorch path (decode_kernels.reference.fused_rope_kv_append_ref) on
    CPU tensors, all host threads, under torch.inference_mode(): whole steps with caches cut to
    64 positions per request."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    q, k, v, kcs, vcs, cos, sin, pos, ri = cpu_inputs(w, seed, CPU_CACHE_LEN)

    def one_step():
        for layer in range(w.layers):
            ref.oracle(q[layer], k[layer], v[layer], pos, cos, sin, kcs[layer], vcs[layer], ri)

    with torch.inference_mode():
        per_step, steps = time_cpu_steps(one_step, seconds, max_steps)
    return {"value": w.bytes_per_step() / per_step / 1e9, "unit": "GB/s", "cores": threads,
            "kind": "reference", "ms_per_step": per_step * 1e3, "steps": steps,
            "sample": f"{steps} whole {w.layers}-layer steps of {w.batch} tokens through the "
                      "reference's PyTorch oracle fused_rope_kv_append_ref on CPU tensors "
                      f"({threads} torch threads, inference_mode); caches cut to {CPU_CACHE_LEN} "
                      "positions per request, which leaves per-token work unchanged"}


def workload_config(w, world):
    """The `config` both arms print, so the driver compares like with like."""
    return dict(w.describe(), **{
        "parallelism": f"batch shard x{world} ({w.batch} sequences and their own caches per GPU)",
        "global_batch": w.batch * world, "seq_len": w.cache_alloc_len})


def strong_scaling_record(bw, tp, world):
    """Per-N records of the two sharded workloads (mistral_b4096 split by batch, llama3_70b_tp
    split by KV head): total work fixed, so per-GPU work shrinks as N grows."""
    out = {}
    for key, r in (("mistral_b4096", bw), ("llama3_70b_tp", tp)):
        if r:
            out[key] = {"n_gpus": world, "us": r["us_per_launch"],
                        "gbs_per_gpu": r["achieved_gbs_per_gpu"], "frac": r["frac_of_peak"],
                        "aggregate_gbs": r["aggregate_gbs"], "shard": r["shard"],
                        "parity": r["parity"]}
    return out


def launch_floor(stream, layers, copy_bytes=0, copy_threads=192, sets=10):
    """Launch floors of a chain of `layers` launches in one CUDA graph, per node:
      graph_us_per_node[_pdl]   empty kernels (the floor the reference measures), without and
                                with programmatic dependent launch;
      dependent_copy_us_per_node  a copy with one layer's memory pattern (copy_bytes read and
                                written, two 16-byte vectors per thread, copy_threads per CTA,
                                source lines pulled toward L2 during the wait, PDL), rotating
                                over `sets` buffer sets larger than L2 like the decode step's
                                inputs: the cost of a chained launch that reads after the
                                previous launch and writes before the next;
      direct_us[_pdl]           empty kernels launched one by one from the host (amortised)."""
    from decode_llm_kernel_b200 import cuda
    ext = cuda.require()
    out = {}
    for pdl in (False, True):
        ext.launch_empty(50, pdl)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ext.launch_empty(2000, pdl)
        torch.cuda.synchronize()
        out[f"direct_us{'_pdl' if pdl else ''}"] = (time.perf_counter() - t0) / 2000 * 1e6
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            ext.launch_empty(1, pdl)
        stream.wait_stream(side)
        with torch.cuda.graph(g):
            ext.launch_empty(layers, pdl)
        for _ in range(20):
            g.replay()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(500):
            g.replay()
        end.record(stream)
        torch.cuda.synchronize()
        key = f"graph_us_per_node{'_pdl' if pdl else ''}"
        out[key] = start.elapsed_time(end) * 1e3 / (500 * layers)
    if copy_bytes:
        out.update(copy_floor(ext, stream, layers, copy_bytes, copy_threads, sets))
    return out


def copy_floor(ext, stream, layers, copy_bytes, threads, sets, replays=200):
    span = layers * copy_bytes
    src = torch.empty(sets * span, dtype=torch.uint8, device="cuda")
    dst = torch.empty_like(src)
    src.random_(0, 255)
    graphs = []
    for s in range(sets):
        chunk_s, chunk_d = src[s * span:(s + 1) * span], dst[s * span:(s + 1) * span]
        ext.launch_copy_probe(chunk_s, chunk_d, copy_bytes, copy_bytes, layers, threads)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ext.launch_copy_probe(chunk_s, chunk_d, copy_bytes, copy_bytes, layers, threads)
        graphs.append(g)
    for i in range(3 * sets):
        graphs[i % sets].replay()
    ms = time_graph_steps(graphs, replays, stream)
    ok = torch.equal(src[:span], dst[:span])
    del graphs, src, dst
    return {"dependent_copy_us_per_node": ms * 1e3 / (replays * layers),
            "dependent_copy": {"bytes_read_per_node": copy_bytes, "threads_per_cta": threads,
                               "prefetch": True, "pdl": True, "copied_correctly": ok}}


def run_reference(args, world, rank):
    """The reference's CPU implementation of the path on the host cores, rank 0 only: its
    PyTorch oracle (decode_kernels.reference.fused_rope_kv_append_ref, installed by
    baseline/build_ref.py) with all host threads under inference_mode; when that is not
    installed, the C/OpenMP port of the same algorithm in oracle/. Same workload, metric, unit
    and config dict as this build's arm; caches cut to 64 positions per request (per-token work
    is unchanged), and each timed step sized so the whole run stays within about two
    minutes."""
    if rank != 0:
        return
    w = WORKLOADS[args.workload]
    ref, why = reference_or_reason()
    threads = os.cpu_count() or 1
    q, k, v, kcs, vcs, cos, sin, pos, ri = cpu_inputs(w, args.seed, CPU_CACHE_LEN)
    if ref is not None:
        torch.set_num_threads(threads)
        kind = "reference"
        what = (f"the reference's PyTorch oracle fused_rope_kv_append_ref on CPU tensors "
                f"({threads} torch threads, inference_mode)")

        def layer_call(layer):
            ref.oracle(q[layer], k[layer], v[layer], pos, cos, sin, kcs[layer], vcs[layer], ri)
    else:
        from oracle import oracle
        kind = "port"
        what = (f"the C/OpenMP port of the reference's algorithm ({threads} threads; the "
                f"reference itself is not installed: {why})")

        def layer_call(layer):
            oracle.fused_rope_kv_append(q[layer], k[layer], v[layer], pos, cos, sin,
                                        kcs[layer], vcs[layer], ri, nthreads=threads)

    with torch.inference_mode():
        layer_call(0)
        t0 = time.perf_counter()
        for layer in range(w.layers):
            layer_call(layer)
        probe_step = time.perf_counter() - t0
        layers_per_step = w.layers
        total = (args.steps + args.warmup) * probe_step
        if total > 120.0:
            layers_per_step = max(1, int(w.layers * 120.0 / total))

        def one_step():
            for layer in range(layers_per_step):
                layer_call(layer)

        for _ in range(args.warmup):
            one_step()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            one_step()
        per = (time.perf_counter() - t0) / args.steps
    value = w.bytes_per_call() * layers_per_step / per / 1e9
    sample = (f"{layers_per_step} of {w.layers} layers x {w.batch} tokens per step through "
              f"{what}; caches cut to {CPU_CACHE_LEN} positions per request")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per * 1e3 * (w.layers / layers_per_step), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": w.dtype_label,
        "data": "synthetic (seeded N(0,1) q/k/v and caches, int positions)",
        "config": workload_config(w, max(1, world)),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    world, rank, local = init_dist(args)
    if args.gpus != world and world > 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.mode in ("bw", "single"):
            local_dev = torch.device("cuda", local)
            torch.cuda.set_device(local_dev)
            peak, _ = measured_hbm_peak()
            name = "mistral_b4096" if args.mode == "bw" else args.probe
            out = single_layer_probe(name, world, rank, local_dev, args.seed, peak,
                                     args.cache_len, args.launches)
            if rank == 0:
                print(json.dumps(out), flush=True)
        elif args.mode == "attention":
            from decode_llm_kernel_b200 import cuda
            cuda.require()
            local_dev = torch.device("cuda", local)
            torch.cuda.set_device(local_dev)
            peak, _ = measured_hbm_peak()
            if rank == 0:
                print(json.dumps(attention_probe(local_dev, args.seed, peak,
                                                 only=args.attention_case)), flush=True)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist
            if dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
