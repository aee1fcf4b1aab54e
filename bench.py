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

Launch: python bench.py [--gpus N --steps K --warmup W]; for N > 1 under torchrun, one rank per
GPU, each owning its own batch shard and caches (weak scaling, no collective on the data path;
NCCL only for the barrier and the max-over-ranks time).
`--impl reference` times the reference's CPU algorithm (the CPU oracle port, all host threads)
on the same workload and prints the same JSON line with impl=reference.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from decode_llm_kernel_b200.harness.configs import WORKLOADS, make_positions  # noqa: E402

FALLBACK_HBM_GBS = 6650.0
# ncu captures (profiles/): DRAM bytes read + written per launch
DECODE32_NCU_DRAM_BYTES = 878848 + 0
MISTRAL_NCU_DRAM_BYTES = 51522560 + 5620480
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
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--mode", choices=["full", "bw", "attention"], default="full",
                   help="bw: only the bandwidth-bound launch loop (for profiling small cases); "
                        "attention: only the fused append + decode attention measurement")
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


def single_layer_probe(name, world, rank, device, seed, peak, cache_len=0, iters=400):
    """One fused launch per call of a single-layer workload (sharded for this rank), input sets
    rotated so they exceed 3x L2, launches replayed from a CUDA graph with programmatic
    dependent launch between them (no launch writes another's positions, indices or tables),
    device time per launch from CUDA events, max over ranks. cache_len > 0 shrinks the caches
    (same per-token work) for profiling runs."""
    from dataclasses import replace
    from decode_llm_kernel_b200.cuda import ops
    w = WORKLOADS[name].shard_for(rank, world)
    if cache_len:
        w = replace(w, cache_alloc_len=cache_len)
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
    rot = w.rotary_dim if w.rotary_dim and w.rotary_dim != w.head_dim else 0

    def call(i):
        q, k, v, p, ri, qo = sets[i % nsets]
        ops.fused_rope_kv_append_ex(q, k, v, p, cos, sin, kc, vc, ri, q_out=qo, pdl=True,
                                    rotary_dim=rot)

    # Launches are replayed from a CUDA graph so host call overhead cannot pace the GPU.
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
    gbs_rank = w.bytes_per_call() / per_launch_s / 1e9
    staged = w.batch >= 512
    out = {"workload": name, "shard": w.shard, "batch_per_gpu": w.batch,
           "q_heads_per_gpu": w.num_q_heads, "kv_heads_per_gpu": w.num_kv_heads,
           "head_dim": w.head_dim, "rotary_dim": w.rotary_dim or w.head_dim,
           "dtype": w.dtype_label, "cache_alloc_len": w.cache_alloc_len, "launches": iters,
           "pdl": True,
           "kernel": ("drk::rope_kv_staged_kernel (TMA bulk copies, 3-stage mbarrier pipeline)"
                      if staged else "drk::rope_kv_kernel (register kernel)"),
           "bytes_per_launch": w.bytes_per_call(), "us_per_launch": per_launch_s * 1e6,
           "achieved_gbs_per_gpu": gbs_rank, "frac_of_peak": gbs_rank / peak,
           "aggregate_gbs": gbs_rank * world, "input_sets": nsets}
    if name == "mistral_b4096" and world == 1:
        out["traffic"] = MISTRAL_NCU_DRAM_BYTES
        out["traffic_note"] = ("ncu, caches cut to 128 positions: reads 51.5 MB = the "
                               "algorithmic reads; 5.6 MB of the 51.4 MB of writes reach DRAM "
                               "within the launch, the rest drains from L2 afterwards")
    del kc, vc, sets
    torch.cuda.empty_cache()
    return out


def bandwidth_probe(world, rank, device, seed, peak, cache_len=0, iters=400):
    """The bandwidth-bound workload (mistral_b4096, sharded by batch)."""
    return single_layer_probe("mistral_b4096", world, rank, device, seed, peak, cache_len, iters)


def run_ours(args, world, rank, local):
    from decode_llm_kernel_b200 import cuda
    from decode_llm_kernel_b200.harness.decode_loop import DecodeStep, StepInputs, pinned_like
    cuda.require()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    w = WORKLOADS[args.workload].shard_for(rank, world)
    if args.cache_len:
        # profiling runs only: smaller caches, same per-token work (one slot per token)
        from dataclasses import replace
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
                                "(878,848 + 0): the reads of q/k/v plus table and slot lines; "
                                "the launch's 0.8 MB of writes stay in L2 until later",
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
               "path": f"DecodeStep.capture_host_pipeline: {depth} steps per graph, each "
                       "copying q/k/v/positions in from pinned host memory, running the 32 "
                       "fused launches and copying q_out back; copies on their own streams; "
                       "wall clock with a sync on both sides"}
        pipe.release()
        del hosts, dev_sets

    floor = None if args.no_floor else launch_floor(stream, w.layers)
    if floor is not None:
        # The layer launch against the graph-node floor: without PDL (an empty kernel per graph
        # node, the floor the reference measures with no PDL in its graphs) and with PDL (the
        # chain this step runs).
        us_launch = per_launch_s * 1e6
        floor["layer_us"] = us_launch
        floor["layer_vs_graph_node"] = us_launch / floor["graph_us_per_node"]
        floor["layer_vs_graph_node_pdl"] = us_launch / floor["graph_us_per_node_pdl"]
    ladder = None if (args.no_ladder or rank != 0) else operator_ladder(device, args.seed)
    del captured, sets, k_caches, v_caches, step
    torch.cuda.empty_cache()
    bw = None if args.no_bw_probe else bandwidth_probe(world, rank, device, args.seed, peak)
    tp = None if args.no_bw_probe else single_layer_probe("llama3_70b_tp", world, rank, device,
                                                          args.seed, peak)
    partial = None
    if not args.no_bw_probe and world == 1:
        partial = single_layer_probe("phi2_partial", world, rank, device, args.seed, peak)
    attention = None
    if not args.no_attention and rank == 0:
        torch.cuda.empty_cache()
        attention = attention_probe(device, args.seed, peak)

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, args.seed, args.cpu_seconds)

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
            "config": dict(w.describe(), **{
                "parallelism": f"batch shard x{world} (64 sequences and own caches per GPU)",
                "global_batch": w.batch * world, "seq_len": w.cache_alloc_len,
                "l2": f"inputs rotate over {nsets} distinct sets "
                      f"({nsets * input_set_bytes(w) / 2**20:.0f} MiB > 3x L2)",
                "pdl": not args.no_pdl}),
            "roofline": roofline, "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks,
            "gpu_launches": args.steps * w.layers, "launch_floor": floor,
            "operator_ladder": ladder,
            "bandwidth_config": bw, "tp_config": tp, "partial_rotary_config": partial,
            "fused_attention": attention,
        }
        print(json.dumps(line), flush=True)


ATTENTION_CASES = ("full_cache_b32", "ragged_b64", "ragged_b64_paged16", "ragged_b64_paged256")


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
      ragged_b64_paged{16,256}: the same over a paged cache (pages shuffled through the block
                       table; the baseline is our paged append, then flash_attn's kv-cache
                       decode with the block table, which takes pages of 256 positions).
    Bytes per call: the K and V rows each token attends over (positions 0..pos), plus q, k, v,
    the appended slots and attn_out. Caches rotate over `sets` sets of 1-2 GiB (> L2).
    `only` names one case to run alone (for a profiler capture)."""
    from decode_llm_kernel_b200.cuda import ops
    from decode_llm_kernel_b200.rope_tables import build_rope_tables
    Hq, Hkv, D, S, dt = 32, 8, 128, 8192, torch.bfloat16
    cos, sin = build_rope_tables(S, D, 500000.0, device=device)
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

    for label, T, full in (("full_cache_b32", 32, True), ("ragged_b64", 64, False)):
        if only is not None and label != only:
            continue
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

        def fused(x):
            return lambda: ops.fused_rope_kv_append_attention(
                x["q"], x["k"], x["v"], x["p"], cos, sin, x["kc"], x["vc"], x["ri"],
                attn_out=x["out"])

        def append(x):
            return lambda: ops.fused_rope_kv_append_ex(x["q"], x["k"], x["v"], x["p"], cos, sin,
                                                       x["kc"], x["vc"], x["ri"], q_out=x["qo"])
        us = graph_us([fused(x) for x in st])
        res = {"T": T, "Hq": Hq, "Hkv": Hkv, "D": D, "cache_alloc_len": S, "dtype": "bf16",
               "positions": "all at S-1" if full else "U[0, S)",
               "bytes_per_call": bytes_call, "fused_us": us,
               "fused_gbs": bytes_call / us / 1e3, "frac_of_hbm_peak": bytes_call / us / 1e3 / peak,
               "kernel": "drk::rope_kv_attention_tc_kernel (tcgen05 + TMA, warp-specialized)"}
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

        def fused_paged(x):
            return lambda: ops.paged_rope_kv_append_attention(
                x["q"], x["k"], x["v"], x["p"], cos, sin, x["kp"], x["vp"], x["table"], x["ri"],
                attn_out=x["out"])
        us = graph_us([fused_paged(x) for x in st])
        res = {"T": T, "block_size": bs, "positions": "U[0, S)", "bytes_per_call": bytes_call,
               "fused_us": us, "fused_gbs": bytes_call / us / 1e3,
               "frac_of_hbm_peak": bytes_call / us / 1e3 / peak}
        try:
            from flash_attn import flash_attn_with_kvcache

            def both(x):
                def run():
                    ops.paged_rope_kv_append(x["q"], x["k"], x["v"], x["p"], cos, sin, x["kp"],
                                             x["vp"], x["table"], x["ri"])
                    flash_attn_with_kvcache(x["qo"].view(T, 1, Hq, D), x["kp"], x["vp"],
                                            cache_seqlens=x["p"] + 1, block_table=x["table"])
                return run
            res["separate_us"] = graph_us([both(x) for x in st])
            res["separate"] = "paged append, then flash_attn_with_kvcache with the block table"
            res["speedup_vs_separate"] = res["separate_us"] / us
        except Exception as e:  # noqa: BLE001 -- an unavailable baseline is reported, not fatal
            res["separate"] = f"unavailable: {type(e).__name__}: {str(e)[:160]}"
        out[f"ragged_b64_paged{bs}"] = res
        del st
        torch.cuda.empty_cache()
    return out


def operator_ladder(device, seed):
    """The reference's operator benchmark at its headline shape, on this build: Llama-3-8B
    heads (32 Q / 8 KV, head_dim 128), batch 8, bf16, cache [8, 4096, 8, 128], eight rotating
    device position sets, every rung through the drop-in ops and the reference's runners, with
    the reference's three timers (benchmarks/benchmark_utils.py:80-126 of the reference). The
    inputs are 200 KB, so like the reference's own rows these are launch-latency numbers."""
    from decode_llm_kernel_b200.harness import impls, timing
    from decode_llm_kernel_b200.harness import positions as pos
    from decode_llm_kernel_b200.harness.workload import Config, build_op_args
    cfg = Config("gqa", 32, 8, 128, 8, 4096, "bf16", pos.RAGGED, theta=500000.0,
                 index_dtype="int32")
    sets = pos.build_position_sets(8, 4096, pos.RAGGED, seed, 8, device, torch.int32)
    args = build_op_args(cfg, device, seed, sets[0])
    nbytes = timing.logical_bytes(args.q, args.k, args.v, args.cos, args.sin, args.k_cache,
                                  args.v_cache)["total_bytes"]
    rows = {}
    for spec in impls.IMPL_SPECS:
        runner = spec.build()
        thunk = runner.make_thunk(args, sets)
        amort = timing.time_amortized_call(thunk, 200, 3000)
        events = timing.time_device_events(thunk, 50, 500)
        synced = timing.time_synchronized_call(thunk, 50, 500)
        med = sorted(events)[len(events) // 2]
        rows[spec.label] = {"amortized_us": amort * 1e3, "event_median_us": med * 1e3,
                            "synchronized_us": synced * 1e3,
                            "logical_gbs_amortized": timing.logical_eff_gbps(nbytes, amort)}
        if hasattr(runner, "release"):
            runner.release()
    return {"workload": "llama3_8b_b8 (batch 8, 32/8 heads, head_dim 128, bf16, theta 5e5)",
            "logical_bytes_per_call": nbytes, "rungs": rows}


def launch_floor(stream, layers):
    """Empty-kernel floor: direct launches (amortised) and a graph of `layers` chained empty
    kernels, with and without programmatic dependent launch."""
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
        out[f"graph_us_per_node{'_pdl' if pdl else ''}"] = start.elapsed_time(end) * 1e3 / (500 * layers)
    return out


def cpu_baseline(w, seed, seconds):
    """The CPU oracle (a port of the reference's PyTorch algorithm) on a bounded sample of the
    workload: whole steps (every layer, every token) with caches cut to 64 positions per request
    -- the op touches one slot per token, so per-token work is unchanged -- on all host
    threads."""
    from oracle import oracle
    from decode_llm_kernel_b200.rope_tables import build_rope_tables
    threads = os.cpu_count() or 1
    S = 64
    g = torch.Generator().manual_seed(seed)
    L, T = w.layers, w.batch
    q = torch.randn(L, T, w.num_q_heads, w.head_dim, generator=g).to(w.dtype)
    k = torch.randn(L, T, w.num_kv_heads, w.head_dim, generator=g).to(w.dtype)
    v = torch.randn(L, T, w.num_kv_heads, w.head_dim, generator=g).to(w.dtype)
    kcs = [torch.randn(T, S, w.num_kv_heads, w.head_dim, generator=g).to(w.dtype)
           for _ in range(L)]
    vcs = [torch.randn(T, S, w.num_kv_heads, w.head_dim, generator=g).to(w.dtype)
           for _ in range(L)]
    cos, sin = build_rope_tables(S, w.rotary_dim or w.head_dim, w.theta)
    pos = torch.randint(0, S, (T,), generator=g)
    ri = torch.arange(T)

    def one_step():
        for layer in range(L):
            oracle.fused_rope_kv_append(q[layer], k[layer], v[layer], pos, cos, sin, kcs[layer],
                                        vcs[layer], ri, nthreads=threads)

    one_step()
    steps, t0 = 0, time.perf_counter()
    while True:
        one_step()
        steps += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= seconds or steps >= 100000:
            break
    per_step = elapsed / steps
    return {"value": w.bytes_per_step() / per_step / 1e9, "unit": "GB/s", "cores": threads,
            "kind": "port", "ms_per_step": per_step * 1e3, "steps": steps,
            "sample": f"{steps} whole {L}-layer steps of {T} tokens through the CPU oracle "
                      f"(C, OpenMP, {threads} threads); caches cut to {S} positions per request "
                      f"and positions drawn in [0, {S}), which leaves per-token work unchanged"}


def run_reference(args, world, rank):
    """The reference's algorithm on the host CPU (the oracle port, all threads), same workload,
    metric and unit; rank 0 only."""
    if rank != 0:
        return
    w = WORKLOADS[args.workload]
    # size each timed step so K + W steps stay within about two minutes
    probe = cpu_baseline(w, args.seed, 0.5)
    per_step_s = probe["ms_per_step"] / 1e3
    total = (args.steps + args.warmup) * per_step_s
    if total > 120.0:
        note = (f"; {args.steps} steps would take {total:.0f} s, so each timed step is "
                f"{args.steps} x a 2-minute budget")
    else:
        note = ""
    from oracle import oracle
    from decode_llm_kernel_b200.rope_tables import build_rope_tables
    threads = os.cpu_count() or 1
    S = 64
    g = torch.Generator().manual_seed(args.seed)
    L, T = w.layers, w.batch
    q = torch.randn(L, T, w.num_q_heads, w.head_dim, generator=g).to(w.dtype)
    k = torch.randn(L, T, w.num_kv_heads, w.head_dim, generator=g).to(w.dtype)
    v = torch.randn(L, T, w.num_kv_heads, w.head_dim, generator=g).to(w.dtype)
    kcs = [torch.randn(T, S, w.num_kv_heads, w.head_dim, generator=g).to(w.dtype)
           for _ in range(L)]
    vcs = [torch.randn(T, S, w.num_kv_heads, w.head_dim, generator=g).to(w.dtype)
           for _ in range(L)]
    cos, sin = build_rope_tables(S, w.rotary_dim or w.head_dim, w.theta)
    pos = torch.randint(0, S, (T,), generator=g)
    ri = torch.arange(T)
    layers_per_step = L
    if total > 120.0:
        layers_per_step = max(1, int(L * 120.0 / total))

    def one_step():
        for layer in range(layers_per_step):
            oracle.fused_rope_kv_append(q[layer], k[layer], v[layer], pos, cos, sin, kcs[layer],
                                        vcs[layer], ri, nthreads=threads)

    for _ in range(args.warmup):
        one_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step()
    elapsed = time.perf_counter() - t0
    per = elapsed / args.steps
    bytes_step = w.bytes_per_call() * layers_per_step
    value = bytes_step / per / 1e9
    sample = (f"{layers_per_step} of {L} layers x {T} tokens per step through the CPU oracle "
              f"(C port of the reference's PyTorch algorithm, OpenMP, {threads} threads); "
              f"caches cut to {S} positions per request{note}")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per * 1e3 * (L / layers_per_step), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": w.dtype_label,
        "data": "synthetic (seeded N(0,1) q/k/v and caches)",
        "config": dict(w.describe(), **{"parallelism": "host CPU, rank 0 only",
                                        "global_batch": w.batch, "seq_len": w.cache_alloc_len}),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
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
        elif args.mode == "bw":
            local_dev = torch.device("cuda", local)
            torch.cuda.set_device(local_dev)
            peak, _ = measured_hbm_peak()
            out = bandwidth_probe(world, rank, local_dev, args.seed, peak, args.cache_len,
                                  args.launches)
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
