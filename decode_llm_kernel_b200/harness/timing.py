"""Byte accounting and the three timers of the reference's harness
(benchmarks/benchmark_utils.py:35-126).

`logical_bytes` is the roofline numerator: reads of q, k, v and the rotary half-rows of cos and
sin, writes of q_rot and of the K and V cache slots. Index reads are excluded, as in the
reference. With partial rotary only rotary_dim/2 cos and sin values are read per token.
"""
import statistics
import time

import torch


def sync():
    torch.cuda.synchronize()


def bytes_per_token(num_q_heads, num_kv_heads, head_dim, elem_bytes, rotary_dim=None):
    r = rotary_dim or head_dim
    return (2 * num_q_heads * head_dim * elem_bytes + 4 * num_kv_heads * head_dim * elem_bytes
            + 2 * (r // 2) * 4)


def logical_bytes(q, k, v, cos, sin, k_cache, v_cache):
    num_tokens, num_q_heads, head_dim = q.shape
    num_kv_heads = k.shape[1]
    half = cos.shape[1] // 2
    reads = {
        "q": num_tokens * num_q_heads * head_dim * q.element_size(),
        "k": num_tokens * num_kv_heads * head_dim * k.element_size(),
        "v": num_tokens * num_kv_heads * head_dim * v.element_size(),
        "cos": num_tokens * half * cos.element_size(),
        "sin": num_tokens * half * sin.element_size(),
    }
    writes = {
        "q_rot": num_tokens * num_q_heads * head_dim * q.element_size(),
        "k_cache": num_tokens * num_kv_heads * head_dim * k_cache.element_size(),
        "v_cache": num_tokens * num_kv_heads * head_dim * v_cache.element_size(),
    }
    read_bytes = sum(reads.values())
    write_bytes = sum(writes.values())
    return {"reads": reads, "writes": writes, "read_bytes": read_bytes,
            "write_bytes": write_bytes, "total_bytes": read_bytes + write_bytes}


def logical_eff_gbps(total_bytes, latency_ms):
    return total_bytes / (latency_ms / 1e3) / 1e9


def time_device_events(fn, warmup, iters):
    """Per-invocation device-timeline ms: CUDA events bracketing each call."""
    for _ in range(warmup):
        fn()
    sync()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    for i in range(iters):
        starts[i].record()
        fn()
        ends[i].record()
    sync()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def time_amortized_call(fn, warmup, iters):
    """Wall time of an unsynchronised loop / iters (ms): steady-state cost per call with
    launches pipelined, not a per-call latency."""
    for _ in range(warmup):
        fn()
    sync()
    t0 = time.perf_counter()
    for _ in range(iters):
        fn()
    sync()
    return (time.perf_counter() - t0) / iters * 1e3


def time_synchronized_call(fn, warmup, iters):
    """Median wall time of individually synchronised calls (ms)."""
    for _ in range(warmup):
        fn()
    sync()
    samples = []
    for _ in range(iters):
        t0 = time.perf_counter()
        fn()
        sync()
        samples.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(samples)


def time_region_events(fn, iters, stream=None):
    """Device ms for `iters` back-to-back calls bracketed by one pair of events."""
    stream = stream or torch.cuda.current_stream()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(iters):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def summarize(samples):
    s = sorted(samples)
    n = len(s)
    return {"median": statistics.median(s), "min": s[0], "p95": s[min(n - 1, int(0.95 * n))],
            "mean": sum(s) / n}
