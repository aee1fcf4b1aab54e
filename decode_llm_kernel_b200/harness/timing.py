"""Byte accounting (the roofline numerator) and the per-call timer.

`logical_bytes` follows the reference's formula (benchmarks/benchmark_utils.py:35-68): reads of
q, k, v and of the rotary half-rows of cos and sin, writes of q_rot and of the K and V cache
slots; index reads are excluded. With partial rotary only rotary_dim/2 cos and sin values are
read per token.

`time_call` reports a call's cost in the three views the reference's results use (an
amortised loop, per-call device events, per-call synchronised wall clock), from one
measurement routine of this package.
"""
import statistics
import time

import torch


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


def time_call(fn, *, warmup=100, iters=1000, stream=None):
    """Cost of `fn()` (which launches work on `stream`, default the current stream), in us:

      amortized_us     wall clock of `iters` calls issued back to back, with one synchronise
                       after the last, divided by `iters`: what a launch-bound caller pays
                       per call in steady state (the reference's headline timer);
      event_median_us  median over calls of the device interval between two events recorded
                       around each call (includes the gaps launch latency leaves);
      synchronized_us  median over calls of the wall clock of one call plus a synchronise.

    Events and wall clocks come from a single pass of `3 * iters` calls after `warmup`."""
    stream = stream or torch.cuda.current_stream()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()

    t0 = time.perf_counter()
    for _ in range(iters):
        fn()
    torch.cuda.synchronize()
    amortized = (time.perf_counter() - t0) / iters

    marks = [torch.cuda.Event(enable_timing=True) for _ in range(2 * iters)]
    for i in range(iters):
        marks[2 * i].record(stream)
        fn()
        marks[2 * i + 1].record(stream)
    torch.cuda.synchronize()
    events = [marks[2 * i].elapsed_time(marks[2 * i + 1]) / 1e3 for i in range(iters)]

    walls = []
    for _ in range(iters):
        t = time.perf_counter()
        fn()
        torch.cuda.synchronize()
        walls.append(time.perf_counter() - t)
    return {"amortized_us": amortized * 1e6,
            "event_median_us": statistics.median(events) * 1e6,
            "synchronized_us": statistics.median(walls) * 1e6,
            "iters": iters}
