"""A multi-layer decode step captured into one CUDA graph.

Each layer is one fused RoPE + KV-append launch into that layer's own K/V cache; all layers
share the step's positions and request indices. Layers after the first are launched with
programmatic dependent launch, so each kernel reads its positions and table rows while the
previous layer's kernel drains (positions and tables are never written by these kernels).
Optionally the step's host<->device traffic is captured in the same graph: q/k/v and
positions are copied in from pinned host buffers and q_out is copied back, so one replay is one
end-to-end decode step. `capture_host_pipeline` captures several such steps in one graph with
the copies on their own streams: step i+1's inputs cross PCIe while step i computes and step
i-1's q_out crosses back, and the layers of successive steps stay in order on one stream.
"""
from dataclasses import dataclass

import torch

from ..cuda import ops


@dataclass
class StepInputs:
    q: torch.Tensor           # [L, T, Hq, D]
    k: torch.Tensor           # [L, T, Hkv, D]
    v: torch.Tensor           # [L, T, Hkv, D]
    positions: torch.Tensor   # [T]
    request_indices: torch.Tensor  # [T]


class CapturedStep:
    def __init__(self, graph, q_out, inputs, host=None, host_q_out=None):
        self.graph = graph
        self.q_out = q_out            # [L, T, Hq, D] on the device
        self.inputs = inputs          # device-side StepInputs the graph reads
        self.host = host              # pinned StepInputs copied in each replay (or None)
        self.host_q_out = host_q_out  # pinned [L, T, Hq, D] copied out each replay (or None)

    def replay(self):
        self.graph.replay()

    def release(self):
        self.graph = None


class DecodeStep:
    def __init__(self, k_caches, v_caches, cos, sin, *, pdl=True, advance_positions=False):
        """advance_positions: end each step with positions += 1 on the device, so a captured
        step can be replayed step after step (each replay appends at the next position)."""
        if len(k_caches) != len(v_caches):
            raise ValueError("one K and one V cache per layer")
        self.k_caches = list(k_caches)
        self.v_caches = list(v_caches)
        self.cos, self.sin = cos, sin
        self.pdl = pdl
        self.advance = advance_positions
        self.layers = len(self.k_caches)

    def run(self, inputs, q_out):
        """Eager launches of every layer (the body that capture() records)."""
        for layer in range(self.layers):
            ops.fused_rope_kv_append_ex(
                inputs.q[layer], inputs.k[layer], inputs.v[layer], inputs.positions, self.cos,
                self.sin, self.k_caches[layer], self.v_caches[layer], inputs.request_indices,
                pdl=self.pdl and layer > 0, q_out=q_out[layer])
        if self.advance:
            ops.advance_positions(inputs.positions, 1, pdl=self.pdl)

    def capture(self, inputs, host=None, warmup=1):
        """Capture one step over device `inputs`. With `host` (pinned StepInputs), the graph
        starts by copying host -> inputs and ends by copying q_out -> a pinned buffer."""
        L, T, Hq, D = inputs.q.shape
        q_out = torch.empty((L, T, Hq, D), dtype=inputs.q.dtype, device=inputs.q.device)
        host_q_out = None
        if host is not None:
            host_q_out = torch.empty((L, T, Hq, D), dtype=inputs.q.dtype, pin_memory=True)
        side = torch.cuda.Stream(device=inputs.q.device)
        side.wait_stream(torch.cuda.current_stream(inputs.q.device))
        saved = inputs.positions.clone() if self.advance else None
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.run(inputs, q_out)
            if saved is not None:
                inputs.positions.copy_(saved)   # warm-up steps must not move the loop
        torch.cuda.current_stream(inputs.q.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            if host is not None:
                for dst, src in ((inputs.q, host.q), (inputs.k, host.k), (inputs.v, host.v),
                                 (inputs.positions, host.positions),
                                 (inputs.request_indices, host.request_indices)):
                    dst.copy_(src, non_blocking=True)
            self.run(inputs, q_out)
            if host is not None:
                host_q_out.copy_(q_out, non_blocking=True)
        return CapturedStep(graph, q_out, inputs, host, host_q_out)

    def capture_host_pipeline(self, device_sets, host_sets, warmup=1):
        """Capture len(device_sets) end-to-end steps in one graph. Step i copies host_sets[i]
        into device_sets[i] on a copy-in stream, runs every layer on the capturing stream after
        its copy and after step i-1's layers, and copies its q_out back into a pinned buffer on a
        copy-out stream. One replay is len(device_sets) decode steps."""
        return _capture_pipeline(self, device_sets, host_sets, warmup)


class CapturedPipeline:
    """Several end-to-end decode steps in one graph (see DecodeStep.capture_host_pipeline)."""

    def __init__(self, graph, q_outs, host_q_outs, steps):
        self.graph = graph
        self.q_outs = q_outs
        self.host_q_outs = host_q_outs
        self.steps = steps

    def replay(self):
        self.graph.replay()

    def release(self):
        self.graph = None


def _capture_pipeline(step, device_sets, host_sets, warmup=1):
    if len(device_sets) != len(host_sets) or not device_sets:
        raise ValueError("one pinned host set per device set")
    dev = device_sets[0].q.device
    q_outs = [torch.empty(d.q.shape, dtype=d.q.dtype, device=dev) for d in device_sets]
    host_q_outs = [torch.empty(d.q.shape, dtype=d.q.dtype, pin_memory=True) for d in device_sets]
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(warmup):
            for d, qo in zip(device_sets, q_outs):
                step.run(d, qo)
    torch.cuda.current_stream(dev).wait_stream(side)
    copy_in = torch.cuda.Stream(device=dev)
    copy_out = torch.cuda.Stream(device=dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        compute = torch.cuda.current_stream(dev)
        copy_in.wait_stream(compute)
        copy_out.wait_stream(compute)
        for d, h, qo, hqo in zip(device_sets, host_sets, q_outs, host_q_outs):
            with torch.cuda.stream(copy_in):
                for dst, src in ((d.q, h.q), (d.k, h.k), (d.v, h.v), (d.positions, h.positions),
                                 (d.request_indices, h.request_indices)):
                    dst.copy_(src, non_blocking=True)
            compute.wait_stream(copy_in)
            step.run(d, qo)
            copy_out.wait_stream(compute)
            with torch.cuda.stream(copy_out):
                hqo.copy_(qo, non_blocking=True)
        compute.wait_stream(copy_in)
        compute.wait_stream(copy_out)
    return CapturedPipeline(graph, q_outs, host_q_outs, len(device_sets))


def pinned_like(inputs):
    """Pinned host copies of a StepInputs (the end-to-end path's source buffers)."""
    def pin(t):
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        h.copy_(t)
        return h
    return StepInputs(pin(inputs.q), pin(inputs.k), pin(inputs.v), pin(inputs.positions),
                      pin(inputs.request_indices))
