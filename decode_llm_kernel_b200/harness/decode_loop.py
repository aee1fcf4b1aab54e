"""A multi-layer decode step captured into one CUDA graph.

Each layer is one fused RoPE + KV-append launch into that layer's own K/V cache; all layers
share the step's positions and request indices. Layers after the first are launched with
programmatic dependent launch, so each kernel reads its positions and table rows while the
previous layer's kernel drains (positions and tables are never written by these kernels).
Optionally the step's host<->device traffic is captured in the same graph: q/k/v and
positions are copied in from pinned host buffers and q_out is copied back, so one replay is one
end-to-end decode step.
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
    def __init__(self, k_caches, v_caches, cos, sin, *, pdl=True):
        if len(k_caches) != len(v_caches):
            raise ValueError("one K and one V cache per layer")
        self.k_caches = list(k_caches)
        self.v_caches = list(v_caches)
        self.cos, self.sin = cos, sin
        self.pdl = pdl
        self.layers = len(self.k_caches)

    def run(self, inputs, q_out):
        """Eager launches of every layer (the body that capture() records)."""
        for layer in range(self.layers):
            ops.fused_rope_kv_append_ex(
                inputs.q[layer], inputs.k[layer], inputs.v[layer], inputs.positions, self.cos,
                self.sin, self.k_caches[layer], self.v_caches[layer], inputs.request_indices,
                pdl=self.pdl and layer > 0, q_out=q_out[layer])

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
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.run(inputs, q_out)
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


def pinned_like(inputs):
    """Pinned host copies of a StepInputs (the end-to-end path's source buffers)."""
    def pin(t):
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        h.copy_(t)
        return h
    return StepInputs(pin(inputs.q), pin(inputs.k), pin(inputs.v), pin(inputs.positions),
                      pin(inputs.request_indices))
