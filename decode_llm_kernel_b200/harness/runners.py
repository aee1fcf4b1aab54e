"""Drivers of a stream of decode calls for the operator ladder: one op, one set of input
tensors, a rotation of device-resident position sets.

  EagerRunner   each call goes through the op's Python binding with the next position set
                (host dispatch + launch every call).
  BoundGraphs   one CUDA graph captured per position set, each bound to its own device
                positions tensor, replayed in rotation: no host-to-device copy and no host
                dispatch on the timed path. (The reference's graph runner keeps a single graph
                and copies each call's positions into its static buffer before the replay,
                benchmarks/impls.py:144-150; with the positions already on the device -- a
                decode loop advances them there, harness/decode_loop.py -- the copy is not
                needed.)

Both take `op(*OpInputs)`: ops.fused_rope_kv_append, ops.separate_rope_kv_append, or the
reference's own ops through its binding. A runner is called with no arguments and returns the
call's q_rot.
"""
import itertools

import torch


class EagerRunner:
    kind = "eager"

    def __init__(self, op, inputs, position_sets):
        self.op = op
        self.inputs = inputs
        self._sets = itertools.cycle(position_sets)

    def __call__(self):
        return self.op(*self.inputs._replace(positions=next(self._sets)))

    def release(self):
        self.inputs = None


class BoundGraphs:
    kind = "graph"

    def __init__(self, op, inputs, position_sets, warmup=2):
        self.outputs = []
        self._graphs = []
        side = torch.cuda.Stream(device=inputs.q.device)
        side.wait_stream(torch.cuda.current_stream(inputs.q.device))
        # warm-up launches (lazy module loads, allocator pools) off the capturing stream
        with torch.cuda.stream(side):
            for p in position_sets:
                for _ in range(warmup):
                    op(*inputs._replace(positions=p))
        torch.cuda.current_stream(inputs.q.device).wait_stream(side)
        for p in position_sets:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                out = op(*inputs._replace(positions=p))
            self._graphs.append(g)
            self.outputs.append(out)
        self._next = itertools.cycle(range(len(self._graphs)))

    def __call__(self):
        i = next(self._next)
        self._graphs[i].replay()
        return self.outputs[i]

    def release(self):
        self._graphs.clear()
        self.outputs.clear()


RUNGS = (
    ("cuda_separate", "separate", EagerRunner),
    ("cuda_fused", "fused", EagerRunner),
    ("graph_cuda_separate", "separate", BoundGraphs),
    ("graph_cuda_fused", "fused", BoundGraphs),
)
