"""Runners and the implementation registry for the custom-kernel rungs
(benchmarks/impls.py:48-224 of the reference).

DirectRunner calls an op through its normal dispatch path. GraphRunner captures the op once
into a CUDA graph (warm-up on a side stream, then capture) and replays it; positions are copied
into a static buffer before each replay, and a change of any other input pointer recaptures.
"""
import itertools
from dataclasses import dataclass

import torch

from .. import cuda
from .workload import make_thunk

CUDA_SEPARATE = "cuda_separate"
CUDA_FUSED = "cuda_fused"
CUDA_BASES = (CUDA_SEPARATE, CUDA_FUSED)
GRAPH_WARMUP = 3


def cuda_impl(base):
    from ..cuda import ops
    if base == CUDA_SEPARATE:
        return ops.separate_rope_kv_append
    if base == CUDA_FUSED:
        return ops.fused_rope_kv_append
    raise ValueError(f"unknown CUDA base {base!r}, expected one of {CUDA_BASES}")


def assert_extension_available(specs):
    needed = sorted({s.label for s in specs if s.base in CUDA_BASES})
    if needed and not cuda.is_available():
        raise ValueError(f"{needed} need the CUDA extension: {cuda.unavailable_reason()}. "
                         f"Build it with '{cuda.BUILD_COMMAND}'.")


class DirectRunner:
    captured = False

    def __init__(self, fn):
        self.fn = fn

    def __call__(self, *op_args):
        return self.fn(*op_args)

    def make_thunk(self, args, position_sets):
        return make_thunk(self.fn, args, position_sets)


class GraphRunner:
    def __init__(self, fn, warmup=GRAPH_WARMUP):
        self.fn = fn
        self.warmup = warmup
        self.capture_count = 0
        self._key = None
        self._graph = None
        self._output = None
        self._static_positions = None
        self._bound_args = None

    @property
    def captured(self):
        return self._graph is not None

    @staticmethod
    def _pointer_key(op_args):
        q, k, v, _, cos, sin, k_cache, v_cache, request_indices = op_args
        return tuple(t.data_ptr() for t in (q, k, v, cos, sin, k_cache, v_cache,
                                            request_indices))

    def _capture(self, op_args):
        self.release()
        q, k, v, positions, cos, sin, k_cache, v_cache, request_indices = op_args
        static_positions = torch.empty_like(positions)
        static_positions.copy_(positions)
        bound = (q, k, v, static_positions, cos, sin, k_cache, v_cache, request_indices)
        current = torch.cuda.current_stream(q.device)
        side = torch.cuda.Stream(device=q.device)
        side.wait_stream(current)
        with torch.cuda.stream(side):
            for _ in range(self.warmup):
                self.fn(*bound)
        current.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            output = self.fn(*bound)
        self._key = self._pointer_key(op_args)
        self._graph = graph
        self._output = output
        self._static_positions = static_positions
        self._bound_args = bound
        self.capture_count += 1

    def __call__(self, *op_args):
        key = self._pointer_key(op_args)
        if key != self._key:
            self._capture(op_args)
        self._static_positions.copy_(op_args[3])
        self._graph.replay()
        return self._output

    def make_thunk(self, args, position_sets):
        cyc = itertools.cycle(position_sets)
        q, k, v = args.q, args.k, args.v
        cos, sin = args.cos, args.sin
        kc, vc, ri = args.k_cache, args.v_cache, args.request_indices

        def run():
            self(q, k, v, next(cyc), cos, sin, kc, vc, ri)
        return run

    def release(self):
        self._output = None
        self._graph = None
        self._static_positions = None
        self._bound_args = None
        self._key = None


@dataclass(frozen=True)
class ImplSpec:
    label: str
    base: str
    graph: bool
    description: str

    def build(self):
        fn = cuda_impl(self.base)
        return GraphRunner(fn) if self.graph else DirectRunner(fn)


IMPL_SPECS = (
    ImplSpec("cuda_separate", CUDA_SEPARATE, False,
             "RoPE kernel then append kernel, k_rot materialized"),
    ImplSpec("cuda_fused", CUDA_FUSED, False,
             "one kernel; k_rot goes straight to its cache slot"),
    ImplSpec("graph_cuda_separate", CUDA_SEPARATE, True,
             "the separate kernels replayed through a CUDA graph"),
    ImplSpec("graph_cuda_fused", CUDA_FUSED, True,
             "the fused kernel replayed through a CUDA graph"),
)
IMPL_LABELS = tuple(s.label for s in IMPL_SPECS)
CUDA_IMPLS = IMPL_LABELS


def resolve_impls(labels):
    by_label = {s.label: s for s in IMPL_SPECS}
    unknown = [lbl for lbl in labels if lbl not in by_label]
    if unknown:
        raise ValueError(f"unknown impl(s) {unknown}, expected any of {list(IMPL_LABELS)}")
    return [by_label[lbl] for lbl in labels]
