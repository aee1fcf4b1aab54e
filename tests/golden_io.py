"""Loads the golden fixtures written by tests/golden/make_golden.py into torch tensors."""
import glob
import json
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16,
          "fp64": torch.float64}


def names():
    return sorted(os.path.splitext(os.path.basename(p))[0]
                  for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def _tensor(a, dt):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dt in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).view(dt)
    return t


class Golden:
    """One fixture: the op's inputs (q/k/v may be strided views), fresh sentinel caches in the
    fixture's cache layout, and the reference's outputs."""

    def __init__(self, name, device="cpu"):
        with np.load(os.path.join(GOLDEN_DIR, f"{name}.npz")) as z:
            data = {k: z[k] for k in z.files}
        self.meta = json.loads(str(data["meta"]))
        m = self.meta
        self.name = name
        self.dtype = dt = DTYPES[m["dtype"]]
        T, Hq, Hkv, D = m["T"], m["Hq"], m["Hkv"], m["D"]
        if m["layout"] == "packed":
            self.q = _tensor(data["q"], dt).reshape(T, Hq, D).to(device)
            self.k = _tensor(data["k"], dt).reshape(T, Hkv, D).to(device)
            self.v = _tensor(data["v"], dt).reshape(T, Hkv, D).to(device)
        else:
            fused = _tensor(data["fused"], dt).reshape(T, (Hq + 2 * Hkv) * D).to(device)
            parts = fused.split([Hq * D, Hkv * D, Hkv * D], dim=-1)
            self.q, self.k, self.v = (p.view(T, -1, D) for p in parts)
            self.fused = fused
        self.positions = torch.from_numpy(data["positions"]).to(device)
        self.request_indices = torch.from_numpy(data["request_indices"]).to(device)
        self.cos = torch.from_numpy(data["cos"]).to(device)
        self.sin = torch.from_numpy(data["sin"]).to(device)
        self.q_out = _tensor(data["q_out"], dt).reshape(T, Hq, D)
        self.k_slots = _tensor(data["k_slots"], dt).reshape(T, Hkv, D)
        self.v_slots = _tensor(data["v_slots"], dt).reshape(T, Hkv, D)
        self.device = device

    def fresh_caches(self):
        """(k_cache, v_cache, k_view, v_view): storage in the fixture's layout and the
        [B, S, Hkv, D] views the op addresses."""
        m = self.meta
        B, S, Hkv, D = m["B"], m["S"], m["Hkv"], m["D"]
        shape = (B, S, Hkv, D) if m["cache_layout"] == "token_major" else (B, Hkv, S, D)
        kc = torch.full(shape, m["sentinel"], dtype=self.dtype, device=self.device)
        vc = torch.full(shape, m["sentinel"], dtype=self.dtype, device=self.device)
        if m["cache_layout"] == "token_major":
            return kc, vc, kc, vc
        return kc, vc, kc.transpose(1, 2), vc.transpose(1, 2)

    def check(self, q_out, k_view, v_view):
        """Bit-exact comparison against the reference outputs; returns a list of failures."""
        m = self.meta
        failures = []
        pos = self.positions.to(torch.int64).cpu()
        ri = self.request_indices.to(torch.int64).cpu()
        q_out, k_view, v_view = q_out.cpu(), k_view.cpu(), v_view.cpu()
        if not bits_equal(q_out, self.q_out):
            failures.append(f"q_out differs in {_count(q_out, self.q_out)} elements")
        if not bits_equal(k_view[ri, pos], self.k_slots):
            failures.append(f"k slots differ in {_count(k_view[ri, pos], self.k_slots)} elements")
        if not bits_equal(v_view[ri, pos], self.v_slots):
            failures.append("v slots are not byte-exact")
        mask = torch.zeros(m["B"], m["S"], dtype=torch.bool)
        mask[ri, pos] = True
        if not (bool((k_view[~mask] == m["sentinel"]).all())
                and bool((v_view[~mask] == m["sentinel"]).all())):
            failures.append("an unaddressed cache slot was modified")
        return failures


_INT_VIEW = {1: torch.int8, 2: torch.int16, 4: torch.int32, 8: torch.int64}


def bits(t):
    """The tensor's storage bits as an integer tensor (so -0.0 != +0.0 and NaNs compare)."""
    return t.contiguous().view(_INT_VIEW[t.element_size()])


def bits_equal(a, b):
    return a.shape == b.shape and a.dtype == b.dtype and torch.equal(bits(a), bits(b))


def _count(a, b):
    if a.shape != b.shape:
        return -1
    return int((bits(a).reshape(-1) != bits(b).reshape(-1)).sum())
