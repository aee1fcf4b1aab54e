"""The seam where a Hugging Face decoder's attention layer calls the fused op.

The reference prices this seam with a patched attention forward ("op_replaced",
benchmarks/rung_patches.py:129-198) that rotates Q/K with its PyTorch oracle and writes the
static cache through its transposed view at the layer's `cumulative_length`. `patch_decoder`
does the same with one call of this package's fused kernel per layer and decode step.

`patch_decoder(model)` swaps the forward of every attention layer of a Llama, Mistral or Phi-3
model (transformers 5.x module layout). A decode step -- one new token per sequence, against a
StaticCache whose layer is a plain full-attention StaticLayer -- then runs, per layer:

  q, k, v   the layer's own projections: q_proj/k_proj/v_proj, or Phi-3's qkv_proj sliced
            three ways; as [B, H, D] views (head_dim contiguous, token stride the projection's
            width), read in place and never copied;
  one call  ops.fused_rope_kv_append_ex: q_rot = RoPE(q), K slot = RoPE(k), V slot = v,
            written through the cache's [B, S, Hkv, D] view of HF's [B, Hkv, S, D] storage
            (strided_cache=True) at the position held in the layer's cumulative_length tensor
            (read on the device, never on the host); then cumulative_length += 1, as
            StaticLayer.update would do;
  attention the model's own attention interface over the whole static cache, unchanged.

RoPE reads fp32 tables built once per model from its rotary embedding (inv_freq and
attention_scaling, the values HF evaluates each step), so the rotation follows the
reference's locked fp32 semantics. HF's own path rotates in the model dtype with cos/sin
rounded to it: in fp32 models the two agree to within an ulp, in bf16 models they differ by
rounding.

Everything else takes the original forward: prefill (more than one new token per sequence),
caches that are not StaticCache full-attention layers (dynamic, sliding-window), an
uninitialised cache layer, rotary embeddings whose frequencies change per step ("dynamic",
"longrope"), and attention modules with extra query/key processing (q_norm/k_norm).
"""
import types

import torch

from .cuda import ops

PATCHED_ATTR = "_drk_original_forward"
_STEPWISE_ROPE = ("dynamic", "longrope")


def rope_tables_from_inv_freq(inv_freq, max_position, scaling=1.0):
    """fp32 (cos, sin) [max_position, 2 * len(inv_freq)] in concat(f, f) rows, computed on
    the CPU from a model's inverse frequencies the way its rotary embedding does per step."""
    inv = inv_freq.detach().to("cpu", torch.float32)
    angles = torch.outer(torch.arange(max_position, dtype=torch.float32), inv)
    both = torch.cat((angles, angles), dim=-1)
    cos, sin = both.cos(), both.sin()
    if scaling != 1.0:
        cos, sin = cos * scaling, sin * scaling
    return cos, sin


class _Tables:
    """The model's fp32 RoPE tables on each device, grown to the longest cache seen."""

    def __init__(self, rotary_emb):
        self.rotary_emb = rotary_emb
        self._by_device = {}

    def get(self, device, rows):
        have = self._by_device.get(device)
        if have is None or have[0].shape[0] < rows:
            cos, sin = rope_tables_from_inv_freq(
                self.rotary_emb.inv_freq, rows,
                float(getattr(self.rotary_emb, "attention_scaling", 1.0)))
            have = (cos.to(device), sin.to(device))
            self._by_device[device] = have
        return have


def _find(model):
    """(decoder layers' attention modules, the rotary embedding) of a transformers model."""
    base = getattr(model, "model", model)
    layers = getattr(base, "layers", None)
    rotary = getattr(base, "rotary_emb", None)
    if layers is None or rotary is None or not hasattr(rotary, "inv_freq"):
        raise ValueError("patch_decoder needs a decoder with .model.layers[i].self_attn and "
                         ".model.rotary_emb (Llama, Mistral, Phi-3)")
    attns = [layer.self_attn for layer in layers]
    for attn in attns:
        has_split = all(hasattr(attn, n) for n in ("q_proj", "k_proj", "v_proj"))
        if not (has_split or hasattr(attn, "qkv_proj")):
            raise ValueError(f"{type(attn).__name__} has neither q/k/v_proj nor qkv_proj")
    return attns, rotary


def _projections(attn, hidden_states):
    """q [B, Hq, D], k and v [B, Hkv, D] for one new token per sequence, as views."""
    B, D = hidden_states.shape[0], attn.head_dim
    hq = attn.config.num_attention_heads
    hkv = attn.config.num_key_value_heads
    x = hidden_states[:, 0]
    if hasattr(attn, "qkv_proj"):
        qkv = attn.qkv_proj(x)
        q = qkv[:, : hq * D]
        k = qkv[:, hq * D:(hq + hkv) * D]
        v = qkv[:, (hq + hkv) * D:]
    else:
        q, k, v = attn.q_proj(x), attn.k_proj(x), attn.v_proj(x)
    return q.view(B, hq, D), k.view(B, hkv, D), v.view(B, hkv, D)


def _make_forward(attn, original, tables, stepwise_rope):
    from transformers.cache_utils import StaticLayer
    rows_cache = {}

    def forward(self, hidden_states, position_embeddings, attention_mask, past_key_values=None,
                **kwargs):
        layer = None
        if past_key_values is not None and hasattr(past_key_values, "layers"):
            layer = past_key_values.layers[self.layer_idx]
        fused = (not stepwise_rope and hidden_states.shape[1] == 1 and hidden_states.is_cuda
                 and type(layer) is StaticLayer and getattr(layer, "is_initialized", False)
                 and not hasattr(self, "q_norm") and not hasattr(self, "k_norm"))
        if not fused:
            return original(hidden_states, position_embeddings, attention_mask,
                            past_key_values=past_key_values, **kwargs)
        B = hidden_states.shape[0]
        q, k, v = _projections(self, hidden_states)
        device = hidden_states.device
        cos, sin = tables.get(device, layer.max_cache_len)
        rows = rows_cache.get((B, device))
        if rows is None:
            rows = torch.arange(B, device=device, dtype=torch.int64)
            rows_cache[(B, device)] = rows
        positions = layer.cumulative_length.expand(B).contiguous()
        rotary = cos.shape[1]
        q_rot = ops.fused_rope_kv_append_ex(
            q, k, v, positions, cos, sin, layer.keys.transpose(1, 2),
            layer.values.transpose(1, 2), rows, strided_cache=True,
            rotary_dim=0 if rotary == self.head_dim else rotary)
        layer.cumulative_length.add_(1)

        from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
        module = __import__(type(self).__module__, fromlist=["eager_attention_forward"])
        interface = ALL_ATTENTION_FUNCTIONS.get_interface(self.config._attn_implementation,
                                                          module.eager_attention_forward)
        attn_output, attn_weights = interface(
            self, q_rot.unsqueeze(2), layer.keys, layer.values, attention_mask,
            dropout=0.0, scaling=self.scaling,
            sliding_window=getattr(self.config, "sliding_window", None), **kwargs)
        attn_output = attn_output.reshape(B, 1, -1).contiguous()
        return self.o_proj(attn_output), attn_weights

    return types.MethodType(forward, attn)


class Patch:
    """Handle of a patched model; restore() puts the original attention forwards back."""

    def __init__(self, attns):
        self.attns = attns

    def restore(self):
        for attn in self.attns:
            if PATCHED_ATTR not in attn.__dict__:
                continue
            previous = attn.__dict__.pop(PATCHED_ATTR)
            if previous is None:
                attn.__dict__.pop("forward", None)     # back to the class's forward
            else:
                attn.forward = previous               # an instance forward set before us
        self.attns = []


def patch_decoder(model):
    """Route the decode steps of every attention layer of `model` through the fused op (see
    the module docstring). Returns a Patch; patching a model twice raises."""
    attns, rotary = _find(model)
    if any(PATCHED_ATTR in a.__dict__ for a in attns):
        raise RuntimeError("this model's attention layers are already patched")
    tables = _Tables(rotary)
    stepwise = getattr(rotary, "rope_type", "default") in _STEPWISE_ROPE
    for attn in attns:
        original = attn.forward
        attn.__dict__[PATCHED_ATTR] = attn.__dict__.get("forward")
        attn.forward = _make_forward(attn, original, tables, stepwise)
    return Patch(attns)
