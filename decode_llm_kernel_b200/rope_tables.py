"""RoPE cos/sin tables in the form the kernels read.

The tables are fp32 [max_position, rotary_dim] with each row laid out as concat(f, f), where
f[i] = position * theta^(-2i/rotary_dim). That is the NeoX / rotate_half convention of the
reference's `build_rope_tables` (decode_kernels/reference/rope_cache.py:3-12); the same fp32
operations are used so a table built here is bit-identical to one built there, which the
golden-fixture tests rely on. The kernels read only the first rotary_dim/2 columns of a row,
because the second half repeats the first.
"""
import torch


def inverse_frequencies(rotary_dim, theta=10000.0, device="cpu"):
    if rotary_dim % 2:
        raise ValueError(f"rotary_dim must be even for split-half RoPE, got {rotary_dim}")
    exponents = torch.arange(0, rotary_dim // 2, dtype=torch.float32, device=device)
    exponents = exponents * 2.0 / rotary_dim
    return 1.0 / (theta ** exponents)


def build_rope_tables(max_position, rotary_dim, theta=10000.0, *, device="cpu",
                      dtype=torch.float32):
    """(cos, sin), each [max_position, rotary_dim]. Built on the CPU and then moved, so the
    values do not depend on the device the caller asks for."""
    inv = inverse_frequencies(rotary_dim, theta)
    t = torch.arange(max_position, dtype=torch.float32)
    angles = torch.outer(t, inv)
    both = torch.cat((angles, angles), dim=-1)
    return both.cos().to(dtype).to(device), both.sin().to(dtype).to(device)
