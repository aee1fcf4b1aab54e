"""The RoPE + KV-append ops, behind the reference's own signatures
(decode_kernels/cuda/ops.py:15-43 of the reference).

Nothing here synchronises, reads device memory on the host, or allocates outside PyTorch's
caching allocator, so every op can be timed at microsecond scale and captured into a CUDA
graph. Out-of-range positions or request indices do not trap: the kernel skips those writes and
records them in a status word that `decode_llm_kernel_b200.cuda.check_status()` reads.
"""
from . import require


def rope_forward(q, k, positions, cos, sin):
    """Split-half RoPE over strided Q and K in one launch. Returns (q_rot, k_rot)."""
    return require().rope_forward(q, k, positions, cos, sin)


def kv_append(k_rot, v, positions, request_indices, k_cache, v_cache):
    """Scatter rotated K and raw V into their cache slots, in place."""
    require().kv_append(k_rot, v, positions, request_indices, k_cache, v_cache)


def separate_rope_kv_append(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices):
    """RoPE kernel then append kernel, with `k_rot` materialised between them: two launches and
    one intermediate, the ablation the fused op is measured against."""
    # One binding call: rope_forward into a fresh k_rot, then the append. A token past the
    # cos/sin table gets no k_rot row from the rope step (a status bit instead), so the append
    # is told the table length and leaves that K slot untouched, as the fused op does; its V
    # slot is still written.
    return require().separate_rope_kv_append(q, k, v, positions, cos, sin, k_cache, v_cache,
                                             request_indices)


def fused_rope_kv_append(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices):
    """One launch: rotate Q into a fresh q_rot, rotate K straight into its cache slot, copy V."""
    return require().fused_rope_kv_append(q, k, v, positions, cos, sin, k_cache, v_cache,
                                          request_indices)


# ---- extensions beyond the reference's surface ----

def fused_rope_kv_append_ex(q, k, v, positions, cos, sin, k_cache, v_cache, request_indices,
                            *, rotary_dim=0, pdl=False, strided_cache=False, inv_freq=None,
                            q_out=None, path="auto", row_splits=0, rows_per_thread=0,
                            staged_stages=0):
    """fused_rope_kv_append with:
    rotary_dim     rotate only the first rotary_dim dims (table [P, rotary_dim]), copy the rest;
    pdl            programmatic dependent launch (indices, block table and table rows read
                   before waiting on the preceding kernel -- the caller guarantees that kernel
                   does not write them);
    strided_cache  caches of any strides with a contiguous last dim, e.g. a head-major
                   [B, Hkv, S, D] cache passed as cache.transpose(1, 2);
    inv_freq       fp32 [rotary_dim/2] device tensor: cos/sin from sincosf in registers
                   (not bit-exact: within the reference's tolerance, almost always 1 ulp);
    q_out          write into this contiguous [T, Hq, D] tensor instead of a fresh one;
    path           "auto" (default), "register" (the register kernel) or "staged" (the
                   bulk-copy kernel that stages tokens through shared memory; refused with a
                   RuntimeError when the layout does not allow it). "auto" takes the staged
                   kernel for large token counts when it can;
    row_splits     register kernel: CTAs that share one token's head rows (0 = chosen by the
                   library from the token count);
    rows_per_thread register kernel: head rows a thread holds, 1 or 3 (0 = chosen);
    staged_stages  bulk-copy kernel: tokens a CTA stages at once, 2..8 (0 = chosen)."""
    return require().fused_rope_kv_append_ex(q, k, v, positions, cos, sin, k_cache, v_cache,
                                             request_indices, rotary_dim, pdl, strided_cache,
                                             inv_freq, q_out, path, row_splits, rows_per_thread,
                                             staged_stages)


def paged_rope_kv_append(q, k, v, positions, cos, sin, k_pages, v_pages, block_table,
                         request_indices, *, rotary_dim=0, pdl=False, path="auto"):
    """Fused RoPE + append into a paged cache: k_pages/v_pages [num_blocks, block_size, Hkv, D],
    block_table [num_requests, max_blocks] (positions' dtype). Token t goes to block
    block_table[ri[t], pos[t] // block_size], row pos[t] % block_size. Returns q_rot."""
    return require().paged_rope_kv_append(q, k, v, positions, cos, sin, k_pages, v_pages,
                                          block_table, request_indices, rotary_dim, pdl, path)


def rope_forward_ex(q, k, positions, cos, sin, *, rotary_dim=0, pdl=False):
    return require().rope_forward_ex(q, k, positions, cos, sin, rotary_dim, pdl)


def kv_append_ex(k_rot, v, positions, request_indices, k_cache, v_cache, *, pdl=False,
                 strided_cache=False, k_position_limit=0):
    """kv_append with PDL, strided caches, and k_position_limit: when > 0, the K row of a token
    whose position is >= it is not written (its V row still is) -- pass the cos/sin table's row
    count when k_rot came from rope_forward, which leaves such rows unwritten."""
    require().kv_append_ex(k_rot, v, positions, request_indices, k_cache, v_cache, pdl,
                           strided_cache, k_position_limit)


def advance_positions(positions, delta=1, *, pdl=False):
    """positions += delta on the device, in place: the step of a captured decode loop, so the
    graph replays without a host-side position copy. With pdl=True it may launch while the
    previous kernel drains and still writes only after that kernel has finished."""
    require().advance_positions(positions, delta, pdl)


def fused_rope_kv_append_attention(q, k, v, positions, cos, sin, k_cache, v_cache,
                                   request_indices, *, scale=None, q_out=None, attn_out=None,
                                   chunk=0, heads_per_cta=0, rotary_dim=0, pdl=False,
                                   strided_cache=False, workspace=None, path="auto",
                                   workspace_zeroed=False):
    """The fused append followed by the decode attention that reads the cache, one launch.

    Appends exactly as fused_rope_kv_append (K slot = RoPE(k), V slot = v), then returns
    attn_out [T, Hq, D] (q's dtype): for each token t and query head h, softmax over cache
    positions 0..pos[t] of request ri[t] of scale * q_rot . K, applied to V, with KV head
    h // (Hq // Hkv) (grouped-query attention). scale defaults to 1/sqrt(head_dim). Each request
    appears at most once per call. q_out, when given, also receives q_rot. chunk and
    heads_per_cta tune the grid (0 = chosen by the library); workspace, when given, is a
    contiguous uint8 device tensor of at least attention_workspace_bytes(...) bytes (same
    tuning and path). path: "auto" (tensor cores for fp16/bf16 with head_dim 64 or 128, CUDA
    cores otherwise), "tensor_cores" or "cuda_cores". workspace_zeroed=True says the given
    workspace's counters are zero, which every call leaves them (unless a bounded wait ran
    out), so a workspace zeroed once can be passed call after call without the per-call
    zeroing."""
    return require().fused_rope_kv_append_attention(
        q, k, v, positions, cos, sin, k_cache, v_cache, request_indices,
        0.0 if scale is None else float(scale), q_out, attn_out, chunk, heads_per_cta,
        rotary_dim, pdl, strided_cache, workspace, path, workspace_zeroed)


def paged_rope_kv_append_attention(q, k, v, positions, cos, sin, k_pages, v_pages, block_table,
                                   request_indices, *, scale=None, q_out=None, attn_out=None,
                                   chunk=0, rotary_dim=0, pdl=False, workspace=None,
                                   workspace_zeroed=False):
    """fused_rope_kv_append_attention over a paged cache: k_pages/v_pages
    [num_blocks, block_size, Hkv, D], block_table [num_requests, max_blocks] (positions' dtype);
    position p of request r lives in block block_table[r, p // block_size], row
    p % block_size. fp16/bf16 with head_dim 64 or 128; block_size a multiple of 8 dividing 128,
    or a multiple of 128. A workspace, when given, holds at least attention_workspace_bytes(...,
    cache_alloc_len=max_blocks * block_size, path="tensor_cores") bytes."""
    return require().paged_rope_kv_append_attention(
        q, k, v, positions, cos, sin, k_pages, v_pages, block_table, request_indices,
        0.0 if scale is None else float(scale), q_out, attn_out, chunk, rotary_dim, pdl,
        workspace, workspace_zeroed)


def attention_workspace_bytes(num_tokens, num_q_heads, num_kv_heads, head_dim, cache_alloc_len,
                              dtype, *, chunk=0, heads_per_cta=0, device=0, path="auto"):
    """Workspace bytes fused_rope_kv_append_attention needs for this shape and tuning."""
    return require().attention_workspace_bytes(num_tokens, num_q_heads, num_kv_heads, head_dim,
                                               cache_alloc_len, dtype, chunk, heads_per_cta,
                                               device, path)


__all__ = ["advance_positions", "attention_workspace_bytes", "fused_rope_kv_append",
           "fused_rope_kv_append_attention", "fused_rope_kv_append_ex", "kv_append",
           "kv_append_ex", "paged_rope_kv_append", "paged_rope_kv_append_attention",
           "rope_forward", "rope_forward_ex",
           "separate_rope_kv_append"]
