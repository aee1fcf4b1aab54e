"""Per-GPU shards of one step's work, and the harness-side gather used to check them.

The op has no exchange step: a token's Q/K/V heads, its cache slot and its table row are all
the GPU needs. Two splits are used:

  kv_head  GPU r owns KV heads [r*Hkv/n, (r+1)*Hkv/n) with their cache slices, and the Q heads
           that attend to them, [r*Hq/n, (r+1)*Hq/n) (Hq/Hkv query heads per KV head).
  batch    GPU r owns requests [r*B/n, (r+1)*B/n): their cache rows and the tokens that write
           them, with request indices rebased to the local rows.

The gather (an all_gather over the process group) reassembles q_out and the written slots on
every rank so a single-device oracle can check them; it is never on the timed path.
"""
import torch


def head_range(total, rank, world):
    if total % world:
        raise ValueError(f"{total} heads do not split over {world} ranks")
    per = total // world
    return rank * per, (rank + 1) * per


def shard_kv_heads(args, rank, world):
    """A rank's view of OpArgs split by KV head: new contiguous tensors for its slice."""
    hq0, hq1 = head_range(args.q.shape[1], rank, world)
    hk0, hk1 = head_range(args.k.shape[1], rank, world)
    return args._replace(
        q=args.q[:, hq0:hq1].contiguous(), k=args.k[:, hk0:hk1].contiguous(),
        v=args.v[:, hk0:hk1].contiguous(),
        k_cache=args.k_cache[:, :, hk0:hk1].contiguous(),
        v_cache=args.v_cache[:, :, hk0:hk1].contiguous())


def owned_requests(batch, rank, world):
    if batch % world:
        raise ValueError(f"batch {batch} does not split over {world} ranks")
    per = batch // world
    return rank * per, (rank + 1) * per


def shard_batch(args, rank, world):
    """A rank's view of OpArgs split by request: its cache rows, the tokens that target them,
    request indices rebased to local rows. Returns (local_args, token_index)."""
    B = args.k_cache.shape[0]
    r0, r1 = owned_requests(B, rank, world)
    ri = args.request_indices.to(torch.int64)
    tokens = torch.nonzero((ri >= r0) & (ri < r1), as_tuple=False).flatten()
    local = args._replace(
        q=args.q[tokens].contiguous(), k=args.k[tokens].contiguous(),
        v=args.v[tokens].contiguous(), positions=args.positions[tokens].contiguous(),
        k_cache=args.k_cache[r0:r1].contiguous(), v_cache=args.v_cache[r0:r1].contiguous(),
        request_indices=(args.request_indices[tokens] - r0).contiguous())
    return local, tokens


def all_gather_cat(tensor, dim, group=None):
    """Concatenate every rank's tensor along dim (equal shapes on all ranks)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    parts = [torch.empty_like(tensor) for _ in range(world)]
    dist.all_gather(parts, tensor.contiguous(), group=group)
    return torch.cat(parts, dim=dim)


def gather_kv_head_shards(q_out, k_cache, v_cache, group=None):
    """Reassemble q_out [T, Hq, D] and the caches [B, S, Hkv, D] from KV-head shards."""
    return (all_gather_cat(q_out, 1, group), all_gather_cat(k_cache, 2, group),
            all_gather_cat(v_cache, 2, group))


def gather_batch_shards(q_out, tokens, k_cache, v_cache, num_tokens, group=None):
    """Reassemble q_out in global token order and the caches from batch shards. Every rank
    must own the same number of tokens (true for the identity and permuted mappings)."""
    q_all = all_gather_cat(q_out, 0, group)
    t_all = all_gather_cat(tokens, 0, group)
    out = torch.empty((num_tokens,) + tuple(q_out.shape[1:]), dtype=q_out.dtype,
                      device=q_out.device)
    out[t_all] = q_all
    return out, all_gather_cat(k_cache, 0, group), all_gather_cat(v_cache, 0, group)
