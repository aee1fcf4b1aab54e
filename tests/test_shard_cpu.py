"""Sharding and gather logic of the multi-GPU path, on CPU: world-size-2 gloo ranks each run
their shard through the CPU oracle (standing in for the GPU kernel), gather, and rank 0 checks
the result bit for bit against the unsharded oracle."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from decode_llm_kernel_b200.harness import positions as pos
from decode_llm_kernel_b200.harness.configs import WORKLOADS
from decode_llm_kernel_b200.harness.inputs import SENTINEL, case, make_inputs


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_workload_shards():
    w = WORKLOADS["llama3_70b_tp"]
    for n in (1, 2, 4, 8):
        s = w.shard_for(0, n)
        assert (s.num_q_heads, s.num_kv_heads) == (64 // n, 8 // n)
        assert s.num_q_heads // s.num_kv_heads == 8
        # each rank re-reads the replicated cos/sin rows: 256 tokens x (40960/n + 512) bytes
        assert s.bytes_per_call() == 256 * (40960 // n + 512)
    m = WORKLOADS["mistral_b4096"]
    assert [m.shard_for(r, 8).batch for r in range(8)] == [512] * 8
    with pytest.raises(ValueError):
        WORKLOADS["llama3_70b_tp"].shard_for(0, 3)
    d = WORKLOADS["llama3_8b_decode32"]
    assert d.shard_for(1, 4) is d      # weak scaling: each GPU runs its own 64-sequence step
    assert d.bytes_per_token() == 25088 and d.bytes_per_step() == 32 * 64 * 25088


def _cfg(mapping):
    return case("gqa", 16, 4, 64, 8, 32, "bf16", pos.RAGGED, request_order=mapping,
                  theta=500000.0)


def _worker(rank, world, port, kind, mapping, result_path):
    import torch.distributed as dist
    from decode_llm_kernel_b200.harness import sharding
    from oracle import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _cfg(mapping)
        p = pos.build_position_sets(8, 32, pos.RAGGED, 1234, 1, "cpu")[0]
        args = make_inputs(cfg, "cpu", 1234, p, cache_fill=SENTINEL)
        if kind == "kv_head":
            local = sharding.shard_kv_heads(args, rank, world)
            q = oracle.fused_rope_kv_append(*local)
            q_all, k_all, v_all = sharding.gather_kv_head_shards(q, local.k_cache, local.v_cache)
        else:
            local, tokens = sharding.shard_batch(args, rank, world)
            q = oracle.fused_rope_kv_append(*local)
            q_all, k_all, v_all = sharding.gather_batch_shards(q, tokens, local.k_cache,
                                                               local.v_cache, 8)
        if rank == 0:
            full = args._replace(k_cache=args.k_cache.clone(), v_cache=args.v_cache.clone())
            q_ref = oracle.fused_rope_kv_append(*full)
            ok = (torch.equal(q_all.view(torch.int16), q_ref.view(torch.int16))
                  and torch.equal(k_all.view(torch.int16), full.k_cache.view(torch.int16))
                  and torch.equal(v_all.view(torch.int16), full.v_cache.view(torch.int16)))
            with open(result_path, "w") as f:
                f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind,mapping", [("kv_head", "identity"), ("batch", "identity"),
                                          ("batch", "shuffled")])
def test_two_gloo_ranks_reassemble_the_unsharded_result(tmp_path, kind, mapping):
    result = tmp_path / "result.txt"
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, kind, mapping, str(result)))
             for r in range(2)]
    for proc in procs:
        proc.start()
    for proc in procs:
        proc.join(timeout=120)
        assert proc.exitcode == 0
    assert result.read_text() == "ok"
