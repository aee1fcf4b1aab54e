"""The sharded multi-GPU path on real GPUs: two processes, one per GPU, each runs its shard of
a batch-split and a KV-head-split workload through the fused kernel; NCCL gathers the results
and rank 0 compares them bit for bit with the CPU oracle on the unsharded problem. Needs at
least two GPUs (skipped otherwise); the same sharding logic is covered on CPU by
tests/test_shard_cpu.py."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    import datetime

    import torch.distributed as dist

    from decode_llm_kernel_b200.cuda import ops
    from decode_llm_kernel_b200.harness import positions as pos
    from decode_llm_kernel_b200.harness import sharding
    from decode_llm_kernel_b200.harness.inputs import SENTINEL, case, make_inputs
    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ok = True
    try:
        for kind, cfg in (("batch", case("gqa", 32, 8, 128, 1024, 64, "fp16", pos.RAGGED,
                                           request_order="shuffled")),
                          ("kv_head", case("gqa70b", 64, 8, 128, 64, 64, "bf16", pos.RAGGED,
                                             theta=500000.0))):
            p = pos.build_position_sets(cfg.batch, cfg.cache_alloc_len, pos.RAGGED, 1234,
                                        1, "cpu")[0]
            full = make_inputs(cfg, "cpu", 1234, p, cache_fill=SENTINEL)
            if kind == "batch":
                local, tokens = sharding.shard_batch(full, rank, world)
            else:
                local = sharding.shard_kv_heads(full, rank, world)
            dev = local._replace(**{f: getattr(local, f).cuda() for f in local._fields})
            q = ops.fused_rope_kv_append(*dev)
            torch.cuda.synchronize()
            if kind == "batch":
                q_all, k_all, v_all = sharding.gather_batch_shards(
                    q, tokens.cuda(), dev.k_cache, dev.v_cache, cfg.batch)
            else:
                q_all, k_all, v_all = sharding.gather_kv_head_shards(q, dev.k_cache, dev.v_cache)
            if rank == 0:
                ref = full._replace(k_cache=full.k_cache.clone(), v_cache=full.v_cache.clone())
                q_ref = oracle.fused_rope_kv_append(*ref)
                ok &= torch.equal(q_all.cpu().view(torch.int16), q_ref.view(torch.int16))
                ok &= torch.equal(k_all.cpu().view(torch.int16), ref.k_cache.view(torch.int16))
                ok &= torch.equal(v_all.cpu().view(torch.int16), ref.v_cache.view(torch.int16))
        if rank == 0:
            with open(result_path, "w") as f:
                f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_two_gpus_reassemble_the_unsharded_result(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    result = tmp_path / "result.txt"
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(result))) for r in range(2)]
    for proc in procs:
        proc.start()
    for proc in procs:
        proc.join(timeout=300)
        assert proc.exitcode == 0
    assert result.read_text() == "ok"
