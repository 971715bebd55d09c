"""Sequence sharding across real GPUs: one shard per process, the candidate
records and the attention partials exchanged by NCCL all-gathers or by
imi_peer_allgather over NVLink peer memory.  Every rank
also runs all the shards in-process (no collective) and must get the same
output.  Needs at least two GPUs (skipped otherwise)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, ws, port, q, peer):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from adaptiveimi_b200 import seqshard
    from adaptiveimi_b200.synthetic import make_layer
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=ws, device_id=dev)
    try:
        heads, G, ctx = 4, 4, 8192
        K, V, Q = make_layer(heads, heads * G, ctx, 128, 64, 5, 500000.0, n_queries=3)
        mid_k, mid_v = K[:, 32:ctx - 64], V[:, 32:ctx - 64]
        plan = seqshard.plan_shards(mid_k.shape[1], ws, 2, 0.1, 32)
        zk = torch.cat([K[:, :32], K[:, ctx - 64:]], 1).contiguous().to(dev)
        zv = torch.cat([V[:, :32], V[:, ctx - 64:]], 1).contiguous().to(dev)
        shards = []
        for r in range(ws):
            s = seqshard.SeqShard(plan, r, heads, G, 96, dev)
            a, b = plan.starts[r], plan.starts[r] + plan.lengths[r]
            s.build(mid_k[:, a:b].contiguous().to(dev), mid_v[:, a:b].contiguous().to(dev), max_iters=6,
                    early_stop_min_iter=6, tol=0.0, early_stop_rel_tol=0.0)
            shards.append(s)
        if peer:
            assert shards[rank].enable_peer_exchange()
        worst = 0.0
        for t in range(Q.shape[0]):
            qd = Q[t].reshape(heads, G, 128).contiguous().to(dev)
            got = seqshard.decode_step([shards[rank]], qd, zk, zv, 96)
            ref = seqshard.decode_step(shards, qd, zk, zv, 96)
            torch.cuda.synchronize()
            worst = max(worst, float((got.float() - ref.float()).abs().max()))
        if peer:
            assert int(shards[rank]._peer["status"].item()) == 0
        q.put((rank, worst))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("peer", [False, True])
def test_two_ranks_match_in_process_shards(peer):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ws, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, q, peer)) for r in range(ws)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(ws))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, worst in res:
        assert worst <= 1e-2, (rank, worst)  # same rows, same kernels; only the combine grouping differs
