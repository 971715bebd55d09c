"""Host logic of the multi-GPU decode path on CPU: KV-head shards and the
max-over-ranks timing reduction, run as two gloo ranks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from adaptiveimi_b200.sharding import max_over_ranks, shard_kv_heads


def test_shards_cover_every_head_once():
    for kv, ws in ((8, 1), (8, 2), (8, 4), (8, 8), (32, 8)):
        heads = []
        for r in range(ws):
            h0, n = shard_kv_heads(kv, ws, r)
            heads.extend(range(h0, h0 + n))
        assert heads == list(range(kv))


def test_uneven_shards_are_rejected():
    with pytest.raises(ValueError):
        shard_kv_heads(8, 3, 0)
    with pytest.raises(ValueError):
        shard_kv_heads(8, 2, 2)


def test_max_over_ranks_without_a_group_is_identity():
    assert max_over_ranks([1.5, 2.0], torch.device("cpu")) == [1.5, 2.0]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, ws, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        h0, n = shard_kv_heads(8, ws, rank)
        # rank r "took" 10 + r ms and built its shard in 100 - r ms
        got = max_over_ranks([10.0 + rank, 100.0 - rank, float(h0)], torch.device("cpu"))
        out.put((rank, h0, n, got))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_reduce():
    ws, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(ws))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [(r, h0, n) for r, h0, n, _ in res] == [(0, 0, 4), (1, 4, 4)]
    for _, _, _, got in res:
        assert got == [11.0, 100.0, 4.0]  # the slowest rank, on every rank
