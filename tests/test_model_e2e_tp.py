"""The tensor-parallel decoder that drives the cache end to end
(adaptiveimi_b200/model_e2e.py) on CPU: two gloo ranks hold slices of the
same random-init model and must generate the same greedy tokens as one rank
holding all of it (dense attention stands in for the IMI cache, which needs a
GPU; the end-to-end IMI run is bench.py --workload qwen72b_e2e)."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from adaptiveimi_b200.model_e2e import DecoderConfig, TPDecoder, generate

CFG = DecoderConfig(layers=2, hidden=64, q_heads=8, kv_heads=2, head_dim=16, intermediate=96, vocab=320)


def _run(ws, rank, port, out):
    if ws > 1:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        torch.manual_seed(0)
        m = TPDecoder(CFG, "cpu", seed=3, attention="dense")
        ids = torch.randint(0, CFG.vocab, (24,), generator=torch.Generator().manual_seed(5))
        r = generate(m, ids, 6)
        out.put((rank, r["tokens"]))
    finally:
        if ws > 1:
            dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_ranks_generate_what_one_rank_generates():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    _run(1, 0, 0, q)
    single = q.get(timeout=60)[1]
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(2, r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert len(single) == 6
    for _, toks in res:
        assert toks == single
