"""Sequence-sharded decode (adaptiveimi_b200/seqshard.py) across two gloo ranks
on CPU: the host logic of ``decode_step`` -- local selection under the global
rules, the all-gather of the candidate records, the merge, the all-gather of
the (o, m, l) partials and the log-sum-exp combine.

The device kernels (select, merge, attention, combine) are replaced by
restatements in numpy that follow their descriptors (include/imi_b200.h:
imi_select_desc.cand_out, imi_merge_desc, imi_attn_desc.o_part/ml_part,
imi_combine_desc); the kernels themselves are covered on one GPU by
tests/test_gpu_seqshard.py.  Checked on every rank: the gathered records are in
rank order, the merged selection over the records equals the oracle's
selection over the whole (unsharded) context, and the combined output equals
an fp64 softmax over the union of the shards' rows."""
import math
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

SHARDS, BG, G, D = 2, 2, 4, 128
SLOTS = (300, 260)         # per-shard slots (padding slot last)
NPROBE, MAX_TOK, PAGES, PAGE = 60, 700, 110, 8
STATIC = 12


def _key(score: np.float32, gid: int) -> np.uint64:
    u = np.float32(score).view(np.uint32)
    o = (~u) if (u & np.uint32(0x80000000)) else (u | np.uint32(0x80000000))
    return np.uint64((int(o) << 32) | (0xFFFFFFFF - gid))


def _walk(entries):
    """entries: (key, size) in descending key order -> the number selected
    (rank, token and page rules, the first violation stops the walk)."""
    tok = pg = 0
    for i, (_, sz) in enumerate(entries):
        p = (sz + PAGE - 1) // PAGE
        if i >= NPROBE or tok >= MAX_TOK or pg + p > PAGES:
            return i
        tok += sz
        pg += p
    return len(entries)


def _shard_data(rank):
    g = np.random.default_rng(100 + rank)
    n = SLOTS[rank]
    scores = g.standard_normal((BG, n)).astype(np.float32)
    sizes = g.integers(1, 30, (BG, n)).astype(np.int64)
    sizes[:, -1] = 0  # the padding slot
    sizes[:, ::37] = 0  # a few empty cells
    offs = np.concatenate([np.zeros((BG, 1), np.int64), np.cumsum(sizes, 1)], 1)
    rows = int(offs[:, -1].max())
    k = g.standard_normal((BG, rows, D)).astype(np.float32)
    v = g.standard_normal((BG, rows, D)).astype(np.float32)
    return scores, sizes, offs, k, v


def _attend(q, k_rows, v_rows):
    """Unnormalised partial: o [G, D], m (log2 units), l."""
    s = (q @ k_rows.T) / math.sqrt(D) / math.log(2.0)
    m = s.max(1) if s.shape[1] else np.full(G, -np.inf)
    w = np.exp2(s - m[:, None]) if s.shape[1] else np.zeros((G, 0))
    return w @ v_rows, m, w.sum(1)


def _worker(rank, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=SHARDS)
    try:
        from adaptiveimi_b200 import seqshard

        key_base = (0, SLOTS[0])
        plan = seqshard.ShardPlan(shards=SHARDS, n_total=2000, starts=(0, 1000), lengths=(1000, 1000),
                                  ks=((16, 16), (16, 16)), n_slots=SLOTS, key_base=key_base, parts=2, nprobe=NPROBE,
                                  max_tokens=MAX_TOK, buffer_pages=PAGES, page_size=PAGE)
        s = seqshard.SeqShard(plan, rank, BG, G, STATIC + 4, torch.device("cpu"))
        scores, sizes, offs, K, V = _shard_data(rank)
        gq = np.random.default_rng(7)
        q = gq.standard_normal((BG, G, D)).astype(np.float32)
        zk = gq.standard_normal((BG, STATIC + 4, D)).astype(np.float32)
        zv = gq.standard_normal((BG, STATIC + 4, D)).astype(np.float32)
        seen = {}

        def select_local(q_, cand_out=None):
            rec = np.zeros((BG, plan.record), np.uint64)
            for h in range(BG):
                cand = [(_key(scores[h, c], key_base[rank] + c), int(sizes[h, c]), c) for c in range(SLOTS[rank])
                        if sizes[h, c] > 0]
                cand.sort(key=lambda e: -int(e[0]))
                ns = _walk([(k, z) for k, z, _ in cand])
                sel = sorted(cand[:ns], key=lambda e: e[2])  # slot order
                for j, (k, z, _) in enumerate(sel):
                    rec[h, j], rec[h, plan.cap + j] = k, z
                cnt = ns
                if ns < len(cand):  # the stop marker
                    rec[h, ns], rec[h, plan.cap + ns] = cand[ns][0], cand[ns][1]
                    cnt += 1
                rec[h, 2 * plan.cap] = cnt
            s.cand.copy_(torch.from_numpy(rec.view(np.int64)))

        def merge(cand_all, static_len):
            allrec = cand_all.numpy().view(np.uint64)
            seen["records"] = allrec.copy()
            s._sel = []
            for h in range(BG):
                union = []
                for r in range(SHARDS):
                    rec = allrec[r, h]
                    for j in range(int(rec[2 * plan.cap])):
                        union.append((rec[j], int(rec[plan.cap + j])))
                union.sort(key=lambda e: -int(e[0]))
                ns = _walk(union)
                mine = sorted(0xFFFFFFFF - (int(k) & 0xFFFFFFFF) - key_base[rank] for k, _ in union[:ns]
                              if key_base[rank] <= 0xFFFFFFFF - (int(k) & 0xFFFFFFFF) < key_base[rank] + SLOTS[rank])
                s._sel.append(mine)
            s._static = static_len if rank == 0 else 0

        def attend(q_, zone_keys, zone_values, partials_out=None):
            blk = s.partials.numpy()
            o_all = blk[:BG * G * 128].reshape(BG, G, 128)
            ml = blk[BG * G * 128:BG * G * 130].reshape(BG, G, 2)
            for h in range(BG):
                rows = [np.arange(offs[h, c], offs[h, c] + sizes[h, c]) for c in s._sel[h]]
                ri = np.concatenate(rows) if rows else np.zeros(0, np.int64)
                kr, vr = K[h][ri], V[h][ri]
                if s._static:
                    kr = np.concatenate([zk[h, :s._static], kr])
                    vr = np.concatenate([zv[h, :s._static], vr])
                o, m, l = _attend(q[h], kr, vr)
                o_all[h], ml[h, :, 0], ml[h, :, 1] = o, m, l

        def combine(parts_all, shards, bg, g, out):
            p = parts_all.numpy()
            o = p[:, :bg * g * 128].reshape(shards, bg, g, 128).astype(np.float64)
            ml = p[:, bg * g * 128:bg * g * 130].reshape(shards, bg, g, 2).astype(np.float64)
            M = ml[..., 0].max(0)
            w = np.exp2(ml[..., 0] - M)
            res = (o * w[..., None]).sum(0) / (ml[..., 1] * w).sum(0)[..., None]
            seen["out"] = res
            out.copy_(torch.from_numpy(res).to(out.dtype))
            return out

        s.select_local, s.merge, s.attend = select_local, merge, attend
        seqshard.combine = combine
        seqshard.decode_step([s], torch.from_numpy(q).to(torch.bfloat16), None, None, STATIC)
        out.put((rank, seen["records"], s._sel, seen["out"]))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def test_two_gloo_ranks_exchange_merge_and_combine():
    from oracle import oracle as O

    port = _free_port()
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, port, qu)) for r in range(SHARDS)]
    for p in procs:
        p.start()
    res = sorted((qu.get(timeout=180) for _ in range(SHARDS)), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    recs = [r[1] for r in res]
    assert np.array_equal(recs[0], recs[1])  # every rank merged the same gathered records
    data = [_shard_data(r) for r in range(SHARDS)]
    gq = np.random.default_rng(7)
    q = gq.standard_normal((BG, G, D)).astype(np.float32)
    zk = gq.standard_normal((BG, STATIC + 4, D)).astype(np.float32)
    zv = gq.standard_normal((BG, STATIC + 4, D)).astype(np.float32)
    for h in range(BG):
        # the union of the shards' selections is the oracle's selection over the
        # concatenated context (global ids, ties to the lower id)
        sc = np.concatenate([data[0][0][h], data[1][0][h]])
        sz = np.concatenate([data[0][1][h], data[1][1][h]]).astype(np.int32)
        ref_sel, _ = O.select(sc, sz, NPROBE, MAX_TOK, PAGES, PAGE, len(sc) - 1)
        got = sorted(list(res[0][2][h]) + [SLOTS[0] + c for c in res[1][2][h]])
        assert got == sorted(int(c) for c in ref_sel), h
        # the combined output: an fp64 softmax over the union of rows
        rows_k, rows_v = [zk[h, :STATIC]], [zv[h, :STATIC]]
        for r in range(SHARDS):
            _, sizes, offs, K, V = data[r]
            for c in res[r][2][h]:
                rows_k.append(K[h][offs[h, c]:offs[h, c] + sizes[h, c]])
                rows_v.append(V[h][offs[h, c]:offs[h, c] + sizes[h, c]])
        kr, vr = np.concatenate(rows_k).astype(np.float64), np.concatenate(rows_v).astype(np.float64)
        s = q[h].astype(np.float64) @ kr.T / math.sqrt(D)
        w = np.exp(s - s.max(1, keepdims=True))
        ref = (w @ vr) / w.sum(1, keepdims=True)
        for r in range(SHARDS):
            assert np.abs(res[r][3][h] - ref).max() < 1e-4
