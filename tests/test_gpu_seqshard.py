"""Sequence sharding on one GPU (every shard in this process): the global
selection over the shards' candidates must equal the oracle's selection over
the union of the shards' cells, and the combined attention must match an fp64
softmax over every selected row plus the steady zone."""
import dataclasses
import math

import numpy as np
import pytest
import torch

from adaptiveimi_b200 import seqshard
from adaptiveimi_b200.synthetic import make_layer
from oracle import oracle as O

pytestmark = pytest.mark.gpu
ATOL_MAX, ATOL_MEAN = 2e-2, 2e-3


def _setup(shards, heads=4, G=4, ctx=8192, seed=5, nprobe=None):
    K, V, Q = make_layer(heads, heads * G, ctx, 128, 64, seed, 500000.0, n_queries=6)
    mid_k, mid_v = K[:, 32:ctx - 64], V[:, 32:ctx - 64]
    n = mid_k.shape[1]
    plan = seqshard.plan_shards(n, shards, 2, 0.1, 32)
    if nprobe is not None:  # a rank-bound selection: every token and page allowed
        plan = dataclasses.replace(plan, nprobe=nprobe, max_tokens=n, buffer_pages=n)
    zone_k = torch.cat([K[:, :32], K[:, ctx - 64:]], 1).contiguous()  # [heads, 96, 128]
    zone_v = torch.cat([V[:, :32], V[:, ctx - 64:]], 1).contiguous()
    local = []
    for r in range(shards):
        s = seqshard.SeqShard(plan, r, heads, G, 96, torch.device("cuda"))
        a, b = plan.starts[r], plan.starts[r] + plan.lengths[r]
        s.build(mid_k[:, a:b].contiguous().cuda(), mid_v[:, a:b].contiguous().cuda(), max_iters=6,
                early_stop_min_iter=6, tol=0.0, early_stop_rel_tol=0.0)
        local.append(s)
    torch.cuda.synchronize()
    return K, V, Q, plan, local, zone_k, zone_v


@pytest.mark.parametrize("shards,nprobe", [(1, None), (2, None), (3, None), (4, 2100), (10, None)])
def test_sharded_selection_and_attention_match_the_union(shards, nprobe):
    # (4, 2100): nprobe above 2048 and 4 * 2101 candidates (the cluster merge
    # refines its boundary bucket in shared memory); (10, None): more shards
    # than a cluster holds, so the one-CTA merge runs
    heads, G = 4, 4
    K, V, Q, plan, local, zone_k, zone_v = _setup(shards, nprobe=nprobe)
    if nprobe is not None:
        assert plan.shards * plan.cap > 8192
    zkd, zvd = zone_k.cuda(), zone_v.cuda()
    cents = [s.index.centroids.cpu().numpy() for s in local]
    masks = [s.index.cell_mask.cpu().numpy() for s in local]
    sizes = [s.index.cell_sizes.cpu().numpy() for s in local]
    lks = [s.index.list_keys.cpu() for s in local]
    lvs = [s.index.list_values.cpu() for s in local]
    offs = [s.index.cell_offsets.cpu().numpy() for s in local]
    for t in range(Q.shape[0]):
        q = Q[t].reshape(heads, G, 128).contiguous()
        out = seqshard.decode_step(local, q.cuda(), zkd, zvd, 96)
        torch.cuda.synchronize()
        qb = O.bf16_bits(q)
        for h in range(heads):
            sc = np.concatenate([O.scores(qb[h], cents[r][h], masks[r][h]) for r in range(shards)])
            sz = np.concatenate([sizes[r][h] for r in range(shards)])
            ref_sel, _ = O.select(sc, sz, plan.nprobe, plan.max_tokens, plan.buffer_pages, 8, sc.shape[0] - 1)
            ref_sel = np.sort(ref_sel)
            krows, vrows = [zone_k[h]], [zone_v[h]]
            for r, s in enumerate(local):
                lo, hi = plan.key_base[r], plan.key_base[r] + plan.n_slots[r]
                exp_r = ref_sel[(ref_sel >= lo) & (ref_sel < hi)] - lo
                cnt = int(s.sel_count[h])
                got_r = s.sel[h, :cnt].cpu().numpy()
                np.testing.assert_array_equal(got_r, exp_r, err_msg=f"t{t} h{h} shard {r}")
                for c in exp_r:
                    krows.append(lks[r][h, offs[r][h, c]:offs[r][h, c + 1]])
                    vrows.append(lvs[r][h, offs[r][h, c]:offs[r][h, c + 1]])
            kk, vv = torch.cat(krows), torch.cat(vrows)
            ref = O.attention(qb[h], O.bf16_bits(kk), O.bf16_bits(vv), 1.0 / math.sqrt(128))
            err = np.abs(out[h].float().cpu().numpy() - ref)
            assert err.max() <= ATOL_MAX and err.mean() <= ATOL_MEAN, (t, h, float(err.max()))


def test_plan_global_rules_and_key_bases():
    plan = seqshard.plan_shards(8096, 3, 2, 0.1, 32)
    assert sum(plan.lengths) == 8096 and plan.starts[0] == 0
    assert plan.key_base == (0, plan.n_slots[0], plan.n_slots[0] + plan.n_slots[1])
    assert plan.nprobe == 102 and plan.max_tokens == 809
