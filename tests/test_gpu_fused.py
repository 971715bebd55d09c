"""The fused decode launch (fused.cu: selection and attention of a layer as one
launch of 8-CTA clusters) against the select kernel + attention kernel pair and
the oracle, through the C ABI (imi_decode_attend with sel->fuse set).

Bar: the selected cells (as a set), the counts and the execution rows (as a
multiset; the fused launch lists cells in rank order, the pair in slot order)
are identical to the two-kernel path, which is bit-exact against the oracle;
the selected cells come out in descending score order (the oracle's rank
order); the attention output is within max-abs 2e-2 / mean-abs 2e-3 of an fp64
softmax over the same rows; repeated launches give identical results."""
import math

import numpy as np
import pytest
import torch

from adaptiveimi_b200 import ops
from adaptiveimi_b200.sizing import RetrievalSizes
from oracle import oracle as O

pytestmark = pytest.mark.gpu
ATOL_MAX, ATOL_MEAN = 2e-2, 2e-3


def _zone(K, V, static_len, cap):
    heads, ctx = K.shape[0], K.shape[1]
    zk = torch.zeros(heads, cap, 128, dtype=torch.bfloat16)
    zv = torch.zeros_like(zk)
    zk[:, :32], zk[:, 32:96] = K[:, :32], K[:, ctx - 64:]
    zv[:, :32], zv[:, 32:96] = V[:, :32], V[:, ctx - 64:]
    return zk, zv


def _run(idx, q, sizes, zk, zv, splits, static_len, fused, bound):
    bg, G, _ = q.shape
    dev = q.device
    cap = sizes.execution_stride
    outs = dict(sel=torch.full((bg, sizes.nprobe), -1, dtype=torch.int32, device=dev),
                cnt=torch.zeros(bg, dtype=torch.int32, device=dev), kept=torch.zeros(bg, dtype=torch.int32, device=dev),
                rows=torch.full((bg, cap), -7, dtype=torch.int32, device=dev),
                rc=torch.zeros(bg, dtype=torch.int32, device=dev),
                out=torch.empty(bg, G, 128, dtype=torch.bfloat16, device=dev))
    ops.decode_attend(q=q, index=idx, nprobe=sizes.nprobe, max_tokens=sizes.max_retrieval_tokens,
                      buffer_pages=sizes.buffer_size, page_size=8, padding_id=idx.n_slots - 1, static_len=static_len,
                      exec_capacity=cap, sel_cells=outs["sel"], sel_count=outs["cnt"], kept_count=outs["kept"],
                      row_index=outs["rows"], row_count=outs["rc"], static_keys=zk, static_values=zv, out=outs["out"],
                      part_o=torch.empty(bg, splits, G, 128, device=dev), part_ml=torch.empty(bg, splits, G, 2, device=dev),
                      counters=torch.zeros(bg, dtype=torch.int32, device=dev), splits=splits, slot_bound=bound,
                      fuse=fused)
    return outs


def _compare(idx, Q, K, V, sizes, splits, bound, queries, static_len=97):
    heads = K.shape[0]
    G = Q.shape[1] // heads
    zk, zv = _zone(K, V, static_len, sizes.static_capacity)
    zkd, zvd = zk.cuda(), zv.cuda()
    lk, lv = idx.list_keys.cpu(), idx.list_values.cpu()
    cents, mask, csz = idx.centroids.cpu().numpy(), idx.cell_mask.cpu().numpy(), idx.cell_sizes.cpu().numpy()
    for t in queries:
        q = Q[t].reshape(heads, G, 128).contiguous().cuda()
        ref = _run(idx, q, sizes, zkd, zvd, splits, static_len, False, bound)
        got = _run(idx, q, sizes, zkd, zvd, splits, static_len, True, bound)
        torch.cuda.synchronize()
        for key in ("cnt", "kept", "rc"):
            assert torch.equal(got[key], ref[key]), (t, key)
        qb = O.bf16_bits(q.cpu())
        for h in range(heads):
            n = int(ref["cnt"][h])
            gs = got["sel"][h, :n].cpu().numpy()
            np.testing.assert_array_equal(np.sort(gs), ref["sel"][h, :n].cpu().numpy(), err_msg=f"{t} {h}")
            # rank order: the oracle's selection walk order
            ref_sel, _ = O.select(O.scores(qb[h], cents[h], mask[h]), csz[h], sizes.nprobe, sizes.max_retrieval_tokens,
                                  sizes.buffer_size, 8, idx.n_slots - 1)
            np.testing.assert_array_equal(gs, np.asarray(ref_sel), err_msg=f"rank order {t} {h}")
            r = int(ref["rc"][h])
            np.testing.assert_array_equal(np.sort(got["rows"][h, :r].cpu().numpy()), np.sort(ref["rows"][h, :r].cpu().numpy()))
            rows = ref["rows"][h, :r].cpu().numpy()
            src, ri = rows >> 30, rows & ((1 << 30) - 1)
            kr = torch.where(torch.from_numpy(src == 1)[:, None], zk[h][torch.from_numpy(np.minimum(ri, zk.shape[1] - 1))],
                             lk[h][torch.from_numpy(np.minimum(ri, lk.shape[1] - 1))])
            vr = torch.where(torch.from_numpy(src == 1)[:, None], zv[h][torch.from_numpy(np.minimum(ri, zv.shape[1] - 1))],
                             lv[h][torch.from_numpy(np.minimum(ri, lv.shape[1] - 1))])
            oref = O.attention(O.bf16_bits(q[h].cpu()), O.bf16_bits(kr), O.bf16_bits(vr), 1.0 / math.sqrt(128))
            err = np.abs(got["out"][h].float().cpu().numpy() - oref)
            assert err.max() <= ATOL_MAX and err.mean() <= ATOL_MEAN, (t, h, float(err.max()))


@pytest.mark.parametrize("splits,bounded", [(16, True), (16, False), (8, True), (144, True)])
def test_fused_matches_two_kernel_path_cfg0(splits, bounded):
    from tests.test_gpu_kernels import _decode_setup

    K, V, Q, k, v, sizes, idx = _decode_setup()
    bound = int(idx.n_active.max()) if bounded else 0
    _compare(idx, Q, K, V, sizes, splits, bound, range(16))


def test_fused_matches_two_kernel_path_cfg1():
    """The benchmarked geometry: 8 101 slots, nprobe 810, 13 097-token budget."""
    from tests.test_gpu_parity_cfg1 import _build
    from tests.test_oracle_pin import cfg1_inputs

    c, K, V, Q, k, v = cfg1_inputs()
    n = k.shape[1]
    sizes = RetrievalSizes.from_capacity(n, 2, 0.1, 32, static_capacity=96 + 16)
    idx = _build(k, v, 2, tuple(c["ks"]), sizes.n_centroids, 6, 0.0, 6, 0.0)
    _compare(idx, Q, K, V, sizes, 72, int(idx.n_active.max()), range(8))


def test_fused_repeated_launches_are_identical():
    from tests.test_gpu_kernels import _decode_setup

    K, V, Q, k, v, sizes, idx = _decode_setup()
    heads, G = 8, 4
    zk, zv = _zone(K, V, 97, sizes.static_capacity)
    zkd, zvd = zk.cuda(), zv.cuda()
    splits = 16
    q = Q[3].reshape(heads, G, 128).contiguous().cuda()
    first = _run(idx, q, sizes, zkd, zvd, splits, 97, True, 0)
    for _ in range(20):
        again = _run(idx, q, sizes, zkd, zvd, splits, 97, True, 0)
    torch.cuda.synchronize()
    assert torch.equal(first["out"], again["out"]) and torch.equal(first["rows"], again["rows"])
