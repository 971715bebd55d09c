"""GPU parity of the CUDA path against the CPU oracle (oracle/imi_oracle.cpp),
through the C ABI (adaptiveimi_b200.ops -> libimi_b200.so).

Bar: bit-exact for the index build (labels, centroids, CSR, list rows), the
cell scores and the selected cell lists; attention within max-abs 2e-2 and
mean-abs 2e-3 of a float64 softmax (the north-star bf16 tolerance).
"""
import ast
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from adaptiveimi_b200 import ops
from adaptiveimi_b200.sizing import RetrievalSizes
from adaptiveimi_b200.synthetic import make_layer
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
ATOL_MAX, ATOL_MEAN = 2e-2, 2e-3


def _build_cfg0(heads=8, ctx=8192, G=4, seed=0, parts=2, ks=(16, 16), iters=10, comps=64, theta=500000.0):
    K, V, Q = make_layer(heads, heads * G, ctx, 128, comps, seed, theta, n_queries=16)
    k = K[:, 32:ctx - 64].contiguous()
    v = V[:, 32:ctx - 64].contiguous()
    return K, V, Q, k, v


def _gpu_build(k, v, parts, ks, iters, n_slots, tol=0.0, min_iter=None, rel_tol=0.0):
    kd, vd = k.cuda(), v.cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    idx = ops.build_index(kd, vd, parts=parts, ks=ks, n_slots=n_slots, max_iters=iters, tol=tol,
                          early_stop_min_iter=iters if min_iter is None else min_iter, early_stop_rel_tol=rel_tol,
                          status=status)
    torch.cuda.synchronize()
    assert int(status) == 0  # no wait of the tensor-core E-step gave up
    return idx


def _check_build_against_oracle(k, v, idx, parts, ks, iters, tol=0.0, min_iter=None, rel_tol=0.0):
    kb, vb = O.bf16_bits(k), O.bf16_bits(v)
    S = 1 if parts == 0 else parts
    na_gpu = idx.n_active.cpu().numpy()
    for h in range(k.shape[0]):
        o = O.build_head(kb[h], vb[h], parts, ks, iters, tol, iters if min_iter is None else min_iter, rel_tol)
        na = o["n_active"]
        assert na == na_gpu[h], f"head {h}: n_active {na_gpu[h]} != {na}"
        for s in range(S):
            np.testing.assert_array_equal(idx.sub_labels[h, s].cpu().numpy(), o["sub_labels"][s], err_msg=f"h{h} s{s}")
            np.testing.assert_array_equal(idx.sub_centroids[h, s, :ks[s]].cpu().numpy(), o["sub_centroids"][s])
        np.testing.assert_array_equal(idx.cell_offsets[h, :na + 1].cpu().numpy(), o["offsets"])
        np.testing.assert_array_equal(idx.cell_sizes[h, :na].cpu().numpy(), np.diff(o["offsets"]))
        assert int(idx.cell_sizes[h, na:].abs().sum()) == 0
        assert bool(idx.cell_mask[h, na:].all()) and not bool(idx.cell_mask[h, :na].any())
        np.testing.assert_array_equal(idx.centroids[h, :na].cpu().numpy(), o["merged"])
        np.testing.assert_array_equal(O.bf16_bits(idx.list_keys[h]), o["list_keys"])
        np.testing.assert_array_equal(O.bf16_bits(idx.list_values[h]), o["list_values"])


def test_build_cfg0_bit_exact():
    _, _, _, k, v = _build_cfg0()
    idx = _gpu_build(k, v, 2, (16, 16), 10, n_slots=1025)
    _check_build_against_oracle(k, v, idx, 2, (16, 16), 10)


@pytest.mark.parametrize("fixture", sorted(p.name for p in GOLD.glob("build_*.npz")))
def test_build_matches_reference_golden(fixture):
    """The device build against the reference's own outputs (golden fixtures)."""
    from tests.test_oracle_pin import _inputs
    z = np.load(GOLD / fixture)
    meta = ast.literal_eval(str(z["meta"]))
    k, v = _inputs(meta)
    parts, ks = meta["parts"], meta["ks"]
    S = 1 if parts == 0 else parts
    n_slots = int(np.prod(ks)) + 1
    idx = _gpu_build(k, v, parts, ks, meta["max_iters"], n_slots, meta["tol"], meta["min_iter"], meta["rel_tol"])
    for h in range(k.shape[0]):
        na = int(z["cluster_counts"][h])
        assert int(idx.n_active[h]) == na
        for s in range(S):
            np.testing.assert_array_equal(idx.sub_labels[h, s].cpu().numpy(), z[f"labels{s + 1}"][h])
            np.testing.assert_array_equal(idx.sub_centroids[h, s, :ks[s]].cpu().numpy(), z[f"centroids{s + 1}"][h])
        np.testing.assert_array_equal(idx.cell_offsets[h, :na + 1].cpu().numpy(), z["cluster_offsets"][h][:na + 1])
        np.testing.assert_array_equal(idx.centroids[h, :na].cpu().numpy(), z["centroids"][h][:na])


def test_build_imi4_and_ivf_against_oracle():
    K, V, _ = make_layer(2, 8, 2600, 128, 48, 3, 1e6, n_queries=1)
    k, v = K[:, :2500].contiguous(), V[:, :2500].contiguous()
    for parts, ks, it in ((4, (3, 4, 5, 2), 6), (0, (70,), 4), (2, (40, 33), 7)):
        n_slots = int(np.prod(ks)) + 1
        idx = _gpu_build(k, v, parts, ks, it, n_slots, 5e-4, 2, 5e-4)
        _check_build_against_oracle(k, v, idx, parts, ks, it, 5e-4, 2, 5e-4)


def test_build_odd_token_count_against_oracle():
    """An odd token count: per-task arrays then start off 16-byte boundaries
    (the early-stop inertia sum reads them with vector loads)."""
    K, V, _ = make_layer(3, 12, 2800, 128, 40, 11, 500000.0, n_queries=1)
    k, v = K[:, :2699].contiguous(), V[:, :2699].contiguous()
    for parts, ks, it, mi in ((2, (24, 21), 8, 2), (4, (3, 4, 3, 2), 5, 5)):
        n_slots = int(np.prod(ks)) + 1
        idx = _gpu_build(k, v, parts, ks, it, n_slots, 5e-4, mi, 5e-4)
        _check_build_against_oracle(k, v, idx, parts, ks, it, 5e-4, mi, 5e-4)


def test_build_strided_model_layout():
    """Keys taken straight from a [T, H, D] prefill tensor (no transpose copy)."""
    K, V, _ = make_layer(4, 16, 3000, 128, 32, 9, 500000.0)
    kt = K.transpose(0, 1).contiguous().cuda()  # [T, H, D]
    vt = V.transpose(0, 1).contiguous().cuda()
    kview = kt[100:2900].transpose(0, 1)        # [H, n, D] strided view
    vview = vt[100:2900].transpose(0, 1)
    idx = ops.build_index(kview, vview, parts=2, ks=(20, 20), n_slots=401, max_iters=5, early_stop_min_iter=5,
                          tol=0.0, early_stop_rel_tol=0.0)
    torch.cuda.synchronize()
    _check_build_against_oracle(K[:, 100:2900].contiguous(), V[:, 100:2900].contiguous(), idx, 2, (20, 20), 5)


def test_similarity_kernel_bit_exact():
    torch.manual_seed(1)
    q = torch.randn(8, 4, 128).to(torch.bfloat16)
    c = torch.randn(8, 1000, 128)
    got = ops.fused_query_group_similarities(q.cuda(), c.cuda()).cpu().numpy()
    qb = O.bf16_bits(q)
    for h in range(8):
        np.testing.assert_array_equal(got[h], O.scores(qb[h], c[h].numpy()))


def _decode_setup(heads=8, G=4, ctx=8192, parts=2, ks=(16, 16), iters=10, budget=0.1, n_slots=None):
    K, V, Q, k, v = _build_cfg0(heads, ctx, G, parts=parts, ks=ks, iters=iters)
    n = k.shape[1]
    sizes = RetrievalSizes.from_capacity(n, parts, budget, 32, static_capacity=96 + 16)
    ns = n_slots or sizes.n_centroids
    idx = _gpu_build(k, v, parts, ks, iters, ns)
    return K, V, Q, k, v, sizes, idx


def _select(idx, q, sizes, static_len, exec_cap, scores=True, slot_bound=0):
    bg = q.shape[0]
    dev = q.device
    sel = torch.full((bg, sizes.nprobe), -1, dtype=torch.int32, device=dev)
    cnt = torch.zeros(bg, dtype=torch.int32, device=dev)
    kept = torch.zeros(bg, dtype=torch.int32, device=dev)
    rows = torch.full((bg, exec_cap), -7, dtype=torch.int32, device=dev)
    rc = torch.zeros(bg, dtype=torch.int32, device=dev)
    sc = torch.zeros((bg, idx.n_slots), dtype=torch.float32, device=dev) if scores else None
    ops.select_cells(q=q, index=idx, nprobe=sizes.nprobe, max_tokens=sizes.max_retrieval_tokens,
                     buffer_pages=sizes.buffer_size, page_size=8, padding_id=idx.n_slots - 1, static_len=static_len,
                     exec_capacity=exec_cap, sel_cells=sel, sel_count=cnt, row_index=rows, row_count=rc,
                     kept_count=kept, scores_out=sc, slot_bound=slot_bound)
    torch.cuda.synchronize()
    return sel, cnt, rows, rc, sc, kept


@pytest.mark.parametrize("bounded", [False, True])
def test_select_matches_oracle_cfg0(bounded):
    """bounded: the selection only visits slots below the largest n_active
    (everything above is padding); the results must not change."""
    K, V, Q, k, v, sizes, idx = _decode_setup()
    bound = int(idx.n_active.max()) if bounded else 0
    heads, G = 8, 4
    static_len = 97
    exec_cap = sizes.buffer_size * 8 + 96 + 16
    cents = idx.centroids.cpu().numpy()
    mask = idx.cell_mask.cpu().numpy()
    csz = idx.cell_sizes.cpu().numpy()
    offs = idx.cell_offsets.cpu().numpy()
    for t in range(16):
        q = Q[t].reshape(heads, G, 128).contiguous()
        sel, cnt, rows, rc, sc, kept = _select(idx, q.cuda(), sizes, static_len, exec_cap, slot_bound=bound)
        qb = O.bf16_bits(q)
        for h in range(heads):
            ref_sc = O.scores(qb[h], cents[h], mask[h])
            np.testing.assert_array_equal(sc[h].cpu().numpy(), ref_sc)
            ref_sel, pre = O.select(ref_sc, csz[h], sizes.nprobe, sizes.max_retrieval_tokens, sizes.buffer_size, 8,
                                    idx.n_slots - 1)
            n_sel = int(cnt[h])
            # selected cells come out in slot order (attention is order-free)
            np.testing.assert_array_equal(sel[h, :n_sel].cpu().numpy(), np.sort(ref_sel))
            assert int(kept[h]) == int((pre != idx.n_slots - 1).sum())
            # row list: static rows, then each selected cell's CSR rows, cells in slot order
            exp = [(1 << 30) | r for r in range(static_len)]
            for c in np.sort(ref_sel):
                exp.extend(range(offs[h, c], offs[h, c] + csz[h, c]))
            assert int(rc[h]) == len(exp)
            np.testing.assert_array_equal(rows[h, :len(exp)].cpu().numpy(), np.array(exp, dtype=np.int64).astype(np.int32))


def test_select_repeatable_under_reruns():
    """The same query, selected many times in both modes, gives the oracle's
    counts every time (a cross-CTA race would show up as a rare mismatch)."""
    K, V, Q, k, v, sizes, idx = _decode_setup()
    heads, G = 8, 4
    exec_cap = sizes.buffer_size * 8 + 96 + 16
    cents, mask, csz = idx.centroids.cpu().numpy(), idx.cell_mask.cpu().numpy(), idx.cell_sizes.cpu().numpy()
    bound = int(idx.n_active.max())
    for t in range(16):
        qb = O.bf16_bits(Q[t].reshape(heads, G, 128))
        exp = []
        for h in range(heads):
            ref_sel, pre = O.select(O.scores(qb[h], cents[h], mask[h]), csz[h], sizes.nprobe,
                                    sizes.max_retrieval_tokens, sizes.buffer_size, 8, idx.n_slots - 1)
            exp.append((len(ref_sel), int((pre != idx.n_slots - 1).sum())))
        qd = Q[t].reshape(heads, G, 128).contiguous().cuda()
        for rep in range(6):
            for bnd in (0, bound):
                _, cnt, _, _, _, kept = _select(idx, qd, sizes, 97, exec_cap, scores=False, slot_bound=bnd)
                got = list(zip(cnt.tolist(), kept.tolist()))
                assert got == exp, (t, rep, bnd)


def _zone(K, V, heads, static_len, cap):
    ctx = K.shape[1]
    zk = torch.zeros(heads, cap, 128, dtype=torch.bfloat16)
    zv = torch.zeros_like(zk)
    zk[:, :32] = K[:, :32]
    zk[:, 32:96] = K[:, ctx - 64:]
    zv[:, :32] = V[:, :32]
    zv[:, 32:96] = V[:, ctx - 64:]
    g = torch.Generator().manual_seed(123)
    extra = static_len - 96
    if extra > 0:
        zk[:, 96:static_len] = torch.randn(heads, extra, 128, generator=g).to(torch.bfloat16)
        zv[:, 96:static_len] = torch.randn(heads, extra, 128, generator=g).to(torch.bfloat16)
    return zk, zv


@pytest.mark.parametrize("splits,fused", [(1, False), (7, True), (37, False), (37, True)])
def test_attention_matches_oracle(splits, fused):
    K, V, Q, k, v, sizes, idx = _decode_setup()
    heads, G = 8, 4
    static_len = 97
    cap = 96 + 16
    exec_cap = sizes.buffer_size * 8 + cap
    zk, zv = _zone(K, V, heads, static_len, cap)
    zkd, zvd = zk.cuda(), zv.cuda()
    lk, lv = idx.list_keys.cpu(), idx.list_values.cpu()
    for t in (0, 5, 11):
        q = Q[t].reshape(heads, G, 128).contiguous()
        qd = q.cuda()
        sel, cnt, rows, rc, _, _ = _select(idx, qd, sizes, static_len, exec_cap, scores=False)
        out = torch.empty(heads, G, 128, dtype=torch.bfloat16, device="cuda")
        part_o = torch.empty(heads, splits, G, 128, device="cuda")
        part_ml = torch.empty(heads, splits, G, 2, device="cuda")
        counters = torch.zeros(heads, dtype=torch.int32, device="cuda") if fused else None
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        ops.sparse_attention(q=qd, row_index=rows, row_count=rc, list_keys=idx.list_keys,
                             list_values=idx.list_values, static_keys=zkd, static_values=zvd, out=out,
                             part_o=part_o, part_ml=part_ml, splits=splits, counters=counters, status=status)
        assert int(status) == 0  # no wait for a row copy gave up
        if fused:
            assert int(counters.abs().sum()) == 0  # the merging CTA re-zeroed the counters
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        rows_c = rows.cpu().numpy()
        for h in range(heads):
            r = rows_c[h, :int(rc[h])]
            src = r >> 30
            ri = r & ((1 << 30) - 1)
            kr = torch.where(torch.from_numpy(src == 1)[:, None], zk[h][torch.from_numpy(np.minimum(ri, cap - 1))],
                             lk[h][torch.from_numpy(np.minimum(ri, lk.shape[1] - 1))])
            vr = torch.where(torch.from_numpy(src == 1)[:, None], zv[h][torch.from_numpy(np.minimum(ri, cap - 1))],
                             lv[h][torch.from_numpy(np.minimum(ri, lv.shape[1] - 1))])
            ref = O.attention(O.bf16_bits(q[h]), O.bf16_bits(kr), O.bf16_bits(vr), 1.0 / math.sqrt(128))
            err = np.abs(got[h] - ref)
            assert err.max() <= ATOL_MAX, (h, err.max())
            assert err.mean() <= ATOL_MEAN, (h, err.mean())


def test_attention_dense_equivalence_full_budget():
    """budget 1.0 and a page buffer large enough that the reference's page
    truncation (ceil(size/8) pages per cell against buffer_size) drops nothing:
    every token is attended, so the result equals dense softmax attention."""
    K, V, Q, k, v = _build_cfg0(heads=2, ctx=2048)
    heads, G = 2, 4
    n = k.shape[1]
    sizes = RetrievalSizes.from_capacity(n, 2, 1.0, 4096, static_capacity=96 + 1)
    idx = _gpu_build(k, v, 2, (16, 16), 4, sizes.n_centroids)
    static_len = 96
    zk, zv = _zone(K, V, heads, static_len, 97)
    exec_cap = sizes.execution_stride
    q = Q[0].reshape(heads, G, 128).contiguous()
    qd = q.cuda()
    sel, cnt, rows, rc, _, _ = _select(idx, qd, sizes, static_len, exec_cap, scores=False)
    assert int(rc[0]) == K.shape[1] and int(rc[1]) == K.shape[1]
    out = torch.empty(heads, G, 128, dtype=torch.bfloat16, device="cuda")
    splits = 16
    ops.sparse_attention(q=qd, row_index=rows, row_count=rc, list_keys=idx.list_keys, list_values=idx.list_values,
                         static_keys=zk.cuda(), static_values=zv.cuda(), out=out,
                         part_o=torch.empty(heads, splits, G, 128, device="cuda"),
                         part_ml=torch.empty(heads, splits, G, 2, device="cuda"), splits=splits)
    torch.cuda.synchronize()
    for h in range(heads):
        ref = O.attention(O.bf16_bits(q[h]), O.bf16_bits(K[h]), O.bf16_bits(V[h]), 1.0 / math.sqrt(128))
        err = np.abs(out[h].float().cpu().numpy() - ref)
        assert err.max() <= ATOL_MAX and err.mean() <= ATOL_MEAN
