"""GPU parity at the benchmarked geometry and at the
S=4 / IVF decode geometries, through the C ABI, against the CPU oracle.

* Build: 2 KV heads x 130 976 middle tokens, k = 90 x 90 (96 TMEM columns, the
  multi-CTA tensor-core E-step), 20 Lloyd iterations with the Llama early-stop
  settings.  Labels, sub-centroids, CSR offsets, merged centroids and list rows
  are bit-exact against the oracle for both heads, and head 0 against the
  reference's own outputs (tests/golden/cfg1_build_digest.npz).
* Decode on that index: 8 101 slots, nprobe 810, a 13 097-token budget, 1 638
  pages; 16 queries.  Scores bit-exact, selected sets equal, row lists exact,
  attention within max-abs 2e-2 / mean-abs 2e-3 of an fp64 softmax.
* S=4 at the config-3 size (k = 10, 10 001 slots, budget 0.05) and IVF
  (subspace_parts 0) decode: the same selection and attention checks.
"""
import math

import numpy as np
import pytest
import torch

from adaptiveimi_b200 import ops
from adaptiveimi_b200.sizing import RetrievalSizes, adaptive_k
from adaptiveimi_b200.synthetic import make_layer
from oracle import oracle as O
from tests.test_oracle_pin import cfg1_inputs, check_cfg1_head0

pytestmark = pytest.mark.gpu
ATOL_MAX, ATOL_MEAN = 2e-2, 2e-3
G = 4  # query heads per KV group at the config-1 geometry


def _build(k, v, parts, ks, n_slots, iters, tol, min_iter, rel_tol):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    idx = ops.build_index(k.cuda(), v.cuda(), parts=parts, ks=ks, n_slots=n_slots, max_iters=iters, tol=tol,
                          early_stop_min_iter=min_iter, early_stop_rel_tol=rel_tol, status=status)
    torch.cuda.synchronize()
    assert int(status) == 0
    return idx


@pytest.fixture(scope="module")
def cfg1():
    c, K, V, Q, k, v = cfg1_inputs()
    n = k.shape[1]
    sizes = RetrievalSizes.from_capacity(n, 2, 0.1, 32, static_capacity=96 + 16)
    assert (sizes.n_centroids, sizes.nprobe, sizes.max_retrieval_tokens, sizes.buffer_size) == (8101, 810, 13097, 1638)
    ks = tuple(c["ks"])
    assert adaptive_k(n, 2) == ks
    idx = _build(k, v, 2, ks, sizes.n_centroids, c["max_iters"], c["tol"], c["min_iter"], c["rel_tol"])
    return c, K, V, Q, k, v, sizes, idx


def _check_build(k, v, idx, parts, ks, iters, tol, min_iter, rel_tol):
    kb, vb = O.bf16_bits(k), O.bf16_bits(v)
    S = 1 if parts == 0 else parts
    outs = []
    for h in range(k.shape[0]):
        o = O.build_head(kb[h], vb[h], parts, ks, iters, tol, min_iter, rel_tol)
        na = o["n_active"]
        assert int(idx.n_active[h]) == na, h
        for s in range(S):
            np.testing.assert_array_equal(idx.sub_labels[h, s].cpu().numpy(), o["sub_labels"][s], err_msg=f"h{h}s{s}")
            np.testing.assert_array_equal(idx.sub_centroids[h, s, :ks[s]].cpu().numpy(), o["sub_centroids"][s])
        np.testing.assert_array_equal(idx.cell_offsets[h, :na + 1].cpu().numpy(), o["offsets"])
        assert bool((idx.cell_offsets[h, na:] == o["offsets"][-1]).all())
        assert bool(idx.cell_mask[h, na:].all()) and not bool(idx.cell_mask[h, :na].any())
        np.testing.assert_array_equal(idx.centroids[h, :na].cpu().numpy(), o["merged"])
        np.testing.assert_array_equal(O.bf16_bits(idx.list_keys[h]), o["list_keys"])
        np.testing.assert_array_equal(O.bf16_bits(idx.list_values[h]), o["list_values"])
        outs.append(o)
    return outs


def test_build_cfg1_geometry_bit_exact(cfg1):
    c, K, V, Q, k, v, sizes, idx = cfg1
    assert idx.iters_run.cpu().tolist() == [[20, 20], [20, 20]]
    _check_build(k, v, idx, 2, tuple(c["ks"]), c["max_iters"], c["tol"], c["min_iter"], c["rel_tol"])
    # head 0 against the reference's own build of the same keys
    na = int(idx.n_active[0])
    check_cfg1_head0([idx.sub_labels[0, s].cpu().numpy() for s in range(2)],
                     [idx.sub_centroids[0, s, :90].cpu().numpy() for s in range(2)],
                     idx.cell_offsets[0, :na + 1].cpu().numpy(), idx.centroids[0, :na].cpu().numpy(),
                     O.bf16_bits(idx.list_keys[0]), O.bf16_bits(idx.list_values[0]), na)


def _zone(K, V, static_len, cap):
    heads, ctx = K.shape[0], K.shape[1]
    zk = torch.zeros(heads, cap, 128, dtype=torch.bfloat16)
    zv = torch.zeros_like(zk)
    zk[:, :32], zk[:, 32:96] = K[:, :32], K[:, ctx - 64:]
    zv[:, :32], zv[:, 32:96] = V[:, :32], V[:, ctx - 64:]
    g = torch.Generator().manual_seed(321)
    extra = static_len - 96
    if extra > 0:
        zk[:, 96:static_len] = torch.randn(heads, extra, 128, generator=g).to(torch.bfloat16)
        zv[:, 96:static_len] = torch.randn(heads, extra, 128, generator=g).to(torch.bfloat16)
    return zk, zv


def _decode_and_check(K, V, Q, idx, sizes, queries, static_len, splits, slot_bound=0):
    """Select + attend every query; compare with the oracle's scores, selection,
    row list and fp64 attention.  Returns the selected counts."""
    heads = K.shape[0]
    G = Q.shape[1] // heads
    cap = sizes.static_capacity
    exec_cap = sizes.execution_stride
    zk, zv = _zone(K, V, static_len, cap)
    zkd, zvd = zk.cuda(), zv.cuda()
    cents, mask = idx.centroids.cpu().numpy(), idx.cell_mask.cpu().numpy()
    csz, offs = idx.cell_sizes.cpu().numpy(), idx.cell_offsets.cpu().numpy()
    lk, lv = idx.list_keys.cpu(), idx.list_values.cpu()
    dev = "cuda"
    counts = []
    for t in queries:
        q = Q[t].reshape(heads, G, 128).contiguous()
        qd = q.cuda()
        sel = torch.full((heads, sizes.nprobe), -1, dtype=torch.int32, device=dev)
        cnt = torch.zeros(heads, dtype=torch.int32, device=dev)
        kept = torch.zeros(heads, dtype=torch.int32, device=dev)
        rows = torch.full((heads, exec_cap), -7, dtype=torch.int32, device=dev)
        rc = torch.zeros(heads, dtype=torch.int32, device=dev)
        sc = torch.zeros((heads, idx.n_slots), dtype=torch.float32, device=dev)
        ops.select_cells(q=qd, index=idx, nprobe=sizes.nprobe, max_tokens=sizes.max_retrieval_tokens,
                         buffer_pages=sizes.buffer_size, page_size=8, padding_id=idx.n_slots - 1,
                         static_len=static_len, exec_capacity=exec_cap, sel_cells=sel, sel_count=cnt,
                         row_index=rows, row_count=rc, kept_count=kept, scores_out=sc, slot_bound=slot_bound)
        out = torch.empty(heads, G, 128, dtype=torch.bfloat16, device=dev)
        ops.sparse_attention(q=qd, row_index=rows, row_count=rc, list_keys=idx.list_keys,
                             list_values=idx.list_values, static_keys=zkd, static_values=zvd, out=out,
                             part_o=torch.empty(heads, splits, G, 128, device=dev),
                             part_ml=torch.empty(heads, splits, G, 2, device=dev), splits=splits,
                             counters=torch.zeros(heads, dtype=torch.int32, device=dev))
        torch.cuda.synchronize()
        qb = O.bf16_bits(q)
        got = out.float().cpu().numpy()
        for h in range(heads):
            ref_sc = O.scores(qb[h], cents[h], mask[h])
            np.testing.assert_array_equal(sc[h].cpu().numpy(), ref_sc, err_msg=f"scores q{t} h{h}")
            ref_sel, pre = O.select(ref_sc, csz[h], sizes.nprobe, sizes.max_retrieval_tokens, sizes.buffer_size, 8,
                                    idx.n_slots - 1)
            n_sel = int(cnt[h])
            np.testing.assert_array_equal(sel[h, :n_sel].cpu().numpy(), np.sort(ref_sel), err_msg=f"q{t} h{h}")
            assert int(kept[h]) == int((pre != idx.n_slots - 1).sum())
            exp = [(1 << 30) | r for r in range(static_len)]
            for cc in np.sort(ref_sel):
                exp.extend(range(offs[h, cc], offs[h, cc] + csz[h, cc]))
            assert int(rc[h]) == len(exp)
            np.testing.assert_array_equal(rows[h, :len(exp)].cpu().numpy(), np.asarray(exp, np.int64).astype(np.int32))
            kr = torch.cat([zk[h, :static_len]] + [lk[h, offs[h, cc]:offs[h, cc] + csz[h, cc]] for cc in ref_sel])
            vr = torch.cat([zv[h, :static_len]] + [lv[h, offs[h, cc]:offs[h, cc] + csz[h, cc]] for cc in ref_sel])
            ref = O.attention(qb[h], O.bf16_bits(kr), O.bf16_bits(vr), 1.0 / math.sqrt(128))
            err = np.abs(got[h] - ref)
            assert err.max() <= ATOL_MAX and err.mean() <= ATOL_MEAN, (t, h, float(err.max()), float(err.mean()))
            counts.append(n_sel)
    return counts


@pytest.mark.parametrize("bounded", [False, True])
def test_decode_cfg1_geometry(cfg1, bounded):
    c, K, V, Q, k, v, sizes, idx = cfg1
    bound = int(idx.n_active.max()) if bounded else 0
    counts = _decode_and_check(K, V, Q, idx, sizes, range(16), static_len=97, splits=48, slot_bound=bound)
    assert min(counts) > 100  # the token budget, not nprobe, ends these selections


def test_select_scores_match_reference_kernel_cfg1(cfg1):
    """The select kernel's fused scores at 8 101 slots against the reference's
    own CUDA scorer (compute_impl.cu:62-103, built from source)."""
    from tests.test_gpu_reference_pins import masked_ref_scores

    c, K, V, Q, k, v, sizes, idx = cfg1
    heads = K.shape[0]
    for t in range(16):
        q = Q[t].reshape(heads, G, 128).contiguous().cuda()
        sc = torch.zeros((heads, idx.n_slots), dtype=torch.float32, device="cuda")
        ops.select_cells(q=q, index=idx, nprobe=sizes.nprobe, max_tokens=sizes.max_retrieval_tokens,
                         buffer_pages=sizes.buffer_size, page_size=8, padding_id=idx.n_slots - 1, static_len=97,
                         exec_capacity=sizes.execution_stride,
                         sel_cells=torch.empty((heads, sizes.nprobe), dtype=torch.int32, device="cuda"),
                         sel_count=torch.empty((heads,), dtype=torch.int32, device="cuda"),
                         row_index=torch.empty((heads, sizes.execution_stride), dtype=torch.int32, device="cuda"),
                         row_count=torch.empty((heads,), dtype=torch.int32, device="cuda"), scores_out=sc)
        torch.cuda.synchronize()
        assert torch.equal(sc.view(torch.int32), masked_ref_scores(q, idx).view(torch.int32)), t


def test_decode_s4_config3_size():
    """S=4 at the config-3 size: k = 10 per subspace (10 000 cells, 10 001 slots),
    budget 0.05, Qwen2.5-7B geometry (theta 1e6, 128-component mixture)."""
    ctx = 131072
    K, V, Q = make_layer(1, 1 * 7, ctx, 128, 128, 1, 1e6, n_queries=4)
    k, v = K[:, 32:ctx - 64].contiguous(), V[:, 32:ctx - 64].contiguous()
    n = k.shape[1]
    ks = adaptive_k(n, 4)
    assert ks == (10, 10, 10, 10)
    sizes = RetrievalSizes.from_capacity(n, 4, 0.05, 32, static_capacity=96 + 16)
    assert (sizes.n_centroids, sizes.nprobe, sizes.max_retrieval_tokens) == (10001, 500, 6548)
    idx = _build(k, v, 4, ks, sizes.n_centroids, 20, 5e-4, 20, 5e-4)
    _check_build(k, v, idx, 4, ks, 20, 5e-4, 20, 5e-4)
    _decode_and_check(K, V, Q, idx, sizes, range(4), static_len=96, splits=32, slot_bound=int(idx.n_active.max()))


def test_decode_ivf():
    """IVF (subspace_parts 0): one k-means of round(n/16) cells over the whole
    head dim; slots sized as the reference's prepare_cache does."""
    ctx = 8192
    K, V, Q = make_layer(2, 8, ctx, 128, 64, 4, 500000.0, n_queries=4)
    k, v = K[:, 32:ctx - 64].contiguous(), V[:, 32:ctx - 64].contiguous()
    n = k.shape[1]
    ks = adaptive_k(n, 0)
    assert ks == (506,)
    sizes = RetrievalSizes.from_capacity(n, 0, 0.1, 32, static_capacity=96 + 16)
    assert sizes.n_centroids == 1025 and sizes.nprobe == 102
    idx = _build(k, v, 0, ks, sizes.n_centroids, 10, 0.0, 10, 0.0)
    _check_build(k, v, idx, 0, ks, 10, 0.0, 10, 0.0)
    _decode_and_check(K, V, Q, idx, sizes, range(4), static_len=100, splits=16)
