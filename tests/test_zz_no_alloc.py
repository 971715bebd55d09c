"""imi_sparse_attention_noalloc: attention for callers that cannot allocate.

Some callers of this library cannot call cudaMalloc (they run inside another
allocator, from a host callback, or in a runtime that forbids device
allocation after start-up), so they cannot hand the attention its scratch
buffers.  The no-alloc entry point uses a fixed array owned by the library
instead.  This test calls it through the C ABI and checks its output against
the regular entry point (imi_sparse_attention, with caller scratch) on two
calls in a row, within the attention tolerance the other tests use.  It sits
in a file of its own that pytest collects last.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from adaptiveimi_b200 import _lib, ops
from adaptiveimi_b200.sizing import RetrievalSizes
from adaptiveimi_b200.synthetic import make_layer

pytestmark = pytest.mark.gpu
ATOL_MAX, ATOL_MEAN = 2e-2, 2e-3


def _setup():
    heads, G, ctx = 4, 4, 4096
    K, V, Q = make_layer(heads, heads * G, ctx, 128, 32, 21, 500000.0, n_queries=2)
    k = K[:, 32:ctx - 64].contiguous().cuda()
    v = V[:, 32:ctx - 64].contiguous().cuda()
    n = k.shape[1]
    sizes = RetrievalSizes.from_capacity(n, 2, 0.1, 32, static_capacity=97)
    idx = ops.build_index(k, v, parts=2, ks=(16, 16), n_slots=sizes.n_centroids, max_iters=5,
                          early_stop_min_iter=5, tol=0.0, early_stop_rel_tol=0.0)
    zk = torch.zeros(heads, 97, 128, dtype=torch.bfloat16, device="cuda")
    zv = torch.zeros_like(zk)
    zk[:, :32], zk[:, 32:96] = K[:, :32].cuda(), K[:, ctx - 64:].cuda()
    zv[:, :32], zv[:, 32:96] = V[:, :32].cuda(), V[:, ctx - 64:].cuda()
    cap = sizes.execution_stride
    qs, rows, rcs = [], [], []
    for t in range(2):
        q = Q[t].reshape(heads, G, 128).contiguous().cuda()
        r = torch.empty(heads, cap, dtype=torch.int32, device="cuda")
        rc = torch.empty(heads, dtype=torch.int32, device="cuda")
        ops.select_cells(q=q, index=idx, nprobe=sizes.nprobe, max_tokens=sizes.max_retrieval_tokens,
                         buffer_pages=sizes.buffer_size, page_size=8, padding_id=idx.n_slots - 1,
                         static_len=96, exec_capacity=cap,
                         sel_cells=torch.empty(heads, sizes.nprobe, dtype=torch.int32, device="cuda"),
                         sel_count=torch.empty(heads, dtype=torch.int32, device="cuda"), row_index=r, row_count=rc)
        qs.append(q)
        rows.append(r)
        rcs.append(rc)
    return idx, zk, zv, qs, rows, rcs, heads, G


def _desc(idx, zk, zv, q, r, rc, out, splits):
    d = _lib.AttnDesc()
    d.bg, d.G, d.splits, d.exec_capacity = q.shape[0], q.shape[1], splits, r.shape[1]
    d.scale = 1.0 / math.sqrt(128)
    d.q, d.row_index, d.row_count = q.data_ptr(), r.data_ptr(), rc.data_ptr()
    d.list_keys, d.list_values, d.list_rows = idx.list_keys.data_ptr(), idx.list_values.data_ptr(), \
        idx.list_keys.shape[1]
    d.static_keys, d.static_values, d.static_rows = zk.data_ptr(), zv.data_ptr(), zk.shape[1]
    d.out = out.data_ptr()
    return d  # part_o / part_ml / counters stay NULL: the no-alloc entry does not read them


@pytest.mark.parametrize("splits", [8, 126])
def test_noalloc_attention_matches_regular_entry_two_calls(splits):
    # 126 splits: 4 groups * 126 * 4 heads * 520 B plus alignment is exactly the
    # 1 MiB array, so the partial outputs reach its last byte
    idx, zk, zv, qs, rows, rcs, heads, G = _setup()
    L = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for t in range(2):  # two calls in a row reuse the same library-owned array
        ref = torch.empty(heads, G, 128, dtype=torch.bfloat16, device="cuda")
        ops.sparse_attention(q=qs[t], row_index=rows[t], row_count=rcs[t], list_keys=idx.list_keys,
                             list_values=idx.list_values, static_keys=zk, static_values=zv, out=ref,
                             part_o=torch.empty(heads, splits, G, 128, device="cuda"),
                             part_ml=torch.empty(heads, splits, G, 2, device="cuda"), splits=splits,
                             counters=torch.zeros(heads, dtype=torch.int32, device="cuda"))
        got = torch.full((heads, G, 128), float("nan"), dtype=torch.bfloat16, device="cuda")
        d = _desc(idx, zk, zv, qs[t], rows[t], rcs[t], got, splits)
        _lib.check(L.imi_sparse_attention_noalloc(ctypes.byref(d), stream), "imi_sparse_attention_noalloc")
        torch.cuda.synchronize()
        err = (got.float() - ref.float()).abs().cpu().numpy()
        assert np.isfinite(err).all()
        assert err.max() <= ATOL_MAX and err.mean() <= ATOL_MEAN, (t, float(err.max()))


def test_noalloc_attention_rejects_requests_beyond_the_array():
    idx, zk, zv, qs, rows, rcs, heads, G = _setup()
    L = _lib.load()
    out = torch.full((heads, G, 128), 7.0, dtype=torch.bfloat16, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for splits in (127, 4096):  # 127: one split past the array; 4096: far past it
        d = _desc(idx, zk, zv, qs[0], rows[0], rcs[0], out, splits)
        rc = L.imi_sparse_attention_noalloc(ctypes.byref(d), stream)
        assert rc != 0
        assert b"scratch" in L.imi_last_error()
    torch.cuda.synchronize()
    assert bool((out.float() == 7.0).all())  # a rejected request launches nothing
