"""Pins against the reference's own CUDA decode scorer.

``fused_query_group_similarity_kernel`` (compute_impl.cu:62-103) is compiled
from the reference source for sm_100a into oracle/_ref/libref_scorer.so by
oracle/build_ref_cuda.py and run here beside the device path:

* ``imi_query_group_similarities`` (the API-compatible scorer) must give the
  same bits;
* the select kernel's fused separable scores (``scores_out``) must give the
  same bits after the reference's ``masked_fill(-inf)`` (retrieval.py:357), on
  the config-0 index; the config-1 geometry is covered in
  tests/test_gpu_parity_cfg1.py with the same helper.
"""
import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from adaptiveimi_b200 import ops

pytestmark = pytest.mark.gpu
LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libref_scorer.so"
_L = None


def ref_lib():
    global _L
    if _L is None:
        if not LIB.exists():
            pytest.skip("oracle/_ref/libref_scorer.so not built (needs the reference checkout at build time)")
        _L = ctypes.CDLL(str(LIB))
        P, i = ctypes.c_void_p, ctypes.c_int
        _L.ref_fused_query_group_similarities_bf16.argtypes = [P, P, P, i, i, i, i, P]
        _L.ref_fused_query_group_similarities_bf16.restype = i
    return _L


def ref_scores(q: torch.Tensor, cents: torch.Tensor) -> torch.Tensor:
    """The reference kernel on device tensors: q [kv, G, D] bf16, cents [kv, n, D] f32."""
    q, cents = q.contiguous(), cents.contiguous()
    kv, G, D = q.shape
    n = cents.shape[1]
    out = torch.empty((kv, n), dtype=torch.float32, device=q.device)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = ref_lib().ref_fused_query_group_similarities_bf16(ctypes.c_void_p(q.data_ptr()),
                                                           ctypes.c_void_p(cents.data_ptr()),
                                                           ctypes.c_void_p(out.data_ptr()), G, n, kv, D, st)
    assert rc == 0
    torch.cuda.synchronize()
    return out


def test_similarity_kernel_matches_reference_kernel():
    g = torch.Generator().manual_seed(7)
    for kv, G, n in ((8, 4, 1025), (4, 7, 8101), (1, 8, 10001)):
        q = torch.randn(kv, G, 128, generator=g).to(torch.bfloat16).cuda()
        c = (torch.randn(kv, n, 128, generator=g) * 0.7).cuda()
        got = ops.fused_query_group_similarities(q, c)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int32), ref_scores(q, c).view(torch.int32)), (kv, G, n)


def masked_ref_scores(q, idx):
    """Reference scores with retrieval.py:357's masked_fill(-inf) over the padded table."""
    s = ref_scores(q, idx.centroids)
    return s.masked_fill(idx.cell_mask.bool(), float("-inf"))


def test_select_scores_match_reference_kernel_cfg0():
    from tests.test_gpu_kernels import _decode_setup, _select

    K, V, Q, k, v, sizes, idx = _decode_setup()
    heads, G = 8, 4
    exec_cap = sizes.buffer_size * 8 + 96 + 16
    for t in range(16):
        q = Q[t].reshape(heads, G, 128).contiguous().cuda()
        _, _, _, _, sc, _ = _select(idx, q, sizes, 97, exec_cap)
        assert torch.equal(sc.view(torch.int32), masked_ref_scores(q, idx).view(torch.int32)), t
