"""ctypes wrapper over ``oracle/_build/libimi_oracle.so``.

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and the
CPU-baseline / reference arm of ``bench.py`` -- never by the product package.
Each wrapper names the reference code it restates (see ``imi_oracle.cpp``).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import build_oracle

_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        path = build_oracle.build()
        L = ctypes.CDLL(str(path))
        P = ctypes.c_void_p
        i, f, u64, d = ctypes.c_int, ctypes.c_float, ctypes.c_uint64, ctypes.c_double
        L.oracle_kmeans.argtypes = [P, i, i, i, u64, i, f, i, f, P, P, P]
        L.oracle_kmeanspp.argtypes = [P, i, i, i, u64, P]
        L.oracle_build_head.argtypes = [P, P, i, i, i, P, i, f, i, f, P, P, P, P, P, P, P, P]
        L.oracle_scores.argtypes = [P, i, i, P, P, i, P]
        L.oracle_scores.restype = None
        L.oracle_select.argtypes = [P, P, i, i, i, i, i, i, P, P]
        L.oracle_attention.argtypes = [P, i, i, P, P, i, d, P]
        L.oracle_attention.restype = None
        L.oracle_async_update.argtypes = [P, i, i, P, i, P, P, P, i, P]
        L.oracle_async_update.restype = None
        _LIB = L
    return _LIB


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the oracle must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def bf16_bits(t) -> np.ndarray:
    """torch bf16 tensor -> uint16 numpy view of its bits (contiguous copy)."""
    import torch

    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def kmeans(data: np.ndarray, k: int, seed: int, max_iters: int, tol=0.0, min_iter=None, rel_tol=0.0):
    """One (head, subspace) k-means; kmeans_core.cpp:351-382."""
    data = np.ascontiguousarray(data, dtype=np.float32)
    n, dim = data.shape
    labels = np.zeros(n, np.int32)
    cent = np.zeros((k, dim), np.float32)
    inertia = np.zeros(1, np.float32)
    it = lib().oracle_kmeans(_p(data), n, dim, k, seed, max_iters, tol, max_iters if min_iter is None else min_iter,
                             rel_tol, _p(labels), _p(cent), _p(inertia))
    return labels, cent, it, float(inertia[0])


def kmeanspp(data: np.ndarray, k: int, seed: int):
    data = np.ascontiguousarray(data, dtype=np.float32)
    n, dim = data.shape
    cent = np.zeros((k, dim), np.float32)
    lib().oracle_kmeanspp(_p(data), n, dim, k, seed, _p(cent))
    return cent


def build_head(keys_bits: np.ndarray, values_bits: np.ndarray, parts: int, ks, max_iters: int, tol=0.0,
               min_iter=None, rel_tol=0.0):
    """IMI build of one head; kmeans_core.cpp:384-772 + reorganize_core.cpp:18-311."""
    keys_bits = np.ascontiguousarray(keys_bits, np.uint16)
    values_bits = np.ascontiguousarray(values_bits, np.uint16)
    n, dim = keys_bits.shape
    S = 1 if parts == 0 else parts
    sub = dim // S
    ks_a = np.asarray(list(ks)[:S], np.int32)
    total = int(np.prod(ks_a.astype(np.int64)))
    sub_labels = np.zeros((S, n), np.int32)
    sub_cent = np.zeros(int(ks_a.sum()) * sub, np.float32)
    final = np.zeros(n, np.int32)
    offsets = np.zeros(min(total, n) + 1, np.int32)
    merged = np.zeros((min(total, n), dim), np.float32)
    lk = np.zeros_like(keys_bits)
    lv = np.zeros_like(values_bits)
    iters = np.zeros(S, np.int32)
    na = lib().oracle_build_head(_p(keys_bits), _p(values_bits), n, dim, parts, _p(ks_a), max_iters, tol,
                                 max_iters if min_iter is None else min_iter, rel_tol, _p(sub_labels), _p(sub_cent),
                                 _p(final), _p(offsets), _p(merged), _p(lk), _p(lv), _p(iters))
    cents = []
    o = 0
    for s in range(S):
        cents.append(sub_cent[o:o + ks_a[s] * sub].reshape(ks_a[s], sub))
        o += ks_a[s] * sub
    return dict(sub_labels=sub_labels, sub_centroids=cents, final_labels=final, n_active=na,
                offsets=offsets[:na + 1], merged=merged[:na], list_keys=lk, list_values=lv, iters=iters)


def scores(q_bits: np.ndarray, cent: np.ndarray, mask: np.ndarray | None = None) -> np.ndarray:
    """compute_impl.cu:62-103 + retrieval.py:357 for one KV group."""
    q_bits = np.ascontiguousarray(q_bits, np.uint16)
    cent = np.ascontiguousarray(cent, np.float32)
    G, dim = q_bits.shape
    n = cent.shape[0]
    out = np.zeros(n, np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, np.uint8)
    lib().oracle_scores(_p(q_bits), G, dim, _p(cent), None if m is None else _p(m), n, _p(out))
    return out


def select(scores_: np.ndarray, sizes: np.ndarray, nprobe: int, max_tokens: int, buffer_pages: int,
           page_size: int = 8, padding_id: int | None = None):
    """retrieval.py:295-303 + wave_buffer_cpu_hotcold.cpp:303-371 for one KV group."""
    scores_ = np.ascontiguousarray(scores_, np.float32)
    sizes = np.ascontiguousarray(sizes, np.int32)
    n = scores_.shape[0]
    pad = n - 1 if padding_id is None else padding_id
    out = np.zeros(n, np.int32)
    pre = np.zeros(min(nprobe, n), np.int32)
    cnt = lib().oracle_select(_p(scores_), _p(sizes), n, nprobe, max_tokens, buffer_pages, page_size, pad, _p(out),
                              _p(pre))
    return out[:cnt], pre


def attention(q_bits: np.ndarray, k_bits: np.ndarray, v_bits: np.ndarray, scale: float) -> np.ndarray:
    """Softmax attention of one KV group (weighted_flash_decoding semantics), fp64."""
    q_bits = np.ascontiguousarray(q_bits, np.uint16)
    k_bits = np.ascontiguousarray(k_bits, np.uint16)
    v_bits = np.ascontiguousarray(v_bits, np.uint16)
    G, dim = q_bits.shape
    out = np.zeros((G, dim), np.float64)
    lib().oracle_attention(_p(q_bits), G, dim, _p(k_bits), _p(v_bits), k_bits.shape[0], scale, _p(out))
    return out


def async_update(keys_bits, shadow, counts, delta_counts, delta_sums, threshold):
    """async_update.py:122-143 for one KV group; updates the arrays in place."""
    keys_bits = np.ascontiguousarray(keys_bits, np.uint16)
    B, dim = keys_bits.shape
    ids = np.zeros(B, np.int32)
    lib().oracle_async_update(_p(keys_bits), B, dim, _p(shadow), shadow.shape[0], _p(counts), _p(delta_counts),
                              _p(delta_sums), threshold, _p(ids))
    return ids
