"""Torch-facing wrappers over the C ABI (one function per entry point).

Tensors are passed by device pointer; every launch goes to the current CUDA
stream of the tensors' device.  Shapes and dtypes are checked here so that
errors surface as Python exceptions with the reference's wording where one
exists.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _lib

_P = ctypes.c_void_p


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else _P(t.data_ptr())


def _stream(dev: torch.device):
    return _P(torch.cuda.current_stream(dev).cuda_stream)


def _need(t: torch.Tensor, dtype, name: str, contiguous=True):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _ks4(ks: Sequence[int]):
    a = (ctypes.c_int32 * 4)()
    for i in range(4):
        a[i] = int(ks[i]) if i < len(ks) else 1
    return a


# ---------------------------------------------------------------------------
# index build
# ---------------------------------------------------------------------------
@dataclass
class IMIIndex:
    """Device-resident IMI index of one layer (all KV groups).

    Layout (bg = KV groups): ``list_keys/list_values`` [bg, list_rows, D] bf16 in
    cell order; ``cell_sizes`` [bg, n_slots] i32; ``cell_offsets`` [bg, n_slots+1]
    i32; ``cell_mask`` [bg, n_slots] u8 (1 = padding / empty); ``cell_code``
    [bg, n_slots] i32 (packed subspace digits); ``centroids`` [bg, n_slots, D]
    f32 (merged, the reference's padded centroid table); ``sub_centroids``
    [bg, S, kmax, D/S] f32; ``sub_labels`` [bg, S, n] i32; ``n_active`` [bg] i32.
    """

    parts: int
    ks: tuple
    kmax: int
    n_tokens: int
    n_slots: int
    list_keys: torch.Tensor
    list_values: torch.Tensor
    cell_sizes: torch.Tensor
    cell_offsets: torch.Tensor
    cell_mask: torch.Tensor
    cell_code: torch.Tensor
    centroids: torch.Tensor
    sub_centroids: torch.Tensor
    sub_labels: torch.Tensor
    n_active: torch.Tensor
    iters_run: torch.Tensor


def build_workspace_size(heads: int, n_tokens: int, dim: int, parts: int, ks: Sequence[int]) -> int:
    L = _lib.load()
    return int(L.imi_build_workspace_size(heads, n_tokens, dim, parts, ctypes.cast(_ks4(ks), _P)))


def build_index(keys: torch.Tensor, values: torch.Tensor, *, parts: int, ks: Sequence[int], n_slots: int,
                max_iters: int = 25, tol: float = 5e-4, early_stop_min_iter: int = 5,
                early_stop_rel_tol: float = 5e-4, list_keys: Optional[torch.Tensor] = None,
                list_values: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None,
                kmax: Optional[int] = None, status: Optional[torch.Tensor] = None,
                phase_ns: Optional[torch.Tensor] = None, ready_event: Optional[torch.cuda.Event] = None) -> IMIIndex:
    """Build the IMI of one layer on the device.

    keys / values: [heads, n, D] bf16 CUDA views whose last dim is contiguous
    (e.g. ``key_states[0, start:end].transpose(0, 1)`` -- no copy is made).
    ``list_keys`` / ``list_values`` ([heads, >= n, D]) receive the rows in cell
    order; allocated when not given.  ``status``: int32 [1] device word, bit 0
    set when the tensor-core E-step gave up (the index is then void).
    ``phase_ns``: int64 [3] device timestamps (k-means start, k-means end,
    reorganize end).  ``ready_event``: an event recorded after keys/values were
    produced on another stream; the build (on the current stream) waits for it.
    """
    if keys.dim() != 3 or keys.shape != values.shape:
        raise ValueError("keys/values must be [kv_heads, tokens, head_dim] and share a shape")
    if keys.dtype != torch.bfloat16 or values.dtype != torch.bfloat16:
        raise ValueError("the IMI build takes bfloat16 keys/values (the reference accepts 16-bit inputs only)")
    if keys.stride(2) != 1 or values.stride(2) != 1 or keys.stride() != values.stride():
        raise ValueError("keys/values need a contiguous last dim and identical strides")
    H, n, D = keys.shape
    dev = keys.device
    S = 1 if parts == 0 else parts
    ks = tuple(int(k) for k in ks[:S])
    kmax = int(kmax or max(ks))
    if list_keys is None:
        list_keys = torch.empty((H, n, D), dtype=keys.dtype, device=dev)
    if list_values is None:
        list_values = torch.empty((H, n, D), dtype=keys.dtype, device=dev)
    out = dict(
        cell_sizes=torch.empty((H, n_slots), dtype=torch.int32, device=dev),
        cell_offsets=torch.empty((H, n_slots + 1), dtype=torch.int32, device=dev),
        cell_mask=torch.empty((H, n_slots), dtype=torch.uint8, device=dev),
        cell_code=torch.full((H, n_slots), -1, dtype=torch.int32, device=dev),
        centroids=torch.empty((H, n_slots, D), dtype=torch.float32, device=dev),
        sub_centroids=torch.zeros((H, S, kmax, D // S), dtype=torch.float32, device=dev),
        sub_labels=torch.empty((H, S, n), dtype=torch.int32, device=dev),
        n_active=torch.zeros((H,), dtype=torch.int32, device=dev),
        iters_run=torch.zeros((H, S), dtype=torch.int32, device=dev),
    )
    wbytes = build_workspace_size(H, n, D, parts, ks)
    if workspace is None or workspace.numel() < wbytes:
        workspace = torch.empty((max(wbytes, 1),), dtype=torch.uint8, device=dev)
    d = _lib.BuildDesc()
    d.heads, d.n_tokens, d.dim, d.parts = H, n, D, parts
    d.ks = _ks4(ks)
    d.keys, d.values = keys.data_ptr(), values.data_ptr()
    d.head_stride, d.token_stride = keys.stride(0), keys.stride(1)
    d.max_iters, d.early_stop_min_iter = int(max_iters), int(early_stop_min_iter)
    d.tol, d.early_stop_rel_tol = float(tol), float(early_stop_rel_tol)
    d.list_keys, d.list_values = list_keys.data_ptr(), list_values.data_ptr()
    d.list_rows = list_keys.shape[1]
    d.n_slots, d.kmax = n_slots, kmax
    for name in ("cell_sizes", "cell_offsets", "cell_mask", "cell_code", "centroids", "sub_centroids",
                 "sub_labels", "n_active", "iters_run"):
        setattr(d, name, out[name].data_ptr())
    d.workspace, d.workspace_bytes = workspace.data_ptr(), workspace.numel()
    d.status = status.data_ptr() if status is not None else None
    d.phase_ns = phase_ns.data_ptr() if phase_ns is not None else None
    d.ready_event = ready_event.cuda_event if ready_event is not None else None
    L = _lib.load()
    with torch.cuda.device(dev):
        _lib.check(L.imi_build_index(ctypes.byref(d), _stream(dev)), "imi_build_index")
    return IMIIndex(parts=parts, ks=ks, kmax=kmax, n_tokens=n, n_slots=n_slots, list_keys=list_keys,
                    list_values=list_values, **out)


# ---------------------------------------------------------------------------
# decode
# ---------------------------------------------------------------------------
def fused_query_group_similarities(query_grouped: torch.Tensor, centroids: torch.Tensor,
                                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Drop-in for gpu_cluster_manager_cpp.fused_query_group_similarities
    (compute_wrappers.cpp:39-104): q [kv, G, D] bf16, centroids [kv, n, D] f32."""
    if not query_grouped.is_cuda or not centroids.is_cuda:
        raise ValueError("query_grouped and centroids must be on GPU")
    if query_grouped.dim() != 3 or centroids.dim() != 3:
        raise ValueError("query_grouped and centroids must be 3D")
    if centroids.dtype != torch.float32:
        raise ValueError("centroids must be FP32")
    if query_grouped.dtype != torch.bfloat16:
        raise ValueError("fused_query_group_similarities: query dtype must be BF16")
    kv, G, D = query_grouped.shape
    n = centroids.shape[1]
    if centroids.shape[0] != kv or centroids.shape[2] != D:
        raise ValueError("centroids kv_heads / dim mismatch")
    q = query_grouped.contiguous()
    c = centroids.contiguous()
    if out is None:
        res = torch.empty((kv, n), dtype=torch.float32, device=q.device)
        stride = n
    else:
        if out.dtype != torch.float32 or out.dim() != 2 or out.size(0) < kv or out.size(1) < n:
            raise ValueError("fused_query_group_similarities: out tensor shape insufficient")
        res = out.narrow(0, 0, kv).narrow(1, 0, n)
        stride = out.stride(0)
    L = _lib.load()
    _lib.check(L.imi_query_group_similarities(_ptr(q), _ptr(c), _ptr(res), kv, G, n, D, stride, _stream(q.device)),
               "imi_query_group_similarities")
    return res


def select_cells(*, q: torch.Tensor, index: IMIIndex, nprobe: int, max_tokens: int, buffer_pages: int,
                 page_size: int, padding_id: int, static_len: int, exec_capacity: int,
                 sel_cells: torch.Tensor, sel_count: torch.Tensor, row_index: torch.Tensor,
                 row_count: torch.Tensor, centroids: Optional[torch.Tensor] = None,
                 cell_dirty: Optional[torch.Tensor] = None, delta_cell_ids: Optional[torch.Tensor] = None,
                 delta_count: Optional[torch.Tensor] = None, kept_count: Optional[torch.Tensor] = None,
                 scores_out: Optional[torch.Tensor] = None, phase_ns: Optional[torch.Tensor] = None,
                 slot_bound: int = 0) -> None:
    """Score cells, choose them (top-nprobe, token budget, page truncation) and
    write the execution row list.  q: [bg, G, D] bf16 contiguous."""
    bg, G, D = q.shape
    d = _lib.SelectDesc()
    d.bg, d.G, d.dim, d.n_slots, d.parts, d.kmax = bg, G, D, index.n_slots, index.parts, index.kmax
    d.ks = _ks4(index.ks)
    d.q = q.data_ptr()
    d.sub_centroids = index.sub_centroids.data_ptr()
    d.cell_code = index.cell_code.data_ptr()
    d.cell_sizes = index.cell_sizes.data_ptr()
    d.cell_offsets = index.cell_offsets.data_ptr()
    d.cell_mask = index.cell_mask.data_ptr()
    d.centroids = (centroids if centroids is not None else index.centroids).data_ptr()
    d.cell_dirty = cell_dirty.data_ptr() if cell_dirty is not None else None
    d.nprobe, d.max_tokens, d.buffer_pages, d.page_size, d.padding_id = nprobe, max_tokens, buffer_pages, \
        page_size, padding_id
    d.static_len = static_len
    d.delta_cell_ids = delta_cell_ids.data_ptr() if delta_cell_ids is not None else None
    d.delta_count = delta_count.data_ptr() if delta_count is not None else None
    d.delta_capacity = delta_cell_ids.shape[1] if delta_cell_ids is not None else 0
    d.exec_capacity = exec_capacity
    d.sel_cells, d.sel_count = sel_cells.data_ptr(), sel_count.data_ptr()
    d.kept_count = kept_count.data_ptr() if kept_count is not None else None
    d.row_index, d.row_count = row_index.data_ptr(), row_count.data_ptr()
    d.scores_out = scores_out.data_ptr() if scores_out is not None else None
    d.phase_ns = phase_ns.data_ptr() if phase_ns is not None else None
    d.slot_bound = int(slot_bound)
    L = _lib.load()
    _lib.check(L.imi_select_cells(ctypes.byref(d), _stream(q.device)), "imi_select_cells")


def default_splits(bg: int, rows_per_group: int, sms: int = 148, exec_capacity: Optional[int] = None) -> int:
    """CTAs per KV group for the split-K attention: one wave (one CTA per SM,
    the kernel's shared-memory ring allows one) and at least 64 rows per CTA.
    ``exec_capacity`` is accepted for callers that pass it; the kernel reads
    the row list straight from global memory, so it no longer bounds the
    split."""
    # one CTA per SM, but at most 48 per group: past that the split merge costs
    # more than the extra streaming width gains (one group on a B200: 13.7 µs at
    # 148 splits, 11.3 µs at 37-74)
    want = max(1, min(48, sms // bg))
    return int(max(1, min(want, (rows_per_group + 63) // 64, 512)))


def sparse_attention(*, q: torch.Tensor, row_index: torch.Tensor, row_count: torch.Tensor,
                     list_keys: torch.Tensor, list_values: torch.Tensor, static_keys: torch.Tensor,
                     static_values: torch.Tensor, out: torch.Tensor, part_o: torch.Tensor, part_ml: torch.Tensor,
                     splits: int, scale: Optional[float] = None, delta_keys: Optional[torch.Tensor] = None,
                     delta_values: Optional[torch.Tensor] = None,
                     counters: Optional[torch.Tensor] = None,
                     status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention of q [bg, G, 128] over the rows named by row_index.
    counters: int32 [bg] zeroed scratch; when given the split merge happens in
    the attention kernel itself (its last CTA per group).
    status: int32 [1] or None (reserved: the kernel has no waits and sets no bit)."""
    bg, G, D = q.shape
    if D != 128:
        raise ValueError("sparse attention supports head_dim 128")
    d = _lib.AttnDesc()
    d.bg, d.G, d.splits, d.exec_capacity = bg, G, splits, row_index.shape[1]
    d.scale = float(scale if scale is not None else 1.0 / math.sqrt(D))
    d.q, d.row_index, d.row_count = q.data_ptr(), row_index.data_ptr(), row_count.data_ptr()
    d.list_keys, d.list_values, d.list_rows = list_keys.data_ptr(), list_values.data_ptr(), list_keys.shape[-2]
    d.static_keys, d.static_values, d.static_rows = static_keys.data_ptr(), static_values.data_ptr(), \
        static_keys.shape[-2]
    if delta_keys is not None:
        d.delta_keys, d.delta_values, d.delta_rows = delta_keys.data_ptr(), delta_values.data_ptr(), \
            delta_keys.shape[-2]
    d.part_o, d.part_ml, d.out = part_o.data_ptr(), part_ml.data_ptr(), out.data_ptr()
    d.counters = counters.data_ptr() if counters is not None else None
    d.status = status.data_ptr() if status is not None else None
    L = _lib.load()
    _lib.check(L.imi_sparse_attention(ctypes.byref(d), _stream(q.device)), "imi_sparse_attention")
    return out


def decode_attend(*, q: torch.Tensor, index: IMIIndex, nprobe: int, max_tokens: int, buffer_pages: int,
                  page_size: int, padding_id: int, static_len: int, exec_capacity: int, sel_cells: torch.Tensor,
                  sel_count: torch.Tensor, row_index: torch.Tensor, row_count: torch.Tensor, static_keys: torch.Tensor,
                  static_values: torch.Tensor, out: torch.Tensor, part_o: torch.Tensor, part_ml: torch.Tensor,
                  counters: torch.Tensor, splits: int, kept_count: Optional[torch.Tensor] = None,
                  slot_bound: int = 0,
                  status: Optional[torch.Tensor] = None, delta_cell_ids: Optional[torch.Tensor] = None,
                  delta_count: Optional[torch.Tensor] = None, delta_keys: Optional[torch.Tensor] = None,
                  delta_values: Optional[torch.Tensor] = None, scores_out: Optional[torch.Tensor] = None,
                  phase_ns: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Selection + attention of one layer through imi_decode_attend (the select
    kernel, then the attention kernel as its programmatic dependent)."""
    bg, G, D = q.shape
    d = _lib.SelectDesc()
    d.bg, d.G, d.dim, d.n_slots, d.parts, d.kmax = bg, G, D, index.n_slots, index.parts, index.kmax
    d.ks = _ks4(index.ks)
    d.q = q.data_ptr()
    d.sub_centroids, d.cell_code = index.sub_centroids.data_ptr(), index.cell_code.data_ptr()
    d.cell_sizes, d.cell_offsets = index.cell_sizes.data_ptr(), index.cell_offsets.data_ptr()
    d.cell_mask, d.centroids = index.cell_mask.data_ptr(), index.centroids.data_ptr()
    d.nprobe, d.max_tokens, d.buffer_pages, d.page_size, d.padding_id = nprobe, max_tokens, buffer_pages, \
        page_size, padding_id
    d.static_len, d.exec_capacity = static_len, exec_capacity
    if delta_cell_ids is not None:
        d.delta_cell_ids, d.delta_count = delta_cell_ids.data_ptr(), delta_count.data_ptr()
        d.delta_capacity = delta_cell_ids.shape[1]
    d.sel_cells, d.sel_count = sel_cells.data_ptr(), sel_count.data_ptr()
    d.kept_count = kept_count.data_ptr() if kept_count is not None else None
    d.row_index, d.row_count = row_index.data_ptr(), row_count.data_ptr()
    d.scores_out = scores_out.data_ptr() if scores_out is not None else None
    d.phase_ns = phase_ns.data_ptr() if phase_ns is not None else None
    d.slot_bound = int(slot_bound)
    a = _lib.AttnDesc()
    a.bg, a.G, a.splits, a.exec_capacity = bg, G, splits, exec_capacity
    a.scale = 1.0 / math.sqrt(D)
    a.q, a.row_index, a.row_count = q.data_ptr(), row_index.data_ptr(), row_count.data_ptr()
    a.list_keys, a.list_values, a.list_rows = index.list_keys.data_ptr(), index.list_values.data_ptr(), \
        index.list_keys.shape[1]
    a.static_keys, a.static_values, a.static_rows = static_keys.data_ptr(), static_values.data_ptr(), \
        static_keys.shape[-2]
    if delta_keys is not None:
        a.delta_keys, a.delta_values, a.delta_rows = delta_keys.data_ptr(), delta_values.data_ptr(), \
            delta_keys.shape[-2]
    a.part_o, a.part_ml, a.out = part_o.data_ptr(), part_ml.data_ptr(), out.data_ptr()
    a.counters = counters.data_ptr()
    a.status = status.data_ptr() if status is not None else None
    L = _lib.load()
    _lib.check(L.imi_decode_attend(ctypes.byref(d), ctypes.byref(a), None, _stream(q.device)), "imi_decode_attend")
    return out


def decode_append(*, new_keys: torch.Tensor, new_values: torch.Tensor, zone_keys: torch.Tensor,
                  zone_values: torch.Tensor, pos: int, batch_keys: Optional[torch.Tensor] = None,
                  batch_values: Optional[torch.Tensor] = None, batch_slot: int = 0) -> None:
    """zone[:, pos] = new (per KV group); optionally also into the async batch slot.
    new_keys: [bg, D] view with contiguous last dim; zone: [bg, rows, D]."""
    bg, D = new_keys.shape
    d = _lib.AppendDesc()
    d.bg, d.dim = bg, D
    d.new_keys, d.new_values, d.src_head_stride = new_keys.data_ptr(), new_values.data_ptr(), new_keys.stride(0)
    d.zone_keys, d.zone_values, d.zone_rows = zone_keys.data_ptr(), zone_values.data_ptr(), zone_keys.shape[-2]
    d.pos = pos
    if batch_keys is not None:
        d.batch_keys, d.batch_values = batch_keys.data_ptr(), batch_values.data_ptr()
        d.batch_cap, d.batch_slot = batch_keys.shape[1], batch_slot
    L = _lib.load()
    _lib.check(L.imi_decode_append(ctypes.byref(d), _stream(new_keys.device)), "imi_decode_append")


def async_assign(*, index: IMIIndex, batch: int, batch_keys: torch.Tensor, batch_values: torch.Tensor,
                 shadow: torch.Tensor, shadow_dirty: torch.Tensor, pending: torch.Tensor, counts: torch.Tensor,
                 delta_counts: torch.Tensor, delta_sums: torch.Tensor, ring_keys: torch.Tensor,
                 ring_values: torch.Tensor, ring_cell_ids: torch.Tensor, ring_write_pos: torch.Tensor,
                 ring_count: torch.Tensor, threshold: int, ids_out: Optional[torch.Tensor] = None,
                 part_best: Optional[torch.Tensor] = None, ring_store: bool = False) -> None:
    """One batched decode-time cell assignment (async_update.py:122-161).
    ring_store: store the batch's rows and cells in the delta ring (False: only
    its position and count advance, as in the reference).
    part_best: int64 scratch [bg, ceil(n_slots / 512), batch] (allocated when absent)."""
    bg = batch_keys.shape[0]
    d = _lib.AsyncDesc()
    d.bg, d.dim, d.n_slots, d.parts, d.kmax = bg, batch_keys.shape[-1], index.n_slots, index.parts, index.kmax
    d.batch, d.batch_cap, d.threshold, d.ring_cap = batch, batch_keys.shape[1], threshold, ring_keys.shape[1]
    d.ks = _ks4(index.ks)
    d.batch_keys, d.batch_values = batch_keys.data_ptr(), batch_values.data_ptr()
    d.sub_centroids, d.cell_code = index.sub_centroids.data_ptr(), index.cell_code.data_ptr()
    d.shadow, d.shadow_dirty, d.pending = shadow.data_ptr(), shadow_dirty.data_ptr(), pending.data_ptr()
    d.counts, d.delta_counts, d.delta_sums = counts.data_ptr(), delta_counts.data_ptr(), delta_sums.data_ptr()
    d.ring_keys, d.ring_values, d.ring_cell_ids = ring_keys.data_ptr(), ring_values.data_ptr(), \
        ring_cell_ids.data_ptr()
    d.ring_write_pos, d.ring_count = ring_write_pos.data_ptr(), ring_count.data_ptr()
    d.ids_out = ids_out.data_ptr() if ids_out is not None else None
    chunks = async_chunks(index.n_slots)
    if part_best is None or part_best.numel() < bg * chunks * batch:
        part_best = torch.empty((bg, chunks, batch), dtype=torch.int64, device=batch_keys.device)
    d.part_best, d.part_chunks = part_best.data_ptr(), chunks
    d.ring_store = 1 if ring_store else 0
    L = _lib.load()
    _lib.check(L.imi_async_assign(ctypes.byref(d), _stream(batch_keys.device)), "imi_async_assign")


def async_chunks(n_slots: int) -> int:
    return (n_slots + 511) // 512


def apply_updates(*, shadow: torch.Tensor, live: torch.Tensor, pending: torch.Tensor,
                  live_dirty: torch.Tensor) -> None:
    bg, n_slots, D = shadow.shape
    d = _lib.ApplyDesc()
    d.bg, d.n_slots, d.dim = bg, n_slots, D
    d.shadow, d.live, d.pending, d.live_dirty = shadow.data_ptr(), live.data_ptr(), pending.data_ptr(), \
        live_dirty.data_ptr()
    L = _lib.load()
    _lib.check(L.imi_apply_updates(ctypes.byref(d), _stream(shadow.device)), "imi_apply_updates")
