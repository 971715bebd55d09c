"""ctypes binding of ``include/imi_b200.h`` (the library's C ABI).

The shared library ``adaptiveimi_b200/lib/libimi_b200.so`` is built in-tree by
``adaptiveimi_b200/csrc/build_lib.py`` (``__graft_entry__.build()`` runs it).
There is no fallback: if the library is missing or fails to load, every entry
point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libimi_b200.so"

i32, i64, f32, sz = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
P = ctypes.c_void_p


class BuildDesc(ctypes.Structure):
    _fields_ = [
        ("heads", i32), ("n_tokens", i32), ("dim", i32), ("parts", i32),
        ("ks", i32 * 4),
        ("keys", P), ("values", P),
        ("head_stride", i64), ("token_stride", i64),
        ("max_iters", i32), ("early_stop_min_iter", i32),
        ("tol", f32), ("early_stop_rel_tol", f32),
        ("list_keys", P), ("list_values", P),
        ("list_rows", i64),
        ("n_slots", i32), ("kmax", i32),
        ("cell_sizes", P), ("cell_offsets", P), ("cell_mask", P), ("cell_code", P),
        ("centroids", P), ("sub_centroids", P), ("sub_labels", P), ("n_active", P), ("iters_run", P),
        ("workspace", P), ("workspace_bytes", sz),
        ("status", P), ("phase_ns", P), ("ready_event", P),
    ]


class SelectDesc(ctypes.Structure):
    _fields_ = [
        ("bg", i32), ("G", i32), ("dim", i32), ("n_slots", i32), ("parts", i32), ("kmax", i32),
        ("ks", i32 * 4),
        ("q", P), ("sub_centroids", P), ("cell_code", P), ("cell_sizes", P), ("cell_offsets", P),
        ("cell_mask", P), ("centroids", P), ("cell_dirty", P),
        ("nprobe", i32), ("max_tokens", i32), ("buffer_pages", i32), ("page_size", i32), ("padding_id", i32),
        ("static_len", i32),
        ("delta_cell_ids", P), ("delta_count", P),
        ("delta_capacity", i32), ("exec_capacity", i32),
        ("sel_cells", P), ("sel_count", P), ("kept_count", P), ("row_index", P), ("row_count", P),
        ("scores_out", P), ("phase_ns", P),
        ("slot_bound", i32), ("key_base", i32), ("cand_out", P),
    ]


class AttnDesc(ctypes.Structure):
    _fields_ = [
        ("bg", i32), ("G", i32), ("splits", i32), ("exec_capacity", i32),
        ("scale", f32),
        ("q", P), ("row_index", P), ("row_count", P),
        ("list_keys", P), ("list_values", P), ("list_rows", i64),
        ("static_keys", P), ("static_values", P), ("static_rows", i64),
        ("delta_keys", P), ("delta_values", P), ("delta_rows", i64),
        ("part_o", P), ("part_ml", P), ("out", P), ("counters", P), ("status", P),
        ("o_part", P), ("ml_part", P),
    ]


class MergeDesc(ctypes.Structure):
    _fields_ = [
        ("bg", i32), ("shards", i32), ("cap", i32), ("rank", i32), ("key_base", i32),
        ("cand", P), ("cell_offsets", P), ("n_slots", i32),
        ("nprobe", i32), ("max_tokens", i32), ("buffer_pages", i32), ("page_size", i32),
        ("static_len", i32), ("exec_capacity", i32),
        ("sel_cells", P), ("sel_count", P), ("row_index", P), ("row_count", P),
    ]


class CombineDesc(ctypes.Structure):
    _fields_ = [("shards", i32), ("bg", i32), ("G", i32), ("part_stride", i64), ("o_parts", P), ("ml_parts", P),
                ("out", P)]


class PeerGatherDesc(ctypes.Structure):
    _fields_ = [("world", i32), ("rank", i32), ("bytes", i64), ("src_peers", P), ("flag_peers", P), ("epoch", P),
                ("ticket", P), ("dst", P), ("status", P)]


class AppendDesc(ctypes.Structure):
    _fields_ = [
        ("bg", i32), ("dim", i32),
        ("new_keys", P), ("new_values", P), ("src_head_stride", i64),
        ("zone_keys", P), ("zone_values", P), ("zone_rows", i64),
        ("pos", i32),
        ("batch_keys", P), ("batch_values", P),
        ("batch_cap", i32), ("batch_slot", i32),
    ]


class AsyncDesc(ctypes.Structure):
    _fields_ = [
        ("bg", i32), ("dim", i32), ("n_slots", i32), ("parts", i32), ("kmax", i32), ("batch", i32),
        ("batch_cap", i32), ("threshold", i32), ("ring_cap", i32),
        ("ks", i32 * 4),
        ("batch_keys", P), ("batch_values", P), ("sub_centroids", P), ("cell_code", P),
        ("shadow", P), ("shadow_dirty", P), ("pending", P), ("counts", P), ("delta_counts", P), ("delta_sums", P),
        ("ring_keys", P), ("ring_values", P), ("ring_cell_ids", P), ("ring_write_pos", P), ("ring_count", P),
        ("ids_out", P), ("part_best", P), ("part_chunks", i32), ("ring_store", i32),
    ]


class ApplyDesc(ctypes.Structure):
    _fields_ = [
        ("bg", i32), ("n_slots", i32), ("dim", i32),
        ("shadow", P), ("live", P), ("pending", P), ("live_dirty", P),
    ]


EXPORTS = (
    "imi_abi_version", "imi_last_error", "imi_build_workspace_size", "imi_build_index",
    "imi_query_group_similarities", "imi_select_cells", "imi_sparse_attention", "imi_decode_append",
    "imi_async_assign", "imi_apply_updates", "imi_decode_attend", "imi_decode_layer",
    "imi_merge_candidates", "imi_combine_partials", "imi_sparse_attention_noalloc", "imi_peer_allgather",
)

_lib = None
_lock = threading.Lock()


class IMIError(RuntimeError):
    """A C-ABI call returned a nonzero status."""


def load():
    """Load the library (once).  Raises when it is missing: there is no fallback."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing; build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "or `python adaptiveimi_b200/csrc/build_lib.py`")
        L = ctypes.CDLL(str(LIB_PATH))
        L.imi_abi_version.restype = ctypes.c_int
        L.imi_last_error.restype = ctypes.c_char_p
        L.imi_build_workspace_size.restype = sz
        L.imi_build_workspace_size.argtypes = [i32, i32, i32, i32, P]
        L.imi_build_index.argtypes = [ctypes.POINTER(BuildDesc), P]
        L.imi_query_group_similarities.argtypes = [P, P, P, i32, i32, i32, i32, i64, P]
        L.imi_select_cells.argtypes = [ctypes.POINTER(SelectDesc), P]
        L.imi_sparse_attention.argtypes = [ctypes.POINTER(AttnDesc), P]
        L.imi_decode_append.argtypes = [ctypes.POINTER(AppendDesc), P]
        L.imi_async_assign.argtypes = [ctypes.POINTER(AsyncDesc), P]
        L.imi_apply_updates.argtypes = [ctypes.POINTER(ApplyDesc), P]
        L.imi_sparse_attention_noalloc.argtypes = [ctypes.POINTER(AttnDesc), P]
        L.imi_decode_attend.argtypes = [ctypes.POINTER(SelectDesc), ctypes.POINTER(AttnDesc),
                                        ctypes.POINTER(ApplyDesc), P]
        L.imi_merge_candidates.argtypes = [ctypes.POINTER(MergeDesc), P]
        L.imi_combine_partials.argtypes = [ctypes.POINTER(CombineDesc), P]
        L.imi_peer_allgather.argtypes = [ctypes.POINTER(PeerGatherDesc), P]
        L.imi_decode_layer.argtypes = [ctypes.POINTER(AppendDesc), ctypes.POINTER(AsyncDesc),
                                       ctypes.POINTER(ApplyDesc), ctypes.POINTER(SelectDesc),
                                       ctypes.POINTER(AttnDesc), P]
        if L.imi_abi_version() != 2:
            raise ImportError("libimi_b200.so ABI version mismatch")
        _lib = L
        return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().imi_last_error()
        raise IMIError(f"{what} failed ({status}): {msg.decode() if msg else ''}")
