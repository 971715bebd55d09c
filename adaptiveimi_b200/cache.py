"""``adpimi_cache``: the reference's IMI KV-cache object, device-resident.

Keeps the public surface of ``cache_hub/adaptive_imi`` (``cache.py:43-518``,
``indexing.py:548-628``, ``runtime.py:9-403``, ``retrieval.py:320-602``,
``async_update.py:7-162``) so the reference's model wrappers drive it
unchanged:

* constructor arguments and sizing attributes (``list_capacity``,
  ``static_capacity``, ``n_centroids``, ``nprobe``, ``buffer_size`` ...);
* ``prefill_update_kv_cache`` builds the layer's IMI on the GPU from the
  prefill K/V already in HBM (no host copy) and fills the steady zone;
* ``prepare_cache`` sizes the decode buffers and switches ``attn_func``;
* ``decode_update_kv_cache`` appends the new token (and feeds the optional
  decode-time cell assignment);
* ``attn_func`` / ``sparse_attention`` scores cells, selects them under the
  token budget and page truncation, and attends over the steady zone, the
  selected cells' rows and matching delta rows, all on the device with no host
  synchronisation.

Differences from the reference that do not change results: the IMI lists live
in HBM, so there is no host page cache (every access is what the reference
calls a miss) and ``execution_buffer_*_dict`` hold the per-group execution row
list instead of copied rows; ``valid_lengths_dict`` holds the row counts.
"""
from __future__ import annotations

import ctypes
import math
import os
from typing import Dict, List, Optional

import torch

from . import _lib, ops
from .imi_adapter import IMIPipeline, IMIRuntimeConfig
from .sizing import RetrievalSizes


class adpimi_cache:  # noqa: N801  (reference class name)
    def __init__(self, valid_start, layer_num: int, batch_size: int, max_length: int, num_key_value_heads: int,
                 num_heads: int, head_dim: int, dtype: torch.dtype, layer_mapping: dict, max_new_length: int,
                 input_length: Optional[int], static_pattern_start: int, static_pattern_end: int, core: int,
                 pages_per_cluster: int, retrieval_budget: float, cache_ratio: float, buffer_cluster_num: int,
                 prefill_bsz: int, num_gpus: int, model_size: int, subspace_parts: int = 4,
                 runtime_config: Optional[Dict[str, Dict[str, object]]] = None) -> None:
        # KV_Cache fields (cache_hub/base.py:9-45)
        self.layer_num = layer_num
        self.batch_size = batch_size
        self.max_length = max_length
        self.kv_head = num_key_value_heads
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.layer_mapping = layer_mapping
        self.prefill_bsz = min(prefill_bsz, batch_size)
        self.context = 0
        self.num_gpus = num_gpus
        self.model_size = model_size
        if batch_size != 1:
            raise ValueError("IMI cache currently supports batch_size=1.")
        if dtype != torch.bfloat16:
            raise ValueError("the B200 IMI cache stores bfloat16 K/V")
        if head_dim != 128:
            raise ValueError("the B200 IMI kernels support head_dim 128")
        self.device_list = sorted(set(self.layer_mapping.values()), key=lambda x: int(x.split(":")[-1]))
        self.valid_start_list = valid_start
        self.static_pattern_start = static_pattern_start
        self.static_pattern_end = static_pattern_end
        self.static_pattern_total = static_pattern_start + static_pattern_end
        self.group_size = self.num_heads // self.kv_head
        self.batch_groups = self.batch_size * self.kv_head
        self.page_size = 8
        self.pages_per_cluster = pages_per_cluster
        self.retrieval_budget = retrieval_budget
        self.cache_ratio = cache_ratio
        self.buffer_cluster_num = buffer_cluster_num
        if subspace_parts not in (0, 2, 4):
            raise ValueError("subspace_parts must be 0, 2 or 4")
        self.subspace_parts = subspace_parts
        self.core = core
        runtime_config = runtime_config or {}
        self.runtime_config = {
            "pipeline": dict(runtime_config.get("pipeline") or {}),
            "kmeans": dict(runtime_config.get("kmeans") or {}),
            "async_update": dict(runtime_config.get("async_update") or {}),
            "prefetch": dict(runtime_config.get("prefetch") or {}),
            "retrieval": dict(runtime_config.get("retrieval") or {}),
        }
        self.input_length = int(input_length) if input_length is not None else self.max_length - max_new_length
        self.actual_gen_len = max_new_length - 1
        self.capacity_input_length = int(self.max_length - max_new_length)
        if self.input_length <= 0:
            raise ValueError(f"input length({self.input_length}) should be larger than 0")
        if self.capacity_input_length <= 0:
            raise ValueError(f"capacity input length({self.capacity_input_length}) should be larger than 0")
        self.list_capacity = max(self.capacity_input_length - self.static_pattern_total, 0)
        self.list_stride = max(self.input_length - self.static_pattern_total, 0)
        self.build_index_when_prefilling = self.list_capacity > 0
        if self.build_index_when_prefilling:
            self.static_capacity = self.static_pattern_total + self.actual_gen_len
            self.static_stride = self.static_pattern_total + self.actual_gen_len
        else:
            self.static_capacity = self.capacity_input_length + self.actual_gen_len
            self.static_stride = self.input_length + self.actual_gen_len
        self.static_capacity = max(self.static_capacity, 1)
        # sizing (runtime.py:31-63), fixed at construction from the capacity
        # runtime_config["retrieval"]["fixed_budget"] = False: top-nprobe cells
        # without a token cap (not a reference mode; see RetrievalSizes)
        self.fixed_budget = bool(self.runtime_config["retrieval"].get("fixed_budget", True))
        self.sizes = RetrievalSizes.from_capacity(self.list_capacity, self.subspace_parts, self.retrieval_budget,
                                                  self.buffer_cluster_num, self.static_capacity, self.page_size,
                                                  fixed_budget=self.fixed_budget)
        self.n_centroids = self.sizes.n_centroids
        self.padding_cluster_id = self.sizes.padding_cluster_id
        self.nprobe = self.sizes.nprobe
        self.max_retrieval_tokens = self.sizes.max_retrieval_tokens
        self.budget_tokens = self.max_retrieval_tokens
        self.buffer_size = self.sizes.buffer_size
        self.execution_stride = self.sizes.execution_stride
        self.retrieval_execution_stride = self.buffer_size * self.page_size
        self.max_retrieval_pages = max((self.max_retrieval_tokens + 7) // 8, 1)
        self.cache_size = 0  # no host page cache: lists are HBM-resident
        self.steady_zone_keys: List[torch.Tensor] = []
        self.steady_zone_values: List[torch.Tensor] = []
        for ldx in range(layer_num):
            dev = self.layer_mapping[str(ldx)]
            self.steady_zone_keys.append(torch.zeros((batch_size, self.kv_head, self.static_capacity, head_dim),
                                                     dtype=dtype, device=dev))
            self.steady_zone_values.append(torch.zeros_like(self.steady_zone_keys[-1]))
        self.list_keys: List[Optional[torch.Tensor]] = [None] * layer_num
        self.list_values: List[Optional[torch.Tensor]] = [None] * layer_num
        self.index: List[Optional[ops.IMIIndex]] = [None] * layer_num
        self.imi_pipelines: List[Optional[IMIPipeline]] = []
        # runtime_config["pipeline"]["async_build"] (default off): the device
        # builds run on one side stream per device, next to the prefill.  Off
        # by default: beside a prefill whose GEMMs hold every SM the build gains
        # nothing (bench.py --workload prefill_overlap)
        self.async_build = bool(self.runtime_config["pipeline"].get("async_build", False))
        self._build_streams: Dict[str, torch.cuda.Stream] = {}
        if self.build_index_when_prefilling and self.async_build and torch.cuda.is_available():
            for dev in self.device_list:
                # high priority: the build is a chain of short dependent kernels;
                # pending CTAs of the prefill's long GEMMs must not hold it back
                self._build_streams[dev] = torch.cuda.Stream(device=torch.device(dev), priority=-1)
        if self.build_index_when_prefilling:
            for ldx in range(layer_num):
                self.imi_pipelines.append(IMIPipeline(
                    layer_idx=ldx, kv_heads=self.kv_head, head_dim=head_dim, dtype=dtype,
                    device_id=int(self.layer_mapping[str(ldx)].split(":")[-1]), max_tokens=self.list_capacity,
                    subspace_parts=self.subspace_parts, n_slots=self.n_centroids,
                    build_stream=self._build_streams.get(self.layer_mapping[str(ldx)]),
                    runtime_config=IMIRuntimeConfig(pipeline=self.runtime_config["pipeline"],
                                                    kmeans=self.runtime_config["kmeans"])))
        else:
            self.imi_pipelines = [None] * layer_num
        self.layer_ready = [False] * layer_num
        self.layer_started = [False] * layer_num
        self.cache_prepared = False
        self.attn_func = self.dense_attention
        # async centroid update (async_update.py; off unless enabled)
        acfg = self.runtime_config["async_update"]
        self.async_update_enabled = bool(acfg.get("enabled", False))
        self.async_update_batch = max(int(acfg.get("batch", 16)), 1)
        self.async_update_threshold = max(int(acfg.get("threshold", 16)), 1)
        self.async_update_delta_tokens = max(int(acfg.get("delta_tokens", 512)), 1)
        # The reference's delta ring never receives its rows (async_update.py:151-157
        # copies into a temporary made by tensor indexing), so by default its rows
        # stay zero with padding ids and only its count grows; "store_delta_rows"
        # stores the batch's keys, values and cells instead.
        self.async_update_store_delta_rows = bool(acfg.get("store_delta_rows", False))
        self._async: List[Optional[Dict[str, object]]] = [None] * layer_num
        # per-device decode buffers (filled by prepare_cache)
        self.execution_buffer_keys_dict: Dict[str, torch.Tensor] = {}
        self.execution_buffer_values_dict: Dict[str, torch.Tensor] = {}
        self.valid_lengths_dict: Dict[str, torch.Tensor] = {}
        self._dec: Dict[str, Dict[str, torch.Tensor]] = {}
        self.splits = ops.default_splits(self.batch_groups, self.max_retrieval_tokens + self.static_capacity,
                                          exec_capacity=self.execution_stride)
        # optional measurement hooks (bench.py): per-call row counts and CUDA
        # events around the attention launch, both on the launching stream
        self._pending = None  # deferred append: (layer, k, v, head stride, pos, batch slot, async batch)
        self._fused = False   # set by prepare_cache: appends ride on the layer's attention call
        self._dev_index = [torch.device(self.layer_mapping[str(i)]).index or 0 for i in range(layer_num)]
        self._rc: List[Optional[torch.Tensor]] = [None] * layer_num
        self.row_count_log: Optional[torch.Tensor] = None
        self.attn_event_log: Optional[list] = None
        self._log_pos = 0

    # ------------------------------------------------------------------------
    # prefill (indexing.py:548-611)
    # ------------------------------------------------------------------------
    def prefill_update_kv_cache(self, query_states, key_states, value_states, layer_idx, start_bdx):
        bsz, seq_len, _, _ = key_states.shape
        if bsz != 1:
            raise ValueError("IMI cache currently supports batch_size=1 for prefilling.")
        valid_start = self.valid_start_list[start_bdx]
        if self.build_index_when_prefilling:
            middle_start = valid_start + self.static_pattern_start
            middle_end = seq_len - self.static_pattern_end
            if middle_end - middle_start <= 0:
                raise ValueError("IMI cache requires a non-empty middle segment.")
            if not self.layer_started[layer_idx]:
                pipe = self.imi_pipelines[layer_idx]
                pipe.start_index_chunked(key_states, value_states, middle_start, middle_end, 0)
                self.index[layer_idx] = pipe.index
                self.list_keys[layer_idx] = pipe.index.list_keys.unsqueeze(0)
                self.list_values[layer_idx] = pipe.index.list_values.unsqueeze(0)
                self.layer_started[layer_idx] = True
            end = start_bdx + bsz
            sp = self.static_pattern_start
            zk, zv = self.steady_zone_keys[layer_idx], self.steady_zone_values[layer_idx]
            zk[start_bdx:end, :, :sp] = key_states[:, valid_start:valid_start + sp].transpose(1, 2)
            zv[start_bdx:end, :, :sp] = value_states[:, valid_start:valid_start + sp].transpose(1, 2)
            zk[start_bdx:end, :, sp:self.static_pattern_total] = \
                key_states[:, seq_len - self.static_pattern_end:seq_len].transpose(1, 2)
            zv[start_bdx:end, :, sp:self.static_pattern_total] = \
                value_states[:, seq_len - self.static_pattern_end:seq_len].transpose(1, 2)
        else:
            end = start_bdx + bsz
            self.steady_zone_keys[layer_idx][start_bdx:end, :, :seq_len].copy_(key_states.transpose(1, 2))
            self.steady_zone_values[layer_idx][start_bdx:end, :, :seq_len].copy_(value_states.transpose(1, 2))
        if layer_idx == self.layer_num - 1 and start_bdx + bsz == self.batch_size:
            self.context += seq_len
            if self.build_index_when_prefilling:
                self.attn_func = self.sparse_attention
            else:
                self.static_pattern_total = seq_len
        return key_states[:, valid_start:, :, :], value_states[:, valid_start:, :, :]

    def sync(self, layer_idx, start_bdx):
        if self._pending is not None:
            self._flush_pending()
        return None

    def capture_cuda_graph(self):
        return None

    def ensure_layer_ready(self, layer_idx: int) -> None:
        """Wait for the layer's device build and check it (indexing.py ensure_layer_ready):
        a build whose device status reports a give-up, or whose cell count
        overflows the slots, raises here, before any decode step reads it."""
        if self.layer_ready[layer_idx] or not self.build_index_when_prefilling:
            return
        if not self.layer_started[layer_idx]:
            raise RuntimeError(f"IMI layer {layer_idx} not started")
        self.imi_pipelines[layer_idx].finish_index(as_host_metadata=False)
        self.layer_ready[layer_idx] = True

    # ------------------------------------------------------------------------
    # decode buffers (runtime.py:11-377)
    # ------------------------------------------------------------------------
    def prepare_cache(self, skip_prefetch: bool = False):
        if not self.build_index_when_prefilling:
            return
        if self.cache_prepared:
            return
        bg, G = self.batch_groups, self.group_size
        for dev in self.device_list:
            rows = torch.zeros((bg, self.execution_stride), dtype=torch.int32, device=dev)
            rc = torch.zeros((bg,), dtype=torch.int32, device=dev)
            self._dec[dev] = dict(
                rows=rows, row_count=rc,
                sel=torch.zeros((bg, self.nprobe), dtype=torch.int32, device=dev),
                sel_count=torch.zeros((bg,), dtype=torch.int32, device=dev),
                kept=torch.zeros((bg,), dtype=torch.int32, device=dev),
                part_o=torch.empty((bg, self.splits, G, self.head_dim), dtype=torch.float32, device=dev),
                part_ml=torch.empty((bg, self.splits, G, 2), dtype=torch.float32, device=dev),
                counters=torch.zeros((bg,), dtype=torch.int32, device=dev),
            )
            self.execution_buffer_keys_dict[dev] = rows
            self.execution_buffer_values_dict[dev] = rows
            self.valid_lengths_dict[dev] = rc
        for ldx in range(self.layer_num):
            self.ensure_layer_ready(ldx)
            if self.async_update_enabled:
                self._init_async(ldx)
        self._descs = [self._make_descs(ldx) for ldx in range(self.layer_num)]
        self._rc = [self._dec[self.layer_mapping[str(ldx)]]["row_count"] for ldx in range(self.layer_num)]
        self.attn_func = self.sparse_attention
        self._fused = True
        self.cache_prepared = True

    def _make_descs(self, ldx: int):
        """Per-layer C-ABI descriptors with every constant field filled in; the
        hot path only writes the per-call pointers and lengths."""
        idx = self.index[ldx]
        dev = self.layer_mapping[str(ldx)]
        buf = self._dec[dev]
        st = self._async[ldx] if self.async_update_enabled else None
        bg, G, D = self.batch_groups, self.group_size, self.head_dim
        sel = _lib.SelectDesc()
        sel.bg, sel.G, sel.dim, sel.n_slots, sel.parts, sel.kmax = bg, G, D, idx.n_slots, idx.parts, idx.kmax
        sel.ks = ops._ks4(idx.ks)
        sel.sub_centroids = idx.sub_centroids.data_ptr()
        sel.cell_code, sel.cell_sizes = idx.cell_code.data_ptr(), idx.cell_sizes.data_ptr()
        sel.cell_offsets, sel.cell_mask = idx.cell_offsets.data_ptr(), idx.cell_mask.data_ptr()
        sel.centroids = (st["live"] if st is not None else idx.centroids).data_ptr()
        sel.cell_dirty = st["live_dirty"].data_ptr() if st is not None else None
        sel.nprobe, sel.max_tokens, sel.buffer_pages = self.nprobe, self.max_retrieval_tokens, self.buffer_size
        sel.page_size, sel.padding_id = self.page_size, self.padding_cluster_id
        sel.delta_cell_ids = st["ring_ids"].data_ptr() if st is not None else None
        sel.delta_count = st["ring_count"].data_ptr() if st is not None else None
        sel.delta_capacity = self.async_update_delta_tokens if st is not None else 0
        sel.exec_capacity = self.execution_stride
        sel.sel_cells, sel.sel_count, sel.kept_count = buf["sel"].data_ptr(), buf["sel_count"].data_ptr(), \
            buf["kept"].data_ptr()
        sel.row_index = buf["rows"].data_ptr()
        # every slot at or above the largest n_active is padding: one host read
        # per layer, here at preparation, lets the selection skip them
        sel.slot_bound = int(idx.n_active.max().item())
        att = _lib.AttnDesc()
        att.bg, att.G, att.splits, att.exec_capacity = bg, G, self.splits, self.execution_stride
        att.scale = 1.0 / math.sqrt(D)
        att.row_index = buf["rows"].data_ptr()
        att.list_keys, att.list_values, att.list_rows = idx.list_keys.data_ptr(), idx.list_values.data_ptr(), \
            idx.list_keys.shape[1]
        zk = self.steady_zone_keys[ldx]
        att.static_keys, att.static_values = zk.data_ptr(), self.steady_zone_values[ldx].data_ptr()
        att.static_rows = self.static_capacity
        if st is not None:
            att.delta_keys, att.delta_values = st["ring_keys"].data_ptr(), st["ring_values"].data_ptr()
            att.delta_rows = self.async_update_delta_tokens
        att.part_o, att.part_ml = buf["part_o"].data_ptr(), buf["part_ml"].data_ptr()
        att.counters = buf["counters"].data_ptr()
        app = None
        if st is not None:
            app = _lib.ApplyDesc()
            app.bg, app.n_slots, app.dim = bg, idx.n_slots, D
            app.shadow, app.live = st["shadow"].data_ptr(), st["live"].data_ptr()
            app.pending, app.live_dirty = st["pending"].data_ptr(), st["live_dirty"].data_ptr()
        ap = _lib.AppendDesc()
        ap.bg, ap.dim = bg, D
        ap.zone_keys, ap.zone_values, ap.zone_rows = zk.data_ptr(), self.steady_zone_values[ldx].data_ptr(), \
            self.static_capacity
        if st is not None:
            ap.batch_keys, ap.batch_values = st["batch_keys"].data_ptr(), st["batch_values"].data_ptr()
            ap.batch_cap = self.async_update_batch
        asd = None
        if st is not None:
            asd = _lib.AsyncDesc()
            asd.bg, asd.dim, asd.n_slots, asd.parts, asd.kmax = bg, D, idx.n_slots, idx.parts, idx.kmax
            asd.batch, asd.batch_cap = self.async_update_batch, self.async_update_batch
            asd.threshold, asd.ring_cap = self.async_update_threshold, self.async_update_delta_tokens
            asd.ks = ops._ks4(idx.ks)
            asd.batch_keys, asd.batch_values = st["batch_keys"].data_ptr(), st["batch_values"].data_ptr()
            asd.sub_centroids, asd.cell_code = idx.sub_centroids.data_ptr(), idx.cell_code.data_ptr()
            asd.shadow, asd.shadow_dirty, asd.pending = st["shadow"].data_ptr(), st["shadow_dirty"].data_ptr(), \
                st["pending"].data_ptr()
            asd.counts, asd.delta_counts = st["counts"].data_ptr(), st["delta_counts"].data_ptr()
            asd.delta_sums = st["delta_sums"].data_ptr()
            asd.ring_keys, asd.ring_values = st["ring_keys"].data_ptr(), st["ring_values"].data_ptr()
            asd.ring_cell_ids, asd.ring_write_pos = st["ring_ids"].data_ptr(), st["ring_pos"].data_ptr()
            asd.ring_count = st["ring_count"].data_ptr()
            asd.ring_store = 1 if self.async_update_store_delta_rows else 0
            asd.part_best, asd.part_chunks = st["part_best"].data_ptr(), ops.async_chunks(idx.n_slots)
        return dict(sel=sel, att=att, app=app, append=ap, **{"async": asd})

    def _init_async(self, ldx: int) -> None:
        idx = self.index[ldx]
        if idx is None:
            return
        dev = idx.centroids.device
        bg, ns, D, R = self.batch_groups, idx.n_slots, self.head_dim, self.async_update_delta_tokens
        self._async[ldx] = dict(
            live=idx.centroids, shadow=idx.centroids.clone(),
            shadow_dirty=torch.zeros((bg, ns), dtype=torch.uint8, device=dev),
            pending=torch.zeros((bg, ns), dtype=torch.uint8, device=dev),
            live_dirty=torch.zeros((bg, ns), dtype=torch.uint8, device=dev),
            counts=idx.cell_sizes.clone(),
            delta_counts=torch.zeros((bg, ns), dtype=torch.int32, device=dev),
            delta_sums=torch.zeros((bg, ns, D), dtype=torch.float32, device=dev),
            batch_keys=torch.zeros((bg, self.async_update_batch, D), dtype=self.dtype, device=dev),
            batch_values=torch.zeros((bg, self.async_update_batch, D), dtype=self.dtype, device=dev),
            ring_keys=torch.zeros((bg, R, D), dtype=self.dtype, device=dev),
            ring_values=torch.zeros((bg, R, D), dtype=self.dtype, device=dev),
            ring_ids=torch.full((bg, R), self.padding_cluster_id, dtype=torch.int32, device=dev),
            ring_pos=torch.zeros((bg,), dtype=torch.int32, device=dev),
            ring_count=torch.zeros((bg,), dtype=torch.int32, device=dev),
            part_best=torch.empty((bg, ops.async_chunks(ns), self.async_update_batch), dtype=torch.int64,
                                  device=dev),
            count=0, pending_flag=False,
        )

    # ------------------------------------------------------------------------
    # decode (runtime.py:378-392, async_update.py:77-162)
    # ------------------------------------------------------------------------
    def decode_update_kv_cache(self, key_states, value_states, layer_idx):
        """key_states/value_states: [B, 1, kv_heads, D].

        Once the cache is prepared the append is deferred: ``attn_func`` issues
        it together with the layer's selection and attention in one
        ``imi_decode_layer`` call (same stream order as two calls).  Any other
        entry point issues a deferred append first."""
        if self._pending is not None:
            self._flush_pending()
        st = self._async[layer_idx] if self.async_update_enabled else None
        nk, nv, stride = self._kv_rows(key_states, value_states)
        pos = self.static_pattern_total
        slot = st["count"] if st is not None else 0
        batch = 0
        if st is not None:
            st["count"] += 1
            if st["count"] >= self.async_update_batch:
                batch = st["count"]
                st["count"] = 0
                st["pending_flag"] = "scheduled"
        rec = (layer_idx, nk, nv, stride, pos, slot, batch)
        if self._fused:
            self._pending = rec
        else:
            self._issue_append(rec)
        if layer_idx == self.layer_num - 1:
            self.context += 1
            self.static_pattern_total += 1
        return None, None

    def _kv_rows(self, key_states, value_states):
        """Base tensors and head stride (elements) of the new token's K/V rows;
        a layout the kernels cannot read in place is copied first."""
        if key_states.shape[0] != 1:
            raise ValueError("decode_update_kv_cache: batch_size 1 only")
        ks, vs = key_states, value_states
        if ks.stride(-1) != 1 or vs.stride(-1) != 1 or ks.stride(2) != vs.stride(2):
            ks, vs = ks.contiguous(), vs.contiguous()
        return ks, vs, ks.stride(2)

    def _fill_append(self, rec):
        layer_idx, nk, nv, stride, pos, slot, batch = rec
        ap = self._descs[layer_idx]["append"] if self.cache_prepared else None
        if ap is None:
            ap = _lib.AppendDesc()
            ap.bg, ap.dim = self.batch_groups, self.head_dim
            ap.zone_keys = self.steady_zone_keys[layer_idx].data_ptr()
            ap.zone_values = self.steady_zone_values[layer_idx].data_ptr()
            ap.zone_rows = self.static_capacity
        ap.new_keys, ap.new_values, ap.src_head_stride = nk.data_ptr(), nv.data_ptr(), stride
        ap.pos = pos
        ap.batch_slot = slot
        return ap

    def _issue_append(self, rec) -> None:
        """Append (and the batched cell assignment when one is due) as their own calls."""
        layer_idx, batch = rec[0], rec[6]
        ap = self._fill_append(rec)
        stream = ctypes.c_void_p(self._stream(layer_idx))
        L = _lib.load()
        _lib.check(L.imi_decode_append(ctypes.byref(ap), stream), "imi_decode_append")
        if batch:
            asd = self._descs[layer_idx]["async"]
            asd.batch = batch
            _lib.check(L.imi_async_assign(ctypes.byref(asd), stream), "imi_async_assign")

    def _flush_pending(self) -> None:
        rec, self._pending = self._pending, None
        if rec is not None:
            self._issue_append(rec)

    def _stream(self, layer_idx: int) -> int:
        return torch._C._cuda_getCurrentRawStream(self._dev_index[layer_idx])

    def _apply_async_centroid_updates(self, layer_idx: int) -> None:
        """Publish the shadow centroids updated by an earlier decode step
        (async_update.py:7-19).  An update scheduled at step t becomes visible at
        the layer's next visit after that step's attention."""
        st = self._async[layer_idx]
        if st is None:
            return
        if st["pending_flag"] == "ready":
            ops.apply_updates(shadow=st["shadow"], live=st["live"], pending=st["pending"],
                              live_dirty=st["live_dirty"])
            st["pending_flag"] = False

    def sparse_attention(self, queries, layer_idx, static_len):
        """retrieval.py:320-602: cell scores, selection under the token budget and
        page truncation, and attention over [steady zone | selected rows | delta
        rows], issued with the layer's deferred append (and, when due, the
        batched cell assignment and centroid publish) as one C-ABI call
        (imi_decode_layer)."""
        if not self.layer_ready[layer_idx]:
            self.ensure_layer_ready(layer_idx)
        q = queries if queries.is_contiguous() else queries.contiguous()
        d = self._descs[layer_idx]
        sel, att = d["sel"], d["att"]
        app_ref = as_ref = None
        rec = self._pending
        if rec is not None:
            if rec[0] == layer_idx:
                self._pending = None
                app_ref = ctypes.byref(self._fill_append(rec))
                if rec[6]:
                    asd = d["async"]
                    asd.batch = rec[6]
                    as_ref = ctypes.byref(asd)
            else:
                self._flush_pending()
        st = self._async[layer_idx] if self.async_update_enabled else None
        apply = None
        if st is not None and st["pending_flag"] == "ready":
            apply = ctypes.byref(d["app"])
            st["pending_flag"] = False
        rc = self._rc[layer_idx]
        if self.row_count_log is not None and self._log_pos < self.row_count_log.shape[0]:
            rc = self.row_count_log[self._log_pos]
            self._log_pos += 1
        out = torch.empty((self.batch_size, 1, self.num_heads, self.head_dim), dtype=self.dtype, device=q.device)
        qp, rcp = q.data_ptr(), rc.data_ptr()
        sel.q = att.q = qp
        sel.row_count = att.row_count = rcp
        sel.static_len = int(static_len)
        att.out = out.data_ptr()
        ev = None
        if self.attn_event_log is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        stream = ctypes.c_void_p(self._stream(layer_idx))
        _lib.check(_lib.load().imi_decode_layer(app_ref, as_ref, apply, ctypes.byref(sel), ctypes.byref(att), stream),
                   "imi_decode_layer")
        if ev is not None:
            ev[1].record()
            self.attn_event_log.append(ev)
        if st is not None and st["pending_flag"] == "scheduled":
            st["pending_flag"] = "ready"
        return out

    def dense_attention(self, queries, layer_idx, static_len):
        """Attention over the first ``static_len`` steady-zone rows (runtime.py:393-403)."""
        if self._pending is not None:
            self._flush_pending()
        dev = queries.device
        bg, G, D = self.batch_groups, self.group_size, self.head_dim
        n = int(static_len) if not torch.is_tensor(static_len) else int(static_len.max())
        rows = torch.arange(n, dtype=torch.int32, device=dev).bitwise_or_(1 << 30).expand(bg, n).contiguous()
        rc = torch.full((bg,), n, dtype=torch.int32, device=dev)
        q = queries.reshape(bg, G, D).contiguous()
        out = torch.empty((bg, G, D), dtype=self.dtype, device=dev)
        splits = ops.default_splits(bg, n)
        zk = self.steady_zone_keys[layer_idx].view(bg, self.static_capacity, D)
        zv = self.steady_zone_values[layer_idx].view(bg, self.static_capacity, D)
        ops.sparse_attention(q=q, row_index=rows, row_count=rc, list_keys=zk, list_values=zv, static_keys=zk,
                             static_values=zv, out=out,
                             part_o=torch.empty((bg, splits, G, D), dtype=torch.float32, device=dev),
                             part_ml=torch.empty((bg, splits, G, 2), dtype=torch.float32, device=dev), splits=splits)
        return out.view(self.batch_size, 1, self.num_heads, self.head_dim)

    # ------------------------------------------------------------------------
    # lifecycle (cache.py:380-454, indexing.py:453-542)
    # ------------------------------------------------------------------------
    def can_reuse_for_next_sequence(self, valid_start, max_new_length: int, input_length: int) -> bool:
        new_list_stride = max(int(input_length) - self.static_pattern_start - self.static_pattern_end, 0)
        if new_list_stride > self.list_capacity:
            return False
        new_static = self.static_pattern_start + self.static_pattern_end + int(max_new_length) - 1
        if new_static > self.static_capacity:
            return False
        return len(valid_start) == len(self.valid_start_list)

    def reset_for_next_sequence(self, valid_start, max_new_length: int, input_length: int) -> None:
        if not self.can_reuse_for_next_sequence(valid_start, max_new_length, input_length):
            raise ValueError("AdaptiveIMI cache shape mismatch; cannot reuse across samples")
        if self._pending is not None:
            self._flush_pending()
        self._fused = False
        self.valid_start_list = valid_start
        self.input_length = int(input_length)
        self.actual_gen_len = int(max_new_length) - 1
        self.list_stride = max(self.input_length - self.static_pattern_start - self.static_pattern_end, 0)
        self.static_pattern_total = self.static_pattern_start + self.static_pattern_end
        self.context = 0
        self.attn_func = self.dense_attention
        self.layer_ready = [False] * self.layer_num
        self.layer_started = [False] * self.layer_num
        self.cache_prepared = False
        self._async = [None] * self.layer_num

    def cleanup(self) -> None:
        self._pending = None
        self._fused = False
        for p in self.imi_pipelines:
            if p is not None:
                p.close()
        self.index = [None] * self.layer_num
        self.list_keys = [None] * self.layer_num
        self.list_values = [None] * self.layer_num
        self._async = [None] * self.layer_num
        self._dec.clear()
