"""Device-side replacement of the reference's IMI build adapter.

Mirrors ``library/AdaptiveIMI/imi_adapter.py`` (``IMIPipeline`` :129-479,
``IMIRuntimeConfig`` :123-126, ``get_imi_kernels`` :114-120): the same method
names, argument meaning and errors, with the build running on the GPU from the
K/V that are already in HBM instead of a D2H copy and CPU k-means
(``LayerPipeline``, layer_pipeline.cpp:430-1401).

Stages follow ``PipelineStage`` (layer_pipeline.hpp:32-40); ``get_pipeline_stats``
keeps the reference's keys (``PipelineStats``, layer_pipeline.hpp:42-53) with the
host-copy stages at zero; ``kmeans_ms`` and ``reorganize_ms`` come from device
timestamps the build takes between its stages on the stream.  A build whose
device status word reports a give-up (or whose cells overflow the slots) goes to
``PipelineStage.Failed`` and ``finish_index`` raises ``RuntimeError``.
"""
from __future__ import annotations

import contextlib
import enum
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch

from . import ops
from .sizing import adaptive_k


class PipelineStage(enum.IntEnum):
    Idle = 0
    Transferring = 1
    Clustering = 2
    Reorganizing = 3
    Writing = 4
    Complete = 5
    Failed = 255


@dataclass
class IMIRuntimeConfig:
    pipeline: Dict[str, object] = field(default_factory=dict)
    kmeans: Dict[str, object] = field(default_factory=dict)


def _kmeans_settings(cfg: Dict[str, object]) -> Dict[str, object]:
    """kmeans sub-dict -> build settings with the reference defaults
    (LayerPipelineRuntimeConfig, layer_pipeline.hpp:142-160)."""
    return dict(
        max_iters=max(1, int(cfg.get("max_iters", 25))),
        tol=max(float(cfg.get("tol", 5e-4)), 0.0),
        early_stop_min_iter=max(1, int(cfg.get("early_stop_min_iter", 5))),
        early_stop_rel_tol=max(float(cfg.get("early_stop_rel_tol", 5e-4)), 0.0),
    )


class _Kernels:
    """``get_imi_kernels()`` result: the device scorer (no CPU fallback)."""

    fused_query_group_similarities = staticmethod(ops.fused_query_group_similarities)


def get_imi_kernels():
    return _Kernels()


@dataclass
class IMIPipeline:
    layer_idx: int
    kv_heads: int
    head_dim: int
    dtype: torch.dtype
    device_id: int
    max_tokens: int
    subspace_parts: int = 2
    runtime_config: IMIRuntimeConfig = field(default_factory=IMIRuntimeConfig)
    enable_direct_write: bool = True
    n_slots: Optional[int] = None
    # a side stream for the build: the build waits for the producer's stream
    # (an event) and then runs next to it, so the prefill of later layers
    # overlaps this layer's k-means (the reference overlaps its host k-means
    # the same way, layer_pipeline.cpp:430-700).  None: the build runs on the
    # caller's stream.
    build_stream: Optional[torch.cuda.Stream] = None

    def __post_init__(self) -> None:
        if self.subspace_parts not in (0, 2, 4):
            raise ValueError("subspace_parts must be 0, 2 or 4")
        self.stage = PipelineStage.Idle
        self.error_message = ""
        self._token_count: Optional[int] = None
        self._keys = None
        self._values = None
        self._staging: Optional[Tuple[torch.Tensor, torch.Tensor]] = None
        self._chunks_seen = 0
        self._done_event: Optional[torch.cuda.Event] = None
        self._status: Optional[torch.Tensor] = None
        self._phase_ns: Optional[torch.Tensor] = None
        self.index: Optional[ops.IMIIndex] = None
        self._last_pipeline_stats: Optional[Dict[str, object]] = None
        self._batch_allocate_cpu_buffer_callback = None
        self._worker_threads = 0

    # -- reference-compatible knobs -------------------------------------------------
    def set_batch_allocate_cpu_buffer_callback(self, callback) -> None:
        self._batch_allocate_cpu_buffer_callback = callback

    def set_worker_threads(self, worker_threads: int) -> None:
        if int(worker_threads) < 1:
            raise ValueError("worker_threads must be >= 1")
        self._worker_threads = int(worker_threads)  # the device build has no CPU workers

    def cancel_pipeline(self) -> None:
        """Drop any build in flight (the launched kernels still retire on the stream)."""
        self._keys = self._values = None
        self._staging = None
        self._token_count = None
        self._done_event = None
        self.stage = PipelineStage.Idle

    def close(self) -> None:
        self.cancel_pipeline()
        self._batch_allocate_cpu_buffer_callback = None
        self.index = None

    # -- build ----------------------------------------------------------------------
    def _device(self) -> torch.device:
        return torch.device("cuda", self.device_id)

    def _ks(self, token_count: int) -> Tuple[int, ...]:
        return adaptive_k(token_count, self.subspace_parts, kmeans_cfg=self.runtime_config.kmeans)

    def _launch(self, keys: torch.Tensor, values: torch.Tensor, list_keys=None, list_values=None) -> None:
        """keys/values: [kv_heads, n, D] views (last dim contiguous) on the device."""
        n = keys.shape[1]
        ks = self._ks(n)
        n_slots = self.n_slots
        if n_slots is None:
            prod = 1
            for k in ks:
                prod *= k
            n_slots = prod + 1
        settings = _kmeans_settings(self.runtime_config.kmeans)
        self.stage = PipelineStage.Clustering
        self.error_message = ""
        dev = self._device()
        # device status word (bit 0: an E-step wait gave up) and the stage
        # timestamps (k-means start / end, reorganize end), read at finish
        self._status = torch.zeros((1,), dtype=torch.int32, device=dev)
        self._phase_ns = torch.zeros((3,), dtype=torch.int64, device=dev)
        self._done_event = torch.cuda.Event()
        side = self.build_stream
        with torch.cuda.device(dev):
            ready = None
            if side is not None:  # keys/values (and the words above) are ready once the caller's stream gets here
                ready = torch.cuda.Event()
                ready.record(torch.cuda.current_stream(dev))
            try:
                with torch.cuda.stream(side) if side is not None else contextlib.nullcontext():
                    self.index = ops.build_index(keys, values, parts=self.subspace_parts, ks=ks, n_slots=n_slots,
                                                 list_keys=list_keys, list_values=list_values, status=self._status,
                                                 phase_ns=self._phase_ns, ready_event=ready, **settings)
                    self._done_event.record()
            except Exception as exc:  # mark_failure (layer_pipeline.cpp:232-236)
                self._mark_failure(str(exc))
                raise RuntimeError(f"IMI pipeline failed: {exc}") from exc
            if side is not None:
                # the producer's tensors (and the words it zeroed) are in use on
                # the side stream until the build is done
                for t in (keys, values, self._status, self._phase_ns, list_keys, list_values):
                    if t is not None:
                        t.record_stream(side)
        self._token_count = n

    def _mark_failure(self, message: str) -> None:
        """layer_pipeline.cpp:232-236: keep the message, stage Failed."""
        self.error_message = message
        self.stage = PipelineStage.Failed

    def _check_device_result(self) -> None:
        """After the build's event: a set status bit or an overflowing cell
        count voids the index (the reference's merge path raises on a head
        whose k-means result is missing, layer_pipeline.cpp:360-402)."""
        st = int(self._status.item())
        if st & 1:
            self._mark_failure("IMI build: a tensor-core E-step wait gave up (device status 0x%x); "
                               "the index is not valid" % st)
            return
        na = int(self.index.n_active.max().item())
        if na > self.index.n_slots - 1:
            self._mark_failure(f"IMI build produced {na} cells for {self.index.n_slots} slots")

    def build_index(self, keys, values, list_keys=None, list_values=None) -> List[Dict[str, object]]:
        self.start_index(keys, values, list_keys, list_values)
        return self.finish_index(list_keys, list_values)

    def start_index(self, keys: torch.Tensor, values: torch.Tensor, list_keys=None, list_values=None) -> None:
        if keys.dim() != 4 or values.dim() != 4:
            raise ValueError("keys/values must be [1, kv_heads, tokens, head_dim]")
        if keys.size(0) != 1 or values.size(0) != 1:
            raise ValueError("IMI pipeline supports batch_size=1")
        if keys.size() != values.size():
            raise ValueError("keys and values must share the same shape")
        if keys.size(1) != self.kv_heads:
            raise ValueError("kv_heads mismatch in IMI pipeline")
        token_count = int(keys.size(2))
        if token_count <= 0:
            raise ValueError("IMI pipeline requires non-empty middle tokens")
        if token_count > self.max_tokens:
            raise ValueError(f"token_count({token_count}) exceeds max_tokens({self.max_tokens})")
        self._launch(keys[0].to(self._device()), values[0].to(self._device()), list_keys, list_values)

    def begin_index_stream(self, token_count: int, submit_chunk_size: int) -> None:
        if token_count <= 0:
            raise ValueError("IMI pipeline requires non-empty middle tokens")
        if token_count > self.max_tokens:
            raise ValueError(f"token_count({token_count}) exceeds max_tokens({self.max_tokens})")
        if submit_chunk_size <= 0:
            raise ValueError("submit_chunk_size must be positive")
        dev = self._device()
        self._staging = (torch.empty((self.kv_heads, token_count, self.head_dim), dtype=torch.bfloat16, device=dev),
                         torch.empty((self.kv_heads, token_count, self.head_dim), dtype=torch.bfloat16, device=dev))
        self._token_count = token_count
        self._chunks_seen = 0
        self.stage = PipelineStage.Transferring

    def submit_index_stream_chunk(self, chunk_keys, chunk_values, chunk_id: int, token_offset: int,
                                  is_last: bool) -> None:
        if chunk_keys.dim() != 4 or chunk_values.dim() != 4:
            raise ValueError("chunk keys/values must be [1, kv_heads, tokens, head_dim]")
        if chunk_keys.size(0) != 1 or chunk_values.size(0) != 1:
            raise ValueError("IMI pipeline supports batch_size=1")
        if chunk_keys.size() != chunk_values.size():
            raise ValueError("chunk keys and values must share the same shape")
        if chunk_keys.size(1) != self.kv_heads:
            raise ValueError("kv_heads mismatch in IMI pipeline")
        if chunk_id < 0:
            raise ValueError("chunk_id must be non-negative")
        if token_offset < 0:
            raise ValueError("token_offset must be non-negative")
        if self._staging is None:
            raise RuntimeError("IMI pipeline failed to submit chunk")
        sk, sv = self._staging
        t = chunk_keys.size(2)
        if token_offset + t > sk.shape[1]:
            raise RuntimeError("IMI pipeline failed to submit chunk")
        sk[:, token_offset:token_offset + t].copy_(chunk_keys[0])
        sv[:, token_offset:token_offset + t].copy_(chunk_values[0])
        self._chunks_seen += 1
        if is_last:
            self._launch(sk, sv)

    def start_index_chunked(self, key_states, value_states, middle_start: int, middle_end: int, chunk_size: int):
        """key_states: [1, seq_len, kv_heads, head_dim]; builds straight from the
        strided view of the middle range (no transpose copy, no host copy)."""
        if key_states.dim() != 4 or value_states.dim() != 4:
            raise ValueError("key_states/value_states must be [1, seq_len, kv_heads, head_dim]")
        if key_states.size(0) != 1 or value_states.size(0) != 1:
            raise ValueError("IMI pipeline supports batch_size=1")
        if key_states.size() != value_states.size():
            raise ValueError("key_states and value_states must share the same shape")
        if key_states.size(2) != self.kv_heads:
            raise ValueError("kv_heads mismatch in IMI pipeline")
        seq_len = int(key_states.size(1))
        if middle_start < 0 or middle_end > seq_len or middle_start >= middle_end:
            raise ValueError("Invalid middle token range for IMI chunked build")
        if middle_end - middle_start > self.max_tokens:
            raise ValueError(f"token_count({middle_end - middle_start}) exceeds max_tokens({self.max_tokens})")
        kv = key_states[0, middle_start:middle_end].transpose(0, 1)
        vv = value_states[0, middle_start:middle_end].transpose(0, 1)
        self._launch(kv, vv)
        return [(kv, vv)]

    def build_index_chunked(self, key_states, value_states, middle_start, middle_end, list_keys, list_values,
                            chunk_size):
        self.start_index_chunked(key_states, value_states, middle_start, middle_end, chunk_size)
        return self.finish_index(list_keys, list_values)

    def wait_ready(self, timeout_sec: float) -> bool:
        """True once the device build has completed and passed its checks;
        False on timeout, before any build, or when the build failed
        (layer_pipeline.cpp:121-137 returns the ready flag, which a failure
        never sets)."""
        if self._done_event is None or self.stage == PipelineStage.Failed:
            return False
        deadline = time.monotonic() + max(0.0, float(timeout_sec))
        while not self._done_event.query():
            if time.monotonic() > deadline:
                return False
            time.sleep(0.0005)
        if self.stage not in (PipelineStage.Complete, PipelineStage.Failed):
            self._check_device_result()
            if self.stage != PipelineStage.Failed:
                self.stage = PipelineStage.Complete
        return self.stage == PipelineStage.Complete

    def finish_index(self, list_keys=None, list_values=None, as_host_metadata: bool = True):
        token_count = self._token_count
        if token_count is None or self.index is None:
            raise RuntimeError("IMI pipeline finish called before start")
        if not self.wait_ready(timeout_sec=max(60.0, token_count / 1024.0 * 5.0)):
            if self.stage == PipelineStage.Failed:
                raise RuntimeError(f"IMI pipeline failed: {self.error_message}")
            raise RuntimeError("IMI pipeline did not finish in time")
        t = [int(x) for x in self._phase_ns.tolist()]
        kmeans_ms = max(0, t[1] - t[0]) / 1e6
        reorganize_ms = max(0, t[2] - t[1]) / 1e6
        idx = self.index
        # PipelineStats keys (layer_pipeline.hpp:42-53).  The host-copy stages
        # do not exist in a device build (0); the reorganize kernels write the
        # list rows directly, so write_ms is part of reorganize_ms.
        self._last_pipeline_stats = {
            "d2h_ms": 0.0, "cpu_copy_ms": 0.0, "kmeans_ms": kmeans_ms, "kmeans_cpu_time_ms": 0.0,
            "kmeans_cpu_util_cores": 0.0, "reorganize_ms": reorganize_ms, "write_ms": 0.0, "kmeans_gate_wait_ms": 0,
            "total_chunks": max(1, self._chunks_seen), "total_tokens": int(token_count),
            "build_ms": kmeans_ms + reorganize_ms,
        }
        if self.build_stream is not None:
            # the index was allocated on the build stream and is read on the
            # caller's stream from here on
            cur = torch.cuda.current_stream(self._device())
            for name in ("list_keys", "list_values", "cell_sizes", "cell_offsets", "cell_mask", "cell_code",
                         "centroids", "sub_centroids", "sub_labels", "n_active", "iters_run"):
                getattr(idx, name).record_stream(cur)
        if list_keys is not None and list_values is not None and list_keys.data_ptr() != idx.list_keys.data_ptr():
            list_keys[0, :, :token_count].copy_(idx.list_keys)
            list_values[0, :, :token_count].copy_(idx.list_values)
        if not as_host_metadata:
            return idx
        na = idx.n_active.cpu()
        out = []
        for h in range(self.kv_heads):
            c = int(na[h])
            out.append({
                "head_idx": h,
                "cluster_sizes": idx.cell_sizes[h, :c].cpu(),
                "cluster_offsets": idx.cell_offsets[h, :c + 1].cpu(),
                "centroids": idx.centroids[h, :c].cpu(),
            })
        return out

    def get_pipeline_stats(self) -> Dict[str, object]:
        return dict(self._last_pipeline_stats or {})

    def get_last_pipeline_stats(self) -> Optional[Dict[str, object]]:
        return None if self._last_pipeline_stats is None else dict(self._last_pipeline_stats)
