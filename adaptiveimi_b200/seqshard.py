"""Sequence sharding of the IMI decode path.

The reference cache lives on one GPU.  For contexts too long for one GPU (and
for more GPUs than KV heads) the middle tokens of the sequence are split into
N contiguous shards, one per GPU.  Each shard builds its own IMI over its
tokens (the reference's adaptive k for the shard's length), and decode runs
this algorithm:

1. every shard scores its cells and selects locally under the *global* rules
   (nprobe, token budget and page budget of the whole context) with ranking
   keys that carry a global cell id (shard offset + slot), so every shard
   orders ties alike.  A shard's part of the global selection is a prefix of
   its own order, so this local selection covers it; the shard also reports
   its stop marker (the highest-ranked cell it left out) so the merge stops
   exactly where the global order stops;
2. the candidate records are all-gathered (one NCCL all-gather of
   ``[bg, 2 * (nprobe + 1) + 1]`` u64 per shard);
3. every shard runs the same merge (the selection's boundary search over the
   union), keeps its own cells above the global boundary and writes its row
   list; the steady zone (static prefix/suffix and appended tokens) belongs to
   shard 0 only;
4. every shard attends over its rows and writes unnormalised (m, l, o)
   partials; these are all-gathered (one NCCL all-gather of ``[bg, G, 130]``
   f32 per shard) and combined by log-sum-exp into the output on every shard.

With one shard the result equals the unsharded path.  The decode-time
centroid update (async assignment) is not used in this mode: a new key's cell
would need a global argmax across shards.

``decode_step`` runs either with one shard per process (``torch.distributed``
initialised, NCCL all-gathers) or with every shard in one process (the
exchange is a tensor that all shards write into), which the single-GPU tests
use.  Limits of the on-chip selection apply: nprobe <= 16384 and shard slots
<= 16384.  The merge keeps up to 8192 candidates (shards * (nprobe + 1)) in
shared memory and searches larger sets in the gathered records directly.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

from . import _lib, ops
from .sizing import RetrievalSizes, adaptive_k


@dataclass(frozen=True)
class ShardPlan:
    shards: int
    n_total: int                 # middle tokens over all shards
    starts: tuple                # middle-token offset of each shard
    lengths: tuple               # middle tokens of each shard
    ks: tuple                    # per-shard k per subspace
    n_slots: tuple               # per-shard slots (padding slot last)
    key_base: tuple              # per-shard global cell-id offset
    parts: int
    nprobe: int                  # the global rules
    max_tokens: int
    buffer_pages: int
    page_size: int

    @property
    def cap(self) -> int:
        return self.nprobe + 1

    @property
    def record(self) -> int:
        return 2 * self.cap + 1


def plan_shards(n_total: int, shards: int, parts: int, retrieval_budget: float, buffer_cluster_num: int,
                page_size: int = 8, kmeans_cfg: Optional[dict] = None) -> ShardPlan:
    """Contiguous shards of the middle tokens and the global selection rules
    (the unsharded context's nprobe, token budget and page budget)."""
    if shards < 1 or n_total < shards:
        raise ValueError(f"cannot split {n_total} tokens into {shards} shards")
    base = n_total // shards
    lengths = [base + (1 if r < n_total % shards else 0) for r in range(shards)]
    starts = [sum(lengths[:r]) for r in range(shards)]
    glob = RetrievalSizes.from_capacity(n_total, parts, retrieval_budget, buffer_cluster_num, 0, page_size)
    ks, slots = [], []
    for n in lengths:
        ks.append(tuple(adaptive_k(n, parts, kmeans_cfg=kmeans_cfg)))
        slots.append(RetrievalSizes.from_capacity(n, parts, retrieval_budget, buffer_cluster_num, 0,
                                                  page_size).n_centroids)
    key_base = [sum(slots[:r]) for r in range(shards)]
    if glob.nprobe > 16384:
        raise ValueError(f"global nprobe {glob.nprobe} > 16384 is beyond the on-chip selection")
    if max(slots) > 16384:
        raise ValueError(f"{max(slots)} slots per shard > 16384: use more shards")
    return ShardPlan(shards=shards, n_total=n_total, starts=tuple(starts), lengths=tuple(lengths), ks=tuple(ks),
                     n_slots=tuple(slots), key_base=tuple(key_base), parts=parts, nprobe=glob.nprobe,
                     max_tokens=glob.max_retrieval_tokens, buffer_pages=glob.buffer_size, page_size=page_size)


class SeqShard:
    """One shard of one layer: its IMI and its decode buffers."""

    def __init__(self, plan: ShardPlan, rank: int, kv_heads: int, G: int, static_capacity: int,
                 device: torch.device):
        self.plan, self.rank, self.bg, self.G = plan, rank, kv_heads, G
        self.dev = torch.device(device)
        self.static_capacity = static_capacity
        # rows this shard may attend: its selected cells, plus the steady zone on shard 0
        self.exec_capacity = plan.buffer_pages * plan.page_size + (static_capacity if rank == 0 else 0)
        self.splits = ops.default_splits(kv_heads, plan.max_tokens + (static_capacity if rank == 0 else 0),
                                         exec_capacity=self.exec_capacity)
        self.index: Optional[ops.IMIIndex] = None
        bg, dev = kv_heads, self.dev
        i32 = torch.int32
        self.cand = torch.zeros((bg, plan.record), dtype=torch.int64, device=dev)
        self.sel = torch.zeros((bg, plan.nprobe), dtype=i32, device=dev)
        self.sel_count = torch.zeros((bg,), dtype=i32, device=dev)
        self.rows = torch.zeros((bg, self.exec_capacity), dtype=i32, device=dev)
        self.row_count = torch.zeros((bg,), dtype=i32, device=dev)
        self.part_o = torch.empty((bg, self.splits, G, 128), dtype=torch.float32, device=dev)
        self.part_ml = torch.empty((bg, self.splits, G, 2), dtype=torch.float32, device=dev)
        self.counters = torch.zeros((bg,), dtype=i32, device=dev)
        # o then (m, l): one contiguous block (a multiple of 4 floats, so each
        # shard's block stays 16-byte aligned when gathered), one all-gather
        self.partials = torch.empty((((bg * G * 130) + 3) // 4 * 4,), dtype=torch.float32, device=dev)
        if rank != 0:  # attends no steady zone, but the kernel wants a buffer
            self._no_zone = torch.zeros((bg, 1, 128), dtype=torch.bfloat16, device=dev)

    # -- prefill --------------------------------------------------------------
    def build(self, keys: torch.Tensor, values: torch.Tensor, *, max_iters: int = 20, tol: float = 5e-4,
              early_stop_min_iter: int = 20, early_stop_rel_tol: float = 5e-4) -> None:
        """keys / values: this shard's middle tokens, [kv_heads, length, 128] bf16."""
        p = self.plan
        if keys.shape[1] != p.lengths[self.rank]:
            raise ValueError(f"shard {self.rank} holds {p.lengths[self.rank]} tokens, got {keys.shape[1]}")
        status = torch.zeros((1,), dtype=torch.int32, device=self.dev)
        self.index = ops.build_index(keys, values, parts=p.parts, ks=p.ks[self.rank], n_slots=p.n_slots[self.rank],
                                     max_iters=max_iters, tol=tol, early_stop_min_iter=early_stop_min_iter,
                                     early_stop_rel_tol=early_stop_rel_tol, status=status)
        self.slot_bound = int(self.index.n_active.max().item())
        if int(status.item()) & 1:
            raise RuntimeError(f"shard {self.rank}: IMI build failed (a tensor-core E-step wait gave up)")
        if self.slot_bound > p.n_slots[self.rank] - 1:
            raise RuntimeError(f"shard {self.rank}: IMI build produced {self.slot_bound} cells for "
                               f"{p.n_slots[self.rank]} slots")

    # -- exchange over NVLink peer memory ---------------------------------------
    def enable_peer_exchange(self, group=None) -> bool:
        """Put this shard's candidate record and partials block in symmetric
        memory (mapped by every rank of `group`, one shard per rank) and
        exchange them with imi_peer_allgather instead of NCCL all-gathers.
        Collective over the group; returns False (NCCL stays) when the block
        sizes do not allow it."""
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        g = group if group is not None else dist.group.WORLD
        world, rank = dist.get_world_size(g), dist.get_rank(g)
        if world != self.plan.shards or rank != self.rank or (self.cand.numel() * 8) % 16 != 0:
            return False
        name = g.group_name
        symm.enable_symm_mem_for_group(name)
        cand = symm.empty(tuple(self.cand.shape), dtype=torch.int64, device=self.dev)
        part = symm.empty(tuple(self.partials.shape), dtype=torch.float32, device=self.dev)
        flags = symm.empty((2, world), dtype=torch.int32, device=self.dev)
        cand.zero_()
        flags.zero_()
        hc, hp, hf = symm.rendezvous(cand, name), symm.rendezvous(part, name), symm.rendezvous(flags, name)
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=g)  # every rank's flags are zero before any exchange
        i64 = torch.int64
        fp = [int(x) for x in hf.buffer_ptrs]
        self.cand, self.partials = cand, part
        self._peer = dict(
            world=world, handles=(hc, hp, hf), keep=(cand, part, flags),
            src=(torch.tensor([int(x) for x in hc.buffer_ptrs], dtype=i64, device=self.dev),
                 torch.tensor([int(x) for x in hp.buffer_ptrs], dtype=i64, device=self.dev)),
            flags=(torch.tensor(fp, dtype=i64, device=self.dev),
                   torch.tensor([x + 4 * world for x in fp], dtype=i64, device=self.dev)),
            counters=torch.zeros((2, 2), dtype=torch.int32, device=self.dev),  # per channel: epoch, ticket
            status=torch.zeros((1,), dtype=torch.int32, device=self.dev),
            # host mirror of the status word, refreshed without a sync after
            # every step's exchanges and checked at the next step
            status_host=torch.zeros((1,), dtype=torch.int32, pin_memory=True),
            bytes=(self.cand.numel() * 8, self.partials.numel() * 4))
        return True

    def exchange_failed(self) -> bool:
        """Whether a peer exchange so far gave up waiting for a peer (synchronises)."""
        pe = getattr(self, "_peer", None)
        return pe is not None and bool(int(pe["status"].item()) & 1)

    def check_exchange(self, lagged: bool = False) -> None:
        """Raise when a peer exchange gave up waiting for a peer: its copy of
        that peer's block was skipped, so the merge or the combine read stale
        data.  lagged=True reads the host mirror that the previous step's
        exchange refreshed (no synchronisation; a failure shows at most one
        step late); otherwise the device word is read."""
        pe = getattr(self, "_peer", None)
        if pe is None:
            return
        bad = int(pe["status_host"][0]) & 1 if lagged else self.exchange_failed()
        if bad:
            raise RuntimeError(f"shard {self.rank}: a peer exchange timed out waiting for a peer "
                               "(the step's candidates or partials are not valid)")

    def peer_allgather(self, channel: int, dst: torch.Tensor) -> None:
        """Channel 0: the candidate records; 1: the partials block."""
        pe = self._peer
        d = _lib.PeerGatherDesc()
        d.world, d.rank, d.bytes = pe["world"], self.rank, pe["bytes"][channel]
        d.src_peers, d.flag_peers = pe["src"][channel].data_ptr(), pe["flags"][channel].data_ptr()
        d.epoch = pe["counters"].data_ptr() + 8 * channel
        d.ticket = d.epoch + 4
        d.dst, d.status = dst.data_ptr(), pe["status"].data_ptr()
        _lib.check(_lib.load().imi_peer_allgather(ctypes.byref(d), ops._stream(self.dev)), "imi_peer_allgather")

    # -- decode ---------------------------------------------------------------
    def select_local(self, q: torch.Tensor, cand_out: Optional[torch.Tensor] = None) -> None:
        """Local selection under the global rules; candidates into cand_out
        (default: this shard's own record buffer)."""
        p, idx = self.plan, self.index
        out = self.cand if cand_out is None else cand_out
        d = _lib.SelectDesc()
        d.bg, d.G, d.dim, d.n_slots, d.parts, d.kmax = self.bg, self.G, 128, idx.n_slots, idx.parts, idx.kmax
        d.ks = ops._ks4(idx.ks)
        d.q = q.data_ptr()
        d.sub_centroids, d.cell_code, d.cell_sizes = idx.sub_centroids.data_ptr(), idx.cell_code.data_ptr(), \
            idx.cell_sizes.data_ptr()
        d.cell_offsets, d.cell_mask, d.centroids = idx.cell_offsets.data_ptr(), idx.cell_mask.data_ptr(), \
            idx.centroids.data_ptr()
        d.nprobe, d.max_tokens, d.buffer_pages = p.nprobe, p.max_tokens, p.buffer_pages
        d.page_size, d.padding_id = p.page_size, idx.n_slots - 1
        d.static_len, d.exec_capacity = 0, p.buffer_pages * p.page_size
        d.sel_cells, d.sel_count = self.sel.data_ptr(), self.sel_count.data_ptr()
        d.slot_bound, d.key_base, d.cand_out = self.slot_bound, p.key_base[self.rank], out.data_ptr()
        _lib.check(_lib.load().imi_select_cells(ctypes.byref(d), ops._stream(self.dev)), "imi_select_cells")

    def merge(self, cand_all: torch.Tensor, static_len: int) -> None:
        """Global boundary over every shard's records ([shards, bg, record]);
        this shard's selected cells and row list."""
        p, idx = self.plan, self.index
        d = _lib.MergeDesc()
        d.bg, d.shards, d.cap, d.rank, d.key_base = self.bg, p.shards, p.cap, self.rank, p.key_base[self.rank]
        d.cand, d.cell_offsets, d.n_slots = cand_all.data_ptr(), idx.cell_offsets.data_ptr(), idx.n_slots
        d.nprobe, d.max_tokens, d.buffer_pages, d.page_size = p.nprobe, p.max_tokens, p.buffer_pages, p.page_size
        d.static_len = int(static_len) if self.rank == 0 else 0
        d.exec_capacity = self.exec_capacity
        d.sel_cells, d.sel_count = self.sel.data_ptr(), self.sel_count.data_ptr()
        d.row_index, d.row_count = self.rows.data_ptr(), self.row_count.data_ptr()
        _lib.check(_lib.load().imi_merge_candidates(ctypes.byref(d), ops._stream(self.dev)), "imi_merge_candidates")

    def attend(self, q: torch.Tensor, zone_keys: Optional[torch.Tensor], zone_values: Optional[torch.Tensor],
               partials_out: Optional[torch.Tensor] = None) -> None:
        """Unnormalised (o, m, l) of this shard's rows into partials_out
        (default: this shard's own block)."""
        idx, bg, G = self.index, self.bg, self.G
        blk = self.partials if partials_out is None else partials_out
        d = _lib.AttnDesc()
        d.bg, d.G, d.splits, d.exec_capacity = bg, G, self.splits, self.exec_capacity
        d.scale = 1.0 / math.sqrt(128)
        d.q, d.row_index, d.row_count = q.data_ptr(), self.rows.data_ptr(), self.row_count.data_ptr()
        d.list_keys, d.list_values, d.list_rows = idx.list_keys.data_ptr(), idx.list_values.data_ptr(), \
            idx.list_keys.shape[1]
        if self.rank == 0:
            d.static_keys, d.static_values, d.static_rows = zone_keys.data_ptr(), zone_values.data_ptr(), \
                zone_keys.shape[-2]
        else:
            d.static_keys = d.static_values = self._no_zone.data_ptr()
            d.static_rows = 1
        d.part_o, d.part_ml, d.counters = self.part_o.data_ptr(), self.part_ml.data_ptr(), self.counters.data_ptr()
        d.o_part, d.ml_part = blk.data_ptr(), blk.data_ptr() + bg * G * 128 * 4
        _lib.check(_lib.load().imi_sparse_attention(ctypes.byref(d), ops._stream(self.dev)), "imi_sparse_attention")


def combine(partials_all: torch.Tensor, shards: int, bg: int, G: int, out: torch.Tensor) -> torch.Tensor:
    """Log-sum-exp combine of [shards, block] partial blocks (o [bg, G, 128]
    then (m, l) [bg, G, 2] at the start of each block) into out [bg, G, 128]."""
    d = _lib.CombineDesc()
    d.shards, d.bg, d.G, d.part_stride = shards, bg, G, partials_all.shape[-1]
    d.o_parts = partials_all.data_ptr()
    d.ml_parts = partials_all.data_ptr() + bg * G * 128 * 4
    d.out = out.data_ptr()
    _lib.check(_lib.load().imi_combine_partials(ctypes.byref(d), ops._stream(out.device)), "imi_combine_partials")
    return out


def decode_step(local: Sequence[SeqShard], q: torch.Tensor, zone_keys: Optional[torch.Tensor],
                zone_values: Optional[torch.Tensor], static_len: int, group=None) -> torch.Tensor:
    """One decode attention of one layer.  q: [bg, G, 128] bf16 (the same on
    every shard); zone_*: the steady zone ([bg, static_capacity, 128]), used by
    shard 0 only.

    ``local`` holds either every shard (all in this process) or this process's
    one shard, with ``torch.distributed`` initialised over the shards."""
    plan = local[0].plan
    bg, G, dev = local[0].bg, local[0].G, local[0].dev
    out = torch.empty((bg, G, 128), dtype=torch.bfloat16, device=dev)
    if len(local) == plan.shards:  # every shard here: the exchange is a shared tensor
        cand_all = torch.empty((plan.shards, bg, plan.record), dtype=torch.int64, device=dev)
        for s in local:
            s.select_local(q, cand_all[s.rank])
        parts_all = torch.empty((plan.shards, local[0].partials.numel()), dtype=torch.float32, device=dev)
        for s in local:
            s.merge(cand_all, static_len)
            s.attend(q, zone_keys, zone_values, parts_all[s.rank])
        return combine(parts_all, plan.shards, bg, G, out)
    if len(local) != 1:
        raise ValueError("pass every shard, or this process's one shard")
    s = local[0]
    peer = getattr(s, "_peer", None) is not None
    if peer:
        s.check_exchange(lagged=True)
    s.select_local(q)
    cand_all = torch.empty((plan.shards, bg, plan.record), dtype=torch.int64, device=dev)
    if peer:
        s.peer_allgather(0, cand_all)
    else:
        # the flat form (output = the inputs concatenated along dim 0) works on
        # every backend, gloo included
        torch.distributed.all_gather_into_tensor(cand_all.view(plan.shards * bg, plan.record), s.cand, group=group)
    s.merge(cand_all, static_len)
    s.attend(q, zone_keys, zone_values)
    parts_all = torch.empty((plan.shards, s.partials.numel()), dtype=torch.float32, device=dev)
    if peer:
        s.peer_allgather(1, parts_all)
        s._peer["status_host"].copy_(s._peer["status"], non_blocking=True)
    else:
        torch.distributed.all_gather_into_tensor(parts_all.view(-1), s.partials, group=group)
    return combine(parts_all, plan.shards, bg, G, out)
