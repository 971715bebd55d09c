"""The reference's page-truncation step driven through its own C++
(``AdpIMI_Index.batch_access``, wave_buffer_cpu_hotcold.cpp:303-371, 897-929,
built from source into oracle/_ref by oracle/build_ref.py).

TEST INFRASTRUCTURE ONLY: used by tests/golden/gen_golden.py's selection
fixture logic and by the CPU-baseline / reference arm of bench.py.
"""
from __future__ import annotations

import numpy as np
import torch


def reference_select(sim: torch.Tensor, sizes: torch.Tensor, nprobe: int, max_tokens: int,
                     padding_id: int) -> torch.Tensor:
    """retrieval.py:295-303 as the same torch calls (topk, gather, cumsum,
    masked_fill) on [bg, n_slots] scores and sizes."""
    topk = torch.topk(sim, nprobe, dim=-1, largest=True, sorted=True)
    sz = torch.gather(sizes, 1, topk.indices)
    valid = sz > 0
    cumsum = torch.cumsum(sz, dim=-1, dtype=torch.int32)
    keep = valid & ((cumsum - sz) < max_tokens)
    return topk.indices.masked_fill(~keep, padding_id)


class PageTruncation:
    """One AdpIMI_Index per call of ``access`` (every page a miss, as on a cold
    cache), over fixed per-group cell metadata."""

    def __init__(self, AI, sizes: torch.Tensor, offsets: torch.Tensor, nprobe: int, buffer_pages: int,
                 threads: int = 2):
        self.AI = AI
        self.bg, self.n_slots = sizes.shape
        self.sizes, self.offsets = sizes.contiguous(), offsets.contiguous()
        self.nprobe, self.buffer_pages = nprobe, buffer_pages
        self.pool = AI.AdpIMI_ThreadPool(threads)
        self.ph = torch.empty(self.bg, 0, 128, dtype=torch.bfloat16)

    def access(self, selected: torch.Tensor):
        """selected: [bg, nprobe] int64 (padding id for dropped entries).
        Returns per group the list of (row start, rows) runs the reference
        would copy for the selected cells that survive page truncation."""
        bg, bp = self.bg, self.buffer_pages
        z = lambda *s: torch.zeros(*s, dtype=torch.int32)  # noqa: E731
        bufs = [z(bg, bp) for _ in range(3)] + [z(bg)] + [z(bg, bp) for _ in range(3)] + [z(bg)] + \
               [z(bg, bp) for _ in range(3)] + [z(bg)]
        idx = self.AI.AdpIMI_Index(1, bg, 128, self.nprobe, 0, 8, self.n_slots, bp, 1, 2, self.pool.get())
        # the index keeps raw pointers to every tensor it is given: keep them alive
        sel = selected.to(torch.int64).contiguous().clone()
        idx.set_indices(*bufs, sel)
        idx.set_kv(self.ph.unsqueeze(0), self.ph.unsqueeze(0), self.ph, self.ph)
        idx.set_cluster_metadata(self.sizes, self.offsets, 0)
        idx.batch_access()
        idx.sync()
        miss_ids, miss_sizes, miss_num = bufs[4], bufs[5], bufs[7]
        runs = []
        for h in range(bg):
            m = int(miss_num[h])
            runs.append(list(zip(miss_ids[h, :m].tolist(), miss_sizes[h, :m].tolist())))
        return runs


def rows_of(runs) -> np.ndarray:
    """Row indices of a group's (start, rows) runs."""
    if not runs:
        return np.zeros(0, np.int64)
    return np.concatenate([np.arange(s, s + n) for s, n in runs])
