"""Index and budget sizing rules of the reference, restated.

* ``adaptive_k`` -- ``calculate_adaptive_k_values`` (layer_pipeline.cpp:177-228)
  with the config overrides of ``merge_all_chunks`` (layer_pipeline.cpp:1131-1163).
* ``RetrievalSizes.from_capacity`` -- ``prepare_cache`` sizing
  (runtime.py:31-63), which also fixes the IVF slot count; the one divergence
  (IVF builds with more cells than k*k) is described at the rule.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional, Tuple


def adaptive_k(seq_len: int, subspace_parts: int, target_cluster_size: int = 16,
               kmeans_cfg: Optional[Dict[str, object]] = None) -> Tuple[int, ...]:
    """k per subspace for a build over ``seq_len`` tokens."""
    cfg = kmeans_cfg or {}
    k1, k2, k3, k4 = (int(cfg.get(f"k{i}", 0) or 0) for i in (1, 2, 3, 4))
    tcs = int(cfg.get("target_cluster_size", cfg.get("cluster_size", target_cluster_size)) or target_cluster_size)
    if tcs <= 0:
        tcs = 16
    if subspace_parts == 0:
        if k1 > 0:
            return (k1,)
    elif subspace_parts == 4 and k1 > 0 and k2 > 0 and k3 > 0 and k4 > 0:
        return (k1, k2, k3, k4)
    elif subspace_parts == 2 and k1 > 0 and k2 > 0:
        return (k1, k2)
    if seq_len <= 0:
        return (1,) * max(1, subspace_parts)
    total = float(seq_len) / tcs
    if subspace_parts == 0:
        return (max(int(_cpp_round(total)), 1),)
    if subspace_parts == 4:
        k = max(int(_cpp_round(total ** 0.25)), 2)
        return (k, k, k, k)
    k = max(int(math.sqrt(total)), 32)
    return (k, k)


def _cpp_round(x: float) -> float:
    """std::round: halves away from zero."""
    return math.floor(x + 0.5) if x >= 0 else -math.floor(-x + 0.5)


@dataclass(frozen=True)
class RetrievalSizes:
    n_centroids: int          # slots per KV group (padding slot = n_centroids - 1)
    padding_cluster_id: int
    nprobe: int
    max_retrieval_tokens: int
    buffer_size: int          # pages
    page_size: int
    static_capacity: int
    execution_stride: int     # rows per KV group in the execution buffer

    @staticmethod
    def from_capacity(list_capacity: int, subspace_parts: int, retrieval_budget: float, buffer_cluster_num: int,
                      static_capacity: int, page_size: int = 8, fixed_budget: bool = True) -> "RetrievalSizes":
        """fixed_budget=False: the token budget is not fixed -- the selection is
        the top nprobe cells (nprobe = the budget ratio of the cell count) with
        neither a token cap nor page truncation.  The reference has no such
        mode (its token budget is always int(budget * capacity)); this rule is
        this library's reading of "budget_ratio without a fixed budget" and is
        not pinned to reference code."""
        n_tokens = max(list_capacity, 1)
        total_clusters = max(int(n_tokens / 16), 1)
        if subspace_parts == 4:
            k = max(int(round(max(n_tokens / 16.0, 1.0) ** 0.25)), 2)
            n_centroids = k ** 4 + 1
        else:
            # prepare_cache (runtime.py:34-39) sizes every mode but S=4 as k*k + 1,
            # IVF included, and it runs before the first layer's metadata is
            # loaded, so _ensure_metadata_buffers' IVF rule (indexing.py:179-181)
            # never fires there.
            k = max(int(math.sqrt(total_clusters)), 32)
            n_centroids = k * k + 1
            if subspace_parts == 0:
                # An IVF build makes up to round(n/16) cells (the build rounds as
                # std::round, layer_pipeline.cpp:177-228).  When that exceeds k*k
                # the reference's metadata copy into k*k + 1 slots fails
                # (indexing.py:128-129, a size mismatch); here the slots widen to
                # hold every cell instead, which is the only divergence.
                ivf_cells = max(int(_cpp_round(n_tokens / 16.0)), 1)
                if ivf_cells > k * k:
                    n_centroids = ivf_cells + 1
        nprobe = max(round((n_centroids - 1) * retrieval_budget), 1)
        nprobe = min(nprobe, n_centroids - 1)
        max_tokens = max(int(retrieval_budget * list_capacity), 1) if fixed_budget else max(list_capacity, 1)
        token_pages = max((max_tokens + page_size - 1) // page_size, 1) if max_tokens > 0 else 0
        buffer_size = max(max(buffer_cluster_num, token_pages), 1)
        return RetrievalSizes(
            n_centroids=n_centroids, padding_cluster_id=n_centroids - 1, nprobe=nprobe,
            max_retrieval_tokens=max_tokens, buffer_size=buffer_size, page_size=page_size,
            static_capacity=static_capacity, execution_stride=buffer_size * page_size + static_capacity)
