"""Sizing rules (runtime.py:31-63, layer_pipeline.cpp:177-228) restated in
adaptiveimi_b200/sizing.py, including the IVF slot count."""
import math

from adaptiveimi_b200.sizing import RetrievalSizes, adaptive_k


def _prepare_cache(list_capacity, parts, budget):
    """The reference's prepare_cache sizing, the same expressions (runtime.py:31-42)."""
    n_tokens = max(list_capacity, 1)
    total_clusters = max(int(n_tokens / 16), 1)
    if parts == 4:
        k = max(int(round(max(n_tokens / 16.0, 1.0) ** 0.25)), 2)
        n_centroids = k ** 4 + 1
    else:
        k = max(int(math.sqrt(total_clusters)), 32)
        n_centroids = k * k + 1
    nprobe = min(max(round((n_centroids - 1) * budget), 1), n_centroids - 1)
    return n_centroids, nprobe


def test_config_sizes():
    s = RetrievalSizes.from_capacity(130976, 2, 0.1, 32, static_capacity=96 + 255)
    assert (s.n_centroids, s.nprobe, s.max_retrieval_tokens, s.buffer_size) == (8101, 810, 13097, 1638)
    assert adaptive_k(130976, 2) == (90, 90)
    s = RetrievalSizes.from_capacity(8096, 2, 0.1, 32, static_capacity=97)
    assert (s.n_centroids, s.nprobe, s.max_retrieval_tokens) == (1025, 102, 809)
    assert adaptive_k(130976, 4) == (10, 10, 10, 10)
    assert adaptive_k(32672, 4) == (7, 7, 7, 7)


def test_every_mode_follows_prepare_cache_where_the_build_fits():
    for cap in (100, 1000, 8096, 16000, 16384, 20000, 65440, 130976):
        for parts in (0, 2, 4):
            for budget in (0.05, 0.1):
                s = RetrievalSizes.from_capacity(cap, parts, budget, 32, static_capacity=97)
                nc, npb = _prepare_cache(cap, parts, budget)
                if parts == 0 and adaptive_k(cap, 0)[0] > nc - 1:
                    continue
                assert (s.n_centroids, s.nprobe) == (nc, npb), (cap, parts, budget)


def test_ivf_slots_widen_only_when_the_build_overflows_prepare_cache():
    # 130 976 tokens: an IVF build makes up to 8 186 cells; prepare_cache's
    # 90 * 90 + 1 slots cannot hold them (the reference fails its metadata copy),
    # so the slots widen to 8 187 and nprobe follows them.
    s = RetrievalSizes.from_capacity(130976, 0, 0.1, 32, static_capacity=97)
    assert adaptive_k(130976, 0) == (8186,)
    assert (s.n_centroids, s.nprobe) == (8187, 819)
    # 8 096 tokens: 506 cells fit prepare_cache's 1 025 slots, which are kept
    s = RetrievalSizes.from_capacity(8096, 0, 0.1, 32, static_capacity=97)
    assert (s.n_centroids, s.nprobe) == (1025, 102)


def test_without_a_fixed_budget_only_nprobe_limits():
    s = RetrievalSizes.from_capacity(81920, 4, 0.05, 32, static_capacity=97, fixed_budget=False)
    k = adaptive_k(81920, 4)[0]
    assert s.n_centroids == k ** 4 + 1 and s.nprobe == round(k ** 4 * 0.05)
    assert s.max_retrieval_tokens == 81920 and s.buffer_size == 81920 // 8
