"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run in a container that has the reference checkout (it builds oracle/_ref from
the reference's own C++ sources with oracle/build_ref.py):

    python tests/golden/gen_golden.py

Each fixture stores (a) a SHA-256 of the seeded synthetic inputs, so a test can
prove it regenerated the same inputs, and (b) the outputs of the reference's own
code on them:

* index builds: ``imi::kmeans_execute{,_4,_ivf}`` + ``imi::reorganize_from_kmeans``
  (kmeans_core.cpp:822-1174, reorganize_core.cpp:313-569), one worker thread;
* cell selection: the reference's torch selection (retrieval.py:295-303, the
  same torch calls) followed by the reference's ``AdpIMI_Index.batch_access``
  page truncation (wave_buffer_cpu_hotcold.cpp:303-371, 897-929).

* the config-1 geometry (one KV head of 130 976 middle tokens, k = 90 x 90,
  the Llama k-means settings: 20 iterations, early stop 20 / 5e-4): the
  reference's labels and sub-centroids stored whole, the CSR offsets, and
  SHA-256 digests of the merged centroids and list rows
  (``cfg1_build_digest.npz``).

The decode scorer (compute_impl.cu:62-103) is CUDA; it is pinned on the GPU box
by running the reference kernel, compiled from its source into oracle/_ref by
oracle/build_ref_cuda.py, against the device scorer
(tests/test_gpu_reference_pins.py).
"""
from __future__ import annotations

import hashlib
import math
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
OUT = Path(__file__).resolve().parent

from adaptiveimi_b200.synthetic import make_layer  # noqa: E402
from oracle import build_ref  # noqa: E402

# name -> (kv_heads, context, components, theta, parts, ks, max_iters, tol, min_iter, rel_tol)
BUILD_CASES = {
    "imi2_k16": (2, 3096, 64, 500000.0, 2, [16, 16], 10, 0.0, 10, 0.0),
    "imi2_earlystop": (2, 3096, 64, 500000.0, 2, [12, 12], 25, 5e-4, 5, 5e-4),
    "imi2_llama_iters": (1, 4096, 64, 500000.0, 2, [20, 20], 20, 5e-4, 20, 5e-4),
    "imi4_k4": (2, 3096, 128, 1e6, 4, [4, 4, 4, 4], 8, 0.0, 8, 0.0),
    "ivf_k40": (2, 3096, 64, 500000.0, 0, [40], 6, 0.0, 6, 0.0),
}


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def case_inputs(heads, ctx, comps, theta, seed=0):
    K, V, Q = make_layer(heads, heads * 4, ctx, 128, comps, seed, theta, n_queries=4)
    k = K[:, 32:ctx - 64].contiguous()
    v = V[:, 32:ctx - 64].contiguous()
    return k, v, Q


def dup_inputs():
    """Heavily duplicated keys: k-means++ sees zero weights, Lloyd sees empty cells."""
    g = torch.Generator().manual_seed(5)
    base = torch.randn(2, 10, 128, generator=g)
    idx = torch.randint(0, 10, (2, 600), generator=g)
    k = torch.gather(base, 1, idx[..., None].expand(-1, -1, 128)).to(torch.bfloat16).contiguous()
    v = torch.randn(2, 600, 128, generator=g).to(torch.bfloat16)
    return k, v


def main():
    build_ref.build()
    sys.path.insert(0, str(ROOT / "oracle" / "_ref"))
    import imi_ref  # noqa: E402
    import AdpIMI_Index as AI  # noqa: E402

    cases = dict(BUILD_CASES)
    for name, (heads, ctx, comps, theta, parts, ks, it, tol, mi, rt) in cases.items():
        k, v, _ = case_inputs(heads, ctx, comps, theta)
        r = imi_ref.build(k, v, parts, ks, it, tol, mi, rt, 1)
        save_build(name, dict(kind="mixture", heads=heads, ctx=ctx, comps=comps, theta=theta, parts=parts, ks=ks,
                              max_iters=it, tol=tol, min_iter=mi, rel_tol=rt), k, v, r)
    k, v = dup_inputs()
    r = imi_ref.build(k, v, 2, [16, 16], 6, 0.0, 6, 0.0, 1)
    save_build("imi2_duplicates", dict(kind="duplicates", heads=2, parts=2, ks=[16, 16], max_iters=6, tol=0.0,
                                       min_iter=6, rel_tol=0.0), k, v, r)
    gen_selection(imi_ref, AI)
    gen_cfg1_digest(imi_ref)


# config-1 geometry: the inputs are head 0 of this call
CFG1 = dict(heads=2, q_heads=8, ctx=131072, comps=64, seed=0, theta=500000.0, ks=[90, 90], max_iters=20,
            tol=5e-4, min_iter=20, rel_tol=5e-4)


def cfg1_inputs():
    c = CFG1
    K, V, Q = make_layer(c["heads"], c["q_heads"], c["ctx"], 128, c["comps"], c["seed"], c["theta"], n_queries=16)
    return K, V, Q, K[:, 32:c["ctx"] - 64].contiguous(), V[:, 32:c["ctx"] - 64].contiguous()


def gen_cfg1_digest(imi_ref):
    c = CFG1
    _, _, _, k, v = cfg1_inputs()
    k0, v0 = k[:1].contiguous(), v[:1].contiguous()
    r = imi_ref.build(k0, v0, 2, c["ks"], c["max_iters"], c["tol"], c["min_iter"], c["rel_tol"], 1)
    na = int(r["cluster_counts"][0])
    np.savez_compressed(
        OUT / "cfg1_build_digest.npz",
        meta=np.array(repr(c)), input_sha=np.array(sha(bits(k0), bits(v0))),
        n_active=np.array(na), labels1=r["labels1"][0].numpy().astype(np.uint8),
        labels2=r["labels2"][0].numpy().astype(np.uint8),
        centroids1=r["centroids1"][0].numpy(), centroids2=r["centroids2"][0].numpy(),
        cluster_offsets=r["cluster_offsets"][0][:na + 1].numpy(),
        merged_sha=np.array(sha(r["centroids"][0][:na].numpy())),
        list_keys_sha=np.array(sha(bits(r["list_keys"][0]))), list_values_sha=np.array(sha(bits(r["list_values"][0]))))
    print("wrote cfg1_build_digest", na)


def save_build(name, meta, k, v, r):
    arrays = {
        "input_sha": np.array(sha(bits(k), bits(v))),
        "meta": np.array(repr(meta)),
        "cluster_counts": r["cluster_counts"].numpy(),
        "cluster_sizes": r["cluster_sizes"].numpy(),
        "cluster_offsets": r["cluster_offsets"].numpy(),
        "centroids": r["centroids"].numpy(),
        "list_keys_sha": np.array([sha(bits(r["list_keys"][h])) for h in range(k.shape[0])]),
        "list_values_sha": np.array([sha(bits(r["list_values"][h])) for h in range(k.shape[0])]),
    }
    for s in range(1, 5):
        if f"labels{s}" in r:
            arrays[f"labels{s}"] = r[f"labels{s}"].numpy()
            arrays[f"centroids{s}"] = r[f"centroids{s}"].numpy()
    np.savez_compressed(OUT / f"build_{name}.npz", **arrays)
    print("wrote", name, r["cluster_counts"].tolist())


def reference_select(sim, sizes, nprobe, max_tokens, padding_id):
    """retrieval.py:295-303, the reference's own torch calls."""
    topk = torch.topk(sim, nprobe, dim=-1, largest=True, sorted=True)
    sz = torch.gather(sizes, 1, topk.indices)
    valid = sz > 0
    cumsum = torch.cumsum(sz, dim=-1, dtype=torch.int32)
    keep = valid & ((cumsum - sz) < max_tokens)
    return topk.indices.masked_fill(~keep, padding_id)


def gen_selection(imi_ref, AI):
    """Config-0 geometry: 8 KV heads, 8192 context, k=16x16, 16 decode queries."""
    heads, G, ctx = 8, 4, 8192
    K, V, Q = make_layer(heads, heads * G, ctx, 128, 64, 0, 500000.0, n_queries=16)
    k = K[:, 32:ctx - 64].contiguous()
    v = V[:, 32:ctx - 64].contiguous()
    r = imi_ref.build(k, v, 2, [16, 16], 10, 0.0, 10, 0.0, 1)
    n = k.shape[1]
    cap = n
    kk = max(int(math.sqrt(max(int(cap / 16), 1))), 32)
    n_slots = kk * kk + 1
    nprobe = min(max(round((n_slots - 1) * 0.1), 1), n_slots - 1)
    max_tokens = max(int(0.1 * cap), 1)
    buffer_pages = max(32, max((max_tokens + 7) // 8, 1))
    counts = r["cluster_counts"]
    sizes = torch.zeros(heads, n_slots, dtype=torch.int32)
    offsets = torch.zeros(heads, n_slots + 1, dtype=torch.int32)
    cents = torch.zeros(heads, n_slots, 128)
    mask = torch.ones(heads, n_slots, dtype=torch.bool)
    mc = r["cluster_sizes"].shape[1]
    sizes[:, :mc] = r["cluster_sizes"]
    offsets[:, :mc + 1] = r["cluster_offsets"]
    offsets[:, mc + 1:] = r["cluster_offsets"][:, -1:]
    cents[:, :mc] = r["centroids"]
    mask[:, :mc] = r["cluster_sizes"] == 0
    # Scores with the scorer's arithmetic (compute_impl.cu:62-103) in fp64-free
    # fp32 fma order: produced by the oracle restatement and stored as inputs.
    from oracle import oracle as O
    sims = np.zeros((16, heads, n_slots), np.float32)
    for t in range(16):
        qb = bits(Q[t].reshape(heads, G, 128))
        for h in range(heads):
            sims[t, h] = O.scores(qb[h], cents[h].numpy(), mask[h].numpy().astype(np.uint8))
    pool = AI.AdpIMI_ThreadPool(2)
    idx = AI.AdpIMI_Index(1, heads, 128, nprobe, 0, 8, n_slots, buffer_pages, 1, 2, pool.get())
    z = lambda *s: torch.zeros(*s, dtype=torch.int32)  # noqa: E731
    bufs = [z(heads, buffer_pages) for _ in range(3)] + [z(heads)] + [z(heads, buffer_pages) for _ in range(3)] + \
           [z(heads)] + [z(heads, buffer_pages) for _ in range(3)] + [z(heads)]
    cluster_ids = torch.zeros(heads, nprobe, dtype=torch.int64)
    idx.set_indices(*bufs, cluster_ids)
    ph = torch.empty(heads, 0, 128, dtype=torch.bfloat16)
    idx.set_kv(ph.unsqueeze(0), ph.unsqueeze(0), ph, ph)
    idx.set_cluster_metadata(sizes, offsets, 0)
    selected_sets = np.full((16, heads, nprobe), -1, np.int32)
    pre = np.zeros((16, heads, nprobe), np.int64)
    for t in range(16):
        sel = reference_select(torch.from_numpy(sims[t]), sizes, nprobe, max_tokens, n_slots - 1)
        pre[t] = sel.numpy()
        # fresh index per query so every access is a cold (all-miss) access
        idx2 = AI.AdpIMI_Index(1, heads, 128, nprobe, 0, 8, n_slots, buffer_pages, 1, 2, pool.get())
        bufs2 = [b.clone() for b in bufs]
        cid = sel.clone()
        idx2.set_indices(*bufs2, cid)
        idx2.set_kv(ph.unsqueeze(0), ph.unsqueeze(0), ph, ph)
        idx2.set_cluster_metadata(sizes, offsets, 0)
        idx2.batch_access()
        idx2.sync()
        miss_ids, miss_sizes, _, miss_num = bufs2[4], bufs2[5], bufs2[6], bufs2[7]
        for h in range(heads):
            starts = miss_ids[h, :int(miss_num[h])].numpy()
            off_h = offsets[h].numpy()
            cells = []
            for s0 in starts:
                c = int(np.searchsorted(off_h[:mc + 1], s0, side="right") - 1)
                # a cell spans several 8-row blocks; record each cell once
                if off_h[c] == s0:
                    cells.append(c)
            selected_sets[t, h, :len(cells)] = cells
    np.savez_compressed(OUT / "select_cfg0.npz", sims=sims, sizes=sizes.numpy(), offsets=offsets.numpy(),
                        pre_trunc=pre, selected=selected_sets,
                        params=np.array([nprobe, max_tokens, buffer_pages, n_slots], np.int64),
                        input_sha=np.array(sha(bits(k), bits(v), bits(Q))))
    print("wrote select_cfg0", nprobe, max_tokens, buffer_pages, n_slots)


if __name__ == "__main__":
    if "--cfg1-only" in sys.argv:
        build_ref.build()
        sys.path.insert(0, str(ROOT / "oracle" / "_ref"))
        import imi_ref  # noqa: E402
        gen_cfg1_digest(imi_ref)
    else:
        main()
