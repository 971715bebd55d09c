"""Pin the CPU oracle (oracle/imi_oracle.cpp) to the reference itself.

* against the committed golden fixtures (tests/golden/*.npz, generated from the
  reference's own C++ by tests/golden/gen_golden.py), always;
* against the reference's C++ built in place (oracle/_ref), when present.
"""
import ast
import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

from adaptiveimi_b200.synthetic import make_layer
from oracle import oracle as O

GOLD = Path(__file__).resolve().parent / "golden"


def _sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _inputs(meta):
    if meta["kind"] == "duplicates":
        g = torch.Generator().manual_seed(5)
        base = torch.randn(2, 10, 128, generator=g)
        idx = torch.randint(0, 10, (2, 600), generator=g)
        k = torch.gather(base, 1, idx[..., None].expand(-1, -1, 128)).to(torch.bfloat16).contiguous()
        v = torch.randn(2, 600, 128, generator=g).to(torch.bfloat16)
        return k, v
    K, V, _ = make_layer(meta["heads"], meta["heads"] * 4, meta["ctx"], 128, meta["comps"], 0, meta["theta"],
                         n_queries=4)
    return K[:, 32:meta["ctx"] - 64].contiguous(), V[:, 32:meta["ctx"] - 64].contiguous()


BUILD_FIXTURES = sorted(p.name for p in GOLD.glob("build_*.npz"))


@pytest.mark.parametrize("fixture", BUILD_FIXTURES)
def test_oracle_build_matches_golden(fixture):
    z = np.load(GOLD / fixture)
    meta = ast.literal_eval(str(z["meta"]))
    k, v = _inputs(meta)
    kb, vb = O.bf16_bits(k), O.bf16_bits(v)
    assert _sha(kb, vb) == str(z["input_sha"]), "synthetic inputs changed; regenerate the golden fixtures"
    parts = meta["parts"]
    S = 1 if parts == 0 else parts
    for h in range(k.shape[0]):
        o = O.build_head(kb[h], vb[h], parts, meta["ks"], meta["max_iters"], meta["tol"], meta["min_iter"],
                         meta["rel_tol"])
        na = o["n_active"]
        assert na == int(z["cluster_counts"][h])
        for s in range(S):
            np.testing.assert_array_equal(o["sub_labels"][s], z[f"labels{s + 1}"][h])
            np.testing.assert_array_equal(o["sub_centroids"][s], z[f"centroids{s + 1}"][h])
        np.testing.assert_array_equal(o["offsets"], z["cluster_offsets"][h][:na + 1])
        np.testing.assert_array_equal(np.diff(o["offsets"]), z["cluster_sizes"][h][:na])
        np.testing.assert_array_equal(o["merged"], z["centroids"][h][:na])
        assert _sha(o["list_keys"]) == str(z["list_keys_sha"][h])
        assert _sha(o["list_values"]) == str(z["list_values_sha"][h])


def test_oracle_selection_matches_golden():
    z = np.load(GOLD / "select_cfg0.npz")
    nprobe, max_tokens, buffer_pages, n_slots = (int(x) for x in z["params"])
    sims, sizes = z["sims"], z["sizes"]
    T, H, _ = sims.shape
    for t in range(T):
        for h in range(H):
            sel, pre = O.select(sims[t, h], sizes[h], nprobe, max_tokens, buffer_pages, 8, n_slots - 1)
            np.testing.assert_array_equal(pre, z["pre_trunc"][t, h])
            ref = z["selected"][t, h]
            ref = ref[ref >= 0]
            np.testing.assert_array_equal(sel, ref)


def test_oracle_scores_arithmetic():
    """The scorer restatement reproduces the g-ordered sum and d-ordered fma chain."""
    rng = np.random.default_rng(0)
    q = torch.from_numpy(rng.standard_normal((4, 128)).astype(np.float32)).to(torch.bfloat16)
    c = rng.standard_normal((50, 128)).astype(np.float32)
    qb = O.bf16_bits(q)
    got = O.scores(qb, c)
    qs = np.zeros(128, np.float32)
    for g in range(4):
        qs = (qs + q[g].float().numpy()).astype(np.float32)
    for i in range(50):
        s = np.float32(0)
        for d in range(128):
            s = np.float32(np.float64(qs[d]) * np.float64(c[i, d]) + np.float64(s))  # fma: exact product, one rounding
        assert got[i] == s


def test_oracle_matches_live_reference(ref_modules):
    imi_ref, _ = ref_modules
    K, V, _ = make_layer(2, 8, 2200, 128, 32, 11, 1e6, n_queries=1)
    k, v = K[:, :2100].contiguous(), V[:, :2100].contiguous()
    for parts, ks in ((2, [8, 9]), (4, [3, 4, 3, 2]), (0, [33])):
        r = imi_ref.build(k, v, parts, ks, 7, 5e-4, 3, 5e-4, 1)
        kb, vb = O.bf16_bits(k), O.bf16_bits(v)
        for h in range(2):
            o = O.build_head(kb[h], vb[h], parts, ks, 7, 5e-4, 3, 5e-4)
            na = o["n_active"]
            assert na == int(r["cluster_counts"][h])
            np.testing.assert_array_equal(o["offsets"], r["cluster_offsets"][h][:na + 1].numpy())
            np.testing.assert_array_equal(o["merged"], r["centroids"][h][:na].numpy())
            np.testing.assert_array_equal(o["list_keys"], O.bf16_bits(r["list_keys"][h]))


def cfg1_inputs():
    """Head 0 of the config-1 geometry (tests/golden/gen_golden.py CFG1)."""
    c = ast.literal_eval(str(np.load(GOLD / "cfg1_build_digest.npz")["meta"]))
    K, V, Q = make_layer(c["heads"], c["q_heads"], c["ctx"], 128, c["comps"], c["seed"], c["theta"], n_queries=16)
    return c, K, V, Q, K[:, 32:c["ctx"] - 64].contiguous(), V[:, 32:c["ctx"] - 64].contiguous()


def check_cfg1_head0(labels, sub_centroids, offsets, merged, list_keys_bits, list_values_bits, n_active):
    """A head-0 build at the config-1 geometry against the reference's own outputs."""
    z = np.load(GOLD / "cfg1_build_digest.npz")
    assert n_active == int(z["n_active"])
    for s in range(2):
        np.testing.assert_array_equal(labels[s], z[f"labels{s + 1}"].astype(np.int32), err_msg=f"labels s{s}")
        np.testing.assert_array_equal(sub_centroids[s], z[f"centroids{s + 1}"], err_msg=f"centroids s{s}")
    np.testing.assert_array_equal(offsets, z["cluster_offsets"])
    assert _sha(np.ascontiguousarray(merged, np.float32)) == str(z["merged_sha"])
    assert _sha(list_keys_bits) == str(z["list_keys_sha"])
    assert _sha(list_values_bits) == str(z["list_values_sha"])


def test_oracle_matches_reference_at_config1_geometry():
    """The oracle at the benchmarked build size (130 976 keys, k = 90 x 90, 20
    Lloyd iterations with the Llama early-stop settings) against the reference's
    outputs on the same keys."""
    c, _, _, _, k, v = cfg1_inputs()
    kb, vb = O.bf16_bits(k[:1]), O.bf16_bits(v[:1])
    assert _sha(kb, vb) == str(np.load(GOLD / "cfg1_build_digest.npz")["input_sha"])
    o = O.build_head(kb[0], vb[0], 2, c["ks"], c["max_iters"], c["tol"], c["min_iter"], c["rel_tol"])
    check_cfg1_head0(o["sub_labels"], o["sub_centroids"], o["offsets"], o["merged"], o["list_keys"],
                     o["list_values"], o["n_active"])


def test_oracle_async_update_matches_reference_torch():
    """The async centroid update restatement (oracle_async_update) against the
    reference's own _schedule_async_update run on CPU torch
    (tests/golden/async_update_ref.npz, made by gen_async_pin.py).

    The reference scores with torch.bmm, the restatement with a d-ordered fma
    chain, so an assignment may differ only where the two best inner products
    are a near-tie: the winner's fp64 score must then be within 1e-6 relative
    of the reference's pick.  Everything downstream of identical assignments
    (scatter_add sums in token order, the thresholded running mean) must be
    bit-identical."""
    from tests.golden.gen_async_pin import pin_inputs

    z = np.load(GOLD / "async_update_ref.npz")
    shadow, counts, keys, _ = pin_inputs()
    thr, B = int(z["threshold"]), int(z["batch"])
    dcounts = np.zeros_like(counts)
    dsums = np.zeros(shadow.shape, np.float32)
    kb = O.bf16_bits(keys)
    mism = 0
    for b in range(z["ids"].shape[0]):
        for h in range(shadow.shape[0]):
            before = shadow[h].astype(np.float64)
            kk = np.ascontiguousarray(kb[h, b * B:(b + 1) * B])
            ids = O.async_update(kk, shadow[h], counts[h], dcounts[h], dsums[h], thr)
            ref = z["ids"][b, h]
            for i in np.nonzero(ids != ref)[0]:
                x = torch.from_numpy(kk[i:i + 1].view(np.int16)).view(torch.bfloat16).double().numpy()[0]
                s_o, s_r = before[ids[i]] @ x, before[ref[i]] @ x
                assert abs(s_o - s_r) <= 1e-6 * max(abs(s_o), abs(s_r), 1e-30), (b, h, i, s_o, s_r)
                mism += 1
    # the reference's delta ring: its count and write position advance, its
    # ids and rows are never written (the quirk the device path reproduces
    # unless store_delta_rows is set)
    n_slots = shadow.shape[1]
    assert (z["ring_ids"] == n_slots - 1).all() and int(z["ring_keys_nonzero"]) == 0
    assert z["ring_count"].tolist() == [64, 64] and z["ring_write_pos"].tolist() == [64, 64]
    assert mism == 0, f"{mism} near-tie assignments"  # none on these inputs
    if mism == 0:
        np.testing.assert_array_equal(shadow, z["shadow"])
        np.testing.assert_array_equal(counts, z["counts"])
        np.testing.assert_array_equal(dcounts, z["delta_counts"])
        np.testing.assert_array_equal(dsums, z["delta_sums"])
