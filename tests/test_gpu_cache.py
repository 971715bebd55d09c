"""End-to-end parity of the drop-in cache API (adpimi_cache + imi_decode_attn)
against a CPU simulation of the reference's decode path built from the oracle:
prefill build, steady zone, decode append, batched decode-time cell assignment
with delayed publication, delta rows, selection and attention.
"""
import math

import numpy as np
import pytest
import torch

from adaptiveimi_b200.attn import imi_decode_attn
from adaptiveimi_b200.cache import adpimi_cache
from adaptiveimi_b200.synthetic import make_layer
from oracle import oracle as O

pytestmark = pytest.mark.gpu


class RefSim:
    """CPU restatement of one layer of the reference cache during decode."""

    def __init__(self, K, V, kv, static_start, static_end, ks, iters, sizes, gen, async_cfg):
        ctx = K.shape[1]
        self.kv = kv
        self.sizes = sizes
        mid_k = K[:, static_start:ctx - static_end].contiguous()
        mid_v = V[:, static_start:ctx - static_end].contiguous()
        kb, vb = O.bf16_bits(mid_k), O.bf16_bits(mid_v)
        ns = sizes["n_slots"]
        self.cent = np.zeros((kv, ns, 128), np.float32)
        self.csz = np.zeros((kv, ns), np.int32)
        self.offs = np.zeros((kv, ns + 1), np.int32)
        self.mask = np.ones((kv, ns), np.uint8)
        self.lk, self.lv = [], []
        for h in range(kv):
            o = O.build_head(kb[h], vb[h], 2, ks, iters)
            na = o["n_active"]
            self.cent[h, :na] = o["merged"]
            self.csz[h, :na] = np.diff(o["offsets"])
            self.offs[h, :na + 1] = o["offsets"]
            self.offs[h, na + 1:] = o["offsets"][-1]
            self.mask[h, :na] = 0
            self.lk.append(o["list_keys"])
            self.lv.append(o["list_values"])
        cap = static_start + static_end + gen
        self.zk = np.zeros((kv, cap, 128), np.uint16)
        self.zv = np.zeros((kv, cap, 128), np.uint16)
        Kb, Vb = O.bf16_bits(K), O.bf16_bits(V)
        self.zk[:, :static_start] = Kb[:, :static_start]
        self.zk[:, static_start:static_start + static_end] = Kb[:, ctx - static_end:]
        self.zv[:, :static_start] = Vb[:, :static_start]
        self.zv[:, static_start:static_start + static_end] = Vb[:, ctx - static_end:]
        self.acfg = async_cfg
        if async_cfg:
            self.shadow = self.cent.copy()
            self.counts = self.csz.copy()
            self.dcounts = np.zeros_like(self.csz)
            self.dsums = np.zeros((kv, ns, 128), np.float32)
            R = async_cfg["delta_tokens"]
            self.ring_k = np.zeros((kv, R, 128), np.uint16)
            self.ring_v = np.zeros((kv, R, 128), np.uint16)
            self.ring_ids = np.full((kv, R), sizes["padding"], np.int32)
            self.ring_pos = 0
            self.ring_count = 0
            self.batch_k, self.batch_v = [], []
            self.state = None  # None / "scheduled" / "ready"

    def append(self, pos, k_bits, v_bits):
        self.zk[:, pos] = k_bits
        self.zv[:, pos] = v_bits
        if not self.acfg:
            return
        self.batch_k.append(k_bits.copy())
        self.batch_v.append(v_bits.copy())
        if len(self.batch_k) >= self.acfg["batch"]:
            bk = np.stack(self.batch_k, 1)  # [kv, B, D]
            bv = np.stack(self.batch_v, 1)
            B = bk.shape[1]
            R = self.acfg["delta_tokens"]
            for h in range(self.kv):
                ids = O.async_update(np.ascontiguousarray(bk[h]), self.shadow[h], self.counts[h], self.dcounts[h],
                                     self.dsums[h], self.acfg["threshold"])
                if not self.acfg.get("store_delta_rows", False):
                    continue  # the reference's ring keeps its zero rows and padding ids
                for b in range(B):
                    p = (self.ring_pos + b) % R
                    self.ring_k[h, p] = bk[h, b]
                    self.ring_v[h, p] = bv[h, b]
                    self.ring_ids[h, p] = ids[b]
            self.ring_pos = (self.ring_pos + B) % R
            self.ring_count = min(self.ring_count + B, R)
            self.batch_k, self.batch_v = [], []
            self.state = "scheduled"

    def attend(self, q_bits, static_len):
        s = self.sizes
        if self.acfg and self.state == "ready":
            self.cent = self.shadow.copy()
            self.state = None
        outs, sels = [], []
        for h in range(self.kv):
            sc = O.scores(q_bits[h], self.cent[h], self.mask[h])
            sel, pre = O.select(sc, self.csz[h], s["nprobe"], s["max_tokens"], s["buffer"], 8, s["padding"])
            rk = [self.zk[h, :static_len]] + [self.lk[h][self.offs[h, c]:self.offs[h, c] + self.csz[h, c]]
                                              for c in sel]
            rv = [self.zv[h, :static_len]] + [self.lv[h][self.offs[h, c]:self.offs[h, c] + self.csz[h, c]]
                                              for c in sel]
            if self.acfg and self.ring_count > 0:
                kept = set(int(x) for x in pre)
                for p in range(self.ring_count):
                    if int(self.ring_ids[h, p]) in kept:
                        rk.append(self.ring_k[h, p:p + 1])
                        rv.append(self.ring_v[h, p:p + 1])
            k_rows = np.concatenate(rk)[:s["exec"]]
            v_rows = np.concatenate(rv)[:s["exec"]]
            outs.append(O.attention(q_bits[h], k_rows, v_rows, 1.0 / math.sqrt(128)))
            sels.append(sel)
        if self.acfg and self.state == "scheduled":
            self.state = "ready"
        return np.stack(outs), sels


@pytest.mark.parametrize("mode", ["off", "reference_ring", "stored_ring"])
def test_cache_decode_matches_reference_simulation(mode):
    """off: no async update.  reference_ring: the reference's behaviour, whose
    delta ring never receives rows (zero rows with padding ids are attended
    whenever the selection holds a dropped entry).  stored_ring: the ring holds
    the batch's rows and cells."""
    torch.manual_seed(0)
    layers, kv, G, ctx, gen = 2, 4, 4, 4096, 24
    async_on = mode != "off"
    acfg = {"enabled": True, "batch": 4, "threshold": 2, "delta_tokens": 16,
            "store_delta_rows": mode == "stored_ring"} if async_on else {}
    cache = adpimi_cache(
        valid_start=[0], layer_num=layers, batch_size=1, max_length=ctx + gen + 1, num_key_value_heads=kv,
        num_heads=kv * G, head_dim=128, dtype=torch.bfloat16, layer_mapping={"0": "cuda:0", "1": "cuda:0"},
        max_new_length=gen + 1, input_length=ctx, static_pattern_start=32, static_pattern_end=64, core=4,
        pages_per_cluster=2, retrieval_budget=0.1, cache_ratio=0.05, buffer_cluster_num=32, prefill_bsz=1,
        num_gpus=1, model_size=8, subspace_parts=2,
        runtime_config={"kmeans": {"k1": 16, "k2": 16, "max_iters": 6, "early_stop_min_iter": 6, "tol": 0.0,
                                   "early_stop_rel_tol": 0.0}, "async_update": acfg})
    sims, means = [], []
    sizes = dict(n_slots=cache.n_centroids, nprobe=cache.nprobe, max_tokens=cache.max_retrieval_tokens,
                 buffer=cache.buffer_size, padding=cache.padding_cluster_id, exec=cache.execution_stride)
    Qs = []
    for l in range(layers):
        K, V, Q = make_layer(kv, kv * G, ctx, 128, 32, 10 + l, 500000.0, n_queries=gen)
        ks = K.transpose(0, 1).unsqueeze(0).cuda()
        vs = V.transpose(0, 1).unsqueeze(0).cuda()
        cache.prefill_update_kv_cache(None, ks, vs, l, 0)
        sims.append(RefSim(K, V, kv, 32, 64, (16, 16), 6, sizes, gen, acfg if async_on else None))
        Qs.append(Q)
    cache.prepare_cache()
    g = torch.Generator().manual_seed(3)
    worst = 0.0
    for t in range(gen):
        for l in range(layers):
            nk = torch.randn(1, 1, kv, 128, generator=g).to(torch.bfloat16)
            nv = torch.randn(1, 1, kv, 128, generator=g).to(torch.bfloat16)
            pos = cache.static_pattern_total
            cache.decode_update_kv_cache(nk.cuda(), nv.cuda(), l)
            sims[l].append(pos, O.bf16_bits(nk[0, 0]), O.bf16_bits(nv[0, 0]))
            q = Qs[l][t].reshape(1, 1, kv * G, 128)
            out = imi_decode_attn(q.cuda(), None, None, l, cache)
            static_len = pos + 1
            ref, ref_sel = sims[l].attend(O.bf16_bits(q.reshape(kv, G, 128)), static_len)
            dev_sel = cache._dec["cuda:0"]["sel"].cpu().numpy()
            dev_cnt = cache._dec["cuda:0"]["sel_count"].cpu().numpy()
            for h in range(kv):
                np.testing.assert_array_equal(np.sort(dev_sel[h, :dev_cnt[h]]), np.sort(ref_sel[h]),
                                              err_msg=f"t{t} l{l} h{h}")
            got = out.reshape(kv, G, 128).float().cpu().numpy()
            err = np.abs(got - ref)
            worst = max(worst, float(err.max()))
            assert err.max() <= 2e-2 and err.mean() <= 2e-3, (t, l, float(err.max()))
    assert cache.context == ctx + gen


def test_build_on_a_side_stream_matches_the_stream_ordered_build():
    """IMIPipeline with a build stream (the cache's async_build option): the build waits for
    the producer's stream, runs beside it, and gives the same index as a build on
    the caller's stream; the producer may drop its K/V right after the call."""
    from adaptiveimi_b200.imi_adapter import IMIPipeline, IMIRuntimeConfig

    kv, G, ctx = 4, 4, 4096
    K, V, _ = make_layer(kv, kv * G, ctx, 128, 32, 31, 500000.0)
    cfg = IMIRuntimeConfig(kmeans={"k1": 16, "k2": 16, "max_iters": 6, "early_stop_min_iter": 6, "tol": 0.0,
                                   "early_stop_rel_tol": 0.0})
    out = []
    for side in (None, torch.cuda.Stream()):
        pipe = IMIPipeline(layer_idx=0, kv_heads=kv, head_dim=128, dtype=torch.bfloat16, device_id=0,
                           max_tokens=ctx, runtime_config=cfg, n_slots=257, build_stream=side)
        ks = K.transpose(0, 1).unsqueeze(0).cuda()
        vs = V.transpose(0, 1).unsqueeze(0).cuda()
        torch.cuda._sleep(2_000_000)  # the producer's stream is still busy when the build is issued
        pipe.start_index_chunked(ks, vs, 32, ctx - 64, 0)
        del ks, vs  # the build keeps the storage alive (record_stream)
        torch.empty(64 << 20, dtype=torch.uint8, device="cuda").fill_(7)  # a reuse attempt of freed blocks
        idx = pipe.finish_index(as_host_metadata=False)
        st = pipe.get_pipeline_stats()
        assert st["kmeans_ms"] > 0 and st["reorganize_ms"] > 0
        out.append(idx)
    a, b = out
    for name in ("cell_sizes", "cell_offsets", "cell_code", "centroids", "list_keys", "list_values"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
