"""Generate tests/golden/async_update_ref.npz: the reference's own async
centroid update (cache_hub/adaptive_imi/async_update.py,
``AdaptiveIMIAsyncUpdateMixin._schedule_async_update``, lines 79-161) run
unchanged on CPU torch over seeded inputs.

The method is loaded from the reference checkout by file path and called on a
small stand-in object that carries exactly the attributes it reads (buffers
shaped as runtime.py:108-160 makes them).  Its CUDA stream and event calls are
the only things replaced: ``torch.cuda.current_stream`` / ``torch.cuda.stream``
become no-ops and the events report completion, so the torch arithmetic itself
-- ``torch.bmm`` over fp32 keys and the shadow centroids, ``argmax``,
``scatter_add_``, the thresholded running mean -- runs as written, on CPU.

Inputs: one IMI per KV group built by the CPU oracle over the first tokens of a
config-0-style layer (S=2, k=12x12, padded to 145 slots, zero padding
centroids), then 64 later keys of the same layer fed as four batches of 16.
Outputs per batch: the cell ids the reference assigned (its ``torch.argmax``
results, recorded as it returns them), then the final shadow centroids, counts
and pending deltas, and the delta ring's state: its ids stay at the padding id
and its rows at zero (its ``tensor[g, pos].copy_(x)`` with a tensor index
writes into a temporary) while its count and write position advance.

Run in a container with the reference checkout:
    python tests/golden/gen_async_pin.py
"""
from __future__ import annotations

import contextlib
import importlib.util
import os
import sys
from pathlib import Path
from unittest import mock

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
OUT = Path(__file__).resolve().parent / "async_update_ref.npz"

from adaptiveimi_b200.synthetic import make_layer  # noqa: E402
from oracle import oracle as O  # noqa: E402

REF = Path(os.environ.get("IMI_REFERENCE_ROOT", "/root/reference"))
KV, CTX, EXTRA, KS, BATCH, THRESHOLD, DELTA = 2, 2048, 64, (12, 12), 16, 3, 512


def pin_inputs():
    """Shadow centroids, counts and decode keys (bf16) -- also used by the test."""
    K, V, _ = make_layer(KV, KV * 4, CTX + EXTRA, 128, 64, 17, 500000.0, n_queries=1)
    n_slots = KS[0] * KS[1] + 1
    shadow = np.zeros((KV, n_slots, 128), np.float32)
    counts = np.zeros((KV, n_slots), np.int32)
    kb, vb = O.bf16_bits(K[:, :CTX]), O.bf16_bits(V[:, :CTX])
    for h in range(KV):
        o = O.build_head(kb[h], vb[h], 2, KS, 8)
        na = o["n_active"]
        shadow[h, :na] = o["merged"]
        counts[h, :na] = np.diff(o["offsets"])
    return shadow, counts, K[:, CTX:].contiguous(), V[:, CTX:].contiguous()


def load_reference_mixin():
    path = REF / "cache_hub" / "adaptive_imi" / "async_update.py"
    spec = importlib.util.spec_from_file_location("ref_async_update", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.AdaptiveIMIAsyncUpdateMixin


class _Done:
    def record(self, *a, **k):
        pass

    def query(self):
        return True


class _Stream:
    def wait_stream(self, *a, **k):
        pass

    def wait_event(self, *a, **k):
        pass


def run_reference(shadow0, counts0, keys, values):
    Mixin = load_reference_mixin()
    n_slots = shadow0.shape[1]
    dev = "cpu"
    st = type("Cache", (), {})()
    st.async_update_enabled = True
    st.batch_groups, st.head_dim = KV, 128
    st.async_update_batch, st.async_update_threshold = BATCH, THRESHOLD
    st.layer_mapping = {"0": dev}
    st.async_update_streams = {dev: _Stream()}
    st.centroids_shadow = [torch.from_numpy(shadow0.copy())]
    st.centroid_counts = [torch.from_numpy(counts0.copy())]
    st.delta_counts = [torch.zeros_like(st.centroid_counts[0])]
    st.delta_sums = [torch.zeros((KV, n_slots, 128), dtype=torch.float32)]
    st.delta_keys = [torch.zeros((KV, DELTA, 128), dtype=torch.bfloat16)]
    st.delta_values = [torch.zeros((KV, DELTA, 128), dtype=torch.bfloat16)]
    st.delta_cluster_ids = [torch.full((KV, DELTA), n_slots - 1, dtype=torch.int64)]
    st.delta_counts_gpu = [torch.zeros((KV,), dtype=torch.int32)]
    st.async_update_buffers = [{
        "keys": torch.empty((KV, BATCH, 128), dtype=torch.bfloat16),
        "values": torch.empty((KV, BATCH, 128), dtype=torch.bfloat16),
        "count": 0, "event": _Done(), "delta_event": _Done(),
        "delta_write_pos": torch.zeros((KV,), dtype=torch.int64),
    }]
    ids = []
    real_argmax = torch.argmax

    def recording_argmax(*a, **k):  # the method's cell ids, as it computes them
        r = real_argmax(*a, **k)
        ids.append(r.clone().numpy())
        return r

    with mock.patch.object(torch.cuda, "current_stream", lambda *a, **k: _Stream()), \
            mock.patch.object(torch.cuda, "stream", lambda *a, **k: contextlib.nullcontext()), \
            mock.patch.object(torch, "argmax", recording_argmax):
        for t in range(keys.shape[1]):
            k_t = keys[:, t].reshape(1, 1, KV, 128)
            v_t = values[:, t].reshape(1, 1, KV, 128)
            Mixin._schedule_async_update(st, 0, k_t, v_t)
    return dict(ids=np.stack(ids).astype(np.int32), shadow=st.centroids_shadow[0].numpy(),
                counts=st.centroid_counts[0].numpy(), delta_counts=st.delta_counts[0].numpy(),
                delta_sums=st.delta_sums[0].numpy(), ring_count=st.delta_counts_gpu[0].numpy(),
                ring_ids=st.delta_cluster_ids[0].numpy(), ring_keys_nonzero=np.array(
                    int(st.delta_keys[0].float().abs().sum() != 0)),
                ring_write_pos=st.async_update_buffers[0]["delta_write_pos"].numpy())


def main():
    shadow0, counts0, keys, values = pin_inputs()
    r = run_reference(shadow0, counts0, keys, values)
    np.savez_compressed(OUT, threshold=np.array(THRESHOLD), batch=np.array(BATCH), **r)
    print("wrote", OUT.name, "batches", r["ids"].shape, "updated cells",
          int((r["counts"] != counts0).sum()))


if __name__ == "__main__":
    main()
