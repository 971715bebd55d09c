"""Host-side behaviour of IMIPipeline (library/AdaptiveIMI/imi_adapter.py:129-479):
argument checks, stage transitions, wait/timeout, cancel, per-stage statistics
and the failure path of a build whose device status word reports a give-up.

No GPU: the device build is replaced by a fake that fills the same output
tensors on the CPU, and CUDA events by a fake whose completion the test
controls."""
import contextlib

import pytest
import torch

from adaptiveimi_b200 import imi_adapter, ops
from adaptiveimi_b200.imi_adapter import IMIPipeline, PipelineStage


class FakeEvent:
    done = True

    def record(self, *a, **k):
        pass

    def query(self):
        return FakeEvent.done


@pytest.fixture
def fake_device(monkeypatch):
    """CPU stand-ins for the CUDA plumbing IMIPipeline touches."""
    calls = {}
    FakeEvent.done = True
    monkeypatch.setattr(imi_adapter.torch.cuda, "Event", FakeEvent)
    monkeypatch.setattr(imi_adapter.torch.cuda, "device", lambda d: contextlib.nullcontext())
    monkeypatch.setattr(IMIPipeline, "_device", lambda self: torch.device("cpu"))

    def fake_build(keys, values, *, parts, ks, n_slots, status=None, phase_ns=None, list_keys=None,
                   list_values=None, **settings):
        H, n, D = keys.shape
        calls.update(parts=parts, ks=ks, n_slots=n_slots, settings=settings)
        if calls.get("fail"):
            status.fill_(1)
        phase_ns.copy_(torch.tensor([1_000_000, 4_500_000, 5_250_000]))
        na = torch.full((H,), calls.get("n_active", 3), dtype=torch.int32)
        sizes = torch.zeros((H, n_slots), dtype=torch.int32)
        sizes[:, :3] = torch.tensor([n - 2, 1, 1])
        offs = torch.zeros((H, n_slots + 1), dtype=torch.int32)
        offs[:, 1:] = sizes.cumsum(1)
        return ops.IMIIndex(parts=parts, ks=tuple(ks), kmax=max(ks), n_tokens=n, n_slots=n_slots,
                            list_keys=keys.clone(), list_values=values.clone(), cell_sizes=sizes,
                            cell_offsets=offs, cell_mask=(sizes == 0).to(torch.uint8),
                            cell_code=torch.zeros((H, n_slots), dtype=torch.int32),
                            centroids=torch.zeros((H, n_slots, D)), sub_centroids=torch.zeros((H, 2, max(ks), D // 2)),
                            sub_labels=torch.zeros((H, 2, n), dtype=torch.int32), n_active=na,
                            iters_run=torch.zeros((H, 2), dtype=torch.int32))

    monkeypatch.setattr(imi_adapter.ops, "build_index", fake_build)
    return calls


def _pipe(**kw):
    args = dict(layer_idx=0, kv_heads=2, head_dim=128, dtype=torch.bfloat16, device_id=0, max_tokens=4096)
    args.update(kw)
    return IMIPipeline(**args)


def _kv(h=2, t=1024, b=1):
    k = torch.randn(b, h, t, 128).to(torch.bfloat16)
    return k, k.clone()


def test_argument_checks_use_the_reference_errors():
    with pytest.raises(ValueError, match="subspace_parts"):
        _pipe(subspace_parts=3)
    p = _pipe()
    with pytest.raises(ValueError, match=r"\[1, kv_heads, tokens, head_dim\]"):
        p.start_index(torch.zeros(2, 8, 128), torch.zeros(2, 8, 128))
    with pytest.raises(ValueError, match="batch_size=1"):
        p.start_index(*_kv(b=2))
    with pytest.raises(ValueError, match="kv_heads mismatch"):
        p.start_index(*_kv(h=3))
    with pytest.raises(ValueError, match="exceeds max_tokens"):
        p.start_index(*_kv(t=5000))
    with pytest.raises(ValueError, match="share the same shape"):
        p.start_index(_kv()[0], _kv(t=512)[0])
    with pytest.raises(ValueError, match="non-empty"):
        p.begin_index_stream(0, 128)
    with pytest.raises(ValueError, match="submit_chunk_size"):
        p.begin_index_stream(128, 0)
    with pytest.raises(RuntimeError, match="failed to submit chunk"):
        p.submit_index_stream_chunk(*_kv(t=8), chunk_id=0, token_offset=0, is_last=False)
    with pytest.raises(ValueError, match="Invalid middle token range"):
        p.start_index_chunked(torch.zeros(1, 64, 2, 128), torch.zeros(1, 64, 2, 128), 40, 20, 0)
    with pytest.raises(ValueError, match="worker_threads"):
        p.set_worker_threads(0)


def test_finish_before_start_and_wait_without_build():
    p = _pipe()
    assert p.stage == PipelineStage.Idle
    assert p.wait_ready(0.0) is False
    with pytest.raises(RuntimeError, match="finish called before start"):
        p.finish_index()


def test_build_completes_with_stage_statistics(fake_device):
    p = _pipe(runtime_config=imi_adapter.IMIRuntimeConfig(kmeans={"k1": 16, "k2": 16, "max_iters": 7}))
    meta = p.build_index(*_kv())
    assert p.stage == PipelineStage.Complete
    assert fake_device["ks"] == (16, 16) and fake_device["n_slots"] == 257
    assert fake_device["settings"]["max_iters"] == 7
    assert [m["head_idx"] for m in meta] == [0, 1]
    assert meta[0]["cluster_offsets"].tolist() == [0, 1022, 1023, 1024]
    st = p.get_pipeline_stats()
    assert st["kmeans_ms"] == pytest.approx(3.5) and st["reorganize_ms"] == pytest.approx(0.75)
    assert st["d2h_ms"] == 0.0 and st["total_tokens"] == 1024 and st["total_chunks"] == 1
    assert p.get_last_pipeline_stats() == st


def test_chunked_stream_submission(fake_device):
    p = _pipe()
    k, v = _kv(t=300)
    p.begin_index_stream(300, 128)
    assert p.stage == PipelineStage.Transferring
    for i, off in enumerate(range(0, 300, 128)):
        p.submit_index_stream_chunk(k[:, :, off:off + 128], v[:, :, off:off + 128], i, off, off + 128 >= 300)
    p.finish_index()
    assert p.get_pipeline_stats()["total_chunks"] == 3
    with pytest.raises(RuntimeError, match="failed to submit chunk"):
        p.begin_index_stream(100, 64)
        p.submit_index_stream_chunk(*_kv(t=128), chunk_id=0, token_offset=0, is_last=True)


def test_device_give_up_fails_the_build(fake_device):
    fake_device["fail"] = True
    p = _pipe()
    p.start_index(*_kv())
    assert p.wait_ready(1.0) is False
    assert p.stage == PipelineStage.Failed
    assert "gave up" in p.error_message
    with pytest.raises(RuntimeError, match="IMI pipeline failed"):
        p.finish_index()


def test_cell_overflow_fails_the_build(fake_device):
    fake_device["n_active"] = 300  # more cells than 16*16 + 1 slots hold
    p = _pipe(runtime_config=imi_adapter.IMIRuntimeConfig(kmeans={"k1": 16, "k2": 16}))
    p.start_index(*_kv())
    with pytest.raises(RuntimeError, match="300 cells for 257 slots"):
        p.finish_index()


def test_wait_timeout_and_cancel(fake_device):
    p = _pipe()
    p.start_index(*_kv())
    FakeEvent.done = False
    assert p.wait_ready(0.01) is False
    assert p.stage == PipelineStage.Clustering
    p.cancel_pipeline()
    assert p.stage == PipelineStage.Idle
    assert p.wait_ready(0.0) is False
    with pytest.raises(RuntimeError, match="finish called before start"):
        p.finish_index()
    FakeEvent.done = True
    p.start_index(*_kv())
    p.finish_index()
    assert p.stage == PipelineStage.Complete


def test_launch_error_marks_failure(fake_device, monkeypatch):
    def boom(*a, **k):
        raise ValueError("workspace too small")

    monkeypatch.setattr(imi_adapter.ops, "build_index", boom)
    p = _pipe()
    with pytest.raises(RuntimeError, match="IMI pipeline failed: workspace too small"):
        p.start_index(*_kv())
    assert p.stage == PipelineStage.Failed and p.wait_ready(0.0) is False
