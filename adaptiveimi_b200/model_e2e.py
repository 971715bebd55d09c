"""End-to-end decoding through the IMI cache: a tensor-parallel Qwen2-style
decoder with random weights (Qwen2.5-72B geometry, 8 GPUs,
one KV head per GPU, a 131 072-token prompt, 128 greedy tokens).

This is the caller of the hot path, written the way the reference's model
wrappers drive the cache (model_hub/base.py:407-544 ``inference``,
model_hub/prefill.py, model_hub/qwen.py): prefill layer by layer with
``prefill_update_kv_cache`` (the IMI of each layer is built on the device from
the K/V the layer just produced), ``prepare_cache`` after the prompt, then per
decode step and layer ``decode_update_kv_cache`` followed by
``imi_decode_attn``.  It has no weights to load (there is no network): every
projection is random-init with the architecture's shapes, so the tokens it
emits mean nothing; the work per token is the real model's.

Tensor parallelism (one process per GPU, NCCL): the query, key and value heads
are split across ranks (Qwen2.5-72B: 64 query / 8 KV heads -> 8 / 1 per GPU),
o_proj and down_proj are row-parallel with an all-reduce after each, the MLP
is column-parallel, the embedding and lm_head are vocab-parallel (greedy
argmax over the ranks' shards).  ``attention`` is pluggable: ``"imi"`` uses
the IMI cache; ``"dense"`` keeps plain K/V and attends to all of it (the CPU
test of the sharding logic uses it).
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class DecoderConfig:
    layers: int = 80
    hidden: int = 8192
    q_heads: int = 64
    kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 29568
    vocab: int = 152064
    rope_theta: float = 1e6
    rms_eps: float = 1e-6

    @staticmethod
    def qwen25_72b() -> "DecoderConfig":
        return DecoderConfig()


def _dist():
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist, dist.get_world_size(), dist.get_rank()
    return None, 1, 0


def _all_reduce(x: torch.Tensor) -> torch.Tensor:
    dist, ws, _ = _dist()
    if ws > 1:
        dist.all_reduce(x)
    return x


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * w.float()).to(x.dtype)


def rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float):
    inv = theta ** (-torch.arange(0, head_dim, 2, dtype=torch.float64, device=positions.device) / head_dim)
    ang = positions.to(torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).to(torch.float32), torch.sin(ang).to(torch.float32)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x: [T, heads, D] (rotate-half form); cos/sin: [T, D/2]."""
    half = x.shape[-1] // 2
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


def _randn(shape, seed: int, device, std: float) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std).to(torch.bfloat16)


class TPDecoder:
    """Random-init tensor-parallel decoder.  Weights come in units that do not
    depend on the world size (one KV group's heads; one eighth of the MLP and
    of the vocabulary), each seeded by (layer, kind, unit), so any world size
    that divides the unit count holds slices of the same model."""

    def __init__(self, cfg: DecoderConfig, device, seed: int = 0, attention: str = "imi", std: float = 0.02):
        _, ws, rank = _dist()
        if cfg.kv_heads % ws or cfg.q_heads % cfg.kv_heads:
            raise ValueError("the KV heads must split evenly over the ranks")
        self.cfg, self.device, self.attention = cfg, torch.device(device), attention
        self.ws, self.rank = ws, rank
        U = cfg.kv_heads                       # units: KV groups
        self.units = list(range(rank * U // ws, (rank + 1) * U // ws))
        self.kvh = len(self.units)             # KV heads on this rank
        self.G = cfg.q_heads // cfg.kv_heads
        self.qh = self.kvh * self.G            # query heads on this rank
        if cfg.intermediate % U or cfg.vocab % U:
            raise ValueError("intermediate size and vocabulary must split into the unit count")
        iu, vu, D, H = cfg.intermediate // U, cfg.vocab // U, cfg.head_dim, cfg.hidden
        dev = self.device
        cat = lambda xs, dim=0: torch.cat(xs, dim)  # noqa: E731
        self.layers = []
        for l in range(cfg.layers):
            wq, wk, wv, bq, bk, bv, wo, gate, up, down = [], [], [], [], [], [], [], [], [], []
            for u in self.units:
                s = (seed * 1000 + l) * 64 + u * 8
                wq.append(_randn((self.G * D, H), s + 0, dev, std))
                wk.append(_randn((D, H), s + 1, dev, std))
                wv.append(_randn((D, H), s + 2, dev, std))
                bq.append(_randn((self.G * D,), s + 3, dev, std))
                bk.append(_randn((D,), s + 4, dev, std))
                bv.append(_randn((D,), s + 5, dev, std))
                wo.append(_randn((H, self.G * D), s + 6, dev, std))
                gu = _randn((2 * iu, H), s + 7, dev, std)
                gate.append(gu[:iu])
                up.append(gu[iu:])
                down.append(_randn((H, iu), s + 7 + 1_000_003, dev, std))
            self.layers.append(dict(
                wqkv=cat(wq + wk + wv), bqkv=cat(bq + bk + bv), wo=cat(wo, 1), gate_up=cat(gate + up),
                down=cat(down, 1), ln1=torch.ones(H, dtype=torch.bfloat16, device=dev),
                ln2=torch.ones(H, dtype=torch.bfloat16, device=dev)))
        self.vocab0 = self.units[0] * vu
        self.embed = cat([_randn((vu, H), (seed * 1000 + 999) * 64 + u, dev, 1.0) for u in self.units])
        self.lm_head = cat([_randn((vu, H), (seed * 1000 + 998) * 64 + u, dev, std) for u in self.units])
        self.norm = torch.ones(H, dtype=torch.bfloat16, device=dev)
        self.cache = None
        self.dense_kv: List[Optional[tuple]] = [None] * cfg.layers
        self._graphs = None
        self.last_hidden: Optional[torch.Tensor] = None   # hidden state after the last decode step

    # -- pieces -------------------------------------------------------------------
    def _embed(self, ids: torch.Tensor) -> torch.Tensor:
        local = ids - self.vocab0
        ok = (local >= 0) & (local < self.embed.shape[0])
        h = self.embed[local.clamp(0, self.embed.shape[0] - 1)] * ok[:, None].to(torch.bfloat16)
        return _all_reduce(h)

    def _qkv(self, lw, x: torch.Tensor, positions: torch.Tensor):
        D = self.cfg.head_dim
        qkv = F.linear(x, lw["wqkv"], lw["bqkv"])
        q = qkv[:, :self.qh * D].view(-1, self.qh, D)
        k = qkv[:, self.qh * D:(self.qh + self.kvh) * D].view(-1, self.kvh, D)
        v = qkv[:, (self.qh + self.kvh) * D:].reshape(-1, self.kvh, D).contiguous()
        cos, sin = rope_cos_sin(positions, D, self.cfg.rope_theta)
        return apply_rope(q, cos, sin), apply_rope(k, cos, sin), v

    def _mlp(self, lw, h: torch.Tensor, chunk: int = 16384) -> None:
        """h += down(silu(gate(x)) * up(x)), x = rms(h); in token chunks, in place."""
        I = lw["down"].shape[1]
        for a in range(0, h.shape[0], chunk):
            x = rms_norm(h[a:a + chunk], lw["ln2"], self.cfg.rms_eps)
            gu = F.linear(x, lw["gate_up"])
            y = F.linear(F.silu(gu[:, :I]) * gu[:, I:], lw["down"])
            h[a:a + chunk] += _all_reduce(y)

    def _greedy(self, h_last: torch.Tensor) -> torch.Tensor:
        """Vocab-parallel greedy token of one position (h_last: [H])."""
        x = rms_norm(h_last[None], self.norm, self.cfg.rms_eps)
        logits = F.linear(x, self.lm_head).float()[0]
        val, idx = logits.max(0)
        dist, ws, _ = _dist()
        if ws == 1:
            return (idx + self.vocab0).view(1)
        pair = torch.stack([val, (idx + self.vocab0).float()])
        allp = torch.empty((ws, 2), dtype=torch.float32, device=pair.device)
        dist.all_gather_into_tensor(allp.view(-1), pair)
        best = int(torch.argmax(allp[:, 0]))  # ties: the lowest rank, i.e. the lowest vocabulary id
        return allp[best, 1].to(torch.int64).view(1)

    # -- attention ------------------------------------------------------------------
    def _prefill_attention(self, l: int, q, k, v) -> torch.Tensor:
        """Causal attention of the prompt (the reference's full prefill attention,
        attn_hub/full.py), then the layer's K/V to the cache, which builds the
        layer's IMI from them on the device.  q: [T, qh, D]; k, v: [T, kvh, D]."""
        o = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None], v.transpose(0, 1)[None],
                                           is_causal=True, enable_gqa=True)
        if self.attention == "imi":
            self.cache.prefill_update_kv_cache(None, k[None], v[None], l, 0)
        else:
            self.dense_kv[l] = (k.clone(), v.clone())
        return o[0].transpose(0, 1).reshape(q.shape[0], -1)

    def _decode_attention(self, l: int, q, k, v) -> torch.Tensor:
        """One new token: the cache append, then the sparse attention
        (attn_hub/sparse_imi.imi_decode_attn).  q: [1, qh, D]; k, v: [1, kvh, D]."""
        if self.attention == "imi":
            from .attn import imi_decode_attn

            self.cache.decode_update_kv_cache(k[None], v[None], l)
            o = imi_decode_attn(q[None], None, None, l, self.cache)
            return o.reshape(1, -1)
        kk, vv = self.dense_kv[l]
        kk, vv = torch.cat([kk, k]), torch.cat([vv, v])
        self.dense_kv[l] = (kk, vv)
        o = F.scaled_dot_product_attention(q.transpose(0, 1)[None], kk.transpose(0, 1)[None], vv.transpose(0, 1)[None],
                                           enable_gqa=True)
        return o[0].transpose(0, 1).reshape(1, -1)

    # -- passes ---------------------------------------------------------------------
    def _layer(self, l: int, h: torch.Tensor, positions: torch.Tensor, prefill: bool) -> None:
        lw = self.layers[l]
        x = rms_norm(h, lw["ln1"], self.cfg.rms_eps)
        q, k, v = self._qkv(lw, x, positions)
        del x
        o = self._prefill_attention(l, q, k, v) if prefill else self._decode_attention(l, q, k, v)
        h += _all_reduce(F.linear(o, lw["wo"]))
        self._mlp(lw, h)

    def prefill(self, ids: torch.Tensor) -> torch.Tensor:
        """ids: [T] prompt token ids -> the first generated token ([1])."""
        h = self._embed(ids)
        pos = torch.arange(ids.shape[0], device=self.device)
        for l in range(self.cfg.layers):
            self._layer(l, h, pos, True)
        return self._greedy(h[-1])

    def decode(self, token: torch.Tensor, position: int) -> torch.Tensor:
        if self._graphs is not None:
            return self._decode_graphed(token, position)
        h = self._embed(token)
        pos = torch.full((1,), position, device=self.device, dtype=torch.int64)
        for l in range(self.cfg.layers):
            self._layer(l, h, pos, False)
        self.last_hidden = h
        return self._greedy(h[0])

    # -- CUDA graphs of a decode step's dense work ----------------------------------
    def _pre(self, l: int):
        """Graph body before the cache: norm, QKV projection, RoPE (static buffers)."""
        lw, D = self.layers[l], self.cfg.head_dim
        x = rms_norm(self._g_h, lw["ln1"], self.cfg.rms_eps)
        qkv = F.linear(x, lw["wqkv"], lw["bqkv"])
        q = qkv[:, :self.qh * D].view(-1, self.qh, D)
        k = qkv[:, self.qh * D:(self.qh + self.kvh) * D].view(-1, self.kvh, D)
        v = qkv[:, (self.qh + self.kvh) * D:].reshape(-1, self.kvh, D).contiguous()
        return apply_rope(q, self._g_cos, self._g_sin), apply_rope(k, self._g_cos, self._g_sin), v

    def _post(self, l: int) -> None:
        """Graph body after the cache: o_proj + all-reduce, the MLP (in place on h)."""
        lw = self.layers[l]
        self._g_h += _all_reduce(F.linear(self._g_o, lw["wo"]))
        self._mlp(lw, self._g_h)

    def capture_decode_graphs(self) -> None:
        """Capture, per layer, the dense work before and after the cache calls as
        two CUDA graphs over static buffers (the hidden state, RoPE cos/sin, the
        attention output), so a decode step is 2 graph launches per layer plus
        the cache's own launches instead of ~50 eager kernel launches per layer.
        The cache calls (append, selection, attention) stay eager: their
        descriptors carry the step's position and the asynchronous centroid
        update schedule, which change from step to step.  For a
        single process only (there are no all-reduces inside the graphs then)."""
        if self.device.type != "cuda":
            raise RuntimeError("decode graphs need a CUDA device")
        if self.ws > 1:
            # An 8-rank run with the all-reduces captured inside these graphs
            # stalled without output on B200 (cause not found), so multi-rank
            # decoding keeps its dense work eager.
            raise RuntimeError("decode graphs are single-process only; tensor-parallel decoding runs eagerly")
        H, D = self.cfg.hidden, self.cfg.head_dim
        dev = self.device
        self._g_h = torch.zeros((1, H), dtype=torch.bfloat16, device=dev)
        self._g_o = torch.zeros((1, self.qh * D), dtype=torch.bfloat16, device=dev)
        self._g_cos = torch.zeros((1, D // 2), dtype=torch.float32, device=dev)
        self._g_sin = torch.zeros((1, D // 2), dtype=torch.float32, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):         # warm-up outside capture (library handles, workspaces)
            for _ in range(3):
                self._pre(0)
                self._post(0)
        torch.cuda.current_stream(dev).wait_stream(side)
        pool = torch.cuda.graph_pool_handle()
        graphs = []
        for l in range(self.cfg.layers):
            ga, gb = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            with torch.cuda.graph(ga, pool=pool):
                qkv = self._pre(l)
            with torch.cuda.graph(gb, pool=pool):
                self._post(l)
            graphs.append((ga, qkv, gb))
        torch.cuda.synchronize(dev)
        self._graphs = graphs

    def _decode_graphed(self, token: torch.Tensor, position: int) -> torch.Tensor:
        self._g_h.copy_(self._embed(token))
        pos = torch.full((1,), position, device=self.device, dtype=torch.int64)
        cos, sin = rope_cos_sin(pos, self.cfg.head_dim, self.cfg.rope_theta)
        self._g_cos.copy_(cos)
        self._g_sin.copy_(sin)
        for l, (ga, (q, k, v), gb) in enumerate(self._graphs):
            ga.replay()
            self._g_o.copy_(self._decode_attention(l, q, k, v))
            gb.replay()
        self.last_hidden = self._g_h
        return self._greedy(self._g_h[0])

    def make_cache(self, prompt_len: int, new_tokens: int, *, budget: float = 0.1, parts: int = 2,
                   kmeans: Optional[dict] = None):
        """The IMI cache of this rank's KV heads (model_hub/base.py:208-256)."""
        from .cache import adpimi_cache

        c = self.cfg
        dev = str(self.device) if self.device.index is not None else f"cuda:{torch.cuda.current_device()}"
        self.cache = adpimi_cache(
            valid_start=[0], layer_num=c.layers, batch_size=1, max_length=prompt_len + new_tokens + 1,
            num_key_value_heads=self.kvh, num_heads=self.qh, head_dim=c.head_dim, dtype=torch.bfloat16,
            layer_mapping={str(i): dev for i in range(c.layers)}, max_new_length=new_tokens + 1,
            input_length=prompt_len, static_pattern_start=32, static_pattern_end=64, core=1, pages_per_cluster=2,
            retrieval_budget=budget, cache_ratio=0.05, buffer_cluster_num=32, prefill_bsz=1, num_gpus=self.ws,
            model_size=72, subspace_parts=parts, runtime_config={"kmeans": dict(kmeans or {})})
        return self.cache


def generate(model: TPDecoder, ids: torch.Tensor, new_tokens: int, graphs: bool = False) -> dict:
    """model_hub/base.py:407-496 ``inference`` with greedy sampling: prefill,
    ``prepare_cache`` (the reference's ``move``), then new_tokens - 1 decode
    steps.  Returns the tokens and the timings (wall clock around synchronised
    device work, as the reference reports them).  ``graphs`` captures the
    dense part of each decode layer as CUDA graphs after ``prepare_cache``
    (counted in the prefill time)."""
    dev = model.device

    def sync():
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)

    sync()
    t0 = time.perf_counter()
    tok = model.prefill(ids)
    out = [tok]
    if model.cache is not None:
        model.cache.prepare_cache()
    if graphs:
        model.capture_decode_graphs()
    sync()
    t1 = time.perf_counter()
    T = ids.shape[0]
    for step in range(new_tokens - 1):
        tok = model.decode(tok, T + step)
        out.append(tok)
    sync()
    t2 = time.perf_counter()
    build_ms = 0.0
    if model.cache is not None:
        for p in model.cache.imi_pipelines:
            st = p.get_pipeline_stats() if p is not None else {}
            build_ms += float(st.get("kmeans_ms", 0.0)) + float(st.get("reorganize_ms", 0.0))
    steps = new_tokens - 1
    return {"tokens": torch.cat(out).tolist(), "prefill_s": t1 - t0, "decode_s": t2 - t1,
            "decode_tokens_per_s": steps / (t2 - t1) if steps > 0 else 0.0, "build_ms": build_ms}
