"""Seeded synthetic KV inputs with the shapes and value distributions of the
benchmark configurations (no dataset or checkpoint is needed or used).

Keys per KV head come from a Gaussian mixture (component means ~ N(0, 1),
within-component std ``spread``), then rotary position embedding (the
rotate-half form used by Llama / Qwen) is applied at their token positions.
Values are N(0, 1).  Decode queries are drawn from the same mixture and
rotated at the positions that follow the context.
"""
from __future__ import annotations

import torch


def rope(x: torch.Tensor, positions: torch.Tensor, theta: float) -> torch.Tensor:
    """Rotate-half RoPE over the last dim.  x: [..., T, D] fp32, positions: [T]."""
    D = x.shape[-1]
    half = D // 2
    inv = theta ** (-torch.arange(0, half, dtype=torch.float64, device=x.device) * 2.0 / D)
    ang = positions.to(torch.float64)[:, None] * inv[None, :]
    cos = torch.cos(ang).to(torch.float32)
    sin = torch.sin(ang).to(torch.float32)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def mixture_keys(kv_heads: int, tokens: int, dim: int, components: int, seed: int, theta: float,
                 spread: float = 0.3, start_pos: int = 0, device="cpu", gen_means=None):
    """[kv_heads, tokens, dim] fp32 keys (mixture + RoPE) and the mixture means."""
    g = torch.Generator(device=device).manual_seed(seed)
    means = gen_means
    if means is None:
        means = torch.randn(kv_heads, components, dim, generator=g, device=device)
    comp = torch.randint(0, components, (kv_heads, tokens), generator=g, device=device)
    noise = torch.randn(kv_heads, tokens, dim, generator=g, device=device) * spread
    x = torch.gather(means, 1, comp[..., None].expand(-1, -1, dim)) + noise
    pos = torch.arange(start_pos, start_pos + tokens, device=device)
    return rope(x, pos, theta), means


def make_layer(kv_heads: int, q_heads: int, context: int, dim: int, components: int, seed: int, theta: float,
               n_queries: int = 1, dtype=torch.bfloat16, device="cpu"):
    """One decoder layer's synthetic K/V for `context` tokens plus decode queries.

    Returns keys, values: [kv_heads, context, dim] (dtype); queries:
    [n_queries, q_heads, dim] (dtype) at positions context .. context+n_queries-1.
    """
    keys, means = mixture_keys(kv_heads, context, dim, components, seed, theta, device=device)
    g = torch.Generator(device=device).manual_seed(seed + 7919)
    values = torch.randn(kv_heads, context, dim, generator=g, device=device)
    G = q_heads // kv_heads
    qk = []
    for t in range(n_queries):
        q, _ = mixture_keys(kv_heads, G, dim, components, seed + 104729 + t, theta, start_pos=0, device=device,
                            gen_means=means)
        # all G query heads of a group sit at the same decode position
        q = rope(mixture_unrotate(q, theta), torch.full((G,), context + t, device=device), theta)
        qk.append(q.reshape(q_heads, dim))
    queries = torch.stack(qk, 0)
    return keys.to(dtype), values.to(dtype), queries.to(dtype)


def mixture_unrotate(x: torch.Tensor, theta: float) -> torch.Tensor:
    """Undo the RoPE that ``mixture_keys`` applied at positions 0..T-1."""
    T = x.shape[-2]
    D = x.shape[-1]
    half = D // 2
    inv = theta ** (-torch.arange(0, half, dtype=torch.float64, device=x.device) * 2.0 / D)
    ang = torch.arange(T, dtype=torch.float64, device=x.device)[:, None] * inv[None, :]
    cos = torch.cos(ang).to(torch.float32)
    sin = torch.sin(ang).to(torch.float32)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos + x2 * sin, x2 * cos - x1 * sin], dim=-1)
