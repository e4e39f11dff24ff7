"""Seeded synthetic activations with the shapes and value distributions of the
benchmark configurations (the reference ships no dataset; its scripts use
``torch.randn``).

* ``lowrank_activation`` -- config-1/2 generator: rank-``signal_rank`` signal
  A(T x s) B(s x H) with A, B ~ N(0,1)/sqrt(s), plus ``noise`` * N(0,1), plus
  ``n_outlier`` random channels scaled by ``outlier_scale``.
* ``heavy_tailed_activation`` -- config-3 generator: Student-t(nu=3) * 0.5.
* ``causal_softmax`` -- config-5 probabilities: causal softmax of N(0,1)/sqrt(128)
  logits.
Generated on the requested device with a torch.Generator seeded per call, so
every rank / test gets reproducible data (seed + rank for sharded runs).
"""
from __future__ import annotations

import math

import torch


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def lowrank_activation(T: int, H: int, *, signal_rank: int = 64, noise: float = 0.05, n_outlier: int = 16,
                       outlier_scale: float = 30.0, seed: int = 0, device="cpu", dtype=torch.bfloat16,
                       outlier_seed: int | None = None):
    """Returns (x, outlier_channels).  The outlier channels are drawn from
    ``outlier_seed`` (default ``seed``) so shards of one activation share them."""
    g = _gen(seed, device)
    a = torch.randn(T, signal_rank, generator=g, device=device) / math.sqrt(signal_rank)
    b = torch.randn(signal_rank, H, generator=g, device=device) / math.sqrt(signal_rank)
    x = a @ b
    x += noise * torch.randn(T, H, generator=g, device=device)
    go = _gen(seed if outlier_seed is None else outlier_seed, "cpu")
    ch = torch.randperm(H, generator=go)[:n_outlier].sort().values
    if n_outlier:
        x[:, ch.to(device)] *= outlier_scale
    return x.to(dtype), ch.to(torch.int32)


def heavy_tailed_activation(T: int, H: int, *, nu: float = 3.0, scale: float = 0.5, seed: int = 0, device="cpu",
                            dtype=torch.bfloat16):
    g = _gen(seed, device)
    z = torch.randn(T, H, generator=g, device=device)
    # chi-square with nu degrees of freedom as a sum of nu squared normals (nu integer)
    chi = torch.zeros(T, H, device=device)
    for _ in range(int(nu)):
        chi += torch.randn(T, H, generator=g, device=device) ** 2
    return (scale * z / torch.sqrt(chi / nu)).to(dtype)


def causal_softmax(B: int, heads: int, S: int, *, head_dim: int = 128, seed: int = 0, device="cpu",
                   dtype=torch.bfloat16):
    g = _gen(seed, device)
    logits = torch.randn(B, heads, S, S, generator=g, device=device) / math.sqrt(head_dim)
    mask = torch.ones(S, S, dtype=torch.bool, device=device).triu(1)
    logits.masked_fill_(mask, float("-inf"))
    return torch.softmax(logits, dim=-1).to(dtype)


def gradient(shape, *, std: float = 0.02, seed: int = 1, device="cpu", dtype=torch.bfloat16):
    g = _gen(seed, device)
    return (std * torch.randn(*shape, generator=g, device=device)).to(dtype)
