"""PyTorch statement of the channel-group encode/decode as the north star
words it (TEST INFRASTRUCTURE ONLY).

An independent checker for oracle/actcomp_oracle.c and the CUDA kernels:
plain float32 torch operations in the order the specification names them,
with no attempt to mirror any kernel's rounding points.

  L        = X @ V                         (projection onto the rank-r basis)
  R        = X - L @ V^T                   (residual, float32)
  outliers = X[:, idx] verbatim;  R[:, idx] = 0
  R        = R rotated per 128-channel block by the (unnormalised) Walsh-Hadamard
             matrix when wht is set
  scale    = absmax over each group of R per token / qmax,  qmax = 2^(bits-1) - 1
  codes    = torch.round(R * (qmax / absmax))   (round half to even)
  X^       = L @ V^T + codes * scale (rotated back, / 128), outliers put back

Reference code this follows: the reference's encode math
(low_rank_extraction_fuse_compression_quantization.py:66-100: residual
x - l@r, scale, round, clamp) with its per-channel scale replaced by the
per-token group absmax of the north star, the channel gather of
extraction_outlier_channel.py:11-14 for the outliers, and the end-to-end
check of low_rank_kernel_accuracy_test.py:6-16.  "Identical V_r": callers pass
the same basis the kernels use (V rounded to bf16, as float32 values).

Only tests/ and bench.py's reporting legs import this module.
"""
from __future__ import annotations

import torch


def hadamard128(device="cpu") -> torch.Tensor:
    """The 128 x 128 Sylvester Hadamard matrix (entries +-1, float32)."""
    h = torch.ones(1, 1, device=device)
    while h.shape[0] < 128:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h


def encode(x: torch.Tensor, V: torch.Tensor, idx, bits: int, group: int, wht: bool = False) -> dict:
    """x (T, H) and V (H, r) float32 (V may have r = 0); idx: outlier channels.

    Returns L (T, r), codes (T, H) int32 signed, scales (T, H/group),
    outliers (T, k), and ``pre`` = the value each code rounds (T, H)."""
    x = x.to(torch.float32)
    T, H = x.shape
    V = V.to(torch.float32)
    r = V.shape[1]
    idx = torch.as_tensor(idx if idx is not None else [], dtype=torch.long)
    if r:
        L = x @ V
        R = x - L @ V.T
    else:
        L = torch.zeros(T, 0)
        R = x.clone()
    outl = x[:, idx].clone()
    R[:, idx] = 0.0
    if wht:
        R = (R.view(T, H // 128, 128) @ hadamard128()).view(T, H)
    qmax = (1 << (bits - 1)) - 1
    Rg = R.view(T, H // group, group)
    amax = Rg.abs().amax(-1, keepdim=True)
    scale = amax / qmax
    rs = torch.where(amax > 0, qmax / torch.where(amax > 0, amax, torch.ones_like(amax)), torch.zeros_like(amax))
    pre = Rg * rs
    codes = torch.round(pre).clamp(-qmax, qmax).to(torch.int32)
    return {"lowrank": L, "codes": codes.view(T, H), "scales": scale.view(T, -1), "outliers": outl,
            "pre": pre.view(T, H)}


def decode(enc: dict, V: torch.Tensor, idx, group: int, wht: bool = False) -> torch.Tensor:
    """Float32 reconstruction X^ from the output of :func:`encode`."""
    codes = enc["codes"].to(torch.float32)
    T, H = codes.shape
    w = (codes.view(T, H // group, group) * enc["scales"].view(T, -1, 1)).view(T, H)
    if wht:
        w = (w.view(T, H // 128, 128) @ hadamard128()).view(T, H) / 128.0
    V = V.to(torch.float32)
    xh = enc["lowrank"] @ V.T + w if V.shape[1] else w
    idx = torch.as_tensor(idx if idx is not None else [], dtype=torch.long)
    xh[:, idx] = enc["outliers"]
    return xh


def rel_fro(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm())


def tie_distance(pre: torch.Tensor) -> torch.Tensor:
    """|frac(pre) - 1/2|: how far each quantiser input sits from a rounding tie."""
    p = pre.double()
    return (p - torch.floor(p) - 0.5).abs()
