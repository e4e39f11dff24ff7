"""torch custom ops (namespace ``actcomp``) over the C ABI.

Each op is functional (returns new tensors), has a fake implementation for
meta/abstract tracing, and launches on the current CUDA stream.  The
reference-named functions in :mod:`actcomp.reference_api` call these ops.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import core, refcompat

_U8, _F32, _BF = torch.uint8, torch.float32, torch.bfloat16


def _empty(shape, dtype, like):
    return torch.empty(shape, dtype=dtype, device=like.device)


# ---------------------------------------------------------------- reference-compatible
@torch.library.custom_op("actcomp::rc_encode", mutates_args=())
def rc_encode(l: torch.Tensor, r: torch.Tensor, x: torch.Tensor, s: torch.Tensor, bits: int, outlier: float,
              flags: int) -> tuple[torch.Tensor, torch.Tensor]:
    return refcompat.encode(l, r, x, s, bits, outlier, flags)


@rc_encode.register_fake
def _(l, r, x, s, bits, outlier, flags):
    B, M, N = x.shape
    return _empty((B, M, N), _BF, x), _empty((B, M, N * bits // 8), _U8, x)


@torch.library.custom_op("actcomp::rc_decode", mutates_args=())
def rc_decode(l: torch.Tensor, r: torch.Tensor, q: torch.Tensor, o: Optional[torch.Tensor], s: torch.Tensor,
              bits: int, flags: int, op: int, y: Optional[torch.Tensor]) -> torch.Tensor:
    return refcompat.decode(l, r, q, o, s, bits, flags, op, y)


@rc_decode.register_fake
def _(l, r, q, o, s, bits, flags, op, y):
    B, M, W = q.shape
    return _empty((B, M, W * 8 // bits), _BF, q)


@torch.library.custom_op("actcomp::lowrank_add", mutates_args=())
def lowrank_add(l: torch.Tensor, r: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    return refcompat.lowrank_add(l, r, x)


@lowrank_add.register_fake
def _(l, r, x):
    return _empty(x.shape, _BF, x)


# ---------------------------------------------------------------- channel-group format
def _basis(basis_t, basis, basis_tile=None):
    if basis is None or basis.numel() == 0:
        return None
    return core.Basis(basis_t, basis, basis_tile)


@torch.library.custom_op("actcomp::cg_encode", mutates_args=())
def cg_encode(x: torch.Tensor, basis_t: Optional[torch.Tensor], basis: Optional[torch.Tensor],
              basis_tile: Optional[torch.Tensor], outlier_idx: Optional[torch.Tensor], bits: int, group: int,
              wht: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    c = core.encode(x, _basis(basis_t, basis, basis_tile), outlier_idx, bits=bits, group=group, wht=wht)
    e = x.new_empty((0,))
    return (c.codes, c.scales, c.lowrank if c.rank else e.to(_F32), c.outliers if c.n_outlier else e)


@cg_encode.register_fake
def _(x, basis_t, basis, basis_tile, outlier_idx, bits, group, wht):
    T = x.numel() // x.shape[-1]
    H = x.shape[-1]
    r = 0 if basis is None else basis.shape[-1]
    k = 0 if outlier_idx is None else outlier_idx.shape[-1]
    return (_empty((T, H * bits // 8), _U8, x), _empty((T, H // group), _F32, x),
            _empty((T, r) if r else (0,), _F32, x), _empty((T, k) if k else (0,), _BF, x))


def _compressed(shape, codes, scales, lowrank, outliers, outlier_idx, basis_t, basis, basis_tile, bits, group, wht):
    batch = shape[0] if len(shape) == 3 else 1
    T, H = shape[-2], shape[-1]
    b = _basis(basis_t, basis, basis_tile)
    k = 0 if outlier_idx is None else outlier_idx.shape[-1]
    return core.Compressed(T, H, bits, group, wht, batch, codes, scales, lowrank if b else None,
                           outliers if k else None, outlier_idx.reshape(batch, -1) if k else None, b)


@torch.library.custom_op("actcomp::cg_consume", mutates_args=())
def cg_consume(shape: list[int], codes: torch.Tensor, scales: torch.Tensor, lowrank: torch.Tensor,
               outliers: torch.Tensor, outlier_idx: Optional[torch.Tensor], basis_t: Optional[torch.Tensor],
               basis: Optional[torch.Tensor], basis_tile: Optional[torch.Tensor], bits: int, group: int, wht: bool,
               op: int, y: Optional[torch.Tensor]) -> torch.Tensor:
    c = _compressed(shape, codes, scales, lowrank, outliers, outlier_idx, basis_t, basis, basis_tile, bits, group,
                    wht)
    if op == 0:
        return core.decode(c).reshape(shape)
    return core._consume(c, op, y.reshape(shape)).reshape(shape)


@cg_consume.register_fake
def _(shape, codes, scales, lowrank, outliers, outlier_idx, basis_t, basis, basis_tile, bits, group, wht, op, y):
    return _empty(tuple(shape), _BF, codes)


@torch.library.custom_op("actcomp::gemm", mutates_args=())
def gemm(a: torch.Tensor, b: torch.Tensor, out_dtype: torch.dtype, activation: str) -> torch.Tensor:
    return core.gemm(a, b, out_dtype, activation)


@torch.library.custom_op("actcomp::gemm_two", mutates_args=())
def gemm_two(a: torch.Tensor, b: torch.Tensor, a2: torch.Tensor, b2: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
    """a @ b + a2 @ b2 (2-D) in one float32 accumulator."""
    return core.gemm(a, b, out_dtype, "", a2, b2)


@gemm_two.register_fake
def _(a, b, a2, b2, out_dtype):
    return a.new_empty((a.shape[0], b.shape[1]), dtype=out_dtype)


@gemm.register_fake
def _(a, b, out_dtype, activation):
    if a.dim() == 3 or b.dim() == 3:
        batch = max(a.shape[0] if a.dim() == 3 else 1, b.shape[0] if b.dim() == 3 else 1)
        return a.new_empty((batch, a.shape[-2], b.shape[-1]), dtype=out_dtype)
    return a.new_empty((a.shape[0], b.shape[1]), dtype=out_dtype)
