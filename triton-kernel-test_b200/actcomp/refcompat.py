"""Reference-compatible format: the reference's own layout and arithmetic.

l (M, K) and r (K, N) are given low-rank factors, s (S, N) per-column scales,
outliers are everything above a threshold (a dense bf16 tensor, returned as
sparse COO like the reference wrapper), codes are packed in 32-column blocks.
Defaults reproduce the Triton kernels of
low_rank_extraction_fuse_compression_quantization.py and
low_rank_extraction_fuse_decompression_dequantization.py; ``flags`` selects the
PyTorch-twin behaviour where the two differ (see include/actcomp.h).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from ._lib import RcArgs, call
from .core import BF16, _need_cuda, _stream

TWIN_LOWRANK = _lib.ACT_RC_TWIN_LOWRANK
HALF_EVEN = _lib.ACT_RC_HALF_EVEN
SCALE_BATCH = _lib.ACT_RC_SCALE_BATCH
ROW_PACK = _lib.ACT_RC_ROW_PACK
OUTLIER_BF16 = _lib.ACT_RC_OUTLIER_BF16
TWIN = TWIN_LOWRANK | HALF_EVEN | SCALE_BATCH | ROW_PACK | OUTLIER_BF16


def _args(l, r, s, bits, flags=0, outlier=0.0) -> RcArgs:
    a = RcArgs()
    a.M, a.K = l.shape
    a.N = r.shape[1]
    a.bits, a.flags, a.outlier = bits, flags, float(outlier)
    a.l, a.r = l.data_ptr(), r.data_ptr()
    if s is not None:
        a.s, a.s_rows = s.data_ptr(), s.shape[0]
    return a


def _lr(l, r):
    if l.shape[1] != r.shape[0]:
        raise ValueError("Incompatible dimensions")  # low_rank_extraction_fuse_compression_quantization.py:120
    return l.to(BF16).contiguous(), r.to(BF16).contiguous()


def _scale(s, N):
    s = s.to(BF16)
    s = s.reshape(-1, N) if s.numel() % N == 0 else s
    return s.contiguous()


def encode(l, r, x, s, bits: int = 8, outlier: float = 5.0, flags: int = 0):
    """Returns (o dense bf16 (B,M,N), q uint8 (B,M,N*bits/8))."""
    _need_cuda(l, r, x, s)
    l, r = _lr(l, r)
    B, M, N = x.shape
    if (M, N) != (l.shape[0], r.shape[1]):
        raise ValueError("x does not match l @ r")
    x = x.to(BF16)
    if x.stride(-1) != 1:
        x = x.contiguous()
    s = _scale(s, N)
    o = torch.empty((B, M, N), dtype=BF16, device=x.device)
    q = torch.empty((B, M, N * bits // 8), dtype=torch.uint8, device=x.device)
    a = _args(l, r, s, bits, flags, outlier)
    a.B = B
    a.x, a.sxb, a.sxm = x.data_ptr(), x.stride(0), x.stride(1)
    a.o, a.q = o.data_ptr(), q.data_ptr()
    call("actcomp_rc_encode", ctypes.byref(a), _stream(x))
    return o, q


def decode(l, r, q, o: Optional[torch.Tensor], s, bits: int = 8, flags: int = 0, op: int = _lib.ACT_OP_DECODE,
           y: Optional[torch.Tensor] = None) -> torch.Tensor:
    """xhat (B,M,N) bf16, or op(xhat, y) for the fused consumers."""
    _need_cuda(l, r, q, s)
    l, r = _lr(l, r)
    B, M, W = q.shape
    N = r.shape[1]
    if W * 8 // bits != N or M != l.shape[0]:
        raise ValueError("q does not match l @ r")
    q = q.contiguous()
    s = _scale(s, N)
    if o is not None:
        o = (o.to_dense() if o.is_sparse else o).to(BF16).contiguous()
    out = torch.empty((B, M, N), dtype=BF16, device=q.device)
    a = _args(l, r, s, bits, flags)
    a.B = B
    a.q, a.o, a.out = q.data_ptr(), 0 if o is None else o.data_ptr(), out.data_ptr()
    if y is not None:
        y = y.to(BF16)
        if y.stride(-1) != 1:
            y = y.contiguous()
        a.x, a.sxb, a.sxm = y.data_ptr(), y.stride(0), y.stride(1)
    call("actcomp_rc_decode", ctypes.byref(a), op, _stream(out))
    return out


def lowrank_add(l, r, x) -> torch.Tensor:
    """bf16(x + l @ r) with binary32 accumulation (low_rank_extraction_speed.py:113)."""
    _need_cuda(l, r, x)
    l, r = _lr(l, r)
    x = x.to(BF16)
    if x.stride(-1) != 1:
        x = x.contiguous()
    B, M, N = x.shape
    out = torch.empty((B, M, N), dtype=BF16, device=x.device)
    a = _args(l, r, None, 8)
    a.B = B
    a.x, a.sxb, a.sxm, a.out = x.data_ptr(), x.stride(0), x.stride(1), out.data_ptr()
    call("actcomp_rc_lowrank_add", ctypes.byref(a), _stream(x))
    return out
