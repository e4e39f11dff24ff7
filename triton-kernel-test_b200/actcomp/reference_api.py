"""The reference's public functions, with their names, signatures and return
types, running on the sm_100a kernels of libactcomp.

Each function cites the reference definition it replaces
(Ther-nullptr/Triton-Kernel-Test, file:line).  Behaviour follows the
reference's Triton kernels; where those are broken the intended result is
computed instead, and the docstring says so.  The ``torch_*`` twins keep the
PyTorch-twin arithmetic (bf16 intermediates, round half to even, per-batch
scales, whole-row packing) through the reference-compat flags.
"""
from __future__ import annotations

import torch

from . import core, ops, refcompat
from .nf4 import dequantize_4bit  # F.dequantize_4bit, low_rank_system_profile_backward.py:58  # noqa: F401
from ._lib import ACT_OP_DECODE, ACT_OP_MUL, ACT_OP_SILU_BWD

_BF = torch.bfloat16


def _assert_lr(l, r):
    # low_rank_extraction_fuse_compression_quantization.py:120-122
    assert l.shape[1] == r.shape[0], "Incompatible dimensions"
    assert l.is_contiguous(), "Matrix A must be contiguous"
    assert r.is_contiguous(), "Matrix B must be contiguous"


# ------------------------------------------------------------------ encode / decode
def low_rank_addition_fuse_compression_quantization(l, r, x, s, quantize_bit=8, outlier=5.):
    """low_rank_extraction_fuse_compression_quantization.py:118.
    Returns (o: sparse COO bf16 (B,M,N) outliers, q: uint8 (B,M,N*bits/8))."""
    _assert_lr(l, r)
    o, q = ops.rc_encode(l, r, x, s, quantize_bit, float(outlier), 0)
    return o.to_sparse(), q  # :149


def torch_low_rank_addition_fuse_compression_quantization(l, r, x, s, quantize_bit=8, outlier=5.):
    """PyTorch twin, :153-171 (per-batch scale, round half to even, whole-row
    packing).  The twin ORs into an uninitialised buffer; here q starts at 0."""
    o, q = ops.rc_encode(l, r, x, s.reshape(-1, x.shape[-1]), quantize_bit, float(outlier), refcompat.TWIN)
    return o.to_sparse(), q


def low_rank_addition_fuse_decompression_dequantization(l, r, q, o, s, quantize_bit=8, outlier=5.):
    """low_rank_extraction_fuse_decompression_dequantization.py:116; o sparse or dense."""
    _assert_lr(l, r)
    return ops.rc_decode(l, r, q, o.to_dense() if o.is_sparse else o, s, quantize_bit, 0, ACT_OP_DECODE, None)


def torch_low_rank_addition_fuse_decompression_dequantization(l, r, q, o, s, quantize_bit=8):
    """PyTorch twin, :155-165."""
    return ops.rc_decode(l, r, q.to(torch.uint8), o.to_dense() if o.is_sparse else o, s, quantize_bit,
                         refcompat.TWIN, ACT_OP_DECODE, None)


def naive_quantization_dequantization(l, r, x, s, quantize_bit=8, outlier=5.):
    """low_rank_kernel_accuracy_test.py:6-16: quantise and reconstruct in one go."""
    N = x.shape[-1]
    s2 = s.reshape(-1, N)
    o, q = ops.rc_encode(l, r, x, s2, quantize_bit, float(outlier), refcompat.TWIN)
    return ops.rc_decode(l, r, q, o, s2, quantize_bit, refcompat.TWIN, ACT_OP_DECODE, None)


def low_rank_addition(l, r, x):
    """low_rank_extraction_speed.py:113: bf16(x + l @ r)."""
    _assert_lr(l, r)
    return ops.lowrank_add(l, r, x)


def torch_low_rank_addition(l, r, x):
    """low_rank_extraction_speed.py:142."""
    return ops.lowrank_add(l, r, x)


# ------------------------------------------------------------------ outlier extraction
def torch_extract_unstructured(x, threshold):
    """extraction_outlier_channel.py:5: (outliers as sparse COO, remainder)."""
    o, rest = core.extract_unstructured(x, float(threshold))
    return o.reshape(x.shape).to_sparse(), rest.reshape(x.shape)


def torch_extract_channel(x, channel_index):
    """extraction_outlier_channel.py:11: (x[:, idx, :], x with those rows zeroed in place)."""
    return core.extract_channel(x, channel_index)


# ------------------------------------------------------------------ elementwise consumers
def torch_hadamard(x, y):
    """extraction_fuse_hadamard.py:5."""
    return core.mul_dense(x, y)


def triton_hadamard(a, b):
    """extraction_fuse_hadamard.py:62."""
    return core.mul_dense(a, b)


def triton_hadamard_fuse_extraction(l, r, q, s, b, quantize_bit=2):
    """extraction_fuse_hadamard.py:185: decode(l, r, q, s) * b, fused."""
    return ops.rc_decode(l, r, q, None, s, quantize_bit, 0, ACT_OP_MUL, b)


def triton_hadamard_add_extraction(l, r, q, s, b, quantize_bit=2):
    """extraction_fuse_hadamard.py:317 (two kernels; the reference returns None,
    this returns the product)."""
    x = ops.rc_decode(l, r, q, None, s, quantize_bit, 0, ACT_OP_DECODE, None)
    return core.mul_dense(x, b)


def torch_silu_backward(x, grad_y):
    """silu_backward.py:6 / extraction_fuse_silu_backward.py:10."""
    return core.silu_backward_dense(x, grad_y)


def triton_silu_backward(x, g):
    """silu_backward.py:54 / extraction_fuse_silu_backward.py:65."""
    return core.silu_backward_dense(x, g)


def triton_silu_backward_fuse_extraction(l, r, q, s, b, quantize_bit=2):
    """extraction_fuse_silu_backward.py:192: SiLU backward at decode(l, r, q, s)
    with upstream gradient b.  (The reference kernel multiplies by the decoded
    value twice, :183-187; this computes the SiLU derivative it intends.)"""
    return ops.rc_decode(l, r, q, None, s, quantize_bit, 0, ACT_OP_SILU_BWD, b)


def triton_silu_backward_add_extraction(l, r, q, s, b, quantize_bit=2):
    """extraction_fuse_silu_backward.py:324 (two kernels; returns the result)."""
    x = ops.rc_decode(l, r, q, None, s, quantize_bit, 0, ACT_OP_DECODE, None)
    return core.silu_backward_dense(x, b)


def torch_gelu_backward(x, grad_y):
    """gelu_backward.py:14."""
    return core.gelu_backward_dense(x, grad_y)


def triton_gelu_backward(x, g):
    """gelu_backward.py:73."""
    return core.gelu_backward_dense(x, g)


def torch_softmax_backward(y, grad_y):
    """softmax_backward.py:6."""
    return core.softmax_backward_dense(y, grad_y)


def triton_softmax_backward(y, grad_y):
    """softmax_backward.py:45 (y is (b, h, n, n))."""
    assert grad_y.shape == y.shape
    return core.softmax_backward_dense(y, grad_y)


# ------------------------------------------------------------------ GEMMs
def leaky_relu(x):
    """triton_matmul.py:169."""
    return torch.where(x >= 0, x, 0.01 * x)


def matmul(a, b, activation=""):
    """triton_matmul.py:178: fp16 C = a @ b (fp32 accumulation, optional leaky_relu)."""
    assert a.shape[1] == b.shape[0], "Incompatible dimensions"
    assert a.is_contiguous(), "Matrix A must be contiguous"
    return ops.gemm(a, b, torch.float16, activation)


def torch_matmul(x, a):
    """extraction_fuse_matmul.py:5."""
    return ops.gemm(x, a, x.dtype, "")


def triton_batched_matmul(x, a):
    """extraction_fuse_matmul.py:59: (B,M,K) @ (B,K,N) in a's dtype."""
    return ops.gemm(x, a, a.dtype, "")


def triton_split_k_matmul(x, a):
    """extraction_fuse_matmul.py:126.  The reference kernel has no split-K
    reduction (tiles overwrite each other); this returns the product it names."""
    return ops.gemm(x, a, a.dtype, "")


def triton_matmul_decompress(q, l, r, s, y, quantize_bit=2):
    """extraction_fuse_matmul.py:224: decode(l, r, q, s) @ y.  The reference
    kernel reads its scratch as codes and never advances l or s (:181-218);
    this computes the product it intends."""
    x = ops.rc_decode(l, r, q, None, s, quantize_bit, 0, ACT_OP_DECODE, None)
    return ops.gemm(x, y.to(_BF), _BF, "")


def triton_matmul_add_extraction(q, l, r, s, y, quantize_bit=2):
    """extraction_fuse_matmul.py:356 (two kernels; returns the result)."""
    return triton_matmul_decompress(q, l, r, s, y, quantize_bit)


# ------------------------------------------------------------------ LoRA driver
def compute_lora(x, w, a, b):
    """low_rank_system_profile_forward.py:8: w(x) + (x @ a) @ b.  w is a
    callable (the reference passes an NF4 Linear) or a (d_in, d_out) weight."""
    y_main = w(x) if callable(w) else _mm(x, w)
    return y_main + _mm(_mm(x, a), b)


def _mm(x, w):
    lead = x.shape[:-1]
    out = ops.gemm(x.reshape(-1, x.shape[-1]).to(_BF).contiguous(), w.to(_BF).contiguous(), _BF, "")
    return out.reshape(*lead, w.shape[-1])


def _pieces3(v):
    """float32 (..., r) -> bf16 (..., 3r): [hi | mid | lo] with hi + mid + lo == v
    exactly (three 8-bit significands hold float32's 24), so that a bf16 tensor
    core product with the pieces accumulates v's exact products in float32."""
    hi = v.to(_BF)
    r1 = v - hi.float()
    mid = r1.to(_BF)
    lo = (r1 - mid.float()).to(_BF)
    return torch.cat([hi, mid, lo], dim=-1)


def _sum3(v, r, dim):
    """(hi + mid) + lo of a product with _pieces3 operands, split along `dim`."""
    h, m, l = v.split(r, dim=dim)
    return (h + m) + l


def compute_lora_gradient(dy, x, w, a, b):
    """low_rank_system_profile_backward.py:14:
    dx = dy (w^T + b^T a^T), da = x^T (dy b^T), db = (x a)^T dy.

    dx is one tensor-core GEMM with two K segments, dy w^T + (dy b^T) a^T, so
    w^T + b^T a^T is never formed; dy b^T and x a are float32 and enter the
    bf16 tensor cores as three exact bf16 pieces, so every product is the
    float32-accumulated value of the formula on the bf16 operands.  x may be a
    dense (B, S, d_in) tensor (da, db per batch, as the reference's batched
    matmuls) or a :class:`actcomp.core.Compressed` activation of B*S tokens
    (da from the fused dequant-GEMM, x a from the reconstruction; da, db over
    all tokens)."""
    B = dy.shape[0] if dy.dim() == 3 else 1
    r = a.shape[-1]
    dy2 = dy.reshape(-1, dy.shape[-1]).to(_BF).contiguous()
    # w is read in place: the GEMM takes either major-ness, so the transposed
    # view dequantize_4bit returns for the frozen base weight is not copied
    a_bf, b_bf, w_bf = a.to(_BF).contiguous(), b.to(_BF).contiguous(), w.to(_BF)
    dyb = ops.gemm(dy2, b_bf.mT, torch.float32, "")          # (BS, r) = dy b^T
    P = _pieces3(dyb)                                         # (BS, 3r)
    a3 = torch.cat([a_bf, a_bf, a_bf], dim=1)                # (d_in, 3r)
    dx = ops.gemm_two(dy2, w_bf.mT, P, a3.mT, _BF)           # dy w^T + (dy b^T) a^T
    dx = dx.reshape(dy.shape[:-1] + (dx.shape[-1],))
    if isinstance(x, core.Compressed):
        da = _sum3(core.weight_grad(x, P, torch.float32), r, 1)
        xa = ops.gemm(core.decode(x).reshape(-1, x.channels), a_bf, torch.float32, "")
        db = _sum3(ops.gemm(_pieces3(xa).mT, dy2, torch.float32, ""), r, 0)
        return dx, da, db
    x3 = x.reshape(B, -1, x.shape[-1]).to(_BF)
    P3 = P.reshape(B, -1, 3 * r)
    da = _sum3(ops.gemm(x3.mT, P3, torch.float32, ""), r, -1)
    xa = ops.gemm(x3, a_bf, torch.float32, "")               # (B, S, r)
    db = _sum3(ops.gemm(_pieces3(xa).mT, dy2.reshape(B, -1, dy2.shape[-1]), torch.float32, ""), r, -2)
    return dx, da, db
