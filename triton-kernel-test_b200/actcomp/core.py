"""Torch-facing API over libactcomp: compressed activations in the channel-group
format, their fused consumers, and the dense helpers.

Every function here allocates its outputs with torch on the input's device,
launches the CUDA kernel on the current stream through the C ABI, and returns
without synchronising.  Inputs must be CUDA tensors; there is no CPU path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field, replace
from typing import Optional

import torch

from . import _lib
from ._lib import CgDesc, EwArgs, GemmArgs, call

BF16 = torch.bfloat16


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> int:
    return 0 if t is None else t.data_ptr()


def _need_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("actcomp kernels run on CUDA tensors only (no CPU fallback)")


# ====================================================================== basis
@dataclass
class Basis:
    """A rank-r basis V (H x r per slice), rounded to bf16 and laid out for the kernels.

    ``basis_t`` (batch, r, H) is V^T for the projection, ``basis`` (batch, H, r)
    is V for the CUDA-core reconstruction, ``basis_tile`` holds V in the
    tensor-core kernels' shared-memory tile layout (include/actcomp.h); without
    it those kernels decline and the CUDA-core kernels run.  All three hold the
    same bf16 values: the format's basis is V rounded to bf16 once."""

    basis_t: torch.Tensor
    basis: torch.Tensor
    basis_tile: Optional[torch.Tensor] = None

    @property
    def rank(self) -> int:
        return self.basis.shape[-1]

    @property
    def channels(self) -> int:
        return self.basis.shape[-2]

    @property
    def batch(self) -> int:
        return self.basis.shape[0]

    def vectors(self) -> torch.Tensor:
        """The basis as float32 (batch, H, r): the exact values every kernel uses."""
        return self.basis.to(torch.float32)

    @staticmethod
    def tile_numel(H: int, r: int, batch: int = 1) -> int:
        rk = 16 if r <= 16 else (32 if r <= 32 else 64)
        return batch * ((H + 127) // 128) * 128 * rk

    @staticmethod
    def from_vectors(V: torch.Tensor) -> "Basis":
        """V: (H, r) or (batch, H, r) float tensor of basis vectors (columns)."""
        _need_cuda(V)
        if V.dim() == 2:
            V = V.unsqueeze(0)
        V = V.to(torch.float32).contiguous()
        b, H, r = V.shape
        bt = torch.empty((b, r, H), dtype=BF16, device=V.device)
        bv = torch.empty((b, H, r), dtype=BF16, device=V.device)
        tile = torch.empty((Basis.tile_numel(H, r, b),), dtype=BF16, device=V.device)  # layout in actcomp.h
        call("actcomp_cg_basis_prepare", V.data_ptr(), H, r, b, bt.data_ptr(), bv.data_ptr(), tile.data_ptr(),
             _stream(V))
        return Basis(bt, bv, tile)

    @staticmethod
    def fit(x: torch.Tensor, rank: int) -> "Basis":
        """Top-``rank`` right singular vectors of x ((T, H) or (batch, T, H)),
        from the eigenvectors of x^T x in float32 (a calibration step, off the
        hot path)."""
        xs = x if x.dim() == 3 else x.unsqueeze(0)
        vs = []
        for xb in xs:
            xf = xb.to(torch.float32)
            g = xf.T @ xf
            _, vec = torch.linalg.eigh(g)
            vs.append(vec[:, -rank:].flip(-1))
        return Basis.from_vectors(torch.stack(vs))


# ====================================================================== compressed activation
@dataclass
class Compressed:
    """One activation (batch x T x H bf16) in the channel-group format.

    Buffers (per slice, back to back): codes (T, H*bits/8) uint8, scales
    (T, H/group) float32, lowrank (T, r) float32 = the projection X . V,
    outliers (T, k) bf16; outlier_idx (batch, k) int32 and the basis are
    shared inputs."""

    tokens: int
    channels: int
    bits: int
    group: int
    wht: bool
    batch: int
    codes: torch.Tensor
    scales: torch.Tensor
    lowrank: Optional[torch.Tensor]
    outliers: Optional[torch.Tensor]
    outlier_idx: Optional[torch.Tensor]
    basis: Optional[Basis]
    _desc: Optional[CgDesc] = field(default=None, repr=False, compare=False)

    @property
    def rank(self) -> int:
        return 0 if self.basis is None else self.basis.rank

    @property
    def n_outlier(self) -> int:
        return 0 if self.outlier_idx is None else self.outlier_idx.shape[-1]

    @property
    def device(self) -> torch.device:
        return self.codes.device

    def buffers(self) -> dict:
        out = {"codes": self.codes, "scales": self.scales}
        if self.rank:
            out["lowrank"] = self.lowrank
        if self.n_outlier:
            out["outliers"] = self.outliers
        return out

    def nbytes(self) -> int:
        """Bytes of the per-activation buffers (what an offload moves)."""
        return sum(t.numel() * t.element_size() for t in self.buffers().values())

    def desc(self) -> CgDesc:
        d = CgDesc()
        d.tokens, d.channels, d.bits, d.group = self.tokens, self.channels, self.bits, self.group
        d.rank, d.n_outlier, d.wht, d.batch = self.rank, self.n_outlier, int(self.wht), self.batch
        d.codes, d.scales = _ptr(self.codes), _ptr(self.scales)
        d.lowrank = _ptr(self.lowrank)
        d.outliers, d.outlier_idx = _ptr(self.outliers), _ptr(self.outlier_idx)
        if self.basis is not None:
            d.basis_t, d.basis = self.basis.basis_t.data_ptr(), self.basis.basis.data_ptr()
            d.basis_tile = _ptr(self.basis.basis_tile)
        return d

    def with_buffers(self, **bufs) -> "Compressed":
        return replace(self, **bufs, _desc=None)


def empty_like_layout(tokens: int, channels: int, *, bits: int, group: int, rank: int, n_outlier: int,
                      batch: int = 1, device=None, pin_memory: bool = False) -> dict:
    """Allocate the per-activation buffers of a channel-group activation."""
    kw = dict(device=device, pin_memory=pin_memory) if pin_memory else dict(device=device)
    T = batch * tokens
    bufs = {
        "codes": torch.empty((T, channels * bits // 8), dtype=torch.uint8, **kw),
        "scales": torch.empty((T, channels // group), dtype=torch.float32, **kw),
        "lowrank": torch.empty((T, rank), dtype=torch.float32, **kw) if rank else None,
        "outliers": torch.empty((T, n_outlier), dtype=BF16, **kw) if n_outlier else None,
    }
    return bufs


def _rows(x: torch.Tensor) -> tuple[torch.Tensor, int, int, int]:
    """View x as (batch, T, H) with unit column stride; returns (x3, batch, T, ld)."""
    x3 = x if x.dim() == 3 else x.unsqueeze(0)
    if x3.stride(-1) != 1 or (x3.shape[0] > 1 and x3.stride(0) != x3.shape[1] * x3.stride(1)):
        x3 = x3.contiguous()
    return x3, x3.shape[0], x3.shape[1], x3.stride(1)


def encode(x: torch.Tensor, basis: Optional[Basis] = None, outlier_idx: Optional[torch.Tensor] = None, *,
           bits: int = 4, group: int = 64, wht: bool = False) -> Compressed:
    """Compress x ((T, H) or (batch, T, H) bf16): projection L = x . V onto the
    basis, residual x - L . V^T with its outlier channels kept verbatim,
    optional 128-wide Walsh-Hadamard rotation of the residual, int4/int8 codes
    with per-token group-absmax scales."""
    _need_cuda(x)
    if x.dtype != BF16:
        raise TypeError("encode expects a bfloat16 activation")
    x3, batch, T, ldx = _rows(x)
    H = x3.shape[2]
    rank = 0 if basis is None else basis.rank
    if basis is not None and (basis.channels != H or basis.batch != batch):
        raise ValueError(f"basis is {basis.batch}x{basis.channels}, activation has {batch} slices of {H} channels")
    k = 0
    if outlier_idx is not None:
        outlier_idx = outlier_idx.to(device=x.device, dtype=torch.int32).reshape(batch, -1).contiguous()
        k = outlier_idx.shape[1]
        if k == 0:
            outlier_idx = None
    bufs = empty_like_layout(T, H, bits=bits, group=group, rank=rank, n_outlier=k, batch=batch, device=x.device)
    c = Compressed(T, H, bits, group, bool(wht), batch, bufs["codes"], bufs["scales"], bufs["lowrank"],
                   bufs["outliers"], outlier_idx, basis)
    d = c.desc()
    call("actcomp_cg_encode", ctypes.byref(d), x3.data_ptr(), ldx, _stream(x))
    return c


def decode(c: Compressed, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Reconstruct the activation (bf16, shape (T, H) or (batch, T, H))."""
    if out is None:
        out = torch.empty((c.batch, c.tokens, c.channels), dtype=BF16, device=c.device)
    d = c.desc()
    call("actcomp_cg_decode", ctypes.byref(d), out.data_ptr(), out.stride(-2), _stream(out))
    return out if c.batch > 1 or out.dim() == 2 else out.squeeze(0)


def _consume(c: Compressed, op: int, y: torch.Tensor) -> torch.Tensor:
    _need_cuda(y)
    y3, batch, T, ldy = _rows(y.to(BF16))
    if batch != c.batch or T != c.tokens or y3.shape[2] != c.channels:
        raise ValueError("second operand shape does not match the compressed activation")
    out = torch.empty((c.batch, c.tokens, c.channels), dtype=BF16, device=c.device)
    d = c.desc()
    call("actcomp_cg_consume", ctypes.byref(d), op, y3.data_ptr(), ldy, out.data_ptr(), out.stride(1), _stream(out))
    return out if y.dim() == 3 else out.squeeze(0)


def mul(c: Compressed, y: torch.Tensor) -> torch.Tensor:
    """xhat * y without materialising xhat (extraction_fuse_hadamard.py:185)."""
    return _consume(c, _lib.ACT_OP_MUL, y)


def silu_backward(c: Compressed, dy: torch.Tensor) -> torch.Tensor:
    """dL/dx of SiLU at the saved activation (extraction_fuse_silu_backward.py:192)."""
    return _consume(c, _lib.ACT_OP_SILU_BWD, dy)


def gelu_backward(c: Compressed, dy: torch.Tensor) -> torch.Tensor:
    """dL/dx of tanh-GELU at the saved activation (gelu_backward.py:14)."""
    return _consume(c, _lib.ACT_OP_GELU_BWD, dy)


def softmax_backward(c: Compressed, dp: torch.Tensor, causal: bool = False,
                     workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """(dP - rowsum(dP * P)) * P with P read from compressed form
    (softmax_backward.py:6).  c holds one S x S slice per (batch, head);
    dp is (..., S, S) with the same number of slices."""
    _need_cuda(dp)
    S = c.channels
    dp3 = dp.to(BF16).reshape(-1, S, S).contiguous()
    if dp3.shape[0] != c.batch or c.tokens != S:
        raise ValueError("dP does not match the compressed probabilities")
    ds = torch.empty_like(dp3)
    d = c.desc()
    if workspace is None:  # partial dot products and row sums of the two tensor-core passes
        workspace = torch.empty((_lib.load().actcomp_cg_softmax_workspace(ctypes.byref(d)),), dtype=torch.uint8,
                                device=dp3.device)
    call("actcomp_cg_softmax_bwd", ctypes.byref(d), dp3.data_ptr(), ds.data_ptr(), S, int(causal),
         workspace.data_ptr(), workspace.numel(), _stream(dp3))
    return ds.reshape(dp.shape)


def weight_grad(c: Compressed, dy: torch.Tensor, out_dtype: torch.dtype = torch.float32,
                workspace: Optional[torch.Tensor] = None, fused: bool = False) -> torch.Tensor:
    """dW = xhat^T dy (H x N) with xhat reconstructed from c, fp32 accumulation
    on the tcgen05 tensor cores (extraction_fuse_matmul.py:224).

    fused=False: the reconstruction into a workspace, then the GEMM
    (actcomp_cg_dw; bit-for-bit the GEMM of decode(c)).  fused=True: the
    dequantisation inside the GEMM's producer and the low-rank and outlier
    terms as their own skinny products (actcomp_cg_dw_fused; about 5e-4
    relative from the former, no T x H workspace)."""
    _need_cuda(dy)
    if c.batch != 1:
        raise ValueError("weight_grad takes a single-slice activation")
    dy = dy.to(BF16)
    if dy.stride(-1) != 1:
        dy = dy.contiguous()
    T, N = dy.shape
    if T != c.tokens:
        raise ValueError("dy rows must equal the activation's tokens")
    dw = torch.empty((c.channels, N), dtype=out_dtype, device=dy.device)
    d = c.desc()
    name = "actcomp_cg_dw_fused" if fused else "actcomp_cg_dw"
    need = getattr(_lib.load(), name + "_workspace")(ctypes.byref(d), N)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty((max(need, 1),), dtype=torch.uint8, device=dy.device)
    call(name, ctypes.byref(d), dy.data_ptr(), N, dy.stride(0), dw.data_ptr(),
         0 if out_dtype == torch.float32 else 1, dw.stride(0), workspace.data_ptr(), workspace.numel(),
         _stream(dy))
    return dw


def select_outlier_channels(x: torch.Tensor, k: int) -> torch.Tensor:
    """The k channels of x (T, H) with the largest absmax, ascending (int32)."""
    _need_cuda(x)
    x = x.to(BF16)
    if x.stride(-1) != 1:
        x = x.contiguous()
    T, H = x.shape
    idx = torch.empty((k,), dtype=torch.int32, device=x.device)
    ws = torch.empty((H,), dtype=torch.float32, device=x.device)
    call("actcomp_cg_channel_topk", x.data_ptr(), T, H, x.stride(0), k, idx.data_ptr(), ws.data_ptr(), _stream(x))
    return idx


def copy_into(dst: Compressed, src: Compressed, stream: Optional[torch.cuda.Stream] = None) -> None:
    """Copy all per-activation buffers of src into dst (same layout), one
    cudaMemcpyAsync per buffer on `stream` (default: current stream)."""
    s = (stream or torch.cuda.current_stream()).cuda_stream
    dd, sd = dst.desc(), src.desc()
    call("actcomp_cg_copy", ctypes.byref(dd), ctypes.byref(sd), s)


# ====================================================================== dense helpers
def _ew(op: int, x: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    _need_cuda(x, g)
    if x.shape != g.shape:
        raise ValueError("shape mismatch")
    x3 = x.reshape((1,) * (3 - x.dim()) + tuple(x.shape)) if x.dim() < 3 else x
    g3 = g.reshape(x3.shape) if g.dim() != 3 else g
    if x3.dim() != 3:
        x3 = x3.reshape(-1, x3.shape[-2], x3.shape[-1])
        g3 = g3.reshape(x3.shape)
    if x3.stride(-1) != 1:
        x3 = x3.contiguous()
    if g3.stride(-1) != 1:
        g3 = g3.contiguous()
    x3 = x3.to(BF16)
    g3 = g3.to(BF16)
    out = torch.empty(x3.shape, dtype=BF16, device=x.device)
    a = EwArgs()
    a.B, a.M, a.N = x3.shape
    a.x, a.sxb, a.sxm = x3.data_ptr(), x3.stride(0), x3.stride(1)
    a.g, a.sgb, a.sgm = g3.data_ptr(), g3.stride(0), g3.stride(1)
    a.out, a.sob, a.som = out.data_ptr(), out.stride(0), out.stride(1)
    call("actcomp_elementwise", ctypes.byref(a), op, _stream(out))
    return out.reshape(x.shape)


def silu_backward_dense(x, g):
    return _ew(_lib.ACT_OP_SILU_BWD, x, g)


def gelu_backward_dense(x, g):
    return _ew(_lib.ACT_OP_GELU_BWD, x, g)


def mul_dense(a, b):
    return _ew(_lib.ACT_OP_MUL, a, b)


def softmax_backward_dense(y: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    _need_cuda(y, g)
    n = y.shape[-1]
    y2 = y.to(BF16).reshape(-1, n).contiguous()
    g2 = g.to(BF16).reshape(-1, n).contiguous()
    out = torch.empty_like(y2)
    call("actcomp_softmax_bwd", y2.data_ptr(), g2.data_ptr(), out.data_ptr(), y2.shape[0], n, n, _stream(y2))
    return out.reshape(y.shape)


def extract_unstructured(x: torch.Tensor, threshold: float):
    _need_cuda(x)
    xc = x.to(BF16).contiguous()
    o = torch.empty_like(xc)
    rest = torch.empty_like(xc)
    call("actcomp_extract_unstructured", xc.data_ptr(), xc.numel(), float(threshold), o.data_ptr(),
         rest.data_ptr(), _stream(xc))
    return o, rest


def extract_channel(x: torch.Tensor, channel_index: torch.Tensor):
    """Gather x[:, idx, :] and zero those rows of x in place."""
    _need_cuda(x)
    if x.dtype != BF16 or not x.is_contiguous() or x.dim() != 3:
        raise ValueError("extract_channel expects a contiguous (B, M, N) bf16 tensor")
    idx = channel_index.to(device=x.device, dtype=torch.int32).contiguous()
    B, M, N = x.shape
    out = torch.empty((B, idx.numel(), N), dtype=BF16, device=x.device)
    call("actcomp_extract_channel", x.data_ptr(), B, M, N, idx.data_ptr(), idx.numel(), out.data_ptr(), _stream(x))
    return out, x


_IN = {torch.bfloat16: 0, torch.float16: 1}
_OUT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def gemm(a: torch.Tensor, b: torch.Tensor, out_dtype: torch.dtype = torch.float32, activation: str = "",
         a2: Optional[torch.Tensor] = None, b2: Optional[torch.Tensor] = None) -> torch.Tensor:
    """C = a @ b (+ a2 @ b2) on tcgen05 for 2-D or batched 3-D bf16/fp16 operands.

    Each operand may be row-major or a transposed view of a row-major tensor
    (K-major or MN-major); other layouts are copied.  The optional second
    product (2-D only) is accumulated with the first in one float32 TMEM
    accumulator: a2 (M x K2) and b2 (K2 x N) are brought to the layouts of a
    and b."""
    _need_cuda(a, b)
    if a.dtype not in _IN or b.dtype != a.dtype:
        raise TypeError("gemm operands must both be bf16 or both fp16")
    batched = a.dim() == 3 or b.dim() == 3
    a3 = a if a.dim() == 3 else a.unsqueeze(0)
    b3 = b if b.dim() == 3 else b.unsqueeze(0)
    batch = max(a3.shape[0], b3.shape[0])
    M, K = a3.shape[1:]
    K2, N = b3.shape[1:]
    if K != K2:
        raise ValueError(f"inner dimensions differ: {K} vs {K2}")

    def layout(t, rows, cols):
        # returns (tensor, kmajor_flag, ld, batch_stride) for a logical rows x cols operand
        if t.stride(-1) == 1 and t.stride(-2) >= cols:
            return t, 1, t.stride(-2), t.stride(0) if t.shape[0] > 1 else 0  # row-major (K contiguous for A)
        if t.stride(-2) == 1 and t.stride(-1) >= rows:
            return t, 0, t.stride(-1), t.stride(0) if t.shape[0] > 1 else 0
        t = t.contiguous()
        return t, 1, t.stride(-2), t.stride(0) if t.shape[0] > 1 else 0

    a3, a_rowmajor, lda, sa = layout(a3, M, K)
    b3, b_rowmajor, ldb, sb = layout(b3, K, N)
    # A row-major (M x K, K contiguous) is K-major; B row-major (K x N) is MN-major
    a_kmajor = a_rowmajor
    b_kmajor = 0 if b_rowmajor else 1
    if batch > 1 and (sa == 0 or sb == 0):
        a3 = a3.expand(batch, M, K).contiguous() if sa == 0 else a3
        b3 = b3.expand(batch, K, N).contiguous() if sb == 0 else b3
        a3, a_rowmajor, lda, sa = layout(a3, M, K)
        b3, b_rowmajor, ldb, sb = layout(b3, K, N)
        a_kmajor, b_kmajor = a_rowmajor, 0 if b_rowmajor else 1
    if (a2 is None) != (b2 is None):
        raise ValueError("a2 and b2 come together")
    if a2 is not None:
        if batched or a2.dim() != 2 or b2.dim() != 2:
            raise ValueError("the second product is 2-D only")
        if a2.dtype != a.dtype or b2.dtype != a.dtype:
            raise TypeError("the second product's operands have the first's dtype")
        K2 = a2.shape[1]
        if a2.shape[0] != M or b2.shape != (K2, N):
            raise ValueError(f"second product shapes {tuple(a2.shape)} x {tuple(b2.shape)} do not give {M} x {N}")
        # same major-ness as the first product's operands
        a2 = a2.contiguous() if a_kmajor else a2.mT.contiguous().mT
        b2 = b2.mT.contiguous().mT if b_kmajor else b2.contiguous()
    c = torch.empty((batch, M, N), dtype=out_dtype, device=a.device)
    g = GemmArgs()
    g.M, g.N, g.K, g.batch = M, N, K, batch
    g.in_dtype, g.c_dtype, g.activation = _IN[a.dtype], _OUT[out_dtype], 1 if activation == "leaky_relu" else 0
    g.a_kmajor, g.b_kmajor = a_kmajor, b_kmajor
    g.A, g.lda, g.sa_batch = a3.data_ptr(), lda, sa
    g.B, g.ldb, g.sb_batch = b3.data_ptr(), ldb, sb
    g.C, g.ldc, g.sc_batch = c.data_ptr(), N, M * N if batch > 1 else 0
    if a2 is not None:
        g.K2 = a2.shape[1]
        g.A2, g.lda2 = a2.data_ptr(), a2.stride(0) if a_kmajor else a2.stride(1)
        g.B2, g.ldb2 = b2.data_ptr(), b2.stride(1) if b_kmajor else b2.stride(0)
    call("actcomp_gemm", ctypes.byref(g), _stream(c))
    return c if batched else c.squeeze(0)


def error_stats(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Accumulate [sum (a-b)^2, sum b^2, max|a-b|, #(a != b)] of two bf16
    tensors into a float64 device vector (for an all-reduce across ranks)."""
    _need_cuda(a, b)
    a = a.to(BF16).contiguous()
    b = b.to(BF16).contiguous()
    if out is None:
        out = torch.zeros(4, dtype=torch.float64, device=a.device)
    call("actcomp_error_stats", a.data_ptr(), b.data_ptr(), a.numel(), out.data_ptr(), _stream(a))
    return out
