"""Python face of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loads ``oracle/_build/libactcomp_oracle.so`` (built from actcomp_oracle.c by
oracle/Makefile) through ctypes and exposes numpy-in/numpy-out functions.  Only
tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may import
this module; the product code under triton-kernel-test_b200/ never does.

bf16 tensors cross this boundary as ``np.uint16`` arrays holding the raw bits.
Every function cites the reference code it restates; the C file header gives
the exact rounding points.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libactcomp_oracle.so")
_lock = threading.Lock()
_lib = None

# Flags of the reference-compat restatement (see actcomp_oracle.c).
RC_TWIN_LOWRANK = 1
RC_HALF_EVEN = 2
RC_SCALE_BATCH = 4
RC_ROW_PACK = 8
RC_OUTLIER_BF16 = 16
#: every PyTorch-twin behaviour at once (low_rank_extraction_speed.py:146-156,
#: low_rank_kernel_accuracy_test.py:6-16, ..._decompression_dequantization.py:155-165)
RC_TWIN = RC_TWIN_LOWRANK | RC_HALF_EVEN | RC_SCALE_BATCH | RC_ROW_PACK | RC_OUTLIER_BF16


def build() -> str:
    """Compile the oracle with oracle/Makefile if the shared object is missing or stale."""
    src = os.path.join(_HERE, "actcomp_oracle.c")
    if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            _lib = ctypes.CDLL(_SO)
    return _lib


def _p(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else ctypes.c_void_p(0)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


I64 = ctypes.c_int64
I32 = ctypes.c_int


# ------------------------------------------------------------------ bf16 helpers
def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even binary32 -> bf16 bits (NaN -> 0x7fc0)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------------ channel-group format
def basis_prepare(V: np.ndarray):
    """V (H x r) float32 -> (Vt bf16 bits r x H, Vb bf16 bits H x r): the basis rounded to bf16."""
    V = _c(V, np.float32)
    H, r = V.shape
    Vt = np.empty((r, H), np.uint16)
    Vb = np.empty((H, r), np.uint16)
    lib().cg_basis_prepare(_p(V), I64(H), I32(r), _p(Vt), _p(Vb))
    return Vt, Vb


def project(X: np.ndarray, Vt: np.ndarray) -> np.ndarray:
    """L = X @ Vt^T, exact sum rounded once to float32 (X bf16 bits or float32)."""
    x_f32 = X.dtype == np.float32
    X = _c(X, np.float32 if x_f32 else np.uint16)
    T, H = X.shape
    r = Vt.shape[0]
    L = np.empty((T, r), np.float32)
    lib().cg_project(_p(X), I32(int(x_f32)), I64(T), I64(H), I64(H), _p(_c(Vt, np.uint16)), I32(r), _p(L))
    return L


def lowrank(L: np.ndarray, Vb: np.ndarray) -> np.ndarray:
    """P = L @ Vb^T, exact sum rounded once to float32 (the low-rank term)."""
    L = _c(L, np.float32)
    T, r = L.shape
    H = Vb.shape[0]
    P = np.empty((T, H), np.float32)
    lib().cg_lowrank(_p(L), _p(_c(Vb, np.uint16)), I64(T), I64(H), I32(r), _p(P))
    return P


def encode_given_lr(X, L, Vb, idx, bits, group, wht):
    """Channel-group encode of X given its projection L -> (codes, scales, outliers)."""
    x_f32 = X.dtype == np.float32
    X = _c(X, np.float32 if x_f32 else np.uint16)
    T, H = X.shape
    r = 0 if L is None else L.shape[1]
    idx = _c(idx if idx is not None else np.zeros(0), np.int32)
    k = idx.shape[0]
    codes = np.empty((T, H * bits // 8), np.uint8)
    scales = np.empty((T, H // group), np.float32)
    outl = np.empty((T, k), np.float32 if x_f32 else np.uint16)
    L_ = _c(L, np.float32) if r else np.zeros((T, 1), np.float32)
    Vb_ = _c(Vb, np.uint16) if r else np.zeros((H, 1), np.uint16)
    lib().cg_encode_given_lr(_p(X), I32(int(x_f32)), I64(T), I64(H), I64(H), _p(L_), _p(Vb_), I32(r), _p(idx),
                             I32(k), I32(bits), I32(group), I32(int(wht)), _p(codes), _p(scales), _p(outl))
    return codes, scales, outl


def encode(X, V_prepared, idx, bits, group, wht):
    """Full channel-group encode: projection (exact sums), residual codes."""
    Vt, Vb = V_prepared
    L = project(X, Vt) if Vt.shape[0] else None
    codes, scales, outl = encode_given_lr(X, L, Vb, idx, bits, group, wht)
    return dict(codes=codes, scales=scales, outliers=outl, lowrank=L)


def decode(codes, scales, L, Vb, outl, idx, H, bits, group, wht, x_f32=False):
    T = codes.shape[0]
    r = 0 if L is None else L.shape[1]
    idx = _c(idx if idx is not None else np.zeros(0), np.int32)
    k = idx.shape[0]
    out = np.empty((T, H), np.float32 if x_f32 else np.uint16)
    L_ = _c(L, np.float32) if r else np.zeros((T, 1), np.float32)
    Vb_ = _c(Vb, np.uint16) if r else np.zeros((H, 1), np.uint16)
    outl_ = _c(outl, np.float32 if x_f32 else np.uint16) if k else np.zeros((T, 1), np.uint16)
    lib().cg_decode(_p(_c(codes, np.uint8)), _p(_c(scales, np.float32)), _p(L_), _p(Vb_), I32(r), _p(outl_),
                    _p(idx), I32(k), I64(T), I64(H), I32(bits), I32(group), I32(int(wht)), I32(int(x_f32)),
                    _p(out))
    return out


def quantizer_inputs(X, L, Vb, idx, bits, group, wht):
    """The value each code rounds, w * (qmax / absmax), in binary64 from the
    oracle's own residual (T x H), for attributing code differences to
    rounding ties."""
    x_f32 = X.dtype == np.float32
    x = (X if x_f32 else bf16_to_f32(X)).astype(np.float32)
    T, H = x.shape
    w = x - lowrank(L, Vb) if L is not None and L.shape[1] else x.copy()
    if idx is not None and len(idx):
        w[:, np.asarray(idx)] = 0.0
    if wht:
        w = w.reshape(T, H // 128, 128)
        m = 1
        while m < 128:  # the oracle's butterfly order, binary32
            w = w.reshape(T, H // 128, 128 // (2 * m), 2, m)
            a, b = w[:, :, :, 0, :].copy(), w[:, :, :, 1, :].copy()
            w[:, :, :, 0, :] = a + b
            w[:, :, :, 1, :] = a - b
            m *= 2
        w = w.reshape(T, H)
    qmax = (1 << (bits - 1)) - 1
    g = np.abs(w).reshape(T, H // group, group).max(-1)
    rs = np.where(g > 0, np.float32(qmax) / np.where(g > 0, g, 1).astype(np.float32), 0).astype(np.float32)
    return w.astype(np.float64) * np.repeat(rs, group, axis=1).astype(np.float64)


def channel_absmax(X):
    X = _c(X, np.uint16)
    T, H = X.shape
    s = np.empty((H,), np.float32)
    lib().cg_channel_absmax(_p(X), I64(T), I64(H), I64(H), _p(s))
    return s


def topk_channels(score, k):
    score = _c(score, np.float32)
    idx = np.empty((k,), np.int32)
    lib().cg_topk_channels(_p(score), I64(score.shape[0]), I32(k), _p(idx))
    return idx


# ------------------------------------------------------------------ consumers
def _unary2(name, x, g):
    x = _c(x, np.uint16)
    g = _c(g, np.uint16)
    out = np.empty_like(x)
    getattr(lib(), name)(_p(x), _p(g), I64(x.size), _p(out))
    return out


def silu_bwd(x, g):
    """silu_backward.py:6-8, binary32 math, one bf16 rounding."""
    return _unary2("orc_silu_bwd", x, g)


def gelu_bwd(x, g):
    """gelu_backward.py:14-21 (tanh approximation), binary32 math."""
    return _unary2("orc_gelu_bwd", x, g)


def mul(a, b):
    """extraction_fuse_hadamard.py:5 elementwise product."""
    return _unary2("orc_mul", a, b)


def softmax_bwd(y, g):
    """softmax_backward.py:6 over the last axis."""
    y = _c(y, np.uint16)
    g = _c(g, np.uint16)
    n = y.shape[-1]
    out = np.empty_like(y)
    lib().orc_softmax_bwd(_p(y), _p(g), I64(y.size // n), I64(n), _p(out))
    return out


def gemm_tn(A, B):
    """C = A^T B, A (K x M) and B (K x N) bf16 bits, binary64 accumulation."""
    A = _c(A, np.uint16)
    B = _c(B, np.uint16)
    K, M = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.float32)
    lib().orc_gemm_tn(_p(A), _p(B), I64(M), I64(N), I64(K), _p(C))
    return C


# ------------------------------------------------------------------ reference-compat
def rc_encode(l, r, x, s, bits, outlier, flags=0):
    """low_rank_addition_fuse_compression_quantization restated (see C header).

    x (B,M,N) bf16 bits, l (M,K), r (K,N), s (S,N).  Returns (o dense bf16 bits,
    q packed uint8, signed codes int32)."""
    x = _c(x, np.uint16)
    B, M, N = x.shape
    K = l.shape[1]
    s = _c(s, np.uint16).reshape(-1, N)
    o = np.empty((B, M, N), np.uint16)
    q = np.empty((B, M, N * bits // 8), np.uint8)
    sc = np.empty((B, M, N), np.int32)
    lib().rc_encode(_p(_c(l, np.uint16)), _p(_c(r, np.uint16)), _p(x), I64(M * N), I64(N), _p(s), I64(s.shape[0]),
                    I64(B), I64(M), I64(N), I32(K), I32(bits), ctypes.c_float(outlier), I32(flags), _p(o), _p(q),
                    _p(sc))
    return o, q, sc


def rc_decode(l, r, q, o, s, bits, flags=0):
    """low_rank_addition_fuse_decompression_dequantization restated; o may be None."""
    q = _c(q, np.uint8)
    B, M, W = q.shape
    N = W * 8 // bits
    K = l.shape[1]
    s = _c(s, np.uint16).reshape(-1, N)
    x = np.empty((B, M, N), np.uint16)
    lib().rc_decode(_p(_c(l, np.uint16)), _p(_c(r, np.uint16)), _p(q), _p(None if o is None else _c(o, np.uint16)),
                    _p(s), I64(s.shape[0]), I64(B), I64(M), I64(N), I32(K), I32(bits), I32(flags), _p(x))
    return x


# ------------------------------------------------------------------ metrics
def rel_fro(a, b) -> float:
    """||a - b||_F / ||b||_F in binary64 (a, b float arrays or bf16 bits)."""
    a = bf16_to_f32(a) if a.dtype == np.uint16 else a
    b = bf16_to_f32(b) if b.dtype == np.uint16 else b
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def unpack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """Channel-group format codes (T x H*bits/8) -> unsigned codes (T x H)."""
    if bits == 8:
        return codes.copy()
    lo = codes & 0xF
    hi = codes >> 4
    return np.stack([lo, hi], axis=-1).reshape(codes.shape[0], -1)


# ------------------------------------------------------------------ parity with tie attribution
def compare_encode(codes, scales, X, L, Vb, idx, bits, group, wht, tie_eps=2e-3, max_frac=1e-4, scale_rtol=1e-4):
    """Compare kernel codes/scales with the oracle's, given the same projection L.

    The kernels sum the low-rank term on the tensor cores in float32 (a few
    ulps from the oracle's exact sum), so a code may differ where the value it
    rounds sits within that distance of a rounding tie.  Returns a dict of
    counts; ``ok`` holds when every differing code is off by one, its oracle
    input lies within ``tie_eps`` of a tie, differing codes are at most
    ``max_frac`` of all codes, and every scale agrees to ``scale_rtol``
    relative (a group's absmax element moves by the same few ulps; with the
    rotation the residual is a sum of 128 such values)."""
    ref_codes, ref_scales, ref_outl = encode_given_lr(X, L, Vb, idx, bits, group, wht)
    off = 1 << (bits - 1)
    a = unpack_codes(np.asarray(codes), bits).astype(np.int32) - off
    b = unpack_codes(ref_codes, bits).astype(np.int32) - off
    diff = a != b
    n_diff = int(diff.sum())
    out = {"codes": int(a.size), "codes_differing": n_diff, "max_code_step": int(np.abs(a - b).max(initial=0)),
           "max_tie_distance": 0.0}
    if n_diff:
        pre = quantizer_inputs(X, L, Vb, idx, bits, group, wht)
        tie = np.abs(pre - np.floor(pre) - 0.5)
        out["max_tie_distance"] = float(tie[diff].max())
    s_a = np.asarray(scales, np.float64)
    s_b = ref_scales.astype(np.float64)
    rel = np.abs(s_a - s_b) / np.maximum(np.abs(s_b), 1e-30)
    out["scales_differing"] = int((s_a != s_b).sum())
    out["max_scale_rel"] = float(rel.max(initial=0.0))
    out["ok"] = (out["max_code_step"] <= 1 and out["max_tie_distance"] < tie_eps and n_diff <= max_frac * a.size
                 and out["max_scale_rel"] < scale_rtol)
    out["ref"] = (ref_codes, ref_scales, ref_outl)
    return out


def _wht_f32(w):
    """The oracle's unnormalised butterflies (stages 1, 2, ..., 64) per 128-channel block, binary32."""
    T, H = w.shape
    w = w.reshape(T, H // 128, 128).copy()
    m = 1
    while m < 128:
        v = w.reshape(T, H // 128, 128 // (2 * m), 2, m)
        a_, b_ = v[:, :, :, 0, :].copy(), v[:, :, :, 1, :].copy()
        v[:, :, :, 0, :] = a_ + b_
        v[:, :, :, 1, :] = a_ - b_
        m *= 2
    return w.reshape(T, H)


def decode_prerounding(codes, scales, L, Vb, H, bits, group, wht):
    """The oracle decode's binary32 value before its bf16 rounding, and the
    magnitude that bounds a float32 evaluation's error: sum_j |L_j V_j| + |w|
    (the low-rank sum often cancels, so its rounding error scales with its
    terms, not with its result)."""
    off = 1 << (bits - 1)
    u = unpack_codes(np.asarray(codes), bits).astype(np.float32) - np.float32(off)
    w = (u * np.repeat(np.asarray(scales, np.float32), group, axis=1)).astype(np.float32)
    if wht:
        w = (_wht_f32(w) * np.float32(0.0078125)).astype(np.float32)
    if L is not None and L.shape[1]:
        P = lowrank(L, Vb)
        terms = np.abs(L.astype(np.float64)) @ np.abs(bf16_to_f32(Vb).astype(np.float64)).T
    else:
        P = np.zeros_like(w)
        terms = 0.0
    return (P + w).astype(np.float32), terms + np.abs(w)


def _bf16_step(f):
    """Spacing of bf16 values at |f| (0 at zero)."""
    m, e = np.frexp(np.abs(f).astype(np.float64))
    return np.where(f == 0, 0.0, np.ldexp(1.0, e - 8))


def compare_decode(xh, ref, codes, scales, L, Vb, idx, H, bits, group, wht, ulps=64, max_frac=1e-3):
    """A kernel decode (bf16 bits) against the oracle's decode of the same
    buffers.  The kernels sum the low-rank term on the tensor cores (a few
    float32 ulps of its terms from the oracle's exact sum), so a kernel value
    may differ from the oracle's where it is the bf16 rounding of some value
    within ``ulps`` ulps of sum_j |L_j V_j| + |w| of the oracle's binary32
    value v (a rounding tie of v).  ``ok`` when every difference is such a case and they are at most
    ``max_frac`` of all values; ``worst`` describes the furthest one."""
    xh = np.asarray(xh, np.uint16)
    ref = np.asarray(ref, np.uint16)
    d = xh != ref
    n = int(d.sum())
    out = {"values": int(xh.size), "differing": n, "max_tie_ulps": 0.0, "ok": True}
    if n:
        v, mag = decode_prerounding(codes, scales, L, Vb, H, bits, group, wht)
        fa = bf16_to_f32(xh[d]).astype(np.float64)
        vd = v[d].astype(np.float64)
        # how far v must move (in ulps of the summands) for fa to be its bf16 rounding
        excess = np.maximum(np.abs(fa - vd) - 0.5 * _bf16_step(fa), 0.0)
        dist = excess / (np.maximum(mag[d].astype(np.float64), 1e-30) * 2.0 ** -24)
        out["max_tie_ulps"] = float(dist.max())
        w = int(np.argmax(dist))
        rows, cols = np.nonzero(d)
        out["worst"] = {"row": int(rows[w]), "col": int(cols[w]), "kernel": float(fa[w]),
                        "oracle": float(bf16_to_f32(ref[d])[w]), "v": float(vd[w]), "mag": float(mag[d][w])}
        out["ok"] = out["max_tie_ulps"] <= ulps and n <= max_frac * xh.size
    return out


def compare_bf16(a, b, max_frac=1e-4):
    """Two bf16 tensors (bit arrays) that should agree except where a float32
    sum of a few ulps' difference crossed a bf16 rounding boundary: differing
    values must be one bf16 step apart and at most ``max_frac`` of all."""
    a = np.asarray(a, np.uint16)
    b = np.asarray(b, np.uint16)
    d = a != b
    n = int(d.sum())
    fa = bf16_to_f32(a[d]).astype(np.float64)
    fb = bf16_to_f32(b[d]).astype(np.float64)
    ulp = np.abs(fb) * 2.0 ** -7  # one bf16 step (7 explicit mantissa bits), upper bound
    step_ok = bool(np.all(np.abs(fa - fb) <= ulp + 1e-38))
    return {"values": int(a.size), "differing": n, "ok": step_ok and n <= max_frac * a.size}


# ------------------------------------------------------------------ NF4 base weight
# bitsandbytes (a third-party dependency of the reference's driver scripts, not
# vendored under the reference and not installed here; no version pinned by the
# reference) quantises the frozen LoRA base weight to NF4
# (low_rank_system_profile_backward.py:31) and dequantises it with
# F.dequantize_4bit(..., quant_type='nf4') (:58).  What follows restates the
# published algorithm (the QLoRA paper's NormalFloat data type and blockwise
# absmax quantisation with optional nested statistics).  No reference test or
# fixture holds NF4 values, so this part of the oracle is "parity unpinned":
# it pins the kernel to this restatement, not to bitsandbytes.

#: quantile offset of the NF4 construction: 1 - (1/32 + 1/30) / 2
NF4_OFFSET = 1.0 - 0.5 * (1.0 / 32.0 + 1.0 / 30.0)


def nf4_code() -> np.ndarray:
    """The 16 NF4 values (float32, ascending): 8 quantiles of N(0, 1) at
    probabilities evenly spaced from NF4_OFFSET down to (not including) 1/2 for
    the positive half, 7 such quantiles for the negative half, and an exact
    zero; normalised so that the extremes are -1 and +1."""
    from statistics import NormalDist

    nd = NormalDist()
    pos = [nd.inv_cdf(p) for p in np.linspace(NF4_OFFSET, 0.5, 9)[:-1]]
    neg = [-nd.inv_cdf(p) for p in np.linspace(NF4_OFFSET, 0.5, 8)[:-1]]
    v = np.array(sorted(pos + [0.0] + neg), dtype=np.float64)
    return (v / np.abs(v).max()).astype(np.float32)


def nf4_quantize(w: np.ndarray, blocksize: int, code: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Blockwise absmax quantisation of w (flattened row-major) to 4-bit indices
    of the nearest code value: returns (packed bytes, value 2j in the high
    nibble of byte j; float32 absmax per block).  Test data only."""
    x = np.ascontiguousarray(w, dtype=np.float32).ravel()
    n = x.size
    nb = -(-n // blocksize)
    pad = np.zeros(nb * blocksize, np.float32)
    pad[:n] = x
    absmax = np.abs(pad.reshape(nb, blocksize)).max(axis=1).astype(np.float32)
    scale = np.where(absmax > 0, absmax, 1.0).astype(np.float32)
    t = (pad.reshape(nb, blocksize) / scale[:, None]).ravel()[:n]
    idx = np.abs(t[:, None] - code[None, :].astype(np.float32)).argmin(axis=1).astype(np.uint8)
    if n % 2:
        idx = np.concatenate([idx, np.zeros(1, np.uint8)])
    packed = ((idx[0::2] << 4) | idx[1::2]).astype(np.uint8)
    return packed, absmax


def nested_stats(absmax: np.ndarray, blocksize2: int, code2: np.ndarray):
    """Nested (double) quantisation of float32 block statistics: offset = mean,
    then blockwise absmax quantisation of (absmax - offset) to the nearest of
    the 256 code2 values.  Returns (absmax_q uint8, absmax2 float32, offset
    float32).  Test data only."""
    a = np.asarray(absmax, np.float32)
    offset = np.float32(a.astype(np.float64).mean())
    d = (a - offset).astype(np.float32)
    nb2 = -(-d.size // blocksize2)
    pad = np.zeros(nb2 * blocksize2, np.float32)
    pad[: d.size] = d
    a2 = np.abs(pad.reshape(nb2, blocksize2)).max(axis=1).astype(np.float32)
    s2 = np.where(a2 > 0, a2, 1.0).astype(np.float32)
    t = (pad.reshape(nb2, blocksize2) / s2[:, None]).ravel()[: d.size]
    q = np.abs(t[:, None] - np.asarray(code2, np.float32)[None, :]).argmin(axis=1).astype(np.uint8)
    return q, a2, offset


def nf4_dequant(packed, n, blocksize, code, absmax=None, absmax_q=None, absmax2=None, code2=None,
                blocksize2=256, offset=0.0) -> np.ndarray:
    """bf16 bits of the n dequantised values, with the rounding points of
    F.dequantize_4bit followed by .to(bfloat16): block statistic in float32
    (nested: code2[q] * absmax2, rounded, plus the offset, rounded), the value
    code[index] * statistic rounded to float32, then to bf16 (nearest even)."""
    packed = np.asarray(packed, np.uint8)
    idx = np.empty(2 * packed.size, np.uint8)
    idx[0::2] = packed >> 4
    idx[1::2] = packed & 15
    idx = idx[:n]
    if absmax_q is not None:
        prod = (np.asarray(code2, np.float32)[np.asarray(absmax_q)] * np.asarray(absmax2, np.float32)[
            np.arange(len(absmax_q)) // blocksize2]).astype(np.float32)
        am = (prod + np.float32(offset)).astype(np.float32)
    else:
        am = np.asarray(absmax, np.float32)
    v = (np.asarray(code, np.float32)[idx] * am[np.arange(n) // blocksize]).astype(np.float32)
    return f32_to_bf16(v)
