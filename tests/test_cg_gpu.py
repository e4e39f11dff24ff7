"""GPU parity of the channel-group format against the CPU oracle.

Protocol:
* the bf16 basis and the outlier values are bit-exact;
* the projection L (a length-H float32 sum on the tensor cores) is within
  (H/16) * 2^-22 * sum |x v| of the oracle's exact sum;
* given the kernel's L, codes and scales equal the oracle's except where the
  quantiser's input sits within 2e-3 of a rounding tie (the tensor cores sum
  the low-rank term L . V^T in their own float32 order, a few ulps from the
  oracle's exact sum); at most 1e-4 of the codes may differ, each by one step;
* the decode of the kernel's buffers equals the oracle's decode of the same
  buffers except for values one bf16 step apart at rounding ties (at most
  1e-3 of them)."""
import numpy as np
import pytest
import torch

from conftest import bits, to_bf16

pytestmark = pytest.mark.gpu


def make_case(O, T, H, r, k, seed=0):
    from actcomp import synthetic

    x, ch = synthetic.lowrank_activation(T, H, signal_rank=24, n_outlier=max(k, 1), seed=seed)
    xb = bits(x)
    V = np.zeros((H, 0), np.float32)
    if r:
        _, _, vt = np.linalg.svd(O.bf16_to_f32(xb).astype(np.float64), full_matrices=False)
        V = vt[:r].T.astype(np.float32)
    idx = O.topk_channels(O.channel_absmax(xb), k) if k else np.zeros(0, np.int32)
    return xb, V, idx


def gpu_encode(xb, V, idx, bits_, group, wht):
    import actcomp

    x = to_bf16(xb)
    basis = actcomp.Basis.from_vectors(torch.from_numpy(V).cuda()) if V.shape[1] else None
    oi = torch.from_numpy(idx).cuda() if len(idx) else None
    c = actcomp.encode(x, basis, oi, bits=bits_, group=group, wht=wht)
    torch.cuda.synchronize()
    return c


CASES = [
    # T, H, r, k, bits, group, wht
    (256, 512, 32, 16, 4, 64, False),   # config-2 style
    (128, 640, 16, 0, 4, 128, True),    # config-3 style (rotation, no outliers)
    (96, 384, 16, 8, 8, 128, False),    # config-1 style (int8 g128)
    (37, 320, 32, 5, 4, 64, False),     # ragged: T not a multiple of anything, H % 128 != 0
    (64, 256, 0, 0, 4, 32, False),      # no low rank, no outliers
    (64, 256, 64, 64, 8, 64, False),    # maximum rank and outlier count
    (50, 1024, 48, 3, 4, 128, True),
    # wide activations (the tensor-core encode splits channels wider than 8192 over a cluster of CTAs)
    (200, 2048, 32, 16, 4, 64, False),
    (130, 4096, 32, 16, 4, 64, False),
    (96, 5120, 16, 0, 4, 128, True),    # config-3 width
    (64, 11008, 32, 16, 4, 64, False),  # config-2 SiLU-input width (row encode, 86 chunks per block)
    (40, 16384, 32, 8, 4, 64, False),   # widest row encode
    (32, 20480, 16, 0, 4, 128, True),   # above 16384 channels: the cluster encode (160 chunks over 8 CTAs)
    # the row encode with the rotation: int8 groups of 64 with outliers, int4 groups of 32
    (100, 2048, 32, 5, 8, 64, True),
    (64, 3072, 16, 9, 4, 32, True),
    (72, 4096, 64, 7, 8, 32, False),
    # the rotated row decode: no low rank (its TMEM scratch columns start at 0)
    # with int8 codes and outliers; several token blocks per CTA range
    (150, 1024, 0, 4, 8, 64, True),
    (3000, 1024, 16, 3, 4, 128, True),
    # the row decode (H a multiple of 512, no rotation): rank 0 with outliers,
    # rank 16 without, rank 48 with an odd outlier count (unaligned outlier rows
    # in the partial last token block), several token blocks per CTA range
    (300, 1024, 0, 5, 4, 64, False),
    (129, 1536, 16, 0, 8, 128, False),
    (260, 2560, 48, 33, 4, 32, False),
    (1100, 512, 32, 16, 4, 64, False),
    # more token blocks than SMs: some CTAs of the row encode take two blocks
    # (separate projection / residual rings, double-buffered low-rank tiles)
    (19277, 1024, 32, 8, 4, 64, False),
    # int8 codes through the two-kernel encode (projection, quantisation)
    (160, 1024, 32, 8, 8, 64, False),
    (90, 768, 16, 4, 8, 32, False),
]


def check_projection(O, xb, L, Vt):
    """L from the kernel against the oracle's exact sums: a float32
    accumulation over H/16 tensor-core steps is within (H/16) * 2^-22 *
    sum |x v| of the exact sum (one ulp of loss per step, truncation included)."""
    L_o = O.project(xb, Vt)
    H = xb.shape[1]
    xf = np.abs(O.bf16_to_f32(xb).astype(np.float64))
    bound = (H / 16) * 2.0 ** -22 * (xf @ np.abs(O.bf16_to_f32(Vt).astype(np.float64)).T) + 1e-30
    err = np.abs(L.astype(np.float64) - L_o)
    assert np.all(err <= bound), f"projection differs from the oracle: max err/bound {float((err / bound).max()):.3f}"
    return L_o


@pytest.mark.parametrize("T,H,r,k,b,g,wht", CASES)
def test_encode_decode_parity(O, T, H, r, k, b, g, wht):
    xb, V, idx = make_case(O, T, H, r, k)
    c = gpu_encode(xb, V, idx, b, g, wht)
    L = Vb = None
    if r:
        Vt, Vb = O.basis_prepare(V)
        assert np.array_equal(bits(c.basis.basis_t[0]), Vt)
        assert np.array_equal(bits(c.basis.basis[0]), Vb)
        L = c.lowrank.cpu().numpy()
        check_projection(O, xb, L, Vt)
    codes, scales = c.codes.cpu().numpy(), c.scales.cpu().numpy()
    cmp = O.compare_encode(codes, scales, xb, L, Vb, idx, b, g, wht)
    assert cmp["ok"], {k_: v for k_, v in cmp.items() if k_ != "ref"}
    outl = cmp["ref"][2]
    if k:
        assert np.array_equal(bits(c.outliers), outl)
    # decode of the GPU buffers
    import actcomp

    xh = bits(actcomp.decode(c))
    ref = O.decode(codes, scales, L, Vb, outl if k else None, idx, H, b, g, wht)
    dcmp = O.compare_decode(xh, ref, codes, scales, L, Vb, idx, H, b, g, wht)
    assert dcmp["ok"], str(dcmp)
    # and the reconstruction is close to the input (without outlier channels an
    # int4 group that holds a x30 channel is coarse, hence the looser bound)
    assert O.rel_fro(xh, xb) < ((0.06 if k else 0.2) if b == 4 else 0.01)


@pytest.mark.parametrize("T,H,r,k,b,g,wht", [CASES[0], CASES[8], CASES[9], CASES[10]])
def test_codes_against_the_oracle_projection(O, T, H, r, k, b, g, wht):
    """End to end: the kernel's codes against the oracle's codes computed from
    the oracle's own projection.  The two projections differ by float32
    summation order only, so the codes may differ only at rounding ties."""
    xb, V, idx = make_case(O, T, H, r, k, seed=11)
    c = gpu_encode(xb, V, idx, b, g, wht)
    Vt, Vb = O.basis_prepare(V)
    L_o = O.project(xb, Vt)
    # the two projections differ by up to ~1e-5 of the terms: the residual (and
    # a group's absmax) moves by that much relative to the low-rank term
    cmp = O.compare_encode(c.codes.cpu().numpy(), c.scales.cpu().numpy(), xb, L_o, Vb, idx, b, g, wht, max_frac=1e-3,
                           scale_rtol=1e-2)
    print(f"T={T} H={H}: codes differing from the oracle's own projection {cmp['codes_differing']} of "
          f"{cmp['codes']}, max tie distance {cmp['max_tie_distance']:.2e}")
    assert cmp["ok"], {k_: v for k_, v in cmp.items() if k_ != "ref"}


@pytest.mark.parametrize("op", ["silu", "gelu", "mul"])
@pytest.mark.parametrize("T,H,r,k,b,g,wht", [CASES[0], CASES[1], CASES[3]])
def test_fused_consumers(O, op, T, H, r, k, b, g, wht):
    import actcomp

    xb, V, idx = make_case(O, T, H, r, k, seed=2)
    c = gpu_encode(xb, V, idx, b, g, wht)
    dy = (torch.randn(T, H, generator=torch.Generator().manual_seed(5)) * 0.02).to(torch.bfloat16)
    fn = {"silu": actcomp.silu_backward, "gelu": actcomp.gelu_backward, "mul": actcomp.mul}[op]
    out = bits(fn(c, dy.cuda()))
    xh = bits(actcomp.decode(c))
    ref = {"silu": O.silu_bwd, "gelu": O.gelu_bwd, "mul": O.mul}[op](xh, bits(dy))
    # exp / reciprocal use the hardware approximations (a few ulp): the bf16
    # outputs differ from the libm oracle only where a rounding boundary falls
    # inside that error
    assert O.rel_fro(out, ref) < 1e-3
    assert (out == ref).mean() > (0.9 if op == "gelu" else 0.999)


@pytest.mark.parametrize("causal", [True, False])
def test_softmax_backward_on_compressed_probabilities(O, causal):
    import actcomp
    from actcomp import synthetic

    B, heads, S = 1, 3, 256
    p = synthetic.causal_softmax(B, heads, S, seed=4) if causal else \
        torch.softmax(torch.randn(B, heads, S, S, generator=torch.Generator().manual_seed(4)), -1).to(torch.bfloat16)
    p3 = p.reshape(-1, S, S)
    Vs = []
    for h in range(p3.shape[0]):
        _, _, vt = np.linalg.svd(p3[h].float().numpy().astype(np.float64), full_matrices=False)
        Vs.append(vt[:32].T.astype(np.float32))
    basis = actcomp.Basis.from_vectors(torch.from_numpy(np.stack(Vs)).cuda())
    c = actcomp.encode(p3.cuda(), basis, None, bits=4, group=64)
    dp = (torch.randn(p3.shape, generator=torch.Generator().manual_seed(6)) * 0.02).to(torch.bfloat16)
    ds = bits(actcomp.softmax_backward(c, dp.cuda(), causal=causal))  # tensor-core passes
    ph = bits(actcomp.decode(c)).reshape(-1, S, S)
    if causal:
        ph = np.where(np.tril(np.ones((S, S), bool)), ph, np.uint16(0))
    ref = O.softmax_bwd(ph, bits(dp))
    assert O.rel_fro(ds, ref) < 1e-3
    # the CUDA-core kernel (no workspace) computes the same
    import ctypes

    from actcomp import _lib

    dpg = dp.cuda().contiguous()
    out = torch.empty_like(dpg)
    d = c.desc()
    assert _lib.load().actcomp_cg_softmax_bwd(ctypes.byref(d), dpg.data_ptr(), out.data_ptr(), S, int(causal), None,
                                                0, torch.cuda.current_stream().cuda_stream) == 0
    assert O.rel_fro(bits(out), ref) < 1e-3


@pytest.mark.parametrize("T,H,N", [(256, 256, 384), (512, 384, 200)])
def test_weight_gradient(O, T, H, N):
    import actcomp

    xb, V, idx = make_case(O, T, H, 32, 8, seed=7)
    c = gpu_encode(xb, V, idx, 4, 64, False)
    dy = (torch.randn(T, N, generator=torch.Generator().manual_seed(8)) * 0.02).to(torch.bfloat16)
    dw = actcomp.weight_grad(c, dy.cuda(), torch.float32).cpu().numpy()
    xh = bits(actcomp.decode(c))
    ref = O.gemm_tn(xh, bits(dy))
    assert O.rel_fro(dw, ref) < 1e-5


def test_channel_topk_matches_oracle(O):
    import actcomp

    xb, _, _ = make_case(O, 200, 768, 0, 0, seed=9)
    for k in (1, 16, 64):
        idx = actcomp.select_outlier_channels(to_bf16(xb), k).cpu().numpy()
        assert list(idx) == list(O.topk_channels(O.channel_absmax(xb), k))


@pytest.mark.parametrize("H", [256, 512, 1024])
def test_batched_slices_are_independent(O, H):
    """batch > 1 with a different basis per slice: every slice's buffers are the
    oracle's encode of that slice with its own basis, and the batch decode of a
    slice is the oracle's decode of that slice's buffers.  (A single-slice
    encode may take another kernel, whose tensor cores sum L in another order,
    so the batch is checked against the oracle, not against single encodes.)"""
    import actcomp

    T, r = 64, 16
    xs, Vs = [], []
    for s in range(3):
        xb, V, _ = make_case(O, T, H, r, 0, seed=20 + s)
        xs.append(xb)
        Vs.append(V)
    basis = actcomp.Basis.from_vectors(torch.from_numpy(np.stack(Vs)).cuda())
    c = actcomp.encode(to_bf16(np.stack(xs)), basis, None, bits=4, group=64)
    torch.cuda.synchronize()
    xh = bits(actcomp.decode(c)).reshape(3, T, H)
    codes = c.codes.cpu().numpy().reshape(3, T, -1)
    scales = c.scales.cpu().numpy().reshape(3, T, -1)
    L = c.lowrank.cpu().numpy().reshape(3, T, r)
    for s in range(3):
        Vt, Vb = O.basis_prepare(Vs[s])
        assert np.array_equal(bits(c.basis.basis_t[s]), Vt)
        check_projection(O, xs[s], L[s], Vt)
        cmp = O.compare_encode(codes[s], scales[s], xs[s], L[s], Vb, None, 4, 64, False)
        assert cmp["ok"], f"slice {s}: {dict((k_, v) for k_, v in cmp.items() if k_ != 'ref')}"
        ref = O.decode(codes[s], scales[s], L[s], Vb, None, None, H, 4, 64, False)
        dcmp = O.compare_decode(xh[s], ref, codes[s], scales[s], L[s], Vb, None, H, 4, 64, False)
        assert dcmp["ok"], f"slice {s}: {dcmp}"


def test_batched_encode_with_outliers_crossing_slices(O):
    """Two slices of 9700 tokens (152 token blocks: some CTAs encode a block of
    each slice, so the per-slice outlier tables change inside a CTA) with a
    different basis and outlier set per slice: every slice matches the oracle
    given the kernel's projection."""
    import actcomp

    T, H, r, k = 9700, 1024, 16, 4
    xs, Vs, idxs = [], [], []
    for s_ in range(2):
        xb, V, idx = make_case(O, T, H, r, k, seed=40 + s_)
        xs.append(xb)
        Vs.append(V)
        idxs.append(idx)
    basis = actcomp.Basis.from_vectors(torch.from_numpy(np.stack(Vs)).cuda())
    oi = torch.from_numpy(np.stack(idxs)).cuda()
    c = actcomp.encode(to_bf16(np.stack(xs)), basis, oi, bits=4, group=64)
    torch.cuda.synchronize()
    codes = c.codes.cpu().numpy().reshape(2, T, -1)
    scales = c.scales.cpu().numpy().reshape(2, T, -1)
    L = c.lowrank.cpu().numpy().reshape(2, T, r)
    outl = bits(c.outliers).reshape(2, T, k)
    for s_ in range(2):
        _, Vb = O.basis_prepare(Vs[s_])
        cmp = O.compare_encode(codes[s_], scales[s_], xs[s_], L[s_], Vb, idxs[s_], 4, 64, False)
        assert cmp["ok"], f"slice {s_}: {dict((k_, v) for k_, v in cmp.items() if k_ != 'ref')}"
        assert np.array_equal(outl[s_], cmp["ref"][2]), f"slice {s_}: outliers differ"
