"""dW = xhat^T dy with the dequantisation inside the GEMM (actcomp_cg_dw_fused).

The fused path evaluates dW = Q^T dy + V (L^T dy), outlier rows = O^T dy, with
Q = bf16((u - 2^(b-1)) s) zero in the outlier channels.  Two checks per case:
the kernel against that formula evaluated in float64 from the compressed
buffers (the GEMM's float32 accumulation is the only difference), and against
the GEMM of the bf16 reconstruction (actcomp_cg_dw): the two round different
things to bf16 (the residual, or the residual plus the low-rank term), about
5e-4 apart on low-rank data and up to ~1.2e-3 when the residual carries an
unextracted outlier channel, so the bar is 2e-3 there, and against the GEMM of
the uncompressed x the fused path must be no further off than the two-kernel
path."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _split_formula(O, c, dy):
    """The fused path's formula in float64 from the compressed buffers."""
    T, H, b, g, r, k = c.tokens, c.channels, c.bits, c.group, c.rank, c.n_outlier
    codes = c.codes.cpu().numpy().reshape(T, -1)
    u = O.unpack_codes(codes, b).astype(np.float32)
    s = np.repeat(c.scales.cpu().numpy().reshape(T, -1), g, axis=1)
    w = ((u - 2 ** (b - 1)).astype(np.float32) * s).astype(np.float32)
    idx = c.outlier_idx.cpu().numpy().reshape(-1) if k else np.zeros(0, np.int64)
    w[:, idx] = 0
    q = O.bf16_to_f32(O.f32_to_bf16(w)).astype(np.float64)
    d = dy.float().cpu().numpy().astype(np.float64)
    out = q.T @ d
    if r:
        L = c.lowrank.cpu().numpy().reshape(T, r).astype(np.float64)
        V = c.basis.basis[0].float().cpu().numpy().astype(np.float64)  # H x r
        out += V @ (L.T @ d)
    if k:
        o = c.outliers.float().cpu().numpy().reshape(T, k).astype(np.float64)
        out[idx] = o.T @ d
    return out


CASES = [  # T, H, N, r, k, bits, group
    (1000, 768, 264, 32, 16, 4, 64),
    (4096, 1024, 512, 16, 8, 4, 32),
    (777, 384, 1000, 0, 0, 4, 128),
    (2048, 512, 256, 32, 0, 8, 64),
    (300, 256, 8, 16, 16, 8, 32),
]


@pytest.mark.parametrize("T,H,N,r,k,bits,group", CASES)
def test_fused_dw_matches_its_formula_and_the_reconstruction_gemm(O, T, H, N, r, k, bits, group):
    import actcomp
    from actcomp import synthetic

    x, _ = synthetic.lowrank_activation(T, H, n_outlier=max(k, 1), seed=T + H, device="cuda")
    basis = actcomp.Basis.fit(x, r) if r else None
    idx = actcomp.select_outlier_channels(x, k) if k else None
    c = actcomp.encode(x, basis, idx, bits=bits, group=group)
    dy = synthetic.gradient((T, N), seed=N, device="cuda")
    fused = actcomp.weight_grad(c, dy, torch.float32, fused=True)
    ref = _split_formula(O, c, dy)
    e = np.linalg.norm(fused.double().cpu().numpy() - ref) / np.linalg.norm(ref)
    assert e < 1e-5, f"fused dW vs its formula: {e:.2e}"
    two = actcomp.weight_grad(c, dy, torch.float32)  # GEMM of the bf16 reconstruction
    e2 = float((fused.double() - two.double()).norm() / two.double().norm())
    assert e2 < 2e-3, f"fused dW vs GEMM of xhat: {e2:.2e}"
    # neither rounding is the truth: against the GEMM of the uncompressed x the
    # fused path is no further off than the reconstruction's GEMM
    gx = actcomp.gemm(x.mT, dy, torch.float32).double()
    e_f = float((fused.double() - gx).norm() / gx.norm())
    e_t = float((two.double() - gx).norm() / gx.norm())
    assert e_f <= 1.02 * e_t + 1e-6, f"fused {e_f:.3e} vs two-kernel {e_t:.3e} from the GEMM of x"
    # bf16 output: the float32 result rounded once
    fb = actcomp.weight_grad(c, dy, torch.bfloat16, fused=True)
    assert torch.equal(fb, fused.to(torch.bfloat16))


def test_fused_dw_refuses_what_it_does_not_cover():
    import ctypes

    import actcomp
    from actcomp import _lib, synthetic

    T, H = 256, 384
    x, _ = synthetic.lowrank_activation(T, H, n_outlier=4, seed=3, device="cuda")
    dy = synthetic.gradient((T, 64), seed=4, device="cuda")
    # the rotated format and an outlier count that is not a multiple of 8
    for kw in (dict(idx=None, wht=True), dict(idx=actcomp.select_outlier_channels(x, 4), wht=False)):
        c = actcomp.encode(x, actcomp.Basis.fit(x, 16), kw["idx"], bits=4, group=64, wht=kw["wht"])
        with pytest.raises(_lib.ActcompError) as ei:
            actcomp.weight_grad(c, dy, torch.float32, fused=True)
        assert ei.value.status == _lib.ACT_E_UNSUPPORTED
    assert _lib.load().actcomp_cg_dw_fused_workspace(None, 64) == 0
    del ctypes
