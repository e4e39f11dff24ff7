"""Parity at the benchmark configurations' full sizes (GPU against the CPU
oracle and the PyTorch north-star checker).

* config 2: 16384 x 4096 and 16384 x 11008 activations, r = 32, k = 16, int4
  group 64; the SiLU backward on the 11008-channel one;
* config 3: 32768 x 5120 heavy-tailed, r = 16, int4 group 128, with and
  without the rotation;
* config 4: dW = Xhat^T dY, 4096 x 11008 x 16384, against a float32 GEMM of the
  decoded activation and (reported) against the bf16 GEMM of the uncompressed X;
* config 5: GELU backward at 65536 x 5120 and softmax backward at S = 2048.

Each prints its figures (pytest -s) -- flip counts with tie distances,
relative errors -- which DESIGN.md quotes.  Protocol as tests/test_cg_gpu.py.
"""
import os
import sys

import numpy as np
import pytest
import torch

from conftest import bits

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def _encode(x, r, k, b, g, wht, calib=4096):
    import actcomp

    basis = actcomp.Basis.fit(x[:calib], r) if r else None
    idx = actcomp.select_outlier_channels(x[:calib], k) if k else None
    c = actcomp.encode(x, basis, idx, bits=b, group=g, wht=wht)
    torch.cuda.synchronize()
    return c, idx


def _check_against_oracle(O, c, xb, idx, b, g, wht, tag):
    """Codes/scales given the kernel's L, projection bound, decode; returns the GPU decode (bf16 bits)."""
    import actcomp

    idx_np = None if idx is None else idx.cpu().numpy()
    L = Vb = None
    if c.rank:
        Vt = bits(c.basis.basis_t[0])
        Vb = bits(c.basis.basis[0])
        L = c.lowrank.cpu().numpy()
        L_o = O.project(xb, Vt)
        xf = np.abs(O.bf16_to_f32(xb))
        bound = (c.channels / 16) * 2.0 ** -22 * (xf @ np.abs(O.bf16_to_f32(Vt)).T).astype(np.float64) + 1e-30
        err = np.abs(L.astype(np.float64) - L_o)
        print(f"{tag}: projection max |L - L_exact| / max |L_exact| = {float(err.max() / np.abs(L_o).max()):.2e}")
        assert np.all(err <= bound), f"{tag}: projection differs (max err/bound {float((err / bound).max()):.3f})"
    codes, scales = c.codes.cpu().numpy(), c.scales.cpu().numpy()
    cmp = O.compare_encode(codes, scales, xb, L, Vb, idx_np, b, g, wht)
    print(f"{tag}: codes {cmp['codes']}, differing {cmp['codes_differing']} (max tie distance "
          f"{cmp['max_tie_distance']:.2e}), scales differing {cmp['scales_differing']}")
    assert cmp["ok"], {k_: v for k_, v in cmp.items() if k_ != "ref"}
    if c.n_outlier:
        assert np.array_equal(bits(c.outliers), cmp["ref"][2])
    xh = bits(actcomp.decode(c))
    ref = O.decode(codes, scales, L, Vb, cmp["ref"][2] if c.n_outlier else None, idx_np, c.channels, b, g, wht)
    dcmp = O.compare_decode(xh, ref, codes, scales, L, Vb, idx_np, c.channels, b, g, wht)
    print(f"{tag}: decode values {dcmp['values']}, differing by one bf16 step at rounding ties "
          f"{dcmp['differing']} (max distance {dcmp['max_tie_ulps']:.1f} ulps)")
    assert dcmp["ok"], str(dcmp)
    return xh


def _check_against_checker(O, NS, c, xb, idx, b, g, wht, tag):
    """End to end against the north-star checker on the identical (bf16) basis."""
    x = torch.from_numpy(O.bf16_to_f32(xb))
    V = c.basis.vectors()[0].cpu() if c.rank else torch.zeros(x.shape[1], 0)
    idx_np = None if idx is None else idx.cpu().numpy()
    ns = NS.encode(x, V, idx_np, b, g, wht)
    xh_ns = NS.decode(ns, V, idx_np, g, wht)
    codes = O.unpack_codes(c.codes.cpu().numpy(), b).astype(np.int32) - (1 << (b - 1))
    diff = codes != ns["codes"].numpy()
    tie = NS.tie_distance(ns["pre"]).numpy()
    import actcomp

    xh = torch.from_numpy(O.bf16_to_f32(bits(actcomp.decode(c))))
    rel = NS.rel_fro(xh, xh_ns)  # includes the bf16 rounding of the kernel's output
    # where the codes agree, both reconstructions rounded to bf16 differ only at rounding ties
    same = torch.from_numpy(~diff)
    xh_ns_bf = xh_ns.to(torch.bfloat16).float()
    rel_same = NS.rel_fro(xh * same, xh_ns_bf * same)
    print(f"{tag}: against the north-star checker: codes differing {int(diff.sum())} of {diff.size} "
          f"(max tie distance {float(tie[diff].max()) if diff.any() else 0.0:.2e}); reconstruction rel-Frobenius "
          f"{rel:.3e} (checker in float32), {NS.rel_fro(xh, xh_ns_bf):.3e} (both bf16), {rel_same:.3e} (both bf16, "
          f"where the codes agree); rel error vs X: kernel {NS.rel_fro(xh, x):.4e}, checker {NS.rel_fro(xh_ns, x):.4e}")
    assert diff.mean() < 1e-4
    if diff.any():
        assert tie[diff].max() < 2e-3
    assert rel_same < 1e-4
    assert rel < 1e-3
    return xh


def test_config2_encode_decode_full_size(O):
    from actcomp import synthetic
    import northstar as NS

    x, _ = synthetic.lowrank_activation(16384, 4096, n_outlier=16, seed=0, device="cuda")
    c, idx = _encode(x, 32, 16, 4, 64, False)
    xb = bits(x)
    _check_against_oracle(O, c, xb, idx, 4, 64, False, "config 2 (16384 x 4096)")
    _check_against_checker(O, NS, c, xb, idx, 4, 64, False, "config 2 (16384 x 4096)")


def test_config2_silu_input_full_size(O):
    import actcomp
    from actcomp import synthetic

    T, H = 16384, 11008
    x, _ = synthetic.lowrank_activation(T, H, n_outlier=16, seed=100, device="cuda")
    c, idx = _encode(x, 32, 16, 4, 64, False)
    xh = _check_against_oracle(O, c, bits(x), idx, 4, 64, False, "config 2 (16384 x 11008)")
    del x
    dy = synthetic.gradient((T, H), seed=7, device="cuda")
    dx = bits(actcomp.silu_backward(c, dy))
    ref = O.silu_bwd(xh, bits(dy))
    rel = O.rel_fro(dx, ref)
    print(f"config 2 SiLU backward 16384 x 11008: rel-Frobenius against the oracle {rel:.2e}, "
          f"equal values {(dx == ref).mean():.6f}")
    assert rel < 1e-3


def test_config3_rotation_full_size(O):
    import actcomp
    from actcomp import synthetic

    T, H = 32768, 5120
    x = synthetic.heavy_tailed_activation(T, H, seed=400, device="cuda")
    xb = bits(x)
    c, _ = _encode(x, 16, 0, 4, 128, True)
    xh_rot = _check_against_oracle(O, c, xb, None, 4, 128, True, "config 3 rotated (32768 x 5120)")
    c2 = actcomp.encode(x, c.basis, None, bits=4, group=128, wht=False)
    xh_plain = bits(actcomp.decode(c2))
    e_rot, e_plain = O.rel_fro(xh_rot, xb), O.rel_fro(xh_plain, xb)
    print(f"config 3: rel error vs X with the rotation {e_rot:.4f}, without {e_plain:.4f}")
    assert e_rot < e_plain  # heavy tails: the rotation spreads them over the block


def test_config4_weight_gradient_full_size(O):
    import actcomp
    from actcomp import synthetic

    T, H, N = 16384, 4096, 11008
    x, _ = synthetic.lowrank_activation(T, H, n_outlier=16, seed=0, device="cuda")
    c, _ = _encode(x, 32, 16, 4, 64, False)
    dy = synthetic.gradient((T, N), seed=11, device="cuda")
    dw = actcomp.weight_grad(c, dy, torch.float32)
    xh = actcomp.decode(c)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = xh.float().T @ dy.float()              # float32 GEMM of the decoded activation
        unc = (x.T @ dy).float()                      # bf16 GEMM of the uncompressed activation
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    rel = float((dw - ref).norm() / ref.norm())
    rel_unc = float((dw - unc).norm() / unc.norm())
    print(f"config 4 dW 4096 x 11008 x 16384: rel-Frobenius against the float32 GEMM of Xhat {rel:.2e}; "
          f"against the bf16 GEMM of the uncompressed X {rel_unc:.4e}")
    assert rel < 1e-4  # float32 accumulation over K = 16384 in two different orders
    assert rel_unc < 0.06


def test_config5_gelu_full_size(O):
    import actcomp
    from actcomp import synthetic

    T, H = 65536, 5120
    x, _ = synthetic.lowrank_activation(T, H, n_outlier=16, seed=200, device="cuda")
    c, idx = _encode(x, 32, 16, 4, 64, False)
    del x
    dy = synthetic.gradient((T, H), seed=13, device="cuda")
    dx = bits(actcomp.gelu_backward(c, dy))
    xh = bits(actcomp.decode(c))
    ref = O.gelu_bwd(xh, bits(dy))
    rel = O.rel_fro(dx, ref)
    print(f"config 5 GELU backward 65536 x 5120: rel-Frobenius against the oracle {rel:.2e}")
    assert rel < 1e-3


@pytest.mark.parametrize("causal", [True])
def test_config5_softmax_full_size(O, causal):
    import actcomp
    from actcomp import synthetic

    heads, S = 4, 2048
    P = synthetic.causal_softmax(1, heads, S, seed=300, device="cuda")[0]
    pf = P[0].float()
    V = torch.linalg.eigh(pf.T @ pf)[1][:, -32:].flip(-1)
    basis = actcomp.Basis.from_vectors(V.unsqueeze(0).expand(heads, S, 32).contiguous())
    c = actcomp.encode(P, basis, None, bits=4, group=64)
    dp = synthetic.gradient((heads, S, S), seed=17, device="cuda")
    ds = bits(actcomp.softmax_backward(c, dp, causal=causal))
    ph = bits(actcomp.decode(c)).reshape(heads, S, S)
    ph = np.where(np.tril(np.ones((S, S), bool)), ph, np.uint16(0))
    ref = O.softmax_bwd(ph, bits(dp))
    rel = O.rel_fro(ds, ref)
    print(f"config 5 causal softmax backward {heads} x {S} x {S}: rel-Frobenius against the oracle {rel:.2e}")
    assert rel < 1e-3
