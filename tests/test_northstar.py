"""The C oracle against an independent PyTorch statement of the north-star math.

oracle/northstar.py states the channel-group encode/decode as the north star
words it -- L = X V, R = X - L V^T in float32, top-k channels verbatim,
per-token group absmax, torch.round -- with no attempt to mirror the oracle's
rounding points.  The two must agree on identical inputs and basis: every
differing code sits at a rounding tie (the two sum L and L V^T in different
orders), and the reconstructions agree far inside the 1e-3 relative
Frobenius bar.  Config 1 (the CPU reference case) runs at its full size."""
import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


@pytest.fixture(scope="module")
def NS():
    import northstar

    return northstar


def _case(T, H, r, k, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((T, 48)) @ rng.standard_normal((48, H))) / 48 + 0.05 * rng.standard_normal((T, H))
    ch = np.sort(rng.choice(H, k, replace=False)).astype(np.int32)
    x[:, ch] *= 30
    _, _, vt = np.linalg.svd(x, full_matrices=False)
    return x.astype(np.float32), ch, vt[:r].T.astype(np.float32)


@pytest.mark.parametrize("bits,group,wht", [(4, 64, False), (8, 128, False), (4, 128, True)])
def test_oracle_codes_match_the_checker_up_to_ties(O, NS, bits, group, wht):
    x, ch, V = _case(512, 1024, 32, 16, seed=bits + group)
    xb = O.f32_to_bf16(x)
    Vt, Vb = O.basis_prepare(V)
    enc = O.encode(xb, (Vt, Vb), ch, bits, group, wht)
    codes = O.unpack_codes(enc["codes"], bits).astype(np.int32) - (1 << (bits - 1))
    xf = torch.from_numpy(O.bf16_to_f32(xb))
    Vbf = torch.from_numpy(O.bf16_to_f32(Vb))
    ns = NS.encode(xf, Vbf, ch, bits, group, wht)
    diff = codes != ns["codes"].numpy()
    tie = NS.tie_distance(ns["pre"]).numpy()
    assert diff.mean() < 1e-4
    assert np.all(np.abs(codes - ns["codes"].numpy()) <= 1)
    if diff.any():
        assert tie[diff].max() < 1e-3
    # the same projection and outliers
    assert np.allclose(enc["lowrank"], ns["lowrank"].numpy(), rtol=1e-5, atol=1e-6 * np.abs(enc["lowrank"]).max())
    assert np.array_equal(O.bf16_to_f32(enc["outliers"]), ns["outliers"].numpy())
    # reconstructions: the oracle's bf16 output against the checker's float32 one
    xh = O.decode(enc["codes"], enc["scales"], enc["lowrank"], Vb, enc["outliers"], ch, 1024, bits, group, wht)
    xh_ns = NS.decode(ns, Vbf, ch, group, wht)
    assert NS.rel_fro(torch.from_numpy(O.bf16_to_f32(xh)), xh_ns) < 1e-3


def test_config1_full_size_report(O):
    """Config 1 at 4096 x 4096 float32 (SVD basis, x50 outliers, int8 g128)."""
    import report_config1

    rep = report_config1.report()
    print(rep)
    assert rep["outliers_verbatim"]
    assert rep["codes_differing_from_checker"] <= 1e-4 * rep["codes"]
    assert rep["max_tie_distance_at_differences"] < 1e-3
    assert rep["rel_fro_oracle_vs_checker"] < 1e-4
    # int8 group-128 quantisation of the residual: the error is small against X
    assert rep["rel_err_oracle_vs_x"] < 3e-3
    assert abs(rep["rel_err_oracle_vs_x"] - rep["rel_err_checker_vs_x"]) < 1e-4
    # the basis rounded to bf16 changes the split between L V^T and R, not the error budget
    assert rep["rel_fro_oracle_vs_checker_fp32_basis"] < 3e-3
