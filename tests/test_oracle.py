"""CPU tests of the oracle: pinned against the reference's own PyTorch functions
(golden fixtures made by tests/golden/make_golden.py), and algebraic checks of
the channel-group restatement that the reference has no code for."""
import numpy as np
import pytest

# ---------------------------------------------------------------- pinned: reference-compatible format


@pytest.mark.parametrize("qb", [1, 2, 4, 8])
@pytest.mark.parametrize("N", [32, 64])
def test_rc_decode_matches_reference_twin(O, golden, qb, N):
    """torch_low_rank_addition_fuse_decompression_dequantization
    (low_rank_extraction_fuse_decompression_dequantization.py:155), bit for bit."""
    k = f"dec_b{qb}_n{N}"
    x = O.rc_decode(golden[k + "_l"], golden[k + "_r"], golden[k + "_q"], golden[k + "_o"], golden[k + "_s"], qb,
                    flags=O.RC_TWIN)
    assert np.array_equal(x, golden[k + "_x"])


@pytest.mark.parametrize("qb", [1, 2, 4, 8])
def test_rc_block32_packing_equals_row_packing_for_one_block(O, golden, qb):
    """With N = 32 the kernel's 32-column blocks and the twin's row interleave coincide."""
    k = f"dec_b{qb}_n32"
    args = (golden[k + "_l"], golden[k + "_r"], golden[k + "_q"], golden[k + "_o"], golden[k + "_s"], qb)
    assert np.array_equal(O.rc_decode(*args, flags=O.RC_TWIN & ~O.RC_ROW_PACK), golden[k + "_x"])


@pytest.mark.parametrize("qb", [8, 4, 2])
def test_rc_end_to_end_matches_naive(O, golden, qb):
    """naive_quantization_dequantization (low_rank_kernel_accuracy_test.py:6), bit for bit."""
    k = f"naive_b{qb}"
    o, q, _ = O.rc_encode(golden[k + "_l"], golden[k + "_r"], golden[k + "_x"], golden[k + "_s"], qb,
                          float(golden[k + "_outlier"]), flags=O.RC_TWIN)
    xh = O.rc_decode(golden[k + "_l"], golden[k + "_r"], q, o, golden[k + "_s"], qb, flags=O.RC_TWIN)
    assert np.array_equal(xh, golden[k + "_xhat"])


@pytest.mark.parametrize("qb", [8, 4, 1])
def test_rc_encode_codes_match_reference_twin(O, golden, qb):
    """torch_low_rank_addition_fuse_compression_quantization (low_rank_extraction_speed.py:146):
    signed codes and dense outliers, bit for bit."""
    k = f"enc_b{qb}"
    o, q, codes = O.rc_encode(golden[k + "_l"], golden[k + "_r"], golden[k + "_x"], golden[k + "_s"], qb,
                              float(golden[k + "_outlier"]), flags=O.RC_TWIN)
    assert np.array_equal(codes, golden[k + "_q"])
    assert np.array_equal(O.bf16_to_f32(o), O.bf16_to_f32(golden[k + "_o"]))


def test_rc_kernel_semantics_differ_from_twin_only_where_documented(O):
    """Half-away vs half-even rounding: x/s = 2.5 exactly -> 3 (kernel) vs 2 (twin)."""
    l = np.zeros((1, 16), np.uint16)
    r = np.zeros((16, 32), np.uint16)
    x = np.full((1, 1, 32), O.f32_to_bf16(np.float32(2.5))[()], np.uint16)
    s = np.full((1, 32), O.f32_to_bf16(np.float32(1.0))[()], np.uint16)
    _, _, c_kernel = O.rc_encode(l, r, x, s, 8, 100.0, flags=0)
    _, _, c_twin = O.rc_encode(l, r, x, s, 8, 100.0, flags=O.RC_HALF_EVEN)
    assert (c_kernel == 3).all() and (c_twin == 2).all()


# ---------------------------------------------------------------- pinned: consumer formulas
@pytest.mark.parametrize("name,fn", [("silu", "silu_bwd"), ("silu2", "silu_bwd"), ("gelu", "gelu_bwd"),
                                     ("mul", "mul")])
def test_consumer_formula_matches_reference_twin(O, golden, name, fn):
    """The reference twin evaluated in fp32 and rounded once to bf16 equals the
    oracle (binary32 formula, one rounding) except at rounding ties of libm."""
    out = getattr(O, fn)(golden["elt_x"], golden["elt_g"])
    ref = O.f32_to_bf16(golden[name + "_f32"])
    assert (out == ref).mean() > 0.999
    assert O.rel_fro(out, golden[name + "_f32"]) < 4e-3  # bf16 output rounding only


def test_softmax_formula_matches_reference_twin(O, golden):
    out = O.softmax_bwd(golden["smax_y"], golden["smax_g"])
    assert (out == O.f32_to_bf16(golden["smax_f32"])).mean() > 0.999


# ---------------------------------------------------------------- channel-group restatement
def _lowrank_x(T, H, r_sig=16, seed=0, n_out=4):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((T, r_sig)) @ rng.standard_normal((r_sig, H))) / r_sig
    x += 0.05 * rng.standard_normal((T, H))
    ch = np.sort(rng.choice(H, n_out, replace=False))
    x[:, ch] *= 30
    return x.astype(np.float32), ch.astype(np.int32)


def _basis(x, r):
    _, _, vt = np.linalg.svd(x.astype(np.float64), full_matrices=False)
    return vt[:r].T.astype(np.float32)


@pytest.mark.parametrize("bits,group,wht", [(4, 64, False), (8, 128, False), (4, 128, True), (4, 32, False)])
def test_cg_roundtrip_error_is_quantisation_error(O, bits, group, wht):
    x, ch = _lowrank_x(64, 256)
    xb = O.f32_to_bf16(x)
    prep = O.basis_prepare(_basis(O.bf16_to_f32(xb), 16))
    enc = O.encode(xb, prep, ch, bits, group, wht)
    xh = O.decode(enc["codes"], enc["scales"], enc["lowrank"], prep[1], enc["outliers"], ch, 256,
                  bits, group, wht)
    err = O.rel_fro(xh, xb)
    assert err < (0.05 if bits == 4 else 0.01)
    # outlier channels are reproduced verbatim
    assert np.array_equal(xh[:, ch], xb[:, ch])
    # codes within the symmetric range
    u = O.unpack_codes(enc["codes"], bits).astype(int) - (1 << (bits - 1))
    assert np.abs(u).max() <= (1 << (bits - 1)) - 1


def test_cg_wht_inverse_is_identity(O):
    """Encode with WHT at 8 bits, no low rank, no outliers: the decode applies
    the inverse rotation, so the error is the 8-bit quantisation error only."""
    rng = np.random.default_rng(1)
    xb = O.f32_to_bf16(rng.standard_normal((8, 256)).astype(np.float32))
    enc = O.encode(xb, (np.zeros((0, 256), np.uint16), np.zeros((256, 0), np.uint16)), None, 8, 128, True)
    xh = O.decode(enc["codes"], enc["scales"], None, None, None, None, 256, 8, 128, True)
    assert O.rel_fro(xh, xb) < 8e-3


def test_cg_lowrank_term_is_the_rounded_exact_sum(O):
    """The low-rank term is L . V^T summed exactly and rounded once: decoding an
    all-zero residual gives bf16(float32(exact L . V^T)), and the residual of
    the encode is x - that term."""
    x, ch = _lowrank_x(16, 128, seed=3)
    xb = O.f32_to_bf16(x)
    Vt, Vb = O.basis_prepare(_basis(O.bf16_to_f32(xb), 16))
    L = O.project(xb, Vt)
    exact = (L.astype(np.float64) @ O.bf16_to_f32(Vb).astype(np.float64).T).astype(np.float32)
    assert np.array_equal(O.lowrank(L, Vb), exact)
    zero_codes = np.full((16, 64), 0x88, np.uint8)
    xh = O.decode(zero_codes, np.zeros((16, 2), np.float32), L, Vb, None, None, 128, 4, 64, False)
    assert np.array_equal(xh, O.f32_to_bf16(exact))
    # the projection is the exact product sum rounded once
    Lx = (O.bf16_to_f32(xb).astype(np.float64) @ O.bf16_to_f32(Vt).astype(np.float64).T).astype(np.float32)
    assert np.array_equal(L, Lx)


def test_topk_channel_selection(O):
    score = np.array([1, 5, 3, 5, 0, 7], np.float32)
    assert list(O.topk_channels(score, 3)) == [1, 3, 5]  # tie 5/5 -> both; ascending
    assert list(O.topk_channels(score, 2)) == [1, 5]     # tie broken to the lower index


def test_fp32_activation_config1_shape(O):
    """Config 1 is CPU-only: fp32 X, int8 group 128, r = 16, k = 8 fp32 outliers."""
    x, ch = _lowrank_x(128, 512, r_sig=32, n_out=8)
    prep = O.basis_prepare(_basis(x, 16))
    enc = O.encode(x, prep, ch, 8, 128, False)
    assert enc["outliers"].dtype == np.float32
    xh = O.decode(enc["codes"], enc["scales"], enc["lowrank"], prep[1], enc["outliers"], ch, 512,
                  8, 128, False, x_f32=True)
    assert np.array_equal(xh[:, ch], x[:, ch])
    assert O.rel_fro(xh, x) < 5e-3


def test_lora_formula_pinned_by_the_reference_fixture(golden):
    """The float64 statement of low_rank_system_profile_backward.py:14-18 used
    by the GPU LoRA tests reproduces the reference's own outputs (fixture made
    by running the reference's compute_lora_gradient)."""
    import torch

    t = {k: torch.from_numpy(golden["lora_" + k]).double() for k in ("x", "dy", "w", "a", "b", "dx", "da", "db")}
    dy, x, w, a, b = t["dy"], t["x"], t["w"], t["a"], t["b"]
    ref = (dy @ (w.mT + b.mT @ a.mT), x.mT @ (dy @ b.mT), (x @ a).mT @ dy)
    for r_, name in zip(ref, ("dx", "da", "db")):
        assert (r_ - t[name]).norm() / t[name].norm() < 1e-5, name
