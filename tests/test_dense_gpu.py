"""GPU tests of the dense helpers and the tcgen05 GEMM."""
import numpy as np
import pytest
import torch

from conftest import bits, to_bf16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,fn", [("silu", "silu_bwd"), ("gelu", "gelu_bwd"), ("mul", "mul")])
def test_elementwise_vs_oracle_and_reference(O, golden, name, fn):
    from actcomp import reference_api as R

    x, g = to_bf16(golden["elt_x"]), to_bf16(golden["elt_g"])
    f = {"silu": R.triton_silu_backward, "gelu": R.triton_gelu_backward, "mul": R.triton_hadamard}[name]
    out = bits(f(x, g))
    ref = getattr(O, fn)(golden["elt_x"], golden["elt_g"])
    assert (out == ref).mean() > (0.9 if name == "gelu" else 0.999)
    assert O.rel_fro(out, ref) < 1e-3
    assert O.rel_fro(out, golden[name + "_f32"]) < 4e-3  # vs the reference twin in fp32


def test_elementwise_strided_inputs(O):
    from actcomp import reference_api as R

    x = torch.randn(3, 40, 96, dtype=torch.bfloat16, device="cuda")[:, ::2, :]
    g = torch.randn(3, 20, 96, dtype=torch.bfloat16, device="cuda")
    out = bits(R.triton_silu_backward(x, g))
    assert (out == O.silu_bwd(bits(x), bits(g))).mean() > 0.999


def test_softmax_backward_dense(O, golden):
    from actcomp import reference_api as R

    out = bits(R.triton_softmax_backward(to_bf16(golden["smax_y"]), to_bf16(golden["smax_g"])))
    assert O.rel_fro(out, O.softmax_bwd(golden["smax_y"], golden["smax_g"])) < 1e-3
    assert O.rel_fro(out, golden["smax_f32"]) < 4e-3


def test_softmax_backward_odd_row_length(O):
    from actcomp import reference_api as R

    y = torch.softmax(torch.randn(2, 2, 511, 511), -1).to(torch.bfloat16)  # softmax_backward.py:63 uses n = 511
    g = torch.randn_like(y)
    out = bits(R.triton_softmax_backward(y.cuda(), g.cuda()))
    assert O.rel_fro(out, O.softmax_bwd(bits(y), bits(g))) < 1e-3


def test_extract_unstructured_and_channel(golden):
    from actcomp import reference_api as R

    a = to_bf16(golden["ext_a"])
    o, rest = R.torch_extract_unstructured(a, float(golden["ext_thr"]))
    assert np.array_equal(bits(o.to_dense()), golden["ext_outlier"])
    assert np.array_equal(bits(rest), golden["ext_rest"])
    ch, rest_c = R.torch_extract_channel(a.clone(), torch.from_numpy(golden["ext_cidx"]))
    assert np.array_equal(bits(ch), golden["ext_channel"])
    assert np.array_equal(bits(rest_c), golden["ext_rest_c"])


def _ref(a, b):
    return a.float() @ b.float()


# (4000, 4864, 136): enough 256 x 256 tiles for the two-accumulator kernel,
# with a partial last M tile and a partial last K step
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 192), (200, 136, 72), (64, 48, 8), (1024, 1000, 520),
                                   (4000, 4864, 136)])
@pytest.mark.parametrize("layout", ["nn", "tn", "nt", "tt"])
def test_gemm_layouts(M, N, K, layout):
    import actcomp

    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    b = torch.randn(K, N, generator=g, device="cuda").to(torch.bfloat16)
    a_in = a if layout[0] == "n" else a.T.contiguous().T   # MN-major view
    b_in = b if layout[1] == "n" else b.T.contiguous().T   # K-major view
    c = actcomp.gemm(a_in, b_in, torch.float32)
    ref = _ref(a, b)
    assert (c - ref).norm() / ref.norm() < 1e-5


@pytest.mark.parametrize("dtype,out", [(torch.float16, torch.float16), (torch.bfloat16, torch.bfloat16),
                                       (torch.float16, torch.float32)])
def test_gemm_dtypes_and_activation(dtype, out):
    import actcomp

    a = torch.randn(256, 128, device="cuda").to(dtype)
    b = torch.randn(128, 384, device="cuda").to(dtype)
    c = actcomp.gemm(a, b, out, activation="leaky_relu")
    ref = torch.nn.functional.leaky_relu(_ref(a, b), 0.01)
    assert c.dtype == out
    assert (c.float() - ref).norm() / ref.norm() < 4e-3


def test_gemm_batched_and_reference_names():
    from actcomp import reference_api as R

    x = torch.randn(4, 256, 128, device="cuda", dtype=torch.bfloat16)
    a = torch.randn(4, 128, 32, device="cuda", dtype=torch.bfloat16)
    for f in (R.triton_batched_matmul, R.triton_split_k_matmul, R.torch_matmul):
        c = f(x, a)
        ref = torch.bmm(x.float(), a.float())
        assert (c.float() - ref).norm() / ref.norm() < 4e-3
    a2 = torch.randn(512, 512, device="cuda", dtype=torch.float16)
    b2 = torch.randn(512, 512, device="cuda", dtype=torch.float16)
    c = R.matmul(a2, b2)
    assert c.dtype == torch.float16
    torch.testing.assert_close(c, (a2.float() @ b2.float()).half(), atol=1e-2, rtol=1e-2)  # triton_matmul.py:232


def _lora_formula(dy, x, w, a, b):
    """low_rank_system_profile_backward.py:14-18 in float64."""
    dy, x, w, a, b = (t.double() for t in (dy, x, w, a, b))
    return dy @ (w.mT + b.mT @ a.mT), x.mT @ (dy @ b.mT), (x @ a).mT @ dy


def _bf(t):
    return t.to(torch.bfloat16).float()


def _check_lora(got, ref):
    """dx (bf16) against the float64 value rounded to bf16: equal but at
    rounding ties; da, db (float32) within float32 accumulation."""
    dx, da, db = got
    rdx, rda, rdb = ref
    e = (dx.double() - rdx.to(torch.bfloat16).double()).norm() / rdx.norm()
    assert e < 2e-4, f"dx {float(e):.2e}"
    for g_, r_, n in ((da, rda, "da"), (db, rdb, "db")):
        e = (g_.double() - r_).norm() / r_.norm()
        assert e < 1e-5, f"{n} {float(e):.2e}"


def test_lora_gradient_matches_reference(golden):
    """The reference's own outputs (fixture) pin the formula; the GPU result
    on the bf16 operands matches the formula on those operands."""
    from actcomp import reference_api as R

    t = {k: torch.from_numpy(golden["lora_" + k]) for k in ("x", "dy", "w", "a", "b")}
    ref = _lora_formula(t["dy"], t["x"], t["w"], t["a"], t["b"])
    for r_, name in zip(ref, ("dx", "da", "db")):
        g_ = torch.from_numpy(golden["lora_" + name]).double()
        assert (r_ - g_).norm() / g_.norm() < 1e-5, name  # the fixture is the reference's float32 run
    tb = {k: _bf(v) for k, v in t.items()}
    got = R.compute_lora_gradient(*(tb[k].cuda() for k in ("dy", "x", "w", "a", "b")))
    _check_lora([g_.cpu() for g_ in got], _lora_formula(tb["dy"], tb["x"], tb["w"], tb["a"], tb["b"]))


def test_lora_gradient_on_a_compressed_activation():
    """x saved compressed (the reference decompresses it before the backward,
    low_rank_system_profile_backward.py:60-62): da through the fused
    dequant-GEMM, x a from the reconstruction, against the formula on the
    decoded activation."""
    import actcomp
    from actcomp import reference_api as R
    from actcomp import synthetic

    S, d_in, d_out, r = 1024, 512, 768, 16
    x, _ = synthetic.lowrank_activation(S, d_in, n_outlier=8, seed=5, device="cuda")
    basis = actcomp.Basis.fit(x, 32)
    c = actcomp.encode(x, basis, actcomp.select_outlier_channels(x, 8), bits=4, group=64)
    g = torch.Generator().manual_seed(6)
    dy = _bf(torch.randn(S, d_out, generator=g))
    w = _bf(torch.randn(d_in, d_out, generator=g) * 0.05)
    a = _bf(torch.randn(d_in, r, generator=g) * 0.1)
    b = _bf(torch.randn(r, d_out, generator=g) * 0.1)
    got = R.compute_lora_gradient(dy.cuda(), c, w.cuda(), a.cuda(), b.cuda())
    xh = actcomp.decode(c).float().cpu()
    _check_lora([g_.cpu() for g_ in got], _lora_formula(dy, xh, w, a, b))


def test_gemm_second_segment():
    """C = A B + A2 B2 in one accumulator, both layouts of each operand."""
    import actcomp

    g = torch.Generator().manual_seed(8)
    M, N, K, K2 = 200, 136, 264, 48
    A, B = _bf(torch.randn(M, K, generator=g)), _bf(torch.randn(K, N, generator=g))
    A2, B2 = _bf(torch.randn(M, K2, generator=g)), _bf(torch.randn(K2, N, generator=g))
    ref = A.double() @ B.double() + A2.double() @ B2.double()
    bf = torch.bfloat16
    for a_t in (False, True):
        for b_t in (False, True):
            a_ = A.cuda().to(bf) if not a_t else A.cuda().to(bf).mT.contiguous().mT
            b_ = B.cuda().to(bf) if not b_t else B.cuda().to(bf).mT.contiguous().mT
            c = actcomp.gemm(a_, b_, torch.float32, "", A2.cuda().to(bf), B2.cuda().to(bf))
            e = (c.double().cpu() - ref).norm() / ref.norm()
            assert e < 1e-6, (a_t, b_t, float(e))


def test_error_stats():
    import actcomp

    a = torch.randn(1000, device="cuda").to(torch.bfloat16)
    b = a.clone()
    b[::10] += 1
    s = actcomp.error_stats(a, b).cpu().numpy()
    e = (a.double() - b.double()).cpu().numpy()
    assert np.isclose(s[0], (e ** 2).sum()) and np.isclose(s[1], (b.double() ** 2).sum().item())
    assert np.isclose(s[2], np.abs(e).max()) and s[3] == (a != b).sum().item()
