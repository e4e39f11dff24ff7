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


def test_lora_gradient_matches_reference(golden):
    from actcomp import reference_api as R

    t = {k: torch.from_numpy(golden["lora_" + k]).cuda() for k in ("x", "dy", "w", "a", "b")}
    dx, da, db = R.compute_lora_gradient(t["dy"], t["x"], t["w"], t["a"], t["b"])
    for got, name in ((dx, "dx"), (da, "da"), (db, "db")):
        ref = torch.from_numpy(golden["lora_" + name]).cuda()
        assert (got.float() - ref).norm() / ref.norm() < 2e-2, name  # bf16 operands vs the fp32 reference


def test_error_stats():
    import actcomp

    a = torch.randn(1000, device="cuda").to(torch.bfloat16)
    b = a.clone()
    b[::10] += 1
    s = actcomp.error_stats(a, b).cpu().numpy()
    e = (a.double() - b.double()).cpu().numpy()
    assert np.isclose(s[0], (e ** 2).sum()) and np.isclose(s[1], (b.double() ** 2).sum().item())
    assert np.isclose(s[2], np.abs(e).max()) and s[3] == (a != b).sum().item()
