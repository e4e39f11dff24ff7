"""NF4 base-weight dequantisation (low_rank_system_profile_backward.py:31,58).

bitsandbytes, which the reference calls for this step, is neither vendored nor
installed, and no reference test holds NF4 values: the oracle restates the
published algorithm (oracle.py, "NF4 base weight") and these tests pin the
kernel to it bit for bit ("parity unpinned" against bitsandbytes itself).
CPU tests cover the restatement and the entry point's argument checks; the
``gpu`` tests compare the kernel with the oracle and run the reference's
backward step on a dequantised weight."""
import ctypes

import numpy as np
import pytest
import torch


# ---------------------------------------------------------------- oracle (CPU)


def test_nf4_code_is_the_normal_float_data_type(O):
    c = O.nf4_code().astype(np.float64)
    assert c.shape == (16,) and np.all(np.diff(c) > 0)
    assert c[0] == -1.0 and c[-1] == 1.0 and c[7] == 0.0  # 7 negative values, zero, 8 positive
    # the positive half: N(0,1) quantiles at evenly spaced probabilities, scaled by the largest
    from statistics import NormalDist

    nd = NormalDist()
    top = nd.inv_cdf(O.NF4_OFFSET)
    for i, p in enumerate(np.linspace(O.NF4_OFFSET, 0.5, 9)[:-1]):
        assert abs(c[15 - i] - nd.inv_cdf(p) / top) < 1e-7
    # the package computes the same float32 table
    from actcomp import nf4

    assert np.array_equal(nf4.nf4_code().numpy(), O.nf4_code())


@pytest.mark.parametrize("blocksize", [64, 256])
def test_nf4_round_trip_error_is_bounded(O, blocksize):
    rng = np.random.default_rng(1)
    w = rng.standard_normal((96, 200)).astype(np.float32)
    code = O.nf4_code()
    packed, absmax = O.nf4_quantize(w, blocksize, code)
    d = O.bf16_to_f32(O.nf4_dequant(packed, w.size, blocksize, code, absmax=absmax)).astype(np.float64)
    am = np.repeat(absmax.astype(np.float64), blocksize)[: w.size]
    half_gap = np.diff(code.astype(np.float64)).max() / 2
    assert np.all(np.abs(d - w.ravel()) <= am * (half_gap + 2 ** -8) + 1e-30)


def test_nf4_nested_statistics_stay_close(O):
    rng = np.random.default_rng(2)
    w = rng.standard_normal(64 * 1024).astype(np.float32)
    code = O.nf4_code()
    packed, absmax = O.nf4_quantize(w, 64, code)
    code2 = np.linspace(-1, 1, 256).astype(np.float32)
    q, a2, off = O.nested_stats(absmax, 256, code2)
    plain = O.bf16_to_f32(O.nf4_dequant(packed, w.size, 64, code, absmax=absmax))
    nest = O.bf16_to_f32(O.nf4_dequant(packed, w.size, 64, code, absmax_q=q, absmax2=a2, code2=code2,
                                       blocksize2=256, offset=off))
    assert np.abs(nest - plain).max() <= 0.02 * np.abs(plain).max()


def test_nf4_entry_point_validates_without_gpu():
    from actcomp import _lib

    lib = _lib.load()
    fake = ctypes.c_void_p(1 << 20)  # aligned, never dereferenced: validation fails first
    call = lambda n, bs, am, amq, out=fake: lib.actcomp_nf4_dequant(  # noqa: E731
        fake, n, bs, fake, am, amq, fake, fake, 256, fake, out, None)
    assert call(0, 64, fake, None) == _lib.ACT_OK                 # nothing to do
    assert call(-1, 64, fake, None) == _lib.ACT_E_INVALID
    assert call(64, 48, fake, None) == _lib.ACT_E_INVALID         # not a power of two
    assert call(64, 64, fake, fake) == _lib.ACT_E_INVALID         # both kinds of statistics
    assert call(64, 64, None, None) == _lib.ACT_E_INVALID         # neither
    assert call(64, 64, fake, None, ctypes.c_void_p((1 << 20) + 8)) == _lib.ACT_E_ALIGN


# ---------------------------------------------------------------- kernel (GPU)


def _case(O, n, blocksize, nested, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(n) * rng.uniform(0.01, 3.0)).astype(np.float32)
    code = O.nf4_code()
    packed, absmax = O.nf4_quantize(w, blocksize, code)
    if not nested:
        return packed, code, dict(absmax=absmax)
    code2 = np.sort(rng.uniform(-1, 1, 256)).astype(np.float32)
    code2[0], code2[-1] = -1.0, 1.0
    q, a2, off = O.nested_stats(absmax, 256, code2)
    return packed, code, dict(absmax_q=q, absmax2=a2, code2=code2, blocksize2=256, offset=off)


def _gpu(lib, packed, n, blocksize, code, st):
    from actcomp import _lib

    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    dp, dc = t(packed), t(code)
    keep = [dp, dc]
    if "absmax" in st:
        am, amq, a2, c2, off, bs2 = t(st["absmax"]), None, None, None, None, 0
    else:
        am = None
        amq, a2, c2 = t(st["absmax_q"]), t(st["absmax2"]), t(st["code2"])
        off, bs2 = t(np.array([st["offset"]], np.float32)), st["blocksize2"]
    keep += [x for x in (am, amq, a2, c2, off) if x is not None]
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    p = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())  # noqa: E731
    st_ = lib.actcomp_nf4_dequant(p(dp), n, blocksize, p(dc), p(am), p(amq), p(a2), p(c2), bs2, p(off),
                                  p(out), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st_ == _lib.ACT_OK, st_
    torch.cuda.synchronize()
    return out.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.gpu
@pytest.mark.parametrize("n,blocksize", [(64 * 1000, 64), (4096 * 37, 128), (1 << 20, 4096), (8 * 977 + 5, 64),
                                         (13, 8), (1, 64)])
@pytest.mark.parametrize("nested", [False, True])
def test_nf4_kernel_matches_oracle(O, n, blocksize, nested):
    from actcomp import _lib

    packed, code, st = _case(O, n, blocksize, nested, seed=n + blocksize)
    got = _gpu(_lib.load(), packed, n, blocksize, code, st)
    ref = O.nf4_dequant(packed, n, blocksize, code, **st)
    assert np.array_equal(got, ref), int((got != ref).sum())


@pytest.mark.gpu
def test_dequantize_4bit_mirrors_the_state_api(O):
    """The bitsandbytes-style call of the reference: a state object with
    absmax / code / blocksize / offset / state2, the packed weight passed
    transposed, the result the transposed (out, in) weight in bf16."""
    from actcomp import nf4

    d_out, d_in = 384, 256
    n = d_out * d_in
    packed, code, st = _case(O, n, 64, True, seed=11)
    ref = torch.from_numpy(O.bf16_to_f32(O.nf4_dequant(packed, n, 64, code, **st)).reshape(d_out, d_in))
    state2 = nf4.QuantState(absmax=torch.from_numpy(st["absmax2"]).cuda(), shape=torch.Size([st["absmax2"].size]),
                            code=torch.from_numpy(st["code2"]).cuda(), blocksize=256)
    state = nf4.QuantState(absmax=torch.from_numpy(st["absmax_q"]).cuda(), shape=torch.Size([d_out, d_in]),
                           code=torch.from_numpy(code).cuda(), blocksize=64,
                           offset=torch.tensor(float(st["offset"])).cuda(), state2=state2)
    weight = torch.from_numpy(packed).cuda().reshape(-1, 1)   # how a 4-bit weight parameter stores it
    w = nf4.dequantize_4bit(weight.t(), state, quant_type="nf4").to(torch.bfloat16)
    assert w.shape == (d_in, d_out) and w.dtype == torch.bfloat16
    assert torch.equal(w.float().cpu(), ref.t())
    w2 = nf4.dequantize_4bit(weight, state)                  # untransposed: the (out, in) weight
    assert w2.shape == (d_out, d_in) and torch.equal(w2.float().cpu(), ref)
    with pytest.raises(ValueError):
        nf4.dequantize_4bit(weight, state, quant_type="fp4")


@pytest.mark.gpu
def test_lora_backward_step_on_an_nf4_base_weight(O):
    """low_rank_system_profile_backward.py:58-62: dequantise the frozen NF4
    weight, then compute_lora_gradient with it; dx against the formula on the
    dequantised weight (no copy of the transposed view is needed)."""
    from actcomp import nf4
    from actcomp import reference_api as R

    S, d_in, d_out, r = 512, 512, 1024, 16
    n = d_out * d_in
    packed, code, st = _case(O, n, 64, False, seed=12)
    state = nf4.QuantState(absmax=torch.from_numpy(st["absmax"]).cuda(), shape=torch.Size([d_out, d_in]),
                           code=torch.from_numpy(code).cuda(), blocksize=64)
    w = R.dequantize_4bit(torch.from_numpy(packed).cuda().reshape(-1, 1).t(), state).to(torch.bfloat16)
    g = torch.Generator().manual_seed(13)
    bf = lambda t: t.to(torch.bfloat16)  # noqa: E731
    dy, x = bf(torch.randn(S, d_out, generator=g)), bf(torch.randn(S, d_in, generator=g))
    a, b = bf(torch.randn(d_in, r, generator=g) * 0.1), bf(torch.randn(r, d_out, generator=g) * 0.1)
    dx, da, db = R.compute_lora_gradient(dy.cuda(), x.cuda(), w, a.cuda(), b.cuda())
    wd, dyd, xd, ad, bd = (t.double() for t in (w.cpu(), dy, x, a, b))
    rdx = dyd @ (wd.mT + bd.mT @ ad.mT)
    e = (dx.double().cpu() - rdx.to(torch.bfloat16).double()).norm() / rdx.norm()
    assert e < 2e-4, float(e)
    rda = xd.mT @ (dyd @ bd.mT)
    assert (da.double().cpu() - rda).norm() / rda.norm() < 1e-5
