"""GPU parity of the reference-compatible kernels: against the reference's own
PyTorch functions (golden fixtures) and against the oracle's restatement of
the Triton kernels, bit for bit."""
import numpy as np
import pytest
import torch

from conftest import bits, to_bf16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qb", [1, 2, 4, 8])
@pytest.mark.parametrize("N", [32, 64])
def test_decode_matches_reference_twin(golden, qb, N):
    from actcomp import refcompat

    k = f"dec_b{qb}_n{N}"
    g = lambda n: to_bf16(golden[k + n])
    q = torch.from_numpy(golden[k + "_q"]).cuda()
    x = refcompat.decode(g("_l"), g("_r"), q, g("_o"), g("_s"), qb, flags=refcompat.TWIN)
    assert np.array_equal(bits(x), golden[k + "_x"])


@pytest.mark.parametrize("qb", [8, 4, 2])
def test_end_to_end_matches_naive(golden, qb):
    from actcomp import reference_api as R

    k = f"naive_b{qb}"
    g = lambda n: to_bf16(golden[k + n])
    xh = R.naive_quantization_dequantization(g("_l"), g("_r"), g("_x"), g("_s"), qb, float(golden[k + "_outlier"]))
    assert np.array_equal(bits(xh), golden[k + "_xhat"])


@pytest.mark.parametrize("qb", [8, 4, 1])
def test_encode_codes_match_reference_twin(O, golden, qb):
    from actcomp import refcompat

    k = f"enc_b{qb}"
    g = lambda n: to_bf16(golden[k + n])
    o, q = refcompat.encode(g("_l"), g("_r"), g("_x"), g("_s"), qb, float(golden[k + "_outlier"]),
                            flags=refcompat.TWIN)
    _, q_ref, _ = O.rc_encode(golden[k + "_l"], golden[k + "_r"], golden[k + "_x"], golden[k + "_s"], qb,
                              float(golden[k + "_outlier"]), flags=O.RC_TWIN)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(O.bf16_to_f32(bits(o)), O.bf16_to_f32(golden[k + "_o"]))


@pytest.mark.parametrize("qb", [1, 2, 4, 8])
@pytest.mark.parametrize("B,M,N,K", [(2, 33, 64, 16), (1, 16, 96, 32), (3, 8, 32, 5),
                                     # the tiled kernels (whole 256-column tiles): ragged row tiles,
                                     # several column tiles, the largest rank
                                     (2, 70, 256, 16), (1, 131, 512, 32), (2, 9, 768, 64)])
def test_kernel_semantics_match_oracle(O, qb, B, M, N, K):
    """Default (Triton-kernel) semantics on non-dyadic data: batch-0 scale,
    half-away rounding, 32-column block packing -- bit for bit."""
    from actcomp import reference_api as R

    rng = np.random.default_rng(qb * 100 + M)
    l = O.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32) * 0.3)
    r = O.f32_to_bf16(rng.standard_normal((K, N)).astype(np.float32) * 0.3)
    x = O.f32_to_bf16(rng.standard_normal((B, M, N)).astype(np.float32) * 2)
    s = O.f32_to_bf16((rng.random((B, N)) * 0.3 + 0.05).astype(np.float32))
    o_ref, q_ref, _ = O.rc_encode(l, r, x, s, qb, 2.5, flags=0)
    o_sp, q = R.low_rank_addition_fuse_compression_quantization(to_bf16(l), to_bf16(r), to_bf16(x), to_bf16(s),
                                                                quantize_bit=qb, outlier=2.5)
    assert o_sp.is_sparse
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(O.bf16_to_f32(bits(o_sp.to_dense())), O.bf16_to_f32(o_ref))
    xh = R.low_rank_addition_fuse_decompression_dequantization(to_bf16(l), to_bf16(r), q, o_sp, to_bf16(s),
                                                               quantize_bit=qb)
    assert np.array_equal(bits(xh), O.rc_decode(l, r, q_ref, o_ref, s, qb, flags=0))


@pytest.mark.parametrize("flags", [1, 2, 4, 16, 1 | 2 | 4 | 16])
@pytest.mark.parametrize("qb", [1, 2, 4, 8])
def test_tiled_kernels_honour_every_flag(O, qb, flags):
    """The twin-semantics flags on the tiled path (N a multiple of 256), bit for
    bit against the oracle; decode also through the fused consumers."""
    from actcomp import _lib, refcompat

    rng = np.random.default_rng(qb * 1000 + flags)
    B, M, N, K = 2, 37, 256, 16
    l = O.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32) * 0.3)
    r = O.f32_to_bf16(rng.standard_normal((K, N)).astype(np.float32) * 0.3)
    x = O.f32_to_bf16(rng.standard_normal((B, M, N)).astype(np.float32) * 2)
    s = O.f32_to_bf16((rng.random((B, N)) * 0.3 + 0.05).astype(np.float32))
    o_ref, q_ref, _ = O.rc_encode(l, r, x, s, qb, 2.5, flags=flags)
    o, q = refcompat.encode(to_bf16(l), to_bf16(r), to_bf16(x), to_bf16(s), qb, 2.5, flags)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(bits(o), o_ref)
    xh = refcompat.decode(to_bf16(l), to_bf16(r), q, o, to_bf16(s), qb, flags)
    ref = O.rc_decode(l, r, q_ref, o_ref, s, qb, flags=flags)
    assert np.array_equal(bits(xh), ref)
    y = O.f32_to_bf16(rng.standard_normal((B, M, N)).astype(np.float32))
    got = refcompat.decode(to_bf16(l), to_bf16(r), q, o, to_bf16(s), qb, flags, op=_lib.ACT_OP_MUL, y=to_bf16(y))
    assert np.array_equal(bits(got), bits(to_bf16(ref) * to_bf16(y)))


def test_fused_consumers_match_unfused(O):
    from actcomp import reference_api as R

    rng = np.random.default_rng(7)
    B, M, N, K = 2, 32, 64, 16
    l = to_bf16(O.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32) * 0.2))
    r = to_bf16(O.f32_to_bf16(rng.standard_normal((K, N)).astype(np.float32) * 0.2))
    q = torch.from_numpy(rng.integers(0, 256, (B, M, N // 4), dtype=np.uint8)).cuda()
    s = to_bf16(O.f32_to_bf16((rng.random((B, N)) + 0.5).astype(np.float32)))
    b = to_bf16(O.f32_to_bf16(rng.standard_normal((B, M, N)).astype(np.float32)))
    fused = R.triton_silu_backward_fuse_extraction(l, r, q, s, b, quantize_bit=2)
    unfused = R.triton_silu_backward_add_extraction(l, r, q, s, b, quantize_bit=2)
    assert torch.equal(fused, unfused)
    fused = R.triton_hadamard_fuse_extraction(l, r, q, s, b, quantize_bit=2)
    assert torch.equal(fused, R.triton_hadamard_add_extraction(l, r, q, s, b, quantize_bit=2))
    xh = R.low_rank_addition_fuse_decompression_dequantization(l, r, q, torch.zeros(B, M, N, dtype=torch.bfloat16,
                                                                                      device="cuda"), s, 2)
    md = R.triton_matmul_decompress(q, l, r, s, b.transpose(1, 2).contiguous()[:, :, :32].contiguous(), 2)
    ref = torch.bmm(xh.float(), b.transpose(1, 2)[:, :, :32].float())
    assert (md.float() - ref).norm() / ref.norm() < 5e-3


def test_low_rank_addition(O):
    from actcomp import reference_api as R

    rng = np.random.default_rng(3)
    l = O.f32_to_bf16(rng.standard_normal((40, 16)).astype(np.float32))
    r = O.f32_to_bf16(rng.standard_normal((16, 72)).astype(np.float32))
    x = O.f32_to_bf16(rng.standard_normal((2, 40, 72)).astype(np.float32))
    out = bits(R.low_rank_addition(to_bf16(l), to_bf16(r), to_bf16(x)))
    d = np.zeros((40, 72), np.float32)
    lf, rf = O.bf16_to_f32(l), O.bf16_to_f32(r)
    for kk in range(16):  # sequential binary32 FMAs: exact in binary64 then rounded once
        d = (lf[:, kk:kk + 1].astype(np.float64) * rf[kk:kk + 1, :] + d).astype(np.float32)
    ref = O.f32_to_bf16(O.bf16_to_f32(x) + d)
    assert (out == ref).mean() > 0.999
