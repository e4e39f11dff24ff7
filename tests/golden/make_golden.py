"""Generate the golden fixtures in tests/golden/ from the reference's own code.

Run in a container where the reference checkout is available (it is not on
the GPU box; the fixtures it writes are committed instead):

    python tests/golden/make_golden.py /path/to/Triton-Kernel-Test

Sources of truth, all executed on the CPU with PyTorch:

* ``torch_low_rank_addition_fuse_decompression_dequantization``
  (low_rank_extraction_fuse_decompression_dequantization.py:155-165), imported.
* ``naive_quantization_dequantization`` (low_rank_kernel_accuracy_test.py:6-16),
  imported.
* ``torch_low_rank_addition_fuse_compression_quantization`` from
  low_rank_extraction_speed.py:146-156 (unpacked int32 codes), imported.  The
  packing twin in low_rank_extraction_fuse_compression_quantization.py:153-171
  calls ``.cuda()`` and cannot run here.
* The PyTorch twins of the consumer kernels (silu_backward.py:6,
  extraction_fuse_silu_backward.py:10, gelu_backward.py:14,
  softmax_backward.py:6, extraction_fuse_hadamard.py:5,
  extraction_outlier_channel.py:5-14, low_rank_system_profile_backward.py:14).
  Those modules launch CUDA work at import time, so only the named function
  definitions are compiled out of each file with ``ast`` and executed.

Inputs are seeded.  The low-rank factors l, r are small dyadic rationals so
that ``l @ r`` is exact in binary32 whatever the summation order, which makes
the reference's bf16 results deterministic and comparable bit for bit.
"""
from __future__ import annotations

import ast
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def load_functions(path: str, names: list[str]) -> dict:
    tree = ast.parse(open(path).read(), filename=path)
    nodes = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    found = {n.name for n in nodes}
    missing = set(names) - found
    if missing:
        raise RuntimeError(f"{path}: functions not found: {missing}")
    ns = {"torch": torch, "F": torch.nn.functional}
    exec(compile(ast.Module(body=nodes, type_ignores=[]), path, "exec"), ns)
    return {n: ns[n] for n in names}


def dyadic(g, shape, lo=-8, hi=8, den=8):
    return (torch.randint(lo, hi + 1, shape, generator=g).float() / den).to(torch.bfloat16)


def main(ref: str) -> None:
    sys.path.insert(0, ref)
    import low_rank_extraction_fuse_decompression_dequantization as dec
    import low_rank_kernel_accuracy_test as acc
    import low_rank_extraction_speed as spd

    g = torch.Generator().manual_seed(0)
    out = {}

    # ---- decode twin, several bit widths; N=32 (single 32-column block) and N=64
    for qb in (1, 2, 4, 8):
        for N in (32, 64):
            B, M, K = 2, 8, 16
            epp = 8 // qb
            l = dyadic(g, (M, K))
            r = dyadic(g, (K, N))
            q = torch.randint(0, 256, (B, M, N // epp), generator=g, dtype=torch.int32).to(torch.uint8)
            o = torch.randn(B, M, N, generator=g).to(torch.bfloat16)
            o = o * (o.abs() > 1.5)
            s = (torch.rand(B, N, generator=g) + 0.5).to(torch.bfloat16)
            x = dec.torch_low_rank_addition_fuse_decompression_dequantization(l, r, q, o.to_sparse(), s, quantize_bit=qb)
            key = f"dec_b{qb}_n{N}"
            out.update({f"{key}_l": bits(l), f"{key}_r": bits(r), f"{key}_q": q.numpy(), f"{key}_o": bits(o),
                        f"{key}_s": bits(s), f"{key}_x": bits(x.to(torch.bfloat16))})

    # ---- naive end-to-end (twin encode + twin decode), int8 and int4/int2
    for qb, outlier in ((8, 5.0), (4, 3.0), (2, 2.5)):
        B, M, N, K = 2, 16, 64, 16
        l = dyadic(g, (M, K), den=16)
        r = dyadic(g, (K, N), den=16)
        x = (torch.randn(B, M, N, generator=g) * 2).to(torch.bfloat16)
        s = (torch.rand(1, N, generator=g) * 0.05 + 0.02).to(torch.bfloat16)
        xh = acc.naive_quantization_dequantization(l, r, x.clone(), s, quantize_bit=qb, outlier=outlier)
        key = f"naive_b{qb}"
        out.update({f"{key}_l": bits(l), f"{key}_r": bits(r), f"{key}_x": bits(x), f"{key}_s": bits(s),
                    f"{key}_xhat": bits(xh.to(torch.bfloat16)), f"{key}_outlier": np.float32(outlier)})

    # ---- twin encode codes (unpacked, signed) and dense outliers
    for qb, outlier in ((8, 4.0), (4, 2.0), (1, 3.0)):
        B, M, N, K = 2, 16, 64, 16
        l = dyadic(g, (M, K), den=16)
        r = dyadic(g, (K, N), den=16)
        x = (torch.randn(B, M, N, generator=g) * 2).to(torch.bfloat16)
        s = (torch.rand(1, N, generator=g) * 0.2 + 0.1).to(torch.bfloat16)
        o, q = spd.torch_low_rank_addition_fuse_compression_quantization(l, r, x.clone(), s, quantize_bit=qb,
                                                                          outlier=outlier)
        key = f"enc_b{qb}"
        out.update({f"{key}_l": bits(l), f"{key}_r": bits(r), f"{key}_x": bits(x), f"{key}_s": bits(s),
                    f"{key}_o": bits(o.to(torch.bfloat16)), f"{key}_q": q.numpy().astype(np.int32),
                    f"{key}_outlier": np.float32(outlier)})

    # ---- consumer twins (functions compiled out of their modules)
    silu = load_functions(os.path.join(ref, "silu_backward.py"), ["torch_silu_backward"])["torch_silu_backward"]
    silu2 = load_functions(os.path.join(ref, "extraction_fuse_silu_backward.py"),
                           ["torch_silu_backward"])["torch_silu_backward"]
    gelu = load_functions(os.path.join(ref, "gelu_backward.py"), ["torch_gelu_backward"])["torch_gelu_backward"]
    smax = load_functions(os.path.join(ref, "softmax_backward.py"),
                          ["torch_softmax_backward"])["torch_softmax_backward"]
    had = load_functions(os.path.join(ref, "extraction_fuse_hadamard.py"), ["torch_hadamard"])["torch_hadamard"]
    ext = load_functions(os.path.join(ref, "extraction_outlier_channel.py"),
                         ["torch_extract_unstructured", "torch_extract_channel"])
    lora = load_functions(os.path.join(ref, "low_rank_system_profile_backward.py"),
                          ["compute_lora_gradient"])["compute_lora_gradient"]

    x = (torch.randn(2, 32, 96, generator=g) * 3).to(torch.bfloat16)
    gy = torch.randn(2, 32, 96, generator=g).to(torch.bfloat16)
    out.update({"elt_x": bits(x), "elt_g": bits(gy),
                "silu_f32": silu(x.float(), gy.float()).numpy(),
                "silu2_f32": silu2(x.float(), gy.float()).numpy(),
                "silu_bf16": bits(silu(x, gy)),
                "gelu_f32": gelu(x.float(), gy.float()).numpy(),
                "gelu_bf16": bits(gelu(x, gy)),
                "mul_f32": had(x.float(), gy.float()).numpy()})

    logits = torch.randn(2, 2, 48, 48, generator=g)
    y = torch.softmax(logits, dim=-1).to(torch.bfloat16)
    gs = torch.randn(2, 2, 48, 48, generator=g).to(torch.bfloat16)
    out.update({"smax_y": bits(y), "smax_g": bits(gs), "smax_f32": smax(y.float(), gs.float()).numpy()})

    a = torch.randn(2, 24, 40, generator=g).to(torch.bfloat16)
    thr = float(torch.kthvalue(a.flatten().float().abs(), int(a.numel() * 0.95)).values)
    o_sp, rest = ext["torch_extract_unstructured"](a.clone(), thr)
    cidx = torch.tensor([3, 7, 20])
    ch, rest_c = ext["torch_extract_channel"](a.clone(), cidx)
    out.update({"ext_a": bits(a), "ext_thr": np.float32(thr), "ext_outlier": bits(o_sp.to_dense()),
                "ext_rest": bits(rest), "ext_cidx": cidx.numpy().astype(np.int32), "ext_channel": bits(ch),
                "ext_rest_c": bits(rest_c)})

    # LoRA gradient consumer: dy (B,S,d2), x (B,S,d1), w (d2? see :15), a (d1,r), b (r,d2)
    d1, d2, S, rr = 32, 48, 16, 16
    xl = torch.randn(2, S, d1, generator=g)
    dyl = torch.randn(2, S, d2, generator=g)
    wl = torch.randn(d1, d2, generator=g) * 0.1   # (d1, d2): the reference passes weight.t() here
    al = torch.randn(d1, rr, generator=g) * 0.1
    bl = torch.randn(rr, d2, generator=g) * 0.1
    dx, da, db = lora(dyl, xl, wl, al, bl)
    out.update({"lora_x": xl.numpy(), "lora_dy": dyl.numpy(), "lora_w": wl.numpy(),
                "lora_a": al.numpy(), "lora_b": bl.numpy(), "lora_dx": dx.numpy(), "lora_da": da.numpy(),
                "lora_db": db.numpy()})

    path = os.path.join(HERE, "reference_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
