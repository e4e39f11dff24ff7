"""Child process of tests/test_bounds_gpu.py: runs ragged shapes through the
library named by ACTCOMP_LIBRARY and saves every output plus the device error
word to the .npz path given as argv[1]."""
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "triton-kernel-test_b200"))


def main(out_path):
    import actcomp
    from actcomp import _lib, refcompat, synthetic

    lib = _lib.load()
    s = torch.cuda.current_stream().cuda_stream
    assert lib.actcomp_clear_device_error(s) == _lib.ACT_OK
    res = {}
    g = torch.Generator(device="cuda").manual_seed(5)
    # channel-group format: ragged token counts, several widths, with and
    # without the rotation, both quantiser widths, outliers
    cases = [(37, 1024, 32, 5, 4, 64, False), (129, 512, 16, 0, 8, 32, False), (300, 1024, 16, 3, 4, 128, True),
             (1100, 2048, 32, 16, 4, 64, False), (70, 384, 16, 4, 8, 128, False)]
    for i, (T, H, r, k, b, gr, wht) in enumerate(cases):
        x, _ = synthetic.lowrank_activation(T, H, n_outlier=max(k, 1), seed=i, device="cuda")
        basis = actcomp.Basis.fit(x, r)
        idx = actcomp.select_outlier_channels(x, k) if k else None
        c = actcomp.encode(x, basis, idx, bits=b, group=gr, wht=wht)
        res[f"codes{i}"] = c.codes.cpu().numpy()
        res[f"scales{i}"] = c.scales.cpu().numpy()
        res[f"xh{i}"] = actcomp.decode(c).view(torch.int16).cpu().numpy()
        dy = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
        res[f"silu{i}"] = actcomp.silu_backward(c, dy).view(torch.int16).cpu().numpy()
        n = 136
        dyw = torch.randn(T, n, device="cuda", generator=g).to(torch.bfloat16)
        res[f"dw{i}"] = actcomp.weight_grad(c, dyw, torch.float32).cpu().numpy()
    # the reference's packed format, per-element and tiled kernels
    for i, (B, M, N, K, qb) in enumerate([(2, 37, 256, 16, 1), (1, 70, 512, 32, 2), (2, 9, 96, 16, 4)]):
        l = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16) * 0.3
        r_ = torch.randn(K, N, device="cuda", generator=g).to(torch.bfloat16) * 0.3
        xx = torch.randn(B, M, N, device="cuda", generator=g).to(torch.bfloat16) * 2
        sc = torch.rand(B, N, device="cuda", generator=g).to(torch.bfloat16) * 0.3 + 0.05
        o, q = refcompat.encode(l, r_, xx, sc, qb, 2.5, 0)
        res[f"rc_q{i}"] = q.cpu().numpy()
        res[f"rc_o{i}"] = o.view(torch.int16).cpu().numpy()
        res[f"rc_x{i}"] = refcompat.decode(l, r_, q, o, sc, qb, 0).view(torch.int16).cpu().numpy()
    import ctypes

    word = ctypes.c_uint32(0)
    st = lib.actcomp_last_device_error(s, ctypes.byref(word))
    res["status"] = np.array([st])
    res["word"] = np.array([word.value])
    np.savez(out_path, **res)


if __name__ == "__main__":
    main(sys.argv[1])
