"""Config 1 of the benchmark (TEST INFRASTRUCTURE ONLY): the CPU reference case.

X = A(4096 x 32) . B(32 x 4096) + 0.1 N(0,1), A and B ~ N(0,1)/sqrt(32), 8
random channels x50, seed 0, float32; V_r = the top-16 right singular vectors
of X; 8 outlier channels kept in float32; residual quantised to int8 with
per-token group-128 absmax scales.  Encodes and decodes it with the C oracle
(the format the kernels implement: V rounded to bf16) and with the PyTorch
north-star checker (oracle/northstar.py), and reports codes and errors:

    python oracle/report_config1.py        # prints one JSON object

tests/test_northstar.py asserts the same figures.
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import northstar as NS  # noqa: E402
import oracle as O  # noqa: E402


def _synthetic():
    path = os.path.join(os.path.dirname(HERE), "triton-kernel-test_b200", "actcomp", "synthetic.py")
    spec = importlib.util.spec_from_file_location("_c1_synthetic", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def config1(T: int = 4096, H: int = 4096):
    S = _synthetic()
    x, ch = S.lowrank_activation(T, H, signal_rank=32, noise=0.1, n_outlier=8, outlier_scale=50.0, seed=0,
                                 dtype=torch.float32)
    V = torch.linalg.svd(x.double(), full_matrices=False).Vh[:16].T.float().contiguous()
    return x, ch.numpy().astype(np.int32), V


def report(T: int = 4096, H: int = 4096) -> dict:
    x, idx, V = config1(T, H)
    bits, group = 8, 128
    # the C oracle (the kernels' format): float32 X, V rounded to bf16
    Vt, Vb = O.basis_prepare(V.numpy())
    enc = O.encode(x.numpy(), (Vt, Vb), idx, bits, group, False)
    xh = O.decode(enc["codes"], enc["scales"], enc["lowrank"], Vb, enc["outliers"], idx, H, bits, group, False,
                  x_f32=True)
    codes = O.unpack_codes(enc["codes"], bits).astype(np.int32) - (1 << (bits - 1))
    # the north-star checker with the identical (bf16-rounded) basis
    Vbf = torch.from_numpy(O.bf16_to_f32(Vb))
    ns = NS.encode(x, Vbf, idx, bits, group)
    xh_ns = NS.decode(ns, Vbf, idx, group)
    diff = codes != ns["codes"].numpy()
    tie = NS.tie_distance(ns["pre"]).numpy()
    # ... and with the float32 SVD basis (no bf16 rounding anywhere)
    ns32 = NS.encode(x, V, idx, bits, group)
    xh_ns32 = NS.decode(ns32, V, idx, group)
    xt = torch.from_numpy(xh)
    return {
        "config": f"config 1: {T} x {H} float32, r=16 (SVD), k=8 outliers x50, int8 group 128",
        "codes": int(codes.size),
        "codes_differing_from_checker": int(diff.sum()),
        "max_tie_distance_at_differences": float(tie[diff].max()) if diff.any() else 0.0,
        "code_histogram_abs": {str(v): int((np.abs(codes) == v).sum()) for v in (0, 1, 2, 4, 8, 16, 32, 64, 127)},
        "rel_err_oracle_vs_x": NS.rel_fro(xt, x),
        "rel_err_checker_vs_x": NS.rel_fro(xh_ns, x),
        "rel_fro_oracle_vs_checker": NS.rel_fro(xt, xh_ns),
        "rel_fro_oracle_vs_checker_fp32_basis": NS.rel_fro(xt, xh_ns32),
        "lowrank_max_rel_diff": float((torch.from_numpy(enc["lowrank"]) - ns["lowrank"]).abs().max()
                                      / ns["lowrank"].abs().max()),
        "outliers_verbatim": bool(np.array_equal(xh[:, idx], x.numpy()[:, idx])),
    }


if __name__ == "__main__":
    print(json.dumps(report()))
