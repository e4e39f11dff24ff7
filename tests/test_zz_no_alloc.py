"""actcomp_cg_dw_static: the weight gradient without a caller workspace.

The decoded activation lives in a device array the library reserves
(ACTCOMP_DW_STATIC_SCRATCH_BYTES); the result must equal actcomp_cg_dw with a
workspace (the existing entry point) on the same inputs, call after call, and
activations whose decoded size exceeds the scratch are rejected before any
launch.  This file is collected last so it also runs after every other test."""
import ctypes

import pytest
import torch

SCRATCH_BYTES = 32 << 20  # ACTCOMP_DW_STATIC_SCRATCH_BYTES in include/actcomp.h


def _desc(tokens, channels):
    from actcomp import _lib

    d = _lib.CgDesc()
    d.tokens, d.channels, d.bits, d.group, d.batch = tokens, channels, 4, 64, 1
    return d


def test_rejects_activation_larger_than_the_scratch():
    """Host-side check: no device work, so it runs without a GPU."""
    from actcomp import _lib

    lib = _lib.load()
    d = _desc(8192, 4096)  # 64 MiB of decoded bf16 > 32 MiB
    assert lib.actcomp_cg_dw_workspace(ctypes.byref(d), 1024) > SCRATCH_BYTES
    st = lib.actcomp_cg_dw_static(ctypes.byref(d), None, 1024, 1024, None, 0, 1024, None)
    assert st == -6  # ACT_E_WORKSPACE
    assert lib.actcomp_strerror(st) == b"workspace missing or too small"
    d0 = _desc(0, 4096)
    assert lib.actcomp_cg_dw_static(ctypes.byref(d0), None, 1024, 1024, None, 0, 1024, None) == -1


@pytest.mark.gpu
@pytest.mark.parametrize("T,H,N,dtype", [(2048, 1024, 768, torch.float32), (4096, 4096, 512, torch.bfloat16)])
def test_static_scratch_matches_workspace_entry_point(T, H, N, dtype):
    import actcomp
    from actcomp import _lib, synthetic

    x, _ = synthetic.lowrank_activation(T, H, seed=5, device="cuda")
    c = actcomp.encode(x, actcomp.Basis.fit(x, 32), actcomp.select_outlier_channels(x, 16), bits=4, group=64)
    dy = synthetic.gradient((T, N), seed=6, device="cuda")
    ref = actcomp.weight_grad(c, dy, dtype)  # actcomp_cg_dw with a torch-allocated workspace
    lib = _lib.load()
    d = c.desc()
    assert lib.actcomp_cg_dw_workspace(ctypes.byref(d), N) <= SCRATCH_BYTES
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # two calls in a row reuse the same scratch
        dw = torch.full((H, N), float("nan"), dtype=dtype, device="cuda")
        st = lib.actcomp_cg_dw_static(ctypes.byref(d), dy.data_ptr(), N, dy.stride(0), dw.data_ptr(),
                                      0 if dtype == torch.float32 else 1, dw.stride(0), stream)
        assert st == 0, lib.actcomp_strerror(st)
        torch.cuda.synchronize()
        err = ((dw.float() - ref.float()).norm() / ref.float().norm()).item()
        assert err < 1e-6, err
