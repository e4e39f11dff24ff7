"""CPU tests of the C ABI: the library loads without a GPU, exports every
entry point include/actcomp.h declares, its ctypes structs match the C layout,
and argument validation happens on the host (no device needed)."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "actcomp.h")


def declared_functions():
    src = open(HEADER).read()
    return re.findall(r"^\s*(?:const char \*|int|size_t)\s*(actcomp_\w+)\(", src, re.M)


def test_library_exports_every_declared_symbol():
    from actcomp import _lib

    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing
    assert set(names) == set(_lib.SIGNATURES), "ctypes signature table out of sync with the header"


def test_abi_version_and_strerror():
    from actcomp import _lib

    lib = _lib.load()
    assert lib.actcomp_abi_version() == _lib.ABI_VERSION == 2
    assert lib.actcomp_strerror(0) == b"ok"
    assert lib.actcomp_strerror(-6) == b"workspace missing or too small"


def test_struct_layout_matches_c():
    """Compile a probe against the header with gcc and compare sizeof/offsetof."""
    from actcomp import _lib

    structs = {"actcomp_cg_desc": _lib.CgDesc, "actcomp_rc_args": _lib.RcArgs, "actcomp_ew_args": _lib.EwArgs,
               "actcomp_gemm_args": _lib.GemmArgs}
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void){"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname}.{fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0;}")
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(c, "w").write("\n".join(lines))
        subprocess.run(["gcc", "-std=c11", c, "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split("\n")
    got = dict(l.split() for l in out if l)
    for cname, py in structs.items():
        assert int(got[cname]) == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert int(got[f"{cname}.{fname}"]) == getattr(py, fname).offset, f"{cname}.{fname}"


def _desc(**kw):
    from actcomp import _lib

    d = _lib.CgDesc()
    d.tokens, d.channels, d.bits, d.group, d.batch = 16, 256, 4, 64, 1
    d.codes, d.scales = 0x1000, 0x2000
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("kw,status", [
    (dict(), -1),                                   # x is NULL
    (dict(bits=3), -2), (dict(group=48), -2), (dict(rank=24), -2), (dict(n_outlier=65), -2),
    (dict(channels=200), -1),                       # not a multiple of the group
    (dict(wht=1, channels=320), -2),                # rotation needs whole 128 blocks
    (dict(codes=0), -1), (dict(codes=0x1001), -3),  # misaligned
    (dict(rank=16), -1),                            # rank without low-rank buffers
])
def test_cg_encode_validation_without_gpu(kw, status):
    from actcomp import _lib

    lib = _lib.load()
    d = _desc(**kw)
    assert lib.actcomp_cg_encode(ctypes.byref(d), None, 256, None) == status


def test_misaligned_activation_is_rejected():
    from actcomp import _lib

    lib = _lib.load()
    d = _desc()
    assert lib.actcomp_cg_encode(ctypes.byref(d), 0x3002, 256, None) == -3
    assert lib.actcomp_cg_encode(ctypes.byref(d), 0x3000, 100, None) == -1  # ld < H


def test_gemm_validation_without_gpu():
    from actcomp import _lib

    lib = _lib.load()
    g = _lib.GemmArgs()
    assert lib.actcomp_gemm(ctypes.byref(g), None) == -1
    g.M = g.N = g.K = 64
    g.batch = 1
    g.A, g.B, g.C = 0x1000, 0x2000, 0x3000
    g.lda, g.ldb, g.ldc = 60, 64, 64  # row stride not 16-byte aligned for TMA
    g.a_kmajor = 1
    assert lib.actcomp_gemm(ctypes.byref(g), None) == -3
    g.lda = 64
    g.c_dtype = 7
    assert lib.actcomp_gemm(ctypes.byref(g), None) == -1


def test_rc_validation_without_gpu():
    from actcomp import _lib

    lib = _lib.load()
    a = _lib.RcArgs()
    assert lib.actcomp_rc_encode(ctypes.byref(a), None) == -1
    a.B, a.M, a.N, a.K, a.bits, a.s_rows = 1, 4, 48, 16, 4, 1
    a.l, a.r, a.s, a.q, a.x, a.o = 1, 2, 3, 4, 5, 6
    assert lib.actcomp_rc_encode(ctypes.byref(a), None) == -2  # 4-bit packing needs N % 32 == 0
    a.bits = 3
    assert lib.actcomp_rc_encode(ctypes.byref(a), None) == -2


def test_dw_workspace_size():
    from actcomp import _lib

    lib = _lib.load()
    d = _desc(tokens=16384, channels=4096)
    assert lib.actcomp_cg_dw_workspace(ctypes.byref(d), 11008) >= 16384 * 4096 * 2


def test_selftest_rejects_bad_poll_counts():
    """Host-side validation of the failure-detection self-test (no launch)."""
    from actcomp import _lib

    lib = _lib.load()
    assert lib.actcomp_selftest_bounded_wait(0, 0, None) == _lib.ACT_E_INVALID
    assert lib.actcomp_selftest_bounded_wait((1 << 24) + 1, 0, None) == _lib.ACT_E_INVALID


def test_fused_dw_validation_and_workspace_without_gpu():
    """actcomp_cg_dw_fused refuses what it does not cover before launching
    anything, and its workspace holds only the low-rank and outlier terms."""
    from actcomp import _lib

    lib = _lib.load()
    T, H, N, r, k = 16384, 4096, 11008, 32, 16
    d = _desc(tokens=T, channels=H, rank=r, n_outlier=k, lowrank=0x4000, basis=0x5000, outliers=0x6000,
              outlier_idx=0x7000, basis_t=0x8000)
    need = lib.actcomp_cg_dw_fused_workspace(ctypes.byref(d), N)
    up = lambda b: (b + 255) // 256 * 256  # noqa: E731
    assert need == up(T * 3 * r * 2) + up(3 * r * N * 4) + up(3 * r * N * 2) + up(H * 3 * r * 2) + up(k * N * 4)
    assert need < T * H * 2 // 10  # against the reconstruction's 134 MB
    call = lambda dd, ws, wsb: lib.actcomp_cg_dw_fused(  # noqa: E731
        ctypes.byref(dd), 0x9000, N, N, 0xA000, 0, N, ws, wsb, None)
    assert call(d, None, 0) == _lib.ACT_E_WORKSPACE                     # no workspace
    assert call(d, 0x10000, need - 1) == _lib.ACT_E_WORKSPACE           # too small
    assert call(_desc(tokens=T, channels=H, wht=1), None, 0) == _lib.ACT_E_UNSUPPORTED   # rotated
    assert call(_desc(tokens=T, channels=H, n_outlier=4, outliers=0x6000, outlier_idx=0x7000), None, 0) == \
        _lib.ACT_E_UNSUPPORTED                                          # outliers not a multiple of 8
    assert call(_desc(tokens=32, channels=H), None, 0) == _lib.ACT_E_UNSUPPORTED         # fewer than 64 tokens
    assert lib.actcomp_cg_dw_fused(ctypes.byref(d), 0x9000, N, N, 0xA000, 2, N, 0x10000, need, None) == \
        _lib.ACT_E_INVALID                                              # output dtype
