"""The bounds-checked build (libactcomp_bc.so, -DACT_BOUNDS_CHECK): every
global store of the tensor-core kernels checks its index against the buffer's
extent and records a bit in the device error word instead of trapping.  Ragged
shapes run through it in a child process; the error word must stay clear and
every output must equal the product library's bit for bit."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _run(lib, out):
    env = dict(os.environ)
    if lib:
        env["ACTCOMP_LIBRARY"] = lib
    else:
        env.pop("ACTCOMP_LIBRARY", None)
    subprocess.run([sys.executable, os.path.join(HERE, "bounds_worker.py"), out], check=True, env=env, timeout=600)
    return dict(np.load(out))


def test_bounds_checked_build_is_clean_and_identical(tmp_path):
    from actcomp import _lib, build

    bc = build.LIB_BC
    assert os.path.exists(bc), "libactcomp_bc.so is built by __graft_entry__.build()"
    checked = _run(bc, str(tmp_path / "bc.npz"))
    plain = _run(None, str(tmp_path / "plain.npz"))
    assert checked["word"][0] == 0 and checked["status"][0] == _lib.ACT_OK
    assert plain["word"][0] == 0
    for key in plain:
        if key in ("word", "status"):
            continue
        assert np.array_equal(checked[key], plain[key]), key
