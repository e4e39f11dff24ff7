"""Multi-process (gloo, world size 2) tests of the token sharding and the
error-statistics reduction, on the CPU.

Each rank encodes and decodes its own shard of the token rows with the CPU
oracle (the same per-row arithmetic the GPU path has), computes the 4-entry
error statistics of its shard and reduces them; the reduced statistics must
equal those of the whole matrix encoded in one piece."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT  # noqa: F401  (puts the package and the oracle on sys.path)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(T=96, H=256, r=16, k=4, seed=3):
    import oracle as O

    rng = np.random.default_rng(seed)
    a = rng.standard_normal((T, 24)) @ rng.standard_normal((24, H)) / 5 + 0.05 * rng.standard_normal((T, H))
    a[:, rng.choice(H, k, replace=False)] *= 20
    xb = O.f32_to_bf16(a.astype(np.float32))
    _, _, vt = np.linalg.svd(O.bf16_to_f32(xb).astype(np.float64), full_matrices=False)
    V = vt[:r].T.astype(np.float32)
    idx = O.topk_channels(O.channel_absmax(xb), k)
    return xb, O.basis_prepare(V), idx


def _stats(O, xb, prep, idx, bits=4, group=64):
    e = O.encode(xb, prep, idx, bits, group, False)
    xh = O.decode(e["codes"], e["scales"], e["lowrank"], prep[1], e["outliers"], idx, xb.shape[1],
                  bits, group, False)
    a = O.bf16_to_f32(xh).astype(np.float64)
    b = O.bf16_to_f32(xb).astype(np.float64)
    d = a - b
    return np.array([(d * d).sum(), (b * b).sum(), np.abs(d).max(initial=0.0), float((a != b).sum())])


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    import oracle as O
    from actcomp import dist as adist

    O.build()
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        xb, prep, idx = _case()
        lo, hi = adist.shard_rows(xb.shape[0], world, rank)
        st = torch.from_numpy(_stats(O, xb[lo:hi], prep, idx))
        adist.reduce_error_stats(st)
        # a second reduction on data every rank knows, to pin the MAX entry
        probe = torch.tensor([rank + 1.0, 10.0 * (rank + 1), 0.5 * (rank + 1), float(rank)], dtype=torch.float64)
        adist.reduce_error_stats(probe)
        out.put((rank, lo, hi, st.numpy().copy(), probe.numpy().copy()))
    finally:
        dist.destroy_process_group()


def test_shard_rows_partition():
    from actcomp.dist import shard_rows

    for n in (0, 1, 7, 64, 16384, 16385):
        for world in (1, 2, 3, 8):
            spans = [shard_rows(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def test_reduce_error_stats_single_process_is_identity():
    from actcomp.dist import reduce_error_stats, relative_error

    s = torch.tensor([4.0, 16.0, 0.25, 3.0], dtype=torch.float64)
    assert torch.equal(reduce_error_stats(s.clone()), s)
    assert relative_error(s) == pytest.approx(0.5)


def test_gloo_world2_sharded_stats_match_whole_matrix(O):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, lo0, hi0, st0, pr0), (r1, lo1, hi1, st1, pr1) = res
    assert (lo0, hi0, lo1) == (0, 48, 48) and hi1 == 96
    xb, prep, idx = _case()
    whole = _stats(O, xb, prep, idx)
    for st in (st0, st1):
        np.testing.assert_allclose(st[[0, 1, 3]], whole[[0, 1, 3]], rtol=1e-12)
        assert st[2] == whole[2]
    for pr in (pr0, pr1):
        np.testing.assert_array_equal(pr, [3.0, 30.0, 1.0, 1.0])
