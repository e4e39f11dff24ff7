"""GPU tests of the asynchronous offload of compressed activations (the
reference's ``o.cpu()`` / ``o_cpu.cuda()`` round trip, offload_forward.py:55 and
offload_backward.py:63): every byte survives device -> pinned host -> device,
and the reloaded activation decodes to exactly the same values."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _compressed(T=512, H=1024, r=32, k=16, bits=4, group=64, seed=0):
    import actcomp
    from actcomp import synthetic

    x, _ = synthetic.lowrank_activation(T, H, seed=seed, device="cuda")
    basis = actcomp.Basis.fit(x, r) if r else None
    idx = actcomp.select_outlier_channels(x, k) if k else None
    return actcomp.encode(x, basis, idx, bits=bits, group=group)


@pytest.mark.parametrize("kw", [dict(), dict(r=0, k=0, bits=8, group=128), dict(T=130, H=640, r=16, k=3)])
def test_offload_reload_roundtrip_is_exact(kw):
    import actcomp

    c = _compressed(**kw)
    ref = actcomp.decode(c)
    off = actcomp.Offloader()
    h = off.offload(c)
    h.done.synchronize()
    assert h.host.codes.device.type == "cpu" and h.host.codes.is_pinned()
    for name, t in c.buffers().items():
        assert torch.equal(getattr(h.host, name), t.cpu()), name
    assert h.nbytes() == c.nbytes()
    del c  # the device buffers may go; the host copy is complete
    c2 = off.reload(h)
    h.wait()
    out = actcomp.decode(c2)
    assert torch.equal(out, ref)


def test_offload_overlaps_and_pools_buffers():
    import actcomp

    cs = [_compressed(seed=s) for s in range(3)]
    refs = [actcomp.decode(c) for c in cs]
    off = actcomp.Offloader()
    hs = [off.offload(c) for c in cs]  # queued back to back on the side stream
    for h in hs:
        h.wait()
    back = [off.reload(h) for h in hs]
    for h in hs:
        off.wait(h)
    for c2, ref in zip(back, refs):
        assert torch.equal(actcomp.decode(c2), ref)
    pinned = hs[0].host.codes.data_ptr()
    for h in hs:
        off.release(h)
    h2 = off.offload(cs[0])  # reuses a pooled pinned buffer set
    h2.done.synchronize()
    assert h2.host.codes.data_ptr() in {h.host.codes.data_ptr() for h in hs}
    assert torch.equal(h2.host.codes, cs[0].codes.cpu())
    assert pinned in {h.host.codes.data_ptr() for h in hs}
