"""Offload of compressed activations to pinned host memory and back.

The reference moves its compressed buffers with synchronous pageable copies:
``o_cpu, q_cpu = o.cpu(), q.cpu()`` after the forward encode
(offload_forward.py:55) and ``o_cpu.cuda(), q_cpu.cuda()`` before the backward
decode (offload_backward.py:63).  Here the same movement runs asynchronously:

* ``Offloader.offload(c)`` starts device->host copies of every per-activation
  buffer of ``c`` (codes, scales, low-rank codes and scale, outlier values) into
  pinned host buffers, on a side stream that first waits for the work already
  queued on the caller's stream (the encode that produced ``c``).  It returns a
  ``HostActivation`` at once.
* ``Offloader.reload(h)`` allocates device buffers and starts the host->device
  copies on the side stream; the returned ``Compressed`` must not be read
  before ``h.wait()`` (or ``Offloader.wait(h)``) has made the caller's stream
  wait for them.  ``decode`` and the fused consumers called after that see the
  reloaded bytes.

The copies are ``cudaMemcpyAsync`` calls issued by ``actcomp_cg_copy`` in
libactcomp (one per buffer); pinned buffers are pooled per layout so a training
loop does not re-pin memory every step.  The basis and the outlier channel
indices are shared inputs and stay on the device.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch

from . import core


def _layout_key(c: core.Compressed) -> tuple:
    return (c.tokens, c.channels, c.bits, c.group, c.rank, c.n_outlier, c.batch)


@dataclass
class HostActivation:
    """A compressed activation whose per-activation buffers live in pinned host
    memory (filled once ``done`` has completed)."""

    meta: core.Compressed  # layout, basis and outlier indices; device buffers dropped
    host: core.Compressed  # the same layout over pinned host buffers
    done: torch.cuda.Event = field(repr=False)

    def ready(self) -> bool:
        return self.done.query()

    def wait(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Make ``stream`` (default: the current stream) wait for the last copy."""
        (stream or torch.cuda.current_stream()).wait_event(self.done)

    def nbytes(self) -> int:
        return self.host.nbytes()


class Offloader:
    """Asynchronous offload / reload of ``Compressed`` activations on one device."""

    def __init__(self, device: Optional[torch.device] = None, stream: Optional[torch.cuda.Stream] = None,
                 pool: bool = True):
        self.device = torch.device(device) if device is not None else torch.device("cuda",
                                                                                   torch.cuda.current_device())
        self.stream = stream or torch.cuda.Stream(self.device)
        self._pool: dict[tuple, list[dict]] = {} if pool else None

    # ------------------------------------------------------------------ host buffers
    def _host_buffers(self, c: core.Compressed) -> dict:
        key = _layout_key(c)
        if self._pool is not None and self._pool.get(key):
            return self._pool[key].pop()
        return core.empty_like_layout(c.tokens, c.channels, bits=c.bits, group=c.group, rank=c.rank,
                                      n_outlier=c.n_outlier, batch=c.batch, device="cpu", pin_memory=True)

    def release(self, h: HostActivation) -> None:
        """Return the pinned buffers of ``h`` to the pool (after its reload completed)."""
        if self._pool is None:
            return
        h.done.synchronize()
        bufs = {k: getattr(h.host, k) for k in ("codes", "scales", "lowrank", "outliers")}
        self._pool.setdefault(_layout_key(h.host), []).append(bufs)

    # ------------------------------------------------------------------ device -> host
    def offload(self, c: core.Compressed) -> HostActivation:
        if c.device.type != "cuda":
            raise ValueError("offload expects a Compressed on a CUDA device")
        host = c.with_buffers(**self._host_buffers(c))
        producer = torch.cuda.current_stream(c.device)
        self.stream.wait_stream(producer)
        with torch.cuda.stream(self.stream):
            core.copy_into(host, c, self.stream)
            done = torch.cuda.Event()
            done.record(self.stream)
        # the device buffers must outlive the copies that read them
        for t in c.buffers().values():
            t.record_stream(self.stream)
        # the layout without the device buffers (so they can be freed)
        empty = lambda t: None if t is None else torch.empty(0, dtype=t.dtype)
        meta = c.with_buffers(codes=empty(c.codes), scales=empty(c.scales), lowrank=empty(c.lowrank),
                              outliers=empty(c.outliers))
        return HostActivation(meta=meta, host=host, done=done)

    # ------------------------------------------------------------------ host -> device
    def reload(self, h: HostActivation) -> core.Compressed:
        m = h.meta
        bufs = core.empty_like_layout(m.tokens, m.channels, bits=m.bits, group=m.group, rank=m.rank,
                                      n_outlier=m.n_outlier, batch=m.batch, device=self.device)
        dev = m.with_buffers(**bufs)
        self.stream.wait_event(h.done)  # the offload copies into the host buffers have finished
        self.stream.wait_stream(torch.cuda.current_stream(self.device))  # the buffers' allocation is ordered
        with torch.cuda.stream(self.stream):
            core.copy_into(dev, h.host, self.stream)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        for t in dev.buffers().values():
            t.record_stream(self.stream)
        h.done = ev
        return dev

    def wait(self, h: HostActivation, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Make ``stream`` (default: the device's current stream) wait for the last copy of ``h``."""
        h.wait(stream or torch.cuda.current_stream(self.device))
