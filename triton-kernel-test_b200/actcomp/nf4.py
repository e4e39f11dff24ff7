"""NF4 base-weight dequantisation on the GPU.

The reference's backward driver keeps the LoRA base weight frozen in NF4
(``bnb.nn.LinearNF4``, low_rank_system_profile_backward.py:31) and, every
step, dequantises it with bitsandbytes' ``F.dequantize_4bit(w.t(), state,
quant_type='nf4').to(torch.bfloat16)`` (:58) before ``compute_lora_gradient``.
:func:`dequantize_4bit` takes the same arguments and returns the same bf16
tensor, computed by one kernel of libactcomp.so (``actcomp_nf4_dequant``).

The state object is read by attribute, so a bitsandbytes ``QuantState`` works
as it is; :class:`QuantState` holds the same fields for callers without
bitsandbytes: ``absmax`` (float32 per block, or uint8 per block when the
statistics are nested), ``shape``, ``code`` (16 floats), ``blocksize``,
``quant_type``, ``offset`` and ``state2`` (the nested statistics' own state:
``absmax`` float32 per ``blocksize`` entries, ``code`` 256 floats).
"""
from __future__ import annotations

from dataclasses import dataclass
from statistics import NormalDist
from typing import Optional

import torch

from . import _lib
from .core import _need_cuda, _ptr, _stream

BF16 = torch.bfloat16

#: quantile offset of the NF4 construction (QLoRA): 1 - (1/32 + 1/30) / 2
NF4_OFFSET = 1.0 - 0.5 * (1.0 / 32.0 + 1.0 / 30.0)


def nf4_code(device=None) -> torch.Tensor:
    """The 16 NF4 values (float32, ascending) by the data type's definition:
    N(0, 1) quantiles at probabilities evenly spaced from NF4_OFFSET towards 1/2
    (8 for the positive half, 7 for the negative half), an exact zero, scaled so
    that the extremes are -1 and +1."""
    nd = NormalDist()
    steps = lambda k: [NF4_OFFSET + (0.5 - NF4_OFFSET) * i / k for i in range(k)]  # noqa: E731
    pos = [nd.inv_cdf(p) for p in steps(8)]
    neg = [-nd.inv_cdf(p) for p in steps(7)]
    v = sorted(pos + [0.0] + neg)
    m = max(abs(x) for x in v)
    return torch.tensor([x / m for x in v], dtype=torch.float32, device=device)


@dataclass
class QuantState:
    """The fields of a 4-bit quantisation state that the dequantisation reads
    (the names of bitsandbytes' QuantState)."""
    absmax: torch.Tensor
    shape: torch.Size
    code: torch.Tensor
    blocksize: int = 64
    quant_type: str = "nf4"
    dtype: torch.dtype = torch.float32
    offset: Optional[torch.Tensor] = None
    state2: Optional["QuantState"] = None


def dequantize_4bit(A: torch.Tensor, quant_state, quant_type: str = "nf4",
                    out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Dequantise a packed NF4 weight to bf16.

    A: the packed indices (uint8, ceil(n/2) bytes, value 2j in the high nibble
    of byte j), of shape (n/2, 1) as the weight parameter stores them or its
    transpose (1, n/2); as bitsandbytes does, the result for a transposed A is
    the transpose of the (quant_state.shape) weight.  Returns bf16 (the
    reference converts the result to bf16 straight away).  Only NF4 data is
    supported; the code table is quant_state.code."""
    if quant_type != "nf4" or getattr(quant_state, "quant_type", "nf4") != "nf4":
        raise ValueError("actcomp.nf4.dequantize_4bit supports quant_type='nf4' only")
    shape = torch.Size(quant_state.shape)
    n = shape.numel()
    dev = A.device
    _need_cuda(A)
    packed = A.reshape(-1)
    if packed.dtype != torch.uint8:
        packed = packed.view(torch.uint8)
    if packed.numel() < (n + 1) // 2:
        raise ValueError(f"packed weight holds {packed.numel()} bytes, {(n + 1) // 2} needed for shape {tuple(shape)}")
    packed = packed.contiguous()
    code = quant_state.code.to(device=dev, dtype=torch.float32).contiguous()
    if code.numel() != 16:
        raise ValueError("the NF4 code table has 16 entries")
    st2 = getattr(quant_state, "state2", None)
    absmax = quant_state.absmax
    nb = -(-n // int(quant_state.blocksize))
    if absmax.numel() < nb:
        raise ValueError(f"{absmax.numel()} block statistics for {nb} blocks")
    am = am_q = am2 = code2 = off = None
    bs2 = 0
    if st2 is not None:
        am_q = absmax.reshape(-1).to(device=dev, dtype=torch.uint8).contiguous()
        am2 = st2.absmax.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
        code2 = st2.code.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
        bs2 = int(st2.blocksize)
        if code2.numel() != 256 or am2.numel() < -(-nb // bs2):
            raise ValueError("nested statistics: 256 code values and one absmax per blocksize2 blocks needed")
        off = quant_state.offset
        off = (torch.zeros(1, dtype=torch.float32, device=dev) if off is None
               else torch.as_tensor(off, dtype=torch.float32, device=dev).reshape(1).contiguous())
    else:
        am = absmax.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    if out is None:
        out = torch.empty(shape, dtype=BF16, device=dev)
    elif out.dtype != BF16 or out.numel() != n or not out.is_contiguous() or out.device != dev:
        raise ValueError("out must be a contiguous bf16 tensor of quant_state.shape on A's device")
    _lib.call("actcomp_nf4_dequant", _ptr(packed), n, int(quant_state.blocksize), _ptr(code), _ptr(am),
              _ptr(am_q), _ptr(am2), _ptr(code2), bs2, _ptr(off), _ptr(out), _stream(out))
    return out.t() if A.dim() == 2 and A.shape[0] == 1 and out.dim() == 2 else out
