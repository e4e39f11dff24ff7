"""actcomp -- B200-native (sm_100a) activation compression.

Compute runs only in libactcomp.so (hand-written CUDA for sm_100a, C ABI in
include/actcomp.h); this package allocates tensors, builds descriptors and
launches through ctypes on the current CUDA stream.

Main entry points:
  Basis, Compressed, encode, decode, mul, silu_backward, gelu_backward,
  softmax_backward, weight_grad, select_outlier_channels   (channel-group format)
  refcompat.encode / refcompat.decode                       (the reference's format)
  reference_api.*                                           (the reference's function names)
  offload.Offloader                                         (pinned-host offload on a side stream)
  nf4.dequantize_4bit                                       (NF4 base weight -> bf16)
  dist.shard_rows / dist.reduce_error_stats                 (token sharding, error-stat all-reduce)
"""
from . import _lib
from .core import (Basis, Compressed, copy_into, decode, encode, error_stats, gelu_backward, gemm, mul,
                   select_outlier_channels, silu_backward, softmax_backward, weight_grad)

from . import dist, nf4, offload
from .offload import HostActivation, Offloader

_lib.load()  # fail loudly at import if the CUDA library is missing

__all__ = ["Basis", "Compressed", "encode", "decode", "mul", "silu_backward", "gelu_backward", "softmax_backward",
           "weight_grad", "select_outlier_channels", "gemm", "error_stats", "copy_into", "Offloader",
           "HostActivation", "dist", "nf4", "offload"]
