"""The compat/ directory mirrors the reference's module names: every public
function the reference's modules define (and its driver scripts import) is
importable from a module of the same name."""
import importlib
import os
import sys

import pytest

from conftest import PKG

REFERENCE_NAMES = {
    "low_rank_extraction_fuse_compression_quantization": ["low_rank_addition_fuse_compression_quantization",
                                                          "torch_low_rank_addition_fuse_compression_quantization"],
    "low_rank_extraction_fuse_decompression_dequantization": [
        "low_rank_addition_fuse_decompression_dequantization",
        "torch_low_rank_addition_fuse_decompression_dequantization"],
    "low_rank_extraction_speed": ["low_rank_addition", "torch_low_rank_addition"],
    "low_rank_kernel_accuracy_test": ["naive_quantization_dequantization"],
    "extraction_outlier_channel": ["torch_extract_unstructured", "torch_extract_channel"],
    "extraction_fuse_hadamard": ["torch_hadamard", "triton_hadamard", "triton_hadamard_fuse_extraction",
                                 "triton_hadamard_add_extraction"],
    "extraction_fuse_silu_backward": ["torch_silu_backward", "triton_silu_backward",
                                      "triton_silu_backward_fuse_extraction", "triton_silu_backward_add_extraction"],
    "extraction_fuse_matmul": ["torch_matmul", "triton_batched_matmul", "triton_split_k_matmul",
                               "triton_matmul_decompress", "triton_matmul_add_extraction"],
    "silu_backward": ["torch_silu_backward", "triton_silu_backward"],
    "gelu_backward": ["torch_gelu_backward", "triton_gelu_backward"],
    "softmax_backward": ["torch_softmax_backward", "triton_softmax_backward"],
    "triton_matmul": ["matmul", "leaky_relu"],
    "low_rank_system_profile_backward": ["compute_lora", "compute_lora_gradient"],
}


@pytest.mark.parametrize("module", sorted(REFERENCE_NAMES))
def test_compat_module_exports_reference_names(module):
    compat = os.path.join(PKG, "compat")
    sys.path.insert(0, compat)
    try:
        mod = importlib.import_module(module)
    finally:
        sys.path.remove(compat)
    for name in REFERENCE_NAMES[module]:
        assert callable(getattr(mod, name)), f"{module}.{name}"
