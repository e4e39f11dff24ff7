"""Drop-in for the reference module ``extraction_fuse_matmul``: the same public names, backed
by libactcomp through :mod:`actcomp.reference_api` (put this directory on
``sys.path`` ahead of the reference's own files)."""
from actcomp.reference_api import torch_matmul, triton_batched_matmul, triton_split_k_matmul, triton_matmul_decompress, triton_matmul_add_extraction  # noqa: F401

__all__ = ['torch_matmul', 'triton_batched_matmul', 'triton_split_k_matmul', 'triton_matmul_decompress', 'triton_matmul_add_extraction']
