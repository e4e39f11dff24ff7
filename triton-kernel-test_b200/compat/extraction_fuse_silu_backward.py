"""Drop-in for the reference module ``extraction_fuse_silu_backward``: the same public names, backed
by libactcomp through :mod:`actcomp.reference_api` (put this directory on
``sys.path`` ahead of the reference's own files)."""
from actcomp.reference_api import torch_silu_backward, triton_silu_backward, triton_silu_backward_fuse_extraction, triton_silu_backward_add_extraction  # noqa: F401

__all__ = ['torch_silu_backward', 'triton_silu_backward', 'triton_silu_backward_fuse_extraction', 'triton_silu_backward_add_extraction']
