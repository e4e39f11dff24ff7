"""Drop-in for the reference module ``extraction_fuse_hadamard``: the same public names, backed
by libactcomp through :mod:`actcomp.reference_api` (put this directory on
``sys.path`` ahead of the reference's own files)."""
from actcomp.reference_api import torch_hadamard, triton_hadamard, triton_hadamard_fuse_extraction, triton_hadamard_add_extraction  # noqa: F401

__all__ = ['torch_hadamard', 'triton_hadamard', 'triton_hadamard_fuse_extraction', 'triton_hadamard_add_extraction']
