"""Drop-in for the reference module ``gelu_backward``: the same public names, backed
by libactcomp through :mod:`actcomp.reference_api` (put this directory on
``sys.path`` ahead of the reference's own files)."""
from actcomp.reference_api import torch_gelu_backward, triton_gelu_backward  # noqa: F401

__all__ = ['torch_gelu_backward', 'triton_gelu_backward']
