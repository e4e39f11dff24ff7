"""Drop-in for the reference module ``triton_matmul``: the same public names, backed
by libactcomp through :mod:`actcomp.reference_api` (put this directory on
``sys.path`` ahead of the reference's own files)."""
from actcomp.reference_api import leaky_relu, matmul  # noqa: F401

__all__ = ['leaky_relu', 'matmul']
