"""Drop-in for the reference module ``low_rank_kernel_accuracy_test``: the same public names, backed
by libactcomp through :mod:`actcomp.reference_api` (put this directory on
``sys.path`` ahead of the reference's own files)."""
from actcomp.reference_api import naive_quantization_dequantization  # noqa: F401

__all__ = ['naive_quantization_dequantization']
