"""Drop-in for the reference module ``extraction_outlier_channel``: the same public names, backed
by libactcomp through :mod:`actcomp.reference_api` (put this directory on
``sys.path`` ahead of the reference's own files)."""
from actcomp.reference_api import torch_extract_unstructured, torch_extract_channel  # noqa: F401

__all__ = ['torch_extract_unstructured', 'torch_extract_channel']
