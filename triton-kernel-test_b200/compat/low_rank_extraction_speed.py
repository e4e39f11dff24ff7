"""Drop-in for the reference module ``low_rank_extraction_speed``: the same public names, backed
by libactcomp through :mod:`actcomp.reference_api` (put this directory on
``sys.path`` ahead of the reference's own files)."""
from actcomp.reference_api import low_rank_addition, torch_low_rank_addition, torch_low_rank_addition_fuse_compression_quantization  # noqa: F401

__all__ = ['low_rank_addition', 'torch_low_rank_addition', 'torch_low_rank_addition_fuse_compression_quantization']
