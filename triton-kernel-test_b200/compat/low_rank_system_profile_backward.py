"""Drop-in for the reference module ``low_rank_system_profile_backward``: the same public names, backed
by libactcomp through :mod:`actcomp.reference_api` (put this directory on
``sys.path`` ahead of the reference's own files)."""
from actcomp.reference_api import compute_lora, compute_lora_gradient  # noqa: F401

__all__ = ['compute_lora', 'compute_lora_gradient']
