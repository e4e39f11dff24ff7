"""Modules named like the reference's files (low_rank_extraction_fuse_compression_quantization,
silu_backward, ...), each re-exporting the reference's public function names from
actcomp.reference_api.  Adding this directory to sys.path lets the reference's own
driver scripts import the B200 implementation unchanged."""
