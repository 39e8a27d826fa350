"""``decode_kernels.testing``: the seeded paged-cache fixtures
(DecodeKernels ``decode_kernels/testing.py:23-77``; same draw order, so the
same seed gives the same cache)."""

from decodekernels_b200.testing import PagedKV, make_paged_kv, make_queries

__all__ = ["PagedKV", "make_paged_kv", "make_queries"]
