"""Compatibility module with the reference's name (kernels_v2_1.py):
``sparse_query_dense_key_attention`` backed by the sm_100a library."""

from hspmn_b200.kernels import sparse_query_dense_key_attention  # noqa: F401
