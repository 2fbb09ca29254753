"""Attention over the K8/V4 paged cache: batch planning, the backend, the eager reference."""
from .backend import K8V4AttentionBackend, K8V4AttentionImpl, K8V4Metadata, K8V4MetadataBuilder  # noqa: F401
from .plan import query_segments, require_decoder, uniform_packed_q_len  # noqa: F401
