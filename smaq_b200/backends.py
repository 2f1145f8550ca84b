"""Concrete attention backend (same name as smaq/backends.py:9-20)."""

from __future__ import annotations

from smaq_b200.core import AttentionBackend
from smaq_b200.score import compute_hybrid_attention


class TorchHybridAttentionBackend(AttentionBackend):
    """Kept for API compatibility: dispatches to the sm_100a hybrid decode kernel."""

    def compute(self, query, store, recent_k, recent_v, num_query_heads, scale=None):
        return compute_hybrid_attention(query=query, store=store, recent_k=recent_k, recent_v=recent_v,
                                        num_query_heads=num_query_heads, scale=scale)
