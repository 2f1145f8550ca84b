"""Hybrid decode attention over compressed history plus the exact recent window.

``compute_hybrid_attention`` keeps the signature and semantics of smaq/score.py:23-72 and runs
as one ``smaq_decode`` call: per query head ``h`` (kv head ``h // (Hq / Hkv)``), one softmax
over ``[history logits || recent logits]`` (fp32), history ignored below
``MIN_HISTORY_FOR_SMAQ`` tokens, each part's weighted value sum cast to the query dtype and the
two parts summed in that dtype.  The ``T`` query rows all attend to the same store, as in the
reference.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from smaq_b200 import ops
from smaq_b200._lib import SMAQ_KEYS_SCALAR
from smaq_b200.core import AttentionBackend
from smaq_b200.store import CompressedKVStore

MIN_HISTORY_FOR_SMAQ = 16


def _decode_call(query: torch.Tensor, store: CompressedKVStore, recent_k: Optional[torch.Tensor],
                 recent_v: Optional[torch.Tensor], num_query_heads: int, scale: Optional[float]):
    """The ``ops.decode`` arguments of one compute_hybrid_attention call (None: nothing to attend)."""
    ops._cuda(query, recent_k, recent_v)
    D = store.head_dim
    Hkv = store.num_kv_heads
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    T = query.shape[0]
    n = store.num_tokens
    has_hist = n >= MIN_HISTORY_FOR_SMAQ
    has_recent = recent_k is not None and recent_k.shape[0] > 0
    if not has_hist and not has_recent:
        return None
    dev = query.device
    q = query.reshape(T, num_query_heads, D)
    if store.capacity == 0:
        # nothing stored yet: a one-token dummy store keeps every pointer valid (never read)
        store._reserve(0, recent_k.dtype if recent_k is not None else query.dtype)
        store._reserve(1, store.dtype)
    view = store.kernel_view()
    bt = torch.zeros((T, 1), dtype=torch.int32, device=dev)
    hist = torch.full((T,), n, dtype=torch.int32, device=dev)
    kw = {}
    strat = store.key_strategy
    if store.key_format == SMAQ_KEYS_SCALAR:
        qz = strat.quantizer
        kw = dict(key_bits=strat.bits, E_inv=qz.E_inv, centroids=qz.centroids, key_norms=view["norms"])
    else:
        # an fp16-valued codebook selects the tensor-core block-VQ kernel (decode-layout rows)
        kw = dict(centroids=strat.quantizer.decoded_centroids, centroids_f16=strat.quantizer.fp16_codebook())
    if has_recent:
        W = recent_k.shape[0]
        rk = recent_k.reshape(1, W, Hkv, D).expand(T, W, Hkv, D)
        rv = recent_v.reshape(1, W, Hkv, D).expand(T, W, Hkv, D)
        rl = torch.full((T,), W, dtype=torch.int32, device=dev)
    else:
        rk = rv = rl = None
    return q, dict(n_kv_heads=Hkv, key_format=store.key_format, key_codes=view["codes"], v_data=view["vdata"],
                   v_scales=view["vscales"], v_zeros=view["vzeros"], hist_len=hist, page_size=view["page_size"],
                   block_table=bt, value_bits=store.value_bits, group_size=store.value_group_size, recent_k=rk,
                   recent_v=rv, recent_len=rl, scale=scale, min_history=MIN_HISTORY_FOR_SMAQ,
                   layout=view["layout"], **kw)


def compute_hybrid_attention(query: torch.Tensor, store: CompressedKVStore, recent_k: Optional[torch.Tensor],
                             recent_v: Optional[torch.Tensor], num_query_heads: int,
                             scale: Optional[float] = None) -> torch.Tensor:
    """``query [T, Hq, D]`` -> ``[T, Hq, D]`` in the query dtype."""
    call = _decode_call(query, store, recent_k, recent_v, num_query_heads, scale)
    if call is None:
        return torch.zeros(query.shape[0], num_query_heads, store.head_dim, device=query.device, dtype=query.dtype)
    q, kw = call
    return ops.decode(q, **kw)


def hybrid_kernel_path(query: torch.Tensor, store: CompressedKVStore, recent_k: Optional[torch.Tensor],
                       recent_v: Optional[torch.Tensor], num_query_heads: int,
                       scale: Optional[float] = None) -> Optional[int]:
    """The decode kernel path compute_hybrid_attention would run for these arguments
    (``ops.PATH_*``; None when there is nothing to attend).  Launches nothing."""
    call = _decode_call(query, store, recent_k, recent_v, num_query_heads, scale)
    if call is None:
        return None
    q, kw = call
    return ops.decode(q, query_path=True, **kw)


class HybridAttentionBackend(AttentionBackend):
    """Attention backend over compressed history and the exact tail (smaq/score.py:141-160)."""

    def compute(self, query, store, recent_k, recent_v, num_query_heads, scale: Optional[float] = None):
        return compute_hybrid_attention(query=query, store=store, recent_k=recent_k, recent_v=recent_v,
                                        num_query_heads=num_query_heads, scale=scale)
