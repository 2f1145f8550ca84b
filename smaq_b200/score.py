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
from smaq_b200.store import KEYS_SHADOW, CompressedKVStore

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
    if store.key_format == KEYS_SHADOW:
        return _shadow_attention(query, store, recent_k, recent_v, num_query_heads, scale)
    call = _decode_call(query, store, recent_k, recent_v, num_query_heads, scale)
    if call is None:
        return torch.zeros(query.shape[0], num_query_heads, store.head_dim, device=query.device, dtype=query.dtype)
    q, kw = call
    return ops.decode(q, **kw)


def _shadow_attention(query: torch.Tensor, store: CompressedKVStore, recent_k: Optional[torch.Tensor],
                      recent_v: Optional[torch.Tensor], num_query_heads: int, scale: Optional[float]) -> torch.Tensor:
    """Hybrid attention with exact history keys (ExactShadowStrategy), smaq/score.py:23-72: the
    history and window logits are fp32 GEMMs (cuBLAS), one fp32 softmax over both, the 2-bit
    history values applied by ``smaq_attend_values`` (dequantization fused), each part cast to
    the query dtype and the parts summed in it."""
    ops._cuda(query, recent_k, recent_v)
    D, Hkv = store.head_dim, store.num_kv_heads
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    T = query.shape[0]
    G = num_query_heads // Hkv
    flat = store.get_flat_cache()
    has_hist = flat is not None and flat.num_tokens >= MIN_HISTORY_FOR_SMAQ
    has_recent = recent_k is not None and recent_k.shape[0] > 0
    if not has_hist and not has_recent:
        return torch.zeros(T, num_query_heads, D, device=query.device, dtype=query.dtype)
    # [Hkv, T*G, D]: query rows grouped by kv head (head h -> kv head h // G)
    q = query.reshape(T, Hkv, G, D).transpose(0, 1).reshape(Hkv, T * G, D).float()
    logits = []
    if has_hist:
        logits.append(torch.matmul(q, flat.key_q.values.float().transpose(-2, -1)) * scale)
    if has_recent:
        logits.append(torch.matmul(q, recent_k.float().permute(1, 2, 0)) * scale)
    w = torch.softmax(torch.cat(logits, -1), dim=-1)

    def back(x):
        return x.reshape(Hkv, T, G, D).transpose(0, 1).reshape(T, num_query_heads, D).to(query.dtype)

    out = None
    n = 0
    if has_hist:
        n = flat.num_tokens
        vq = flat.value_q
        out = back(ops.attend_values(w[..., :n], vq.data, vq.scales, vq.zeros, bits=store.value_bits,
                                     group_size=store.value_group_size, head_dim=D, out_dtype=torch.float32))
    if has_recent:
        o_r = back(torch.matmul(w[..., n:], recent_v.float().transpose(0, 1)))
        out = o_r if out is None else out + o_r
    return out


def hybrid_kernel_path(query: torch.Tensor, store: CompressedKVStore, recent_k: Optional[torch.Tensor],
                       recent_v: Optional[torch.Tensor], num_query_heads: int,
                       scale: Optional[float] = None) -> Optional[int]:
    """The decode kernel path compute_hybrid_attention would run for these arguments
    (``ops.PATH_*``; None when there is nothing to attend or the keys are exact shadows, which
    take no decode kernel).  Launches nothing."""
    if store.key_format == KEYS_SHADOW:
        return None
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
