"""vLLM integration: capture K/V writes of attention layers, keep the recent tokens exact in a
ring buffer, compress older tokens into a CompressedKVStore, and answer decode steps from
compressed history plus the exact window.

Same public API as ``smaq.integration.vllm`` (smaq/integration/vllm.py:1-476): the mode
constants and ``set_mode``/``get_mode``, ``LayerConfig``/``LayerState``, ``install_hooks``,
``free_kv_cache``, ``get_stats``.  The hooks wrap an attention implementation's
``do_kv_cache_update`` (when present) and ``forward``; the decode path runs
``compute_hybrid_attention`` of this package (the device kernels), prefill stays with the
wrapped implementation unless ``no_alloc`` is set.  MLA layers are recognised and passed
through, as in the reference.  The mode is process-global and not thread-safe, as in the
reference.
"""

from __future__ import annotations

import logging
import math
import types
from dataclasses import dataclass, field
from typing import Callable, Optional

import torch
import torch.nn.functional as F

from ..capture import KVCaptureEngine
from ..score import MIN_HISTORY_FOR_SMAQ, compute_hybrid_attention
from ..store import CompressedKVStore

logger = logging.getLogger("smaq.integration.vllm")

MODE_OFF = "off"
MODE_CAPTURE_ONLY = "capture_only"
MODE_HYBRID = "hybrid"
MODE_FULL_SMAQ = "full_smaq"
_VALID_MODES = (MODE_OFF, MODE_CAPTURE_ONLY, MODE_HYBRID, MODE_FULL_SMAQ)

_GLOBAL_MODE = MODE_CAPTURE_ONLY


def set_mode(mode: str):
    global _GLOBAL_MODE
    if mode not in _VALID_MODES:
        raise ValueError(f"Invalid mode: {mode}. Valid: {_VALID_MODES}")
    _GLOBAL_MODE = mode
    logger.info("[SMAQ] Mode set to %s", mode)


def get_mode() -> str:
    return _GLOBAL_MODE


@dataclass
class LayerConfig:
    """Per-layer settings (smaq/integration/vllm.py:49-62)."""

    head_dim: int
    num_kv_heads: int
    num_query_heads: int
    Sigma_q: Optional[torch.Tensor] = None
    key_bits: int = 3
    value_bits: int = 2
    value_group_size: int = 32
    ring_capacity: int = 128
    layer_idx: int = 0
    backend_kind: str = "flash"
    device: torch.device = field(default_factory=lambda: torch.device("cuda"))


@dataclass
class LayerState:
    """Per-layer runtime state: the compressed store and the capture engine feeding it."""

    config: LayerConfig
    store: CompressedKVStore
    engine: KVCaptureEngine
    _log_count: int = 0

    @property
    def supports_hybrid(self) -> bool:
        return self.config.backend_kind == "flash"

    def reset(self):
        self.engine.reset()
        self._log_count = 0


def _create_layer_state(cfg: LayerConfig) -> LayerState:
    store = CompressedKVStore(head_dim=cfg.head_dim, num_kv_heads=cfg.num_kv_heads, Sigma_q=cfg.Sigma_q,
                              key_bits=cfg.key_bits, value_bits=cfg.value_bits,
                              value_group_size=cfg.value_group_size, device=cfg.device, layer_idx=cfg.layer_idx)
    engine = KVCaptureEngine(store=store, ring_capacity=cfg.ring_capacity, device=cfg.device)
    return LayerState(config=cfg, store=store, engine=engine)


def _infer_num_query_heads(attn_module, impl) -> int:
    for value in (getattr(attn_module, "num_heads", None), getattr(attn_module, "num_attention_heads", None),
                  getattr(impl, "num_heads", None)):
        if value:
            return int(value)
    return int(impl.num_kv_heads)


def _is_mla_impl(impl) -> bool:
    return hasattr(impl, "forward_mqa") and hasattr(impl, "do_kv_cache_update") and not hasattr(impl, "forward")


def _ingest(state: LayerState, key: torch.Tensor, value: torch.Tensor, num_tokens: int):
    """One token is a decode step; more are a prefill chunk."""
    if num_tokens <= 1:
        state.engine.ingest_decode(key, value, num_tokens)
    else:
        state.engine.ingest_prefill(key, value, num_tokens)


def _make_patched_kv_update(orig_fn: Callable, state: LayerState, no_alloc: bool = False):
    """Wrap ``do_kv_cache_update``: keep vLLM's own write unless no_alloc, then capture."""

    def patched(self_impl, layer, key, value, kv_cache, slot_mapping):
        if not no_alloc:
            orig_fn(self_impl, layer, key, value, kv_cache, slot_mapping)
        if _GLOBAL_MODE == MODE_OFF:
            return
        _ingest(state, key, value, slot_mapping.shape[0])

    return patched


def _no_alloc_prefill_attention(state: LayerState, self_impl, query, key, value, attn_metadata):
    """Causal attention over the prefill chunk itself (the paged cache does not exist)."""
    n = attn_metadata.num_actual_tokens
    cfg = state.config
    q, k, v = query[:n], key[:n], value[:n]
    if q.dim() == 2:
        q = q.view(n, cfg.num_query_heads, cfg.head_dim)
    if k.dim() == 2:
        k = k.view(n, cfg.num_kv_heads, cfg.head_dim)
        v = v.view(n, cfg.num_kv_heads, cfg.head_dim)
    if cfg.num_query_heads != cfg.num_kv_heads:
        rep = cfg.num_query_heads // cfg.num_kv_heads
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    scale = getattr(self_impl, "scale", 1.0 / math.sqrt(cfg.head_dim))
    out = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None], v.transpose(0, 1)[None],
                                         is_causal=True, scale=scale)
    return out[0].transpose(0, 1)


def _emit(result: torch.Tensor, query: torch.Tensor, output, state: LayerState, n: int):
    """Return the attention result the way the wrapped forward would: into ``output`` when
    given, else shaped like the query."""
    flat = result.reshape(n, state.config.num_query_heads * state.config.head_dim).to(query.dtype)
    if output is not None:
        dst = output[:n]
        dst.copy_(result.to(dst.dtype) if dst.dim() == 3 else flat.to(dst.dtype))
        return output
    return result.to(query.dtype) if query.dim() == 3 else flat


def _make_patched_forward(orig_fn: Callable, state: LayerState, no_alloc: bool = False,
                          capture_in_forward: bool = False):
    """Wrap ``forward``: capture (when the impl has no separate KV update), then serve decode
    steps from compressed history + exact window in hybrid mode."""

    def patched(self_impl, layer, query, key, value, kv_cache, attn_metadata, output=None, output_scale=None,
                output_block_scale=None):
        mode = _GLOBAL_MODE

        def passthrough():
            return orig_fn(self_impl, layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                           output_block_scale)

        if capture_in_forward and mode != MODE_OFF and attn_metadata is not None:
            n = getattr(attn_metadata, "num_actual_tokens", key.shape[0])
            _ingest(state, key[:n], value[:n], n)
        if mode in (MODE_OFF, MODE_CAPTURE_ONLY) or attn_metadata is None:
            return passthrough()
        n = attn_metadata.num_actual_tokens
        if attn_metadata.max_query_len > 1:  # prefill
            if no_alloc:
                return _emit(_no_alloc_prefill_attention(state, self_impl, query, key, value, attn_metadata), query,
                             output, state, n)
            return passthrough()
        if mode == MODE_HYBRID and state.supports_hybrid:
            flat = state.store.get_flat_cache()
            if flat is not None and flat.num_tokens >= MIN_HISTORY_FOR_SMAQ:
                q = query[:n]
                if q.dim() == 2:
                    q = q.view(n, state.config.num_query_heads, state.config.head_dim)
                recent = state.engine.ring.peek()
                result = compute_hybrid_attention(query=q, store=state.store,
                                                  recent_k=recent[0] if recent else None,
                                                  recent_v=recent[1] if recent else None,
                                                  num_query_heads=state.config.num_query_heads,
                                                  scale=getattr(self_impl, "scale", None))
                return _emit(result, query, output, state, n)
        if no_alloc:  # nothing to attend to yet and no paged cache to fall back on
            n = getattr(attn_metadata, "num_actual_tokens", query.shape[0])
            if query.dim() == 3:
                return torch.zeros_like(query[:n])
            return torch.zeros(n, state.config.num_query_heads * state.config.head_dim, dtype=query.dtype,
                               device=query.device)
        return passthrough()

    return patched


def _make_patched_mla_update(orig_fn: Callable, state: LayerState):
    """MLA KV writes pass through (the reference has no MLA path yet)."""

    def patched(self_impl, kv_c_normed, k_pe, kv_cache, slot_mapping, kv_cache_dtype, k_scale):
        orig_fn(self_impl, kv_c_normed, k_pe, kv_cache, slot_mapping, kv_cache_dtype, k_scale)
        if state._log_count < 1:
            logger.info("[SMAQ] MLA update observed on layer %s; MLA path is not active yet.", state.config.layer_idx)
            state._log_count += 1

    return patched


def _make_patched_mla_forward(orig_fn: Callable, state: LayerState):
    def patched(self_impl, q, kv_c_and_k_pe_cache, attn_metadata, layer):
        return orig_fn(self_impl, q, kv_c_and_k_pe_cache, attn_metadata, layer)

    return patched


def _bind(impl, name: str, fn: Callable):
    setattr(impl, name, types.MethodType(lambda self, *a, _fn=fn, **kw: _fn(self, *a, **kw), impl))


def install_hooks(model_runner, calibration_covariances: Optional[dict[str, torch.Tensor]] = None,
                  key_bits: int = 3, value_bits: int = 2, value_group_size: int = 32, ring_capacity: int = 128,
                  initial_layers_count: int = 4, initial_layers_key_bits: int | None = None,
                  mode: str = MODE_CAPTURE_ONLY, no_alloc: bool = False) -> dict[str, LayerState]:
    """Hook every attention layer of ``model_runner.compilation_config.static_forward_context``.
    The first ``initial_layers_count`` layers get ``initial_layers_key_bits`` (default
    key_bits + 1, at most 4)."""
    global _GLOBAL_MODE
    _GLOBAL_MODE = mode
    if initial_layers_key_bits is None:
        initial_layers_key_bits = min(key_bits + 1, 4)
    ctx = model_runner.compilation_config.static_forward_context
    device = model_runner.device
    states: dict[str, LayerState] = {}
    idx = 0
    for name, attn in ctx.items():
        impl = getattr(attn, "impl", None)
        if impl is None or getattr(impl, "num_kv_heads", None) is None:
            continue
        if hasattr(impl, "head_size"):
            head_dim = int(impl.head_size)
        elif hasattr(impl, "kv_lora_rank"):
            head_dim = int(impl.kv_lora_rank)
        else:
            continue
        kind = "mla" if _is_mla_impl(impl) else "flash"
        cfg = LayerConfig(head_dim=head_dim, num_kv_heads=int(impl.num_kv_heads),
                          num_query_heads=_infer_num_query_heads(attn, impl),
                          Sigma_q=(calibration_covariances or {}).get(name) if calibration_covariances else None,
                          key_bits=initial_layers_key_bits if idx < initial_layers_count else key_bits,
                          value_bits=value_bits, value_group_size=min(value_group_size, head_dim),
                          ring_capacity=ring_capacity, layer_idx=idx, backend_kind=kind, device=device)
        state = _create_layer_state(cfg)
        states[name] = state
        if kind == "flash":
            separate_update = hasattr(impl, "do_kv_cache_update")
            if separate_update:
                _bind(impl, "do_kv_cache_update",
                      _make_patched_kv_update(impl.do_kv_cache_update.__func__, state, no_alloc=no_alloc))
            _bind(impl, "forward", _make_patched_forward(impl.forward.__func__, state, no_alloc=no_alloc,
                                                         capture_in_forward=not separate_update))
        else:
            if hasattr(impl, "do_kv_cache_update"):
                _bind(impl, "do_kv_cache_update", _make_patched_mla_update(impl.do_kv_cache_update.__func__, state))
            if hasattr(impl, "forward_mqa"):
                _bind(impl, "forward_mqa", _make_patched_mla_forward(impl.forward_mqa.__func__, state))
        impl._smaq_layer_state = state
        idx += 1
    model_runner._smaq_layer_states = states
    model_runner._smaq_no_alloc = no_alloc
    logger.info("[SMAQ] Hooks installed on %s layers (mode=%s, no_alloc=%s)", len(states), mode, no_alloc)
    return states


def free_kv_cache(model_runner) -> int:
    """Replace the paged KV cache tensors of hooked flash layers by a 1-byte tensor; returns the
    bytes released."""
    states = getattr(model_runner, "_smaq_layer_states", None)
    if not states:
        logger.warning("[SMAQ] No layer states found, nothing to free")
        return 0
    ctx = model_runner.compilation_config.static_forward_context
    tiny = torch.zeros(1, dtype=torch.int8, device=model_runner.device)
    hooked = [name for name, st in states.items() if st.supports_hybrid and name in ctx]
    ptrs = set()
    freed = 0
    for name in hooked:
        kv = getattr(ctx[name], "kv_cache", None)
        if kv and len(kv) > 0:
            ptrs.add(kv[0].data_ptr())
            freed += kv[0].nelement() * kv[0].element_size()
            kv[0] = tiny
    for i, entry in enumerate(model_runner.kv_caches):
        if isinstance(entry, list):
            for j, t in enumerate(entry):
                if hasattr(t, "data_ptr") and t.data_ptr() in ptrs:
                    entry[j] = tiny
        elif hasattr(entry, "data_ptr") and entry.data_ptr() in ptrs:
            model_runner.kv_caches[i] = tiny
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    logger.info("[SMAQ] Freed %.0f MB KV cache", freed / 1e6)
    return freed


def get_stats(model_runner) -> dict:
    """Per-layer and total compressed/buffered token counts and store bytes."""
    states = getattr(model_runner, "_smaq_layer_states", None)
    if not states:
        return {}
    stats = {}
    tot_c = tot_b = tot_m = 0
    for name, st in states.items():
        c, b, m = st.store.num_tokens, st.engine.ring.size, st.store.memory_bytes()
        tot_c, tot_b, tot_m = tot_c + c, tot_b + b, tot_m + m
        stats[name] = {"compressed_tokens": c, "buffered_tokens": b, "memory_bytes": m,
                       "supports_hybrid": st.supports_hybrid}
    stats["_totals"] = {"compressed_tokens": tot_c, "buffered_tokens": tot_b, "memory_bytes": tot_m,
                        "layers": len(states)}
    return stats
