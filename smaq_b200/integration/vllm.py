"""vLLM integration: batched SMAQ decode over vLLM's paged KV cache.

Public names follow ``smaq.integration.vllm`` (smaq/integration/vllm.py): the mode constants
with ``set_mode``/``get_mode``, ``LayerConfig``, ``LayerState``, ``install_hooks``,
``free_kv_cache`` and ``get_stats``.  The design is this package's own:

* every hooked attention layer owns a ``PagedCompressedCache`` (integration/paged.py) whose
  pages mirror vLLM's cache blocks; each KV write of a step (all sequences, one flat slot per
  token) is quantized into the same slots with one ``smaq_append`` launch;
* a decode step of the whole batch (every sequence one new token) is one ``smaq_decode`` launch
  that follows vLLM's block table: compressed history from the pages, the exact window from
  vLLM's own cache, with the reference's ring rule deciding the split per sequence;
* prefill and mixed prefill/decode steps run vLLM's own attention (the reference does the same
  for prefill); their prompt lengths are recorded for the ring rule.

The same two entry points (``LayerState.on_kv_update`` / ``LayerState.on_forward``) serve the
registered attention backend (integration/vllm_backend.py) and the monkey-patch hooks of
``install_hooks``.

``no_alloc`` (vLLM's cache freed) keeps the reference's single-sequence behaviour: one compressed
store and one exact ring per layer (capture.py), decode through ``compute_hybrid_attention``, and
prefill attention over the chunk itself (this package's decode kernel, ``ops.causal_attention``).  Without vLLM's cache there is no per-sequence exact
window to read, so that mode serves one sequence at a time.  MLA layers are recognised and
passed through, as in the reference.  The mode is process-global.
"""

from __future__ import annotations

import logging
import math
import types
from dataclasses import dataclass, field
from typing import Callable, Optional

import torch
from .. import ops
from ..capture import KVCaptureEngine
from ..score import MIN_HISTORY_FOR_SMAQ, compute_hybrid_attention
from ..store import CompressedKVStore
from .paged import PagedCompressedCache

logger = logging.getLogger("smaq.integration.vllm")

MODE_OFF = "off"
MODE_CAPTURE_ONLY = "capture_only"
MODE_HYBRID = "hybrid"
MODE_FULL_SMAQ = "full_smaq"
_VALID_MODES = (MODE_OFF, MODE_CAPTURE_ONLY, MODE_HYBRID, MODE_FULL_SMAQ)

_mode = MODE_CAPTURE_ONLY


def set_mode(mode: str):
    global _mode
    if mode not in _VALID_MODES:
        raise ValueError(f"Invalid mode: {mode}. Valid: {_VALID_MODES}")
    _mode = mode


def get_mode() -> str:
    return _mode


@dataclass
class LayerConfig:
    """Per-layer settings (fields of smaq/integration/vllm.py's LayerConfig)."""

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


def _emit(result: torch.Tensor, query: torch.Tensor, output: Optional[torch.Tensor], n: int, hq: int, d: int):
    """The attention result as the wrapped forward returns it: written into ``output`` when
    given, else shaped like the query."""
    if output is not None:
        dst = output[:n]
        dst.copy_(result.reshape(dst.shape).to(dst.dtype))
        return output
    if query.dim() == 3:
        return result.to(query.dtype)
    return result.reshape(n, hq * d).to(query.dtype)


def _causal_chunk_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """Causal attention of a prefill chunk over itself, ``[n, H, D]`` in and out, on this
    package's decode kernel (``ops.causal_attention``): grouped query heads read their shared
    KV head directly, with no expanded copy of K and V and no library attention kernel."""
    return ops.causal_attention(q, k, v, scale)


class LayerState:
    """Runtime state of one hooked attention layer (the role of smaq/integration/vllm.py's
    LayerState): the paged compressed cache, or in ``no_alloc`` mode the single-sequence store
    and exact ring."""

    def __init__(self, config: LayerConfig, no_alloc: bool = False):
        self.config = config
        self.no_alloc = no_alloc
        self.cache: Optional[PagedCompressedCache] = None
        self.tokens_written = 0
        self.store: Optional[CompressedKVStore] = None
        self.engine: Optional[KVCaptureEngine] = None
        if no_alloc:
            self.store = CompressedKVStore(head_dim=config.head_dim, num_kv_heads=config.num_kv_heads,
                                           Sigma_q=config.Sigma_q, key_bits=config.key_bits,
                                           value_bits=config.value_bits, value_group_size=config.value_group_size,
                                           device=config.device, layer_idx=config.layer_idx)
            self.engine = KVCaptureEngine(store=self.store, ring_capacity=config.ring_capacity, device=config.device)

    @property
    def supports_hybrid(self) -> bool:
        return self.config.backend_kind == "flash"

    def reset(self):
        self.tokens_written = 0
        if self.engine is not None:
            self.engine.reset()
        if self.cache is not None:
            self.cache.prompt_len.zero_()

    def memory_bytes(self) -> int:
        if self.store is not None:
            return self.store.memory_bytes()
        return self.cache.device_bytes() if self.cache is not None else 0

    def compressed_tokens(self) -> int:
        return self.store.num_tokens if self.store is not None else self.tokens_written

    def buffered_tokens(self) -> int:
        return self.engine.ring.size if self.engine is not None else 0

    def _ensure_cache(self, kv_cache: torch.Tensor) -> Optional[PagedCompressedCache]:
        if self.cache is None:
            cfg = self.config
            if kv_cache is None or kv_cache.dim() != 5:
                raise ValueError("SMAQ paged mode needs vLLM's [2, num_blocks, block_size, Hkv, D] KV cache")
            if kv_cache.element_size() == 1:
                # quantized (fp8) vLLM caches: the exact window would be fp8; leave the layer to vLLM
                if not getattr(self, "_unsupported_logged", False):
                    logger.warning("[SMAQ] layer %d: KV cache dtype %s not served (8-bit caches are left to vLLM)", cfg.layer_idx,
                                   kv_cache.dtype)
                    self._unsupported_logged = True
                return None
            self.cache = PagedCompressedCache(kv_cache.shape[1], kv_cache.shape[2], cfg.num_kv_heads, cfg.head_dim,
                                              key_bits=cfg.key_bits, value_bits=cfg.value_bits,
                                              group_size=cfg.value_group_size, capacity=cfg.ring_capacity,
                                              Sigma_q=cfg.Sigma_q, dtype=kv_cache.dtype, device=kv_cache.device)
        return self.cache

    # ------------------------------------------------------------------ entry points
    def on_kv_update(self, key: torch.Tensor, value: torch.Tensor, kv_cache: Optional[torch.Tensor],
                     slot_mapping: torch.Tensor) -> None:
        """After vLLM's own cache write (skipped in no_alloc mode): quantize the step's tokens."""
        if _mode == MODE_OFF:
            return
        n = slot_mapping.shape[0]
        if self.no_alloc:
            k, v = key[:n], value[:n]
            if k.dim() == 2:
                k = k.view(n, self.config.num_kv_heads, self.config.head_dim)
                v = v.view(n, self.config.num_kv_heads, self.config.head_dim)
            if n <= 1:
                self.engine.ingest_decode(k, v, n)
            else:
                self.engine.ingest_prefill(k, v, n)
        else:
            cache = self._ensure_cache(kv_cache)
            if cache is None:
                return
            cache.write(key, value, slot_mapping)
        self.tokens_written += n

    def on_forward(self, impl, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                   kv_cache: Optional[torch.Tensor], attn_metadata, output: Optional[torch.Tensor],
                   capture: bool = False):
        """The SMAQ answer for this step, or None to run vLLM's own attention."""
        if _mode == MODE_OFF or attn_metadata is None:
            return None
        cfg = self.config
        n = attn_metadata.num_actual_tokens
        if capture:  # implementations whose forward also writes the cache
            slots = getattr(attn_metadata, "slot_mapping", None)
            if slots is None:
                slots = torch.arange(n, device=key.device)
            self.on_kv_update(key, value, kv_cache, slots[:n])
        scale = getattr(impl, "scale", 1.0 / math.sqrt(cfg.head_dim))
        prefill = attn_metadata.max_query_len > 1
        if self.no_alloc:
            return self._forward_single(query, key, value, attn_metadata, output, n, prefill, scale)
        if prefill:
            if self.cache is not None and getattr(attn_metadata, "block_table", None) is not None:
                qsl = attn_metadata.query_start_loc
                B = qsl.shape[0] - 1
                self.cache.note_prompts(attn_metadata.block_table[:B], attn_metadata.seq_lens[:B], qsl[1:] - qsl[:-1])
            return None
        if _mode != MODE_HYBRID or not self.supports_hybrid or self.cache is None:
            return None
        q = query[:n]
        if q.dim() == 2:
            q = q.view(n, cfg.num_query_heads, cfg.head_dim)
        res = self.cache.decode(q, kv_cache, attn_metadata.block_table, attn_metadata.seq_lens, scale=scale)
        return _emit(res, query, output, n, cfg.num_query_heads, cfg.head_dim)

    def _forward_single(self, query, key, value, attn_metadata, output, n, prefill, scale):
        """no_alloc: one sequence, served from this layer's store and ring (or the chunk itself)."""
        cfg = self.config
        q = query[:n]
        if q.dim() == 2:
            q = q.view(n, cfg.num_query_heads, cfg.head_dim)
        if prefill:
            k, v = key[:n], value[:n]
            if k.dim() == 2:
                k = k.view(n, cfg.num_kv_heads, cfg.head_dim)
                v = v.view(n, cfg.num_kv_heads, cfg.head_dim)
            return _emit(_causal_chunk_attention(q, k, v, scale), query, output, n, cfg.num_query_heads, cfg.head_dim)
        if _mode == MODE_HYBRID and self.supports_hybrid and self.store.num_tokens >= MIN_HISTORY_FOR_SMAQ:
            recent = self.engine.ring.peek()
            res = compute_hybrid_attention(query=q, store=self.store, recent_k=recent[0] if recent else None,
                                           recent_v=recent[1] if recent else None,
                                           num_query_heads=cfg.num_query_heads, scale=scale)
            return _emit(res, query, output, n, cfg.num_query_heads, cfg.head_dim)
        # nothing compressed yet and no paged cache to fall back on
        return _emit(torch.zeros(n, cfg.num_query_heads, cfg.head_dim, dtype=query.dtype, device=query.device),
                     query, output, n, cfg.num_query_heads, cfg.head_dim)


# ---------------------------------------------------------------------- hook installation
def _query_heads(attn_module, impl) -> int:
    for v in (getattr(attn_module, "num_heads", None), getattr(attn_module, "num_attention_heads", None),
              getattr(impl, "num_heads", None)):
        if v:
            return int(v)
    return int(impl.num_kv_heads)


def _is_mla(impl) -> bool:
    return hasattr(impl, "forward_mqa") and hasattr(impl, "do_kv_cache_update") and not hasattr(impl, "forward")


def _rebind(impl, name: str, make: Callable[[Callable], Callable]) -> None:
    """Replace bound method ``name`` of ``impl`` by ``make(original bound method)``."""
    orig = getattr(impl, name)
    wrapped = make(orig)
    setattr(impl, name, types.MethodType(lambda self, *a, **kw: wrapped(*a, **kw), impl))


def _hook_flash(impl, state: LayerState, no_alloc: bool) -> None:
    separate = hasattr(impl, "do_kv_cache_update")

    if separate:
        def make_update(orig):
            def update(layer, key, value, kv_cache, slot_mapping):
                if not no_alloc:
                    orig(layer, key, value, kv_cache, slot_mapping)
                state.on_kv_update(key, value, kv_cache, slot_mapping)
            return update
        _rebind(impl, "do_kv_cache_update", make_update)

    def make_forward(orig):
        def forward(layer, query, key, value, kv_cache, attn_metadata, output=None, *rest, **kw):
            res = state.on_forward(impl, query, key, value, kv_cache, attn_metadata, output, capture=not separate)
            return res if res is not None else orig(layer, query, key, value, kv_cache, attn_metadata, output,
                                                    *rest, **kw)
        return forward
    _rebind(impl, "forward", make_forward)


def install_hooks(model_runner, calibration_covariances: Optional[dict[str, torch.Tensor]] = None,
                  key_bits: int = 3, value_bits: int = 2, value_group_size: int = 32, ring_capacity: int = 128,
                  initial_layers_count: int = 4, initial_layers_key_bits: int | None = None,
                  mode: str = MODE_CAPTURE_ONLY, no_alloc: bool = False) -> dict[str, LayerState]:
    """Hook every attention layer of ``model_runner.compilation_config.static_forward_context``
    (the API of smaq/integration/vllm.py's install_hooks).  The first ``initial_layers_count``
    layers use ``initial_layers_key_bits`` (default key_bits + 1, at most 4)."""
    set_mode(mode)
    if initial_layers_key_bits is None:
        initial_layers_key_bits = min(key_bits + 1, 4)
    states: dict[str, LayerState] = {}
    for name, attn in model_runner.compilation_config.static_forward_context.items():
        impl = getattr(attn, "impl", None)
        if impl is None or getattr(impl, "num_kv_heads", None) is None:
            continue
        head_dim = getattr(impl, "head_size", None) or getattr(impl, "kv_lora_rank", None)
        if head_dim is None:
            continue
        idx = len(states)
        mla = _is_mla(impl)
        cfg = LayerConfig(head_dim=int(head_dim), num_kv_heads=int(impl.num_kv_heads),
                          num_query_heads=_query_heads(attn, impl),
                          Sigma_q=(calibration_covariances or {}).get(name),
                          key_bits=initial_layers_key_bits if idx < initial_layers_count else key_bits,
                          value_bits=value_bits, value_group_size=min(value_group_size, int(head_dim)),
                          ring_capacity=ring_capacity, layer_idx=idx, backend_kind="mla" if mla else "flash",
                          device=model_runner.device)
        state = LayerState(cfg, no_alloc=no_alloc and not mla)
        if not mla:
            _hook_flash(impl, state, no_alloc)
        else:
            logger.info("[SMAQ] layer %s is MLA: passed through", name)
        impl._smaq_layer_state = state
        states[name] = state
    model_runner._smaq_layer_states = states
    model_runner._smaq_no_alloc = no_alloc
    logger.info("[SMAQ] hooks on %d layers (mode=%s, no_alloc=%s)", len(states), mode, no_alloc)
    return states


def free_kv_cache(model_runner) -> int:
    """Swap the KV cache tensors of hooked flash layers for a 1-byte tensor (no_alloc serving);
    returns the bytes released."""
    states = getattr(model_runner, "_smaq_layer_states", None)
    if not states:
        logger.warning("[SMAQ] no hooked layers: nothing to free")
        return 0
    ctx = model_runner.compilation_config.static_forward_context
    tiny = torch.zeros(1, dtype=torch.int8, device=model_runner.device)
    released, freed = set(), 0
    for name, st in states.items():
        kv = getattr(ctx.get(name), "kv_cache", None)
        if st.supports_hybrid and kv:
            released.add(kv[0].data_ptr())
            freed += kv[0].nelement() * kv[0].element_size()
            kv[0] = tiny

    def swap(t):
        return tiny if hasattr(t, "data_ptr") and t.data_ptr() in released else t

    for i, entry in enumerate(model_runner.kv_caches):
        if isinstance(entry, list):
            entry[:] = [swap(t) for t in entry]
        else:
            model_runner.kv_caches[i] = swap(entry)
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    logger.info("[SMAQ] released %.0f MB of KV cache", freed / 1e6)
    return freed


def get_stats(model_runner) -> dict:
    """Per-layer and total token counts and bytes (keys of smaq/integration/vllm.py's get_stats)."""
    states = getattr(model_runner, "_smaq_layer_states", None)
    if not states:
        return {}
    stats = {name: {"compressed_tokens": st.compressed_tokens(), "buffered_tokens": st.buffered_tokens(),
                    "memory_bytes": st.memory_bytes(), "supports_hybrid": st.supports_hybrid}
             for name, st in states.items()}
    stats["_totals"] = {k: sum(s[k] for s in stats.values()) for k in ("compressed_tokens", "buffered_tokens",
                                                                       "memory_bytes")}
    stats["_totals"]["layers"] = len(states)
    return stats
