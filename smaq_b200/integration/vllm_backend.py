"""SMAQ as a registered vLLM attention backend (vLLM >= 0.22 backend registry).

``register(...)`` installs ``SmaqAttentionBackend`` under ``AttentionBackendEnum.CUSTOM``; an
engine started with ``attention_backend="CUSTOM"`` then builds every decoder attention layer
with ``SmaqAttentionImpl``.  The backend is vLLM's FlashAttention backend (same KV cache shape,
metadata builder and prefill kernels) whose implementation adds the SMAQ path of
``integration.vllm.LayerState``: every cache write is also quantized into the layer's paged
compressed cache, and decode-only steps are answered by one ``smaq_decode`` launch over the
batch.  No method of vLLM is patched.

The settings (key bits, exact-window capacity, optional per-layer query covariances) are
process-wide and must be set before the engine builds its layers.  Importing this module
without vLLM leaves ``SmaqAttentionBackend``/``SmaqAttentionImpl`` undefined and ``register``
raising ``ImportError``.
"""

from __future__ import annotations

import itertools
from typing import Optional

import torch

from . import vllm as _hooks

_settings = {"key_bits": 3, "value_bits": 2, "value_group_size": 32, "ring_capacity": 128,
             "initial_layers_count": 4, "initial_layers_key_bits": None, "covariances": None}
_layer_counter = itertools.count()

try:
    from vllm.v1.attention.backends.flash_attn import FlashAttentionBackend, FlashAttentionImpl
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend
except ImportError:  # vLLM absent
    FlashAttentionBackend = FlashAttentionImpl = None


def _layer_config(impl, idx: int, device: torch.device) -> _hooks.LayerConfig:
    s = _settings
    init_bits = s["initial_layers_key_bits"] or min(s["key_bits"] + 1, 4)
    cov = (s["covariances"] or {}).get(idx)
    return _hooks.LayerConfig(head_dim=int(impl.head_size), num_kv_heads=int(impl.num_kv_heads),
                              num_query_heads=int(impl.num_heads), Sigma_q=cov,
                              key_bits=init_bits if idx < s["initial_layers_count"] else s["key_bits"],
                              value_bits=s["value_bits"], value_group_size=min(s["value_group_size"],
                                                                               int(impl.head_size)),
                              ring_capacity=s["ring_capacity"], layer_idx=idx, device=device)


if FlashAttentionImpl is not None:

    class SmaqAttentionImpl(FlashAttentionImpl):
        """FlashAttention plus the SMAQ paged path (``LayerState`` of integration.vllm)."""

        def __init__(self, *args, **kwargs):
            super().__init__(*args, **kwargs)
            self._smaq_idx = next(_layer_counter)
            self._smaq_state: Optional[_hooks.LayerState] = None

        def _state(self, device: torch.device) -> _hooks.LayerState:
            if self._smaq_state is None:
                self._smaq_state = _hooks.LayerState(_layer_config(self, self._smaq_idx, device))
            return self._smaq_state

        def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
            super().do_kv_cache_update(layer, key, value, kv_cache, slot_mapping)
            if kv_cache is not None and kv_cache.dim() == 5:
                self._state(kv_cache.device).on_kv_update(key, value, kv_cache, slot_mapping)

        def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                    output_block_scale=None):
            if self._smaq_state is not None and output_scale is None and output_block_scale is None:
                res = self._smaq_state.on_forward(self, query, key, value, kv_cache, attn_metadata, output)
                if res is not None:
                    return res
            return super().forward(layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                                   output_block_scale)

    class SmaqAttentionBackend(FlashAttentionBackend):
        @staticmethod
        def get_name() -> str:
            return "CUSTOM"

        @staticmethod
        def get_impl_cls():
            return SmaqAttentionImpl


def register(key_bits: int = 3, value_bits: int = 2, value_group_size: int = 32, ring_capacity: int = 128,
             initial_layers_count: int = 4, initial_layers_key_bits: Optional[int] = None,
             covariances: Optional[dict[int, torch.Tensor]] = None, mode: str = _hooks.MODE_HYBRID) -> str:
    """Register ``SmaqAttentionBackend`` as vLLM's CUSTOM attention backend and set the SMAQ
    mode; returns the backend's class path.  ``covariances``: per-layer query covariance by
    layer index (layers in construction order)."""
    if FlashAttentionImpl is None:
        raise ImportError("vLLM is not installed")
    _settings.update(key_bits=key_bits, value_bits=value_bits, value_group_size=value_group_size,
                     ring_capacity=ring_capacity, initial_layers_count=initial_layers_count,
                     initial_layers_key_bits=initial_layers_key_bits, covariances=covariances)
    _hooks.set_mode(mode)
    path = f"{SmaqAttentionBackend.__module__}.{SmaqAttentionBackend.__qualname__}"
    register_backend(AttentionBackendEnum.CUSTOM, path)
    return path
