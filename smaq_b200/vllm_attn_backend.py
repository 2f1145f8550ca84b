"""Legacy entry points of ``smaq.vllm_attn_backend`` (smaq/vllm_attn_backend.py): the three old
mode names, ``install_smaq_hooks``, ``enable_no_alloc`` and ``free_kv_cache``, all served by
``integration.vllm``.  New code can register the attention backend instead
(``integration.vllm_backend.register``), which patches nothing.
"""

from __future__ import annotations

import logging

from .integration import vllm as _iv

logger = logging.getLogger("smaq.attn")

MODE_SHADOW = "shadow"          # capture only
MODE_ACCUMULATE = "accumulate"  # capture only (the reference's default)
MODE_ACTIVE = "active"          # SMAQ decode
_MODES = {MODE_SHADOW: _iv.MODE_CAPTURE_ONLY, MODE_ACCUMULATE: _iv.MODE_CAPTURE_ONLY,
          MODE_ACTIVE: _iv.MODE_HYBRID}

_legacy_mode = MODE_ACCUMULATE
_no_alloc_settings = None


def set_mode(mode: str):
    global _legacy_mode
    if mode not in _MODES:
        raise ValueError(f"Invalid mode: {mode}. Valid: {tuple(_MODES)}")
    _legacy_mode = mode
    _iv.set_mode(_MODES[mode])


def get_mode() -> str:
    return _legacy_mode


def install_smaq_hooks(model_runner, calibration_covariances=None, key_bits: int = 3, value_bits: int = 2,
                       value_group_size: int = 32, buffer_size: int = 128, initial_layers_count: int = 4,
                       initial_layers_key_bits: int | None = None, mode: str = MODE_ACCUMULATE,
                       no_alloc: bool = False):
    """``integration.vllm.install_hooks`` under a legacy mode name; ``buffer_size`` is the
    exact-window capacity."""
    global _legacy_mode
    if mode not in _MODES:
        raise ValueError(f"Invalid mode: {mode}. Valid: {tuple(_MODES)}")
    states = _iv.install_hooks(model_runner, calibration_covariances=calibration_covariances, key_bits=key_bits,
                               value_bits=value_bits, value_group_size=value_group_size, ring_capacity=buffer_size,
                               initial_layers_count=initial_layers_count,
                               initial_layers_key_bits=initial_layers_key_bits, mode=_MODES[mode], no_alloc=no_alloc)
    _legacy_mode = mode
    model_runner._smaq_states = states
    return states


def _share_kv_targets(runner, kv_caches: dict) -> None:
    """Layers that reuse another layer's KV cache see the target's tensor in ``kv_caches``."""
    for name, target in getattr(runner, "shared_kv_cache_layers", {}).items():
        if name not in kv_caches and target in kv_caches:
            kv_caches[name] = kv_caches[target]


def enable_no_alloc(calibration_covariances=None, key_bits: int = 3, value_bits: int = 2, buffer_size: int = 128,
                    initial_layers_count: int = 4):
    """Make every vLLM worker install the hooks (active, no_alloc) while the engine sizes its KV
    cache.  Inert without vLLM.  The layout update of the model runner is wrapped with vLLM
    0.22's signature ``(self, kv_caches, kernel_block_sizes)``; extra arguments pass through."""
    global _no_alloc_settings
    _no_alloc_settings = dict(calibration_covariances=calibration_covariances, key_bits=key_bits,
                              value_bits=value_bits, buffer_size=buffer_size, initial_layers_count=initial_layers_count)
    try:
        from vllm.v1.executor.abstract import Executor
        from vllm.v1.worker.gpu_model_runner import GPUModelRunner
    except ImportError:
        logger.warning("[SMAQ] vLLM is not installed; enable_no_alloc is inert.")
        return
    if getattr(Executor, "_smaq_patched", False):
        return
    if not getattr(GPUModelRunner, "_smaq_layout_patch", False):
        layout = GPUModelRunner._update_hybrid_attention_mamba_layout

        def layout_update(self, kv_caches, *args, **kwargs):
            _share_kv_targets(self, kv_caches)
            return layout(self, kv_caches, *args, **kwargs)

        GPUModelRunner._update_hybrid_attention_mamba_layout = layout_update
        GPUModelRunner._smaq_layout_patch = True
    specs = Executor.get_kv_cache_specs

    def get_kv_cache_specs(self):
        cfg = _no_alloc_settings
        if cfg is not None:
            def on_worker(worker):
                st = install_smaq_hooks(worker.model_runner, calibration_covariances=cfg["calibration_covariances"],
                                        key_bits=cfg["key_bits"], value_bits=cfg["value_bits"],
                                        buffer_size=cfg["buffer_size"], initial_layers_count=cfg["initial_layers_count"],
                                        mode=MODE_ACTIVE, no_alloc=True)
                return {"hooks": len(st)}
            try:
                self.collective_rpc(on_worker)
            except Exception as exc:  # the engine keeps serving without the hooks
                logger.exception("[SMAQ] collective_rpc failed during no-alloc install: %s", exc)
        return specs(self)

    Executor.get_kv_cache_specs = get_kv_cache_specs
    Executor._smaq_patched = True


def free_kv_cache(model_runner):
    """``integration.vllm.free_kv_cache``."""
    return _iv.free_kv_cache(model_runner)
