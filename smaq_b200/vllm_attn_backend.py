"""SMAQ attention backend entry points for vLLM (smaq/vllm_attn_backend.py:1-154): legacy mode
names mapped onto ``integration.vllm``, hook installation, the no-alloc engine patch and
``free_kv_cache``."""

from __future__ import annotations

import logging

from .integration import vllm as _backend

logger = logging.getLogger("smaq.attn")

MODE_SHADOW = "shadow"
MODE_ACCUMULATE = "accumulate"
MODE_ACTIVE = "active"
_VALID_MODES = (MODE_SHADOW, MODE_ACCUMULATE, MODE_ACTIVE)

_LEGACY_TO_NEW = {
    MODE_SHADOW: _backend.MODE_CAPTURE_ONLY,
    MODE_ACCUMULATE: _backend.MODE_CAPTURE_ONLY,
    MODE_ACTIVE: _backend.MODE_HYBRID,
}

_GLOBAL_MODE = MODE_ACCUMULATE
_SMAQ_NO_ALLOC_CONFIG = None


def set_mode(mode: str):
    global _GLOBAL_MODE
    if mode not in _VALID_MODES:
        raise ValueError(f"Invalid mode: {mode}. Valid: {_VALID_MODES}")
    _GLOBAL_MODE = mode
    _backend.set_mode(_LEGACY_TO_NEW[mode])


def get_mode() -> str:
    return _GLOBAL_MODE


def install_smaq_hooks(model_runner, calibration_covariances=None, key_bits: int = 3, value_bits: int = 2,
                       value_group_size: int = 32, buffer_size: int = 128, initial_layers_count: int = 4,
                       initial_layers_key_bits: int | None = None, mode: str = MODE_ACCUMULATE,
                       no_alloc: bool = False):
    """Install the hooks with a legacy mode name; ``buffer_size`` is the exact-window ring."""
    global _GLOBAL_MODE
    states = _backend.install_hooks(model_runner, calibration_covariances=calibration_covariances,
                                    key_bits=key_bits, value_bits=value_bits, value_group_size=value_group_size,
                                    ring_capacity=buffer_size, initial_layers_count=initial_layers_count,
                                    initial_layers_key_bits=initial_layers_key_bits,
                                    mode=_LEGACY_TO_NEW.get(mode, _backend.MODE_CAPTURE_ONLY), no_alloc=no_alloc)
    _GLOBAL_MODE = mode
    model_runner._smaq_states = states
    model_runner._smaq_no_alloc = no_alloc
    return states


def enable_no_alloc(calibration_covariances=None, key_bits: int = 3, value_bits: int = 2, buffer_size: int = 128,
                    initial_layers_count: int = 4):
    """Patch vLLM's executor so every worker installs the hooks (active, no_alloc) while the
    engine sizes its KV cache.  Inert when vLLM is not importable."""
    global _SMAQ_NO_ALLOC_CONFIG
    _SMAQ_NO_ALLOC_CONFIG = dict(calibration_covariances=calibration_covariances, key_bits=key_bits,
                                 value_bits=value_bits, buffer_size=buffer_size,
                                 initial_layers_count=initial_layers_count)
    try:
        from vllm.v1.executor.abstract import Executor
        from vllm.v1.worker.gpu_model_runner import GPUModelRunner
    except ImportError:
        logger.warning("[SMAQ] vLLM is not installed; enable_no_alloc is inert.")
        return
    if hasattr(Executor, "_smaq_patched"):
        return
    if not hasattr(GPUModelRunner, "_smaq_layout_patch"):
        orig_layout = GPUModelRunner._update_hybrid_attention_mamba_layout

        def layout_update(self, kv_caches):
            # layers that share a KV cache with another layer see the target's tensor
            for name, target in getattr(self, "shared_kv_cache_layers", {}).items():
                if name not in kv_caches and target in kv_caches:
                    kv_caches[name] = kv_caches[target]
            return orig_layout(self, kv_caches)

        GPUModelRunner._update_hybrid_attention_mamba_layout = layout_update
        GPUModelRunner._smaq_layout_patch = True
    orig_specs = Executor.get_kv_cache_specs

    def get_kv_cache_specs(self):
        cfg = _SMAQ_NO_ALLOC_CONFIG
        if cfg is None:
            return orig_specs(self)

        def install_on_worker(worker):
            states = install_smaq_hooks(worker.model_runner, calibration_covariances=cfg["calibration_covariances"],
                                        key_bits=cfg["key_bits"], value_bits=cfg["value_bits"],
                                        buffer_size=cfg["buffer_size"],
                                        initial_layers_count=cfg["initial_layers_count"], mode=MODE_ACTIVE,
                                        no_alloc=True)
            return {"hooks": len(states)}

        try:
            self.collective_rpc(install_on_worker)
        except Exception as exc:  # the engine keeps working without the hooks
            logger.exception("[SMAQ] collective_rpc failed during no-alloc install: %s", exc)
        return orig_specs(self)

    Executor.get_kv_cache_specs = get_kv_cache_specs
    Executor._smaq_patched = True
    logger.info("[SMAQ] Patched Executor for automatic no-alloc hook installation")


def free_kv_cache(model_runner):
    """Free the paged KV cache of hooked layers (integration.vllm.free_kv_cache)."""
    return _backend.free_kv_cache(model_runner)
