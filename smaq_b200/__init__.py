"""smaq_b200: B200-native (sm_100a) implementation of SMAQ's compressed-KV hot path.

The modules mirror the reference package ``smaq`` (gauravsaini/smaq) for the hot path:
``quantizer``, ``weighted_scalar``, ``block_vq``, ``kv_cache``, ``store``, ``score``, ``capture``, ``strategies``,
``core``, ``calibration``, ``vllm_attn_backend`` / ``integration.vllm``.  Compute runs in
``libsmaq_b200.so`` (C ABI in ``include/smaq_b200.h``); there is no CPU fallback.

``install_as_smaq()`` registers this package under the name ``smaq`` so code written against
the reference imports it unchanged.
"""

from __future__ import annotations

import importlib
import sys

__version__ = "0.1.0"

_MIRRORED = ("ssf", "core", "calibration", "layout", "quantizer", "triton_kernels", "weighted_scalar", "block_vq",
             "kv_cache", "strategies", "store", "score", "capture", "backends")


def install_as_smaq() -> None:
    """Make ``import smaq`` / ``import smaq.<module>`` resolve to this package."""
    pkg = sys.modules[__name__]
    sys.modules["smaq"] = pkg
    for name in _MIRRORED + ("vllm_attn_backend", "integration", "integration.vllm"):
        try:
            mod = importlib.import_module(f"{__name__}.{name}")
        except ImportError:
            continue
        sys.modules[f"smaq.{name}"] = mod


def __getattr__(name):
    # lazy re-exports of the reference's top-level names
    table = {
        "SMAQQuantizer": "quantizer", "SMAQQuantized": "quantizer", "SMAQBlockVQ": "block_vq",
        "BlockVQQuantized": "block_vq", "SMAQKVCache": "kv_cache", "CompressedKVStore": "store",
        "compute_hybrid_attention": "score", "KVCaptureEngine": "capture", "RingBuffer": "capture",
        "SMAQFullMetricScalarStrategy": "strategies", "SMAQBlockVQStrategy": "strategies",
        "IdentityMetricStrategy": "strategies", "SMAQFullMetricStrategy": "strategies",
        "SMAQDiagonalMetricState": "strategies", "IdentityScalarStrategy": "strategies",
        "SMAQDiagonalMetricStrategy": "strategies", "ExactShadowStrategy": "strategies",
        "ExactShadowQuantized": "strategies", "RotationAdapter": "weighted_scalar",
        "SMAQWeightedRotationQuantizer": "weighted_scalar", "build_codebook": "weighted_scalar",
        "build_rotated_diagonal_metric_scales": "weighted_scalar",
        "build_block_diagonal_metric_scales": "weighted_scalar", "IdentityCalibrationProvider": "calibration",
        "StaticCalibrationProvider": "calibration", "TorchHybridAttentionBackend": "backends",
        "AttentionBackend": "core", "CacheBackend": "core", "CacheCapabilities": "core",
        "CalibrationProvider": "core", "LayoutInfo": "core", "MetricStrategy": "core",
        "QuantizationStrategy": "core", "ModelLayoutAdapter": "core",
        "GenericModelLayoutAdapter": "layout", "QwenModelLayoutAdapter": "layout",
        "GemmaModelLayoutAdapter": "layout", "infer_model_layout_adapter": "layout",
    }
    if name in table:
        return getattr(importlib.import_module(f"{__name__}.{table[name]}"), name)
    raise AttributeError(name)
