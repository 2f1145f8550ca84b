"""The reference's own test file (test_generic_core.py:42-86) checks calibration providers,
the Gemma / Qwen layout adapters and the CacheCapabilities fields; the same checks run here
against this package, with shape-only stand-ins for tensors as the reference uses, plus the
adapter inference and head-dim resolution it does not test."""

import types

import pytest

from smaq_b200.calibration import IdentityCalibrationProvider, StaticCalibrationProvider
from smaq_b200.core import CacheCapabilities, LayoutInfo
from smaq_b200.layout import (GemmaModelLayoutAdapter, GenericModelLayoutAdapter, QwenModelLayoutAdapter,
                              infer_model_layout_adapter)


def shaped(*shape):
    return types.SimpleNamespace(shape=shape)


def test_identity_provider_has_no_covariance():
    assert IdentityCalibrationProvider().get_sigma_q(layer_idx=0, head_dim=128) is None


def test_static_provider_by_index_and_by_name():
    p = StaticCalibrationProvider({0: "sigma0", "layer_1": "sigma1"})
    assert p.get_sigma_q(layer_idx=0, head_dim=64) == "sigma0"
    assert p.get_sigma_q(layer_idx=1, head_dim=64) == "sigma1"


def test_gemma_widened_keys_are_unified():
    info = GemmaModelLayoutAdapter().normalize_kv(shaped(1, 8, 16, 256), shaped(1, 8, 16, 256),
                                                  expected_head_dim=128)
    assert isinstance(info, LayoutInfo)
    assert info.adapter_name == "gemma" and info.unified_kv and info.effective_head_dim == 256


def test_qwen_standard_shape():
    info = QwenModelLayoutAdapter().normalize_kv(shaped(1, 8, 16, 128), shaped(1, 8, 16, 128),
                                                 expected_head_dim=128)
    assert info.adapter_name == "qwen" and not info.unified_kv and info.effective_head_dim == 128


def test_generic_reports_both_widths_and_no_expectation():
    info = GenericModelLayoutAdapter().normalize_kv(shaped(4, 192), shaped(4, 128))
    assert (info.observed_key_dim, info.observed_value_dim, info.effective_head_dim) == (192, 128, 192)
    assert info.unified_kv is False


def test_capabilities_fields():
    caps = CacheCapabilities(strategy_name="diag", metric_name="smaq_diagonal_metric", quantization_name="scalar",
                             compressed_history=True, compressed_history_shadow_only=False, values_compressed=True,
                             decode_uses_compressed_keys=True, decode_uses_compressed_values=False)
    assert caps.strategy_name == "diag" and caps.compressed_history and not caps.compressed_history_shadow_only


def test_adapter_inference_and_head_dim():
    Gemma3ForCausalLM = type("Gemma3ForCausalLM", (), {})
    Qwen2Model = type("Qwen2Model", (), {})
    assert infer_model_layout_adapter(Gemma3ForCausalLM()).name == "gemma"
    assert infer_model_layout_adapter(Qwen2Model()).name == "qwen"
    assert infer_model_layout_adapter(object()).name == "generic"
    model = types.SimpleNamespace(layers=[types.SimpleNamespace(self_attn=types.SimpleNamespace(head_dim=96)),
                                          types.SimpleNamespace(self_attn=types.SimpleNamespace(hidden_size=4096,
                                                                                                num_heads=32)),
                                          types.SimpleNamespace()])
    a = GenericModelLayoutAdapter()
    assert [a.resolve_head_dim(model, i) for i in range(3)] == [96, 128, 128]


def test_layout_module_is_mirrored():
    import sys
    import smaq_b200
    saved = {k: v for k, v in sys.modules.items() if k == "smaq" or k.startswith("smaq.")}
    try:
        smaq_b200.install_as_smaq()
        import smaq.layout
        assert smaq.layout.GemmaModelLayoutAdapter is GemmaModelLayoutAdapter
    finally:
        for k in [k for k in sys.modules if k == "smaq" or k.startswith("smaq.")]:
            del sys.modules[k]
        sys.modules.update(saved)
    with pytest.raises(TypeError):
        from smaq_b200.core import ModelLayoutAdapter
        ModelLayoutAdapter()


def test_top_level_names_of_the_reference_package():
    """Every name smaq/__init__.py re-exports resolves on this package."""
    import smaq_b200
    names = """TorchHybridAttentionBackend IdentityCalibrationProvider StaticCalibrationProvider BlockVQQuantized
    SMAQBlockVQ AttentionBackend CacheBackend CacheCapabilities CalibrationProvider LayoutInfo MetricStrategy
    ModelLayoutAdapter QuantizationStrategy KVCaptureEngine RingBuffer SMAQKVCache GemmaModelLayoutAdapter
    GenericModelLayoutAdapter QwenModelLayoutAdapter infer_model_layout_adapter SMAQQuantized SMAQQuantizer
    compute_hybrid_attention ExactShadowStrategy IdentityMetricStrategy IdentityScalarStrategy SMAQBlockVQStrategy
    SMAQDiagonalMetricState SMAQDiagonalMetricStrategy SMAQFullMetricScalarStrategy SMAQFullMetricStrategy
    CompressedKVStore RotationAdapter SMAQWeightedRotationQuantizer build_rotated_diagonal_metric_scales
    build_block_diagonal_metric_scales build_codebook""".split()
    missing = [n for n in names if not hasattr(smaq_b200, n)]
    assert not missing, missing
