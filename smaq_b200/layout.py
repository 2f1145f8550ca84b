"""Model KV-layout adapters (same names and results as smaq/layout.py:10-60).

Bookkeeping only: they read the last dimension of the key and value tensors a layer produces
and report it as a ``LayoutInfo``; nothing on the compute path depends on them.
"""

from __future__ import annotations

from typing import Any

from smaq_b200.core import LayoutInfo, ModelLayoutAdapter


def _widths(keys: Any, values: Any) -> tuple[int, int]:
    return int(keys.shape[-1]), int(values.shape[-1])


class GenericModelLayoutAdapter(ModelLayoutAdapter):
    """The observed key width is the head dim; a width other than the expected one is
    reported as a unified KV layout."""

    name = "generic"

    def normalize_kv(self, keys: Any, values: Any, expected_head_dim: int | None = None) -> LayoutInfo:
        kd, vd = _widths(keys, values)
        return LayoutInfo(adapter_name=self.name, effective_head_dim=kd, observed_key_dim=kd, observed_value_dim=vd,
                          unified_kv=expected_head_dim is not None and kd != expected_head_dim)


class QwenModelLayoutAdapter(GenericModelLayoutAdapter):
    """Qwen models: standard KV shapes, reported under their own name."""

    name = "qwen"


class GemmaModelLayoutAdapter(GenericModelLayoutAdapter):
    """Gemma models: keys may arrive wider than the configured head dim (unified KV)."""

    name = "gemma"


_BY_FAMILY = (("gemma", GemmaModelLayoutAdapter), ("qwen", QwenModelLayoutAdapter))


def infer_model_layout_adapter(model: Any) -> ModelLayoutAdapter:
    """Pick the adapter from the model's class and module names (Gemma before Qwen)."""
    tag = f"{type(model).__module__} {type(model).__name__}".lower()
    for family, cls in _BY_FAMILY:
        if family in tag:
            return cls()
    return GenericModelLayoutAdapter()
