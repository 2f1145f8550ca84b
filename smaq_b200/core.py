"""Backend-agnostic contracts of the SMAQ cache (same names and methods as smaq/core.py:20-173).

``QuantizationStrategy`` is the plugin interface the store and the attention code dispatch
through; the two concrete strategies on the hot path live in ``smaq_b200.strategies``.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import Any, Optional


@dataclass(frozen=True)
class CacheCapabilities:
    """What a cache/backend does at runtime (smaq/core.py:20-31)."""

    strategy_name: str
    metric_name: str
    quantization_name: str
    compressed_history: bool
    compressed_history_shadow_only: bool
    values_compressed: bool
    decode_uses_compressed_keys: bool
    decode_uses_compressed_values: bool


@dataclass(frozen=True)
class LayoutInfo:
    """Normalised view of a model's KV layout (smaq/core.py:34-43)."""

    adapter_name: str
    effective_head_dim: int
    observed_key_dim: int
    observed_value_dim: int
    unified_kv: bool = False


class CalibrationProvider(ABC):
    """Source of per-layer query covariance."""

    @abstractmethod
    def get_sigma_q(self, layer_idx: int, head_dim: int, device: Any | None = None) -> Any | None:
        ...


class MetricStrategy(ABC):
    """Owns query-aware transforms and their calibration state."""

    name: str = "metric"

    @abstractmethod
    def fit(self, calibration_queries: Any, calibration_keys: Any | None = None) -> "MetricStrategy":
        ...

    @abstractmethod
    def export_state(self) -> dict[str, Any]:
        ...


class QuantizationStrategy(ABC):
    """Owns the compressed key layout and score-time reconstruction (smaq/core.py:71-124)."""

    name: str = "quantization"
    metric_name: str = "metric"
    quantization_name: str = "quantization"

    @property
    def capabilities(self) -> CacheCapabilities:
        # the flags the reference reports for a compressed-history strategy
        return CacheCapabilities(
            strategy_name=self.name,
            metric_name=self.metric_name,
            quantization_name=self.quantization_name,
            compressed_history=True,
            compressed_history_shadow_only=False,
            values_compressed=True,
            decode_uses_compressed_keys=True,
            decode_uses_compressed_values=False,
        )

    def fit(self, calibration_queries: Any, calibration_keys: Any | None = None) -> "QuantizationStrategy":
        return self

    @property
    def supports_kernel(self) -> bool:
        return False

    @abstractmethod
    def quantize(self, keys: Any) -> Any: ...

    @abstractmethod
    def dequantize(self, quantized: Any) -> Any: ...

    @abstractmethod
    def attention_score(self, query: Any, quantized: Any, scale: float | None = None, **kwargs: Any) -> Any: ...

    @abstractmethod
    def flatten_quantized(self, quantized: Any) -> Any: ...

    @abstractmethod
    def concat_quantized(self, chunks: list[Any]) -> Any: ...

    @abstractmethod
    def select_head(self, quantized: Any, head_idx: int) -> Any: ...

    @abstractmethod
    def memory_bytes(self, quantized: Any) -> int: ...


class AttentionBackend(ABC):
    """Attention over compressed history plus an optional exact tail."""

    @abstractmethod
    def compute(self, query: Any, store: Any, recent_k: Any | None, recent_v: Any | None,
                num_query_heads: int, scale: Optional[float] = None) -> Any:
        ...


class CacheBackend(ABC):
    """Owns prefill/decode append, flush and history storage."""

    @property
    @abstractmethod
    def capabilities(self) -> CacheCapabilities:
        ...


class ModelLayoutAdapter(ABC):
    """Per-model-family view of the KV tensors a layer hands over (smaq/core.py:152-173):
    which head dim the cache should use, and whether keys arrive widened or unified."""

    name: str = "generic"

    def resolve_head_dim(self, model: Any, layer_idx: int) -> int:
        attn = getattr(model.layers[layer_idx], "self_attn", None)
        if attn is None:
            return 128
        if hasattr(attn, "head_dim"):
            return int(attn.head_dim)
        if hasattr(attn, "hidden_size") and hasattr(attn, "num_heads"):
            return int(attn.hidden_size // attn.num_heads)
        return 128

    @abstractmethod
    def normalize_kv(self, keys: Any, values: Any, expected_head_dim: int | None = None) -> LayoutInfo:
        ...
