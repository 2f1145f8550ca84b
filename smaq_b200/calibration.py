"""Query-covariance providers (same interface as smaq/calibration.py:10-27)."""

from __future__ import annotations

from typing import Any, Mapping

from smaq_b200.core import CalibrationProvider


class IdentityCalibrationProvider(CalibrationProvider):
    """No calibration: callers fall back to the identity covariance."""

    def get_sigma_q(self, layer_idx: int, head_dim: int, device: Any | None = None) -> Any | None:
        return None


class StaticCalibrationProvider(CalibrationProvider):
    """Precomputed covariances keyed by layer index or by ``"layer_<idx>"``."""

    def __init__(self, per_layer: Mapping[Any, Any]):
        self.per_layer = dict(per_layer)

    def get_sigma_q(self, layer_idx: int, head_dim: int, device: Any | None = None) -> Any | None:
        if layer_idx in self.per_layer:
            return self.per_layer[layer_idx]
        return self.per_layer.get(f"layer_{layer_idx}")
