"""Key quantization strategies on the hot path (same classes as smaq/strategies.py).

Scalar-code strategies (``IdentityScalarStrategy`` and its subclasses
``SMAQFullMetricScalarStrategy`` and ``SMAQDiagonalMetricStrategy``) share the
``SMAQQuantized`` format.  Their quantizers expose ``E`` / ``E_inv`` / ``centroids`` /
``decision_boundaries``, so the scalar-key append and decode kernels serve all three.
``SMAQBlockVQStrategy`` is served by the block-VQ kernels.  ``ExactShadowStrategy`` keeps the
history's keys unquantized (values stay 2-bit): a validation mode that measures what key
compression costs.  Its scores are a plain GEMM (cuBLAS); the compressed values are applied
by the fused attend kernel (``smaq_attend_values``).
"""

from __future__ import annotations

from typing import Any, NamedTuple

import torch

from smaq_b200.block_vq import BlockVQQuantized, SMAQBlockVQ
from smaq_b200.core import MetricStrategy, QuantizationStrategy
from smaq_b200.quantizer import SMAQQuantized, SMAQQuantizer
from smaq_b200.ssf import build_smaq_metric
from smaq_b200.weighted_scalar import RotationAdapter


def _dev(device):
    return torch.device(device) if device is not None else torch.device("cuda" if torch.cuda.is_available() else "cpu")


class IdentityMetricStrategy(MetricStrategy):
    name = "identity"

    def __init__(self, dim: int, device: torch.device | None = None):
        self.dim = dim
        self.device = _dev(device)
        self.sigma_q = torch.eye(dim, dtype=torch.float32, device=self.device)

    def fit(self, calibration_queries: Any, calibration_keys: Any | None = None) -> "IdentityMetricStrategy":
        return self

    def export_state(self) -> dict[str, Any]:
        return {"Sigma_q": self.sigma_q}


def _centered_cov(q: torch.Tensor) -> torch.Tensor:
    q = q.float()
    qc = q - q.mean(dim=0, keepdim=True)
    return qc.T @ qc / max(1, qc.shape[0])


class SMAQFullMetricStrategy(MetricStrategy):
    name = "smaq_full_metric"

    def __init__(self, dim: int, Sigma_q: torch.Tensor | None = None, device: torch.device | None = None):
        self.dim = dim
        self.device = _dev(device)
        self.sigma_q = Sigma_q if Sigma_q is not None else torch.eye(dim, dtype=torch.float32, device=self.device)
        self.E, self.E_inv = build_smaq_metric(self.sigma_q.to(torch.float32), c=5.0)

    def fit(self, calibration_queries: Any, calibration_keys: Any | None = None) -> "SMAQFullMetricStrategy":
        self.sigma_q = _centered_cov(calibration_queries)
        self.E, self.E_inv = build_smaq_metric(self.sigma_q, c=5.0)
        return self

    def export_state(self) -> dict[str, Any]:
        return {"Sigma_q": self.sigma_q, "E": self.E, "E_inv": self.E_inv}


class SMAQDiagonalMetricState(MetricStrategy):
    name = "smaq_diagonal_metric"

    def __init__(self, dim: int, Sigma_q: torch.Tensor | None = None, device: torch.device | None = None):
        self.dim = dim
        self.device = _dev(device)
        self.sigma_q = Sigma_q if Sigma_q is not None else torch.eye(dim, dtype=torch.float32, device=self.device)

    def fit(self, calibration_queries: Any, calibration_keys: Any | None = None) -> "SMAQDiagonalMetricState":
        self.sigma_q = _centered_cov(calibration_queries)
        return self

    def export_state(self) -> dict[str, Any]:
        return {"Sigma_q": self.sigma_q}


class IdentityScalarStrategy(QuantizationStrategy):
    """Scalar codes with no metric: identity rotation, unit scales, midpoint codebook
    (smaq/strategies.py:100-138)."""

    name = "identity_scalar"
    metric_name = "identity"
    quantization_name = "scalar"

    def __init__(self, dim: int, bits: int = 3, device: torch.device | None = None):
        self.quantizer = RotationAdapter(dim=dim, bits=bits, coord_scales=torch.ones(dim), device=device)
        self.bits = bits

    def quantize(self, keys: Any) -> Any:
        return self.quantizer.quantize(keys)

    def dequantize(self, quantized: Any) -> Any:
        return self.quantizer.dequantize(quantized)

    def attention_score(self, query: Any, quantized: Any, scale: float | None = None, **kwargs: Any) -> Any:
        return self.quantizer.attention_score(query, quantized, scale=scale)

    def flatten_quantized(self, quantized: SMAQQuantized) -> SMAQQuantized:
        ix, nm = quantized.indices, quantized.norms
        return SMAQQuantized(indices=ix.reshape(-1, ix.shape[-2], ix.shape[-1]).contiguous(),
                             norms=nm.reshape(-1, nm.shape[-1]).contiguous(), bits=quantized.bits)

    def concat_quantized(self, chunks: list[SMAQQuantized]) -> SMAQQuantized:
        return SMAQQuantized(indices=torch.cat([c.indices for c in chunks], dim=-2),
                             norms=torch.cat([c.norms for c in chunks], dim=-1), bits=chunks[0].bits)

    def select_head(self, quantized: SMAQQuantized, head_idx: int) -> SMAQQuantized:
        return SMAQQuantized(indices=quantized.indices[head_idx], norms=quantized.norms[head_idx],
                             bits=quantized.bits)

    def memory_bytes(self, quantized: SMAQQuantized) -> int:
        # the reference's accounting: one byte per packed code byte, two per norm
        return quantized.indices.nelement() + quantized.norms.nelement() * 2


class SMAQFullMetricScalarStrategy(IdentityScalarStrategy):
    """Scalar metric-aware key codes (smaq/strategies.py:141-166)."""

    name = "smaq_full_metric_scalar"
    metric_name = "smaq_full_metric"

    def __init__(self, dim: int, bits: int = 3, Sigma_q: torch.Tensor | None = None,
                 device: torch.device | None = None, dtype: torch.dtype = torch.float32):
        self.quantizer = SMAQQuantizer(dim=dim, bits=bits, Sigma_q=Sigma_q, device=device, dtype=dtype)
        self.bits = bits

    @property
    def supports_kernel(self) -> bool:
        return True

    def fit(self, calibration_queries: Any, calibration_keys: Any | None = None) -> "SMAQFullMetricScalarStrategy":
        self.quantizer.fit(calibration_queries)
        return self

    def attention_score(self, query: Any, quantized: Any, scale: float | None = None, **kwargs: Any) -> Any:
        return self.quantizer.attention_score(query, quantized, scale=scale,
                                              use_kernel=kwargs.get("use_kernel", False))


class SMAQDiagonalMetricStrategy(IdentityScalarStrategy):
    """Diagonal approximation of the SMAQ metric in a rotation basis (smaq/strategies.py:169-192)."""

    name = "smaq_diagonal_metric"
    metric_name = "smaq_diagonal_metric"

    def __init__(self, dim: int, bits: int = 3, Sigma_q: torch.Tensor | None = None,
                 rotation: torch.Tensor | None = None, device: torch.device | None = None,
                 dtype: torch.dtype = torch.float32):
        self.quantizer = RotationAdapter(dim=dim, bits=bits, Sigma_q=Sigma_q, rotation=rotation, device=device,
                                         dtype=dtype)
        self.bits = bits


class SMAQBlockVQStrategy(QuantizationStrategy):
    """Block-VQ key codes (smaq/strategies.py:195-255)."""

    name = "smaq_block_vq"
    metric_name = "smaq_full_metric"
    quantization_name = "block_vq"

    def __init__(self, head_dim: int, block_dim: int = 8, n_centroids: int = 256, c: float = 5.0,
                 device: torch.device | None = None, dtype: torch.dtype = torch.float32):
        self.quantizer = SMAQBlockVQ(head_dim=head_dim, block_dim=block_dim, n_centroids=n_centroids, c=c,
                                     device=device, dtype=dtype)

    def fit(self, calibration_queries: Any, calibration_keys: Any | None = None) -> "SMAQBlockVQStrategy":
        keys = calibration_keys if calibration_keys is not None else calibration_queries
        self.quantizer.fit(keys, calibration_queries)
        return self

    def quantize(self, keys: Any) -> Any:
        return self.quantizer.quantize(keys)

    def dequantize(self, quantized: Any) -> Any:
        return self.quantizer.dequantize(quantized)

    def attention_score(self, query: Any, quantized: Any, scale: float | None = None, **kwargs: Any) -> Any:
        return self.quantizer.attention_score(query, quantized, scale=scale)

    def flatten_quantized(self, quantized: BlockVQQuantized) -> BlockVQQuantized:
        ix = quantized.indices
        return BlockVQQuantized(indices=ix.reshape(-1, ix.shape[-2], ix.shape[-1]).contiguous(),
                                n_blocks=quantized.n_blocks, block_dim=quantized.block_dim)

    def concat_quantized(self, chunks: list[BlockVQQuantized]) -> BlockVQQuantized:
        return BlockVQQuantized(indices=torch.cat([c.indices for c in chunks], dim=-2),
                                n_blocks=chunks[0].n_blocks, block_dim=chunks[0].block_dim)

    def select_head(self, quantized: BlockVQQuantized, head_idx: int) -> BlockVQQuantized:
        return BlockVQQuantized(indices=quantized.indices[head_idx], n_blocks=quantized.n_blocks,
                                block_dim=quantized.block_dim)

    def memory_bytes(self, quantized: BlockVQQuantized) -> int:
        return quantized.indices.nelement() * quantized.indices.element_size()


class ExactShadowQuantized(NamedTuple):
    """Unquantized keys ``[..., N, D]`` standing in for codes (smaq/strategies.py:70-83)."""

    values: torch.Tensor


class ExactShadowStrategy(QuantizationStrategy):
    """Exact history keys (smaq/strategies.py:258-298): the history half of the cache keeps
    its keys as stored, so attention differs from full precision only by the value codes."""

    name = "exact_shadow"
    metric_name = "identity"
    quantization_name = "shadow_exact"

    @property
    def capabilities(self):
        from smaq_b200.core import CacheCapabilities
        return CacheCapabilities(strategy_name=self.name, metric_name=self.metric_name,
                                 quantization_name=self.quantization_name, compressed_history=False,
                                 compressed_history_shadow_only=True, values_compressed=False,
                                 decode_uses_compressed_keys=False, decode_uses_compressed_values=False)

    def quantize(self, keys: Any) -> Any:
        return ExactShadowQuantized(values=keys.detach().clone())

    def dequantize(self, quantized: Any) -> Any:
        return quantized.values

    def attention_score(self, query: Any, quantized: Any, scale: float | None = None, **kwargs: Any) -> Any:
        s = torch.matmul(query.float(), quantized.values.float().transpose(-2, -1))
        if scale is not None:
            s = s * scale
        return s.to(query.dtype)

    def flatten_quantized(self, quantized: ExactShadowQuantized) -> ExactShadowQuantized:
        v = quantized.values
        return ExactShadowQuantized(values=v.reshape(-1, v.shape[-2], v.shape[-1]).contiguous())

    def concat_quantized(self, chunks: list[ExactShadowQuantized]) -> ExactShadowQuantized:
        return ExactShadowQuantized(values=torch.cat([c.values for c in chunks], dim=-2))

    def select_head(self, quantized: ExactShadowQuantized, head_idx: int) -> ExactShadowQuantized:
        return ExactShadowQuantized(values=quantized.values[head_idx])

    def memory_bytes(self, quantized: ExactShadowQuantized) -> int:
        return quantized.values.nelement() * quantized.values.element_size()
