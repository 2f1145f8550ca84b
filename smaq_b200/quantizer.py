"""Scalar metric-aware key quantizer (API of smaq/quantizer.py, compute on sm_100a).

``SMAQQuantizer.quantize`` runs the CUDA kernel behind ``smaq_quantize_keys_scalar``: per
key ``norm = ||k||`` (key dtype), ``k_unit = k / (norm + 1e-10)`` (key dtype),
``y = k_unit @ E^T`` (fp32), code = number of decision boundaries strictly below ``y``,
packed LSB-first ``max(1, 8 // bits)`` codes per byte (smaq/quantizer.py:34-46, :138-145).
The codebook is the Gaussian-quantile table of smaq/quantizer.py:96-119, computed on the
CPU in fp32 so every device holds bit-identical tables.
"""

from __future__ import annotations

import math
from typing import NamedTuple

import torch

from smaq_b200 import ops
from smaq_b200._lib import SMAQ_KEYS_SCALAR
from smaq_b200.ssf import build_smaq_metric


class SMAQQuantized(NamedTuple):
    """Bit-packed key codes ``(..., ceil(D / (8 // bits)))`` uint8 and per-key norms ``(...)``."""

    indices: torch.Tensor
    norms: torch.Tensor
    bits: int


def _pack_indices(indices: torch.Tensor, bits: int) -> torch.Tensor:
    """Pack codes ``(..., D)`` into bytes, ``max(1, 8 // bits)`` per byte, LSB first."""
    per = max(1, 8 // bits)
    d = indices.shape[-1]
    width = -(-d // per) * per
    x = indices.to(torch.int32)
    if width != d:
        x = torch.nn.functional.pad(x, (0, width - d))
    x = x.reshape(*x.shape[:-1], width // per, per)
    acc = torch.zeros(x.shape[:-1], dtype=torch.int32, device=x.device)
    for i in range(per):
        acc |= x[..., i] << (i * bits)
    return acc.to(torch.uint8)


def _unpack_indices(packed: torch.Tensor, bits: int, d: int) -> torch.Tensor:
    """Inverse of ``_pack_indices``: int64 codes ``(..., d)``."""
    per = max(1, 8 // bits)
    p = packed.to(torch.int64).unsqueeze(-1)
    sh = torch.arange(per, device=packed.device, dtype=torch.int64) * bits
    codes = (p >> sh) & ((1 << bits) - 1)
    return codes.reshape(*packed.shape[:-1], -1)[..., :d]


def _normal_ppf(probs: torch.Tensor) -> torch.Tensor:
    """Standard normal quantile function."""
    return torch.erfinv(2.0 * probs - 1.0) * math.sqrt(2.0)


def gaussian_codebook(bits: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(centroids [2^bits], boundaries [2^bits + 1] with +-inf ends), fp32 on the CPU."""
    n = 2 ** bits
    mids = torch.linspace(0.0, 1.0, n + 2, dtype=torch.float32)[1:-1]
    centroids = _normal_ppf(mids)
    edges = torch.linspace(0.0, 1.0, n + 1, dtype=torch.float32).clamp(1e-6, 1.0 - 1e-6)
    bnd = _normal_ppf(edges)
    bnd[0] = -float("inf")
    bnd[-1] = float("inf")
    return centroids, bnd


def _default_device(device):
    if device is not None:
        return torch.device(device)
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


class SMAQQuantizer(torch.nn.Module):
    """Spectral metric-aware scalar quantizer (constructor and buffers of smaq/quantizer.py:63-119)."""

    def __init__(self, dim: int, Sigma_q: torch.Tensor | None = None, bits: int = 3,
                 device: torch.device | None = None, dtype: torch.dtype = torch.float32,
                 E: torch.Tensor | None = None, E_inv: torch.Tensor | None = None):
        super().__init__()
        self.dim = dim
        self.bits = bits
        self.device = _default_device(device)
        if E is None or E_inv is None:
            sig = Sigma_q if Sigma_q is not None else torch.eye(dim, dtype=torch.float32)
            E, E_inv = build_smaq_metric(sig.to(torch.float32), c=5.0)
        self.register_buffer("E", E.to(self.device, dtype=dtype))
        self.register_buffer("E_inv", E_inv.to(self.device, dtype=dtype))
        cent, bnd = gaussian_codebook(bits)
        self.register_buffer("centroids", cent.to(self.device, dtype=dtype))
        self.register_buffer("boundaries", bnd.to(self.device, dtype=dtype))
        self.register_buffer("decision_boundaries", self.boundaries[1:-1].contiguous())

    def fit(self, calibration_queries: torch.Tensor) -> "SMAQQuantizer":
        """Refit ``E`` from the centered covariance of calibration queries (quantizer.py:121-129)."""
        q = calibration_queries.detach().to("cpu", torch.float32)
        qc = q - q.mean(dim=0, keepdim=True)
        sigma = qc.T @ qc / max(1, qc.shape[0])
        E, E_inv = build_smaq_metric(sigma, c=5.0)
        self.E.copy_(E.to(self.E.device, self.E.dtype))
        self.E_inv.copy_(E_inv.to(self.E_inv.device, self.E_inv.dtype))
        return self

    def rotate_query(self, query: torch.Tensor) -> torch.Tensor:
        """``query.float() @ E_inv^T`` -- the decode kernel does this in its prologue."""
        return torch.matmul(query.float(), self.E_inv.T)

    def quantize(self, k: torch.Tensor) -> SMAQQuantized:
        """Compress keys ``(..., dim)`` on the GPU."""
        codes, norms = ops.quantize_keys_scalar(k, self.E, self.decision_boundaries, self.bits)
        return SMAQQuantized(indices=codes, norms=norms, bits=self.bits)

    def dequantize(self, q: SMAQQuantized) -> torch.Tensor:
        """Reconstruct keys ``centroids[codes] @ E_inv^T * norm`` (a debugging view, not the decode path)."""
        y = self.centroids[_unpack_indices(q.indices, q.bits, self.dim)]
        return (torch.matmul(y.float(), self.E_inv.T) * q.norms.unsqueeze(-1)).to(self.E.dtype)

    def attention_score(self, query: torch.Tensor, quantized_key: SMAQQuantized, scale: float | None = None,
                        use_kernel: bool = False) -> torch.Tensor:
        """Scores ``(q @ E_inv^T) . centroids[codes] * norm [* scale]`` in the query dtype
        (smaq/quantizer.py:154-184), one ``smaq_key_scores`` launch; ``use_kernel`` is accepted
        for the reference's signature (the kernel always runs)."""
        return ops.key_scores(query, key_format=SMAQ_KEYS_SCALAR, scale=scale, key_codes=quantized_key.indices,
                              key_norms=quantized_key.norms, key_bits=quantized_key.bits, E_inv=self.E_inv,
                              centroids=self.centroids)

    def forward(self, k: torch.Tensor) -> torch.Tensor:
        return self.dequantize(self.quantize(k))
