"""Rotation + per-dimension-scale scalar key quantizer (API of smaq/weighted_scalar.py).

``RotationAdapter`` quantizes ``z = (k_unit @ R^T) * s`` against a scalar codebook and scores
``q_r = (q @ R^T) / s`` against ``centroids[codes] * norm`` (smaq/weighted_scalar.py:139-383).
Both transforms are linear maps, so the adapter hands the sm_100a kernels the fused matrices

    E     = diag(s) R        (keys:    k_unit @ E^T     = (k_unit @ R^T) * s)
    E_inv = diag(1 / s) R    (queries: q @ E_inv^T      = (q @ R^T) / s)

and the same kernels that serve ``SMAQQuantizer`` serve it: the tensor-core rotation and
code-packing append kernel, and the fused scalar-key decode.  The stored format is the
reference's ``SMAQQuantized`` (LSB-first packed codes + per-key norms).  Fusing ``s`` into the
matrix moves the fp32 rounding point of each coordinate; codes are therefore exact outside
the same fp32 rounding band as ``SMAQQuantizer``'s.

The codebook, the diagonal-metric scales and the calibration (``fit``) are host-side setup,
evaluated on the CPU in fp32 like ``smaq_b200.ssf`` so every device holds identical tables.
"""

from __future__ import annotations

import torch

from smaq_b200 import ops
from smaq_b200._lib import SMAQ_KEYS_SCALAR
from smaq_b200.quantizer import SMAQQuantized, _normal_ppf, _unpack_indices
from smaq_b200.ssf import ssf_log


def _default_device(device):
    if device is not None:
        return torch.device(device)
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


def build_codebook(bits: int, device: torch.device, dtype: torch.dtype, centroids: torch.Tensor | None = None,
                   boundaries: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Scalar codebook (smaq/weighted_scalar.py:22-51).

    Default centroids are the Gaussian quantiles at ``linspace(0, 1, 2^bits + 2)[1:-1]``.  The
    default boundaries are ``[-inf, midpoints of adjacent centroids, +inf]``.  External
    centroids / boundaries are used as given.
    """
    if centroids is None:
        probs = torch.linspace(0.0, 1.0, (2 ** bits) + 2, dtype=torch.float32)[1:-1]
        centroids = _normal_ppf(probs)
    centroids = centroids.to(device=device, dtype=dtype)
    if boundaries is None:
        full = torch.empty(centroids.shape[0] + 1, device=device, dtype=dtype)
        full[0] = -float("inf")
        full[-1] = float("inf")
        full[1:-1] = 0.5 * (centroids[:-1] + centroids[1:])
        boundaries = full
    else:
        boundaries = boundaries.to(device=device, dtype=dtype)
    return centroids, boundaries


def _shaped_metric(sigma: torch.Tensor, c: float) -> torch.Tensor:
    lam, V = torch.linalg.eigh(sigma)
    return V @ torch.diag(ssf_log(lam, c=c)) @ V.T


def build_rotated_diagonal_metric_scales(Sigma_q: torch.Tensor, rotation=None, c: float = 5.0,
                                         min_scale: float = 1e-6) -> torch.Tensor:
    """Per-dimension scales ``s`` of the diagonal approximation of the SMAQ metric in the
    rotated basis (smaq/weighted_scalar.py:54-87).

    ``M = V diag(ssf(lambda)) V^T`` for ``(lambda, V) = eigh(Sigma_q)``; with a rotation ``R``
    (a matrix, or a callable applied to the identity) ``M <- R M R^T``.  Then
    ``s = sqrt(clamp(diag M, min_scale))`` normalised to geometric mean 1.  fp32, on the CPU,
    returned on Sigma_q's device.
    """
    dev = Sigma_q.device
    metric = _shaped_metric(Sigma_q.detach().to("cpu", torch.float32), c)
    if rotation is not None:
        if callable(rotation):
            rotation = rotation(torch.eye(Sigma_q.shape[0], dtype=torch.float32))
        R = rotation.detach().to("cpu", torch.float32)
        metric = R @ metric @ R.T
    scales = metric.diagonal().clamp(min=min_scale).sqrt()
    log_s = torch.log(scales)
    return torch.exp(log_s - log_s.mean()).to(dev)


def build_block_diagonal_metric_scales(Sigma_q: torch.Tensor, block_size: int = 2, c: float = 5.0,
                                       min_scale: float = 1e-6) -> torch.Tensor:
    """Per-coordinate scales for block-diagonal rotations (smaq/weighted_scalar.py:90-136):
    the shaped metric of each ``block_size`` diagonal block of ``Sigma_q``, its diagonal's
    square root normalised to geometric mean 1 per block; a ragged tail gets scale 1."""
    dev = Sigma_q.device
    sig = Sigma_q.detach().to("cpu", torch.float32)
    dim = sig.shape[0]
    parts = []
    for b in range(dim // block_size):
        sl = slice(b * block_size, (b + 1) * block_size)
        s = _shaped_metric(sig[sl, sl], c).diagonal().clamp(min=min_scale).sqrt()
        log_s = torch.log(s)
        parts.append(torch.exp(log_s - log_s.mean()))
    if dim % block_size:
        parts.append(torch.ones(dim - (dim // block_size) * block_size, dtype=torch.float32))
    return torch.cat(parts).to(dev)


class RotationAdapter(torch.nn.Module):
    """Rotation-based scalar quantizer with per-dimension scales (smaq/weighted_scalar.py:139-383).

    Buffers as in the reference: ``rotation`` ``R``, ``coord_scales`` ``s``,
    ``inv_coord_scales`` ``1 / max(s, 1e-6)``, ``centroids``, ``boundaries`` (with the
    infinite ends) and ``decision_boundaries``.  Also ``E`` / ``E_inv``, the fused matrices the
    kernels use (module docstring).
    """

    def __init__(self, dim: int, bits: int = 3, Sigma_q: torch.Tensor | None = None,
                 rotation: torch.Tensor | None = None, coord_scales: torch.Tensor | None = None, c: float = 5.0,
                 device: torch.device | None = None, dtype: torch.dtype = torch.float32,
                 centroids: torch.Tensor | None = None, boundaries: torch.Tensor | None = None):
        super().__init__()
        self.dim = dim
        self.bits = bits
        self.device = _default_device(device)
        if rotation is None:
            rotation = torch.eye(dim, dtype=torch.float32)
        rotation = rotation.to(device=self.device, dtype=dtype)
        if coord_scales is None:
            if Sigma_q is None:
                Sigma_q = torch.eye(dim, dtype=torch.float32)
            coord_scales = build_rotated_diagonal_metric_scales(Sigma_q, rotation=rotation.to(torch.float32), c=c)
        coord_scales = coord_scales.to(device=self.device, dtype=dtype)
        cent, full = build_codebook(bits, self.device, dtype, centroids=centroids, boundaries=boundaries)
        self.register_buffer("rotation", rotation)
        self.register_buffer("coord_scales", coord_scales)
        self.register_buffer("inv_coord_scales", 1.0 / coord_scales.clamp(min=1e-6))
        self.register_buffer("centroids", cent)
        self.register_buffer("boundaries", full)
        self.register_buffer("decision_boundaries", full[1:-1].contiguous())
        R = rotation.to(torch.float32)
        self.register_buffer("E", coord_scales.to(torch.float32)[:, None] * R)
        self.register_buffer("E_inv", self.inv_coord_scales.to(torch.float32)[:, None] * R)
        self._c = c
        self._Sigma_q = Sigma_q

    @classmethod
    def fit(cls, dim: int, bits: int, calibration_queries: torch.Tensor, calibration_keys: torch.Tensor,
            rotation: torch.Tensor | None = None, c_values: list[float] | None = None,
            use_rotation_values: list[bool] | None = None, device: torch.device | None = None,
            dtype: torch.dtype = torch.float32, centroids: torch.Tensor | None = None,
            boundaries: torch.Tensor | None = None) -> tuple["RotationAdapter", dict]:
        """Grid-search the shaping constant ``c`` and rotation-or-identity by held-out logit MSE
        ``mean(((q . (k - k_hat)))^2)`` (smaq/weighted_scalar.py:229-340).  The first half of
        the calibration pairs gives ``Sigma_q = Q^T Q / n`` (uncentred), the second half scores.
        Keys are quantized by the sm_100a kernel; ties keep the first candidate."""
        c_values = c_values or [0.5, 1.0, 2.0, 5.0, 10.0, 20.0, 50.0]
        use_rotation_values = use_rotation_values or [True, False]
        device = _default_device(device)
        n = calibration_queries.shape[0]
        mid = n // 2
        q_cal = calibration_queries[:mid]
        q_val, k_val = calibration_queries[mid:], calibration_keys[mid:]
        Sigma_q = (q_cal.T @ q_cal) / mid
        eye = torch.eye(dim, dtype=torch.float32, device=device)
        rotation = eye if rotation is None else rotation.to(device=device, dtype=dtype)

        def logit_mse(q, k, k_hat):
            return ((q * (k - k_hat)).sum(dim=1) ** 2).mean().item()

        best = (float("inf"), 5.0, True)
        results = []
        for use_rot in use_rotation_values:
            rot = rotation if use_rot else eye
            for c_val in c_values:
                ad = cls(dim=dim, bits=bits, Sigma_q=Sigma_q, rotation=rot, c=c_val, device=device, dtype=dtype,
                         centroids=centroids, boundaries=boundaries)
                k_hat = ad.dequantize(ad.quantize(k_val))
                lmse = logit_mse(q_val.float(), k_val.float(), k_hat.float())
                results.append({"c": c_val, "use_rotation": use_rot, "lmse": lmse})
                if lmse < best[0]:
                    best = (lmse, c_val, use_rot)
        best_lmse, best_c, best_rot = best
        adapter = cls(dim=dim, bits=bits, Sigma_q=Sigma_q, rotation=rotation if best_rot else eye, c=best_c,
                      device=device, dtype=dtype, centroids=centroids, boundaries=boundaries)
        return adapter, {"best_c": best_c, "best_use_rotation": best_rot, "best_lmse": best_lmse,
                         "all_results": results}

    def rotate_query(self, query: torch.Tensor) -> torch.Tensor:
        """``(query @ R^T) / s`` in fp32 (the decode kernel does this in its prologue via E_inv)."""
        return torch.matmul(query.float(), self.rotation.T.float()) * self.inv_coord_scales.float()

    def quantize(self, k: torch.Tensor) -> SMAQQuantized:
        """Compress keys ``(..., dim)`` on the GPU: norms, unit keys, ``k_unit @ E^T``, codes, packing."""
        codes, norms = ops.quantize_keys_scalar(k, self.E, self.decision_boundaries, self.bits)
        return SMAQQuantized(indices=codes, norms=norms, bits=self.bits)

    def dequantize(self, q: SMAQQuantized) -> torch.Tensor:
        """``((centroids[codes] / s) @ R) * norm`` in the rotation's dtype (a debugging view)."""
        y = self.centroids[_unpack_indices(q.indices, q.bits, self.dim)].float() * self.inv_coord_scales.float()
        return (torch.matmul(y, self.rotation.float()) * q.norms.unsqueeze(-1)).to(self.rotation.dtype)

    def attention_score(self, query: torch.Tensor, quantized_key: SMAQQuantized,
                        scale: float | None = None) -> torch.Tensor:
        """Scores ``rotate_query(q) . centroids[codes] * norm [* scale]`` in the query dtype,
        one ``smaq_key_scores`` launch (the rotation and coordinate scales fused in E_inv)."""
        return ops.key_scores(query, key_format=SMAQ_KEYS_SCALAR, scale=scale, key_codes=quantized_key.indices,
                              key_norms=quantized_key.norms, key_bits=quantized_key.bits, E_inv=self.E_inv,
                              centroids=self.centroids)

    def forward(self, k: torch.Tensor) -> torch.Tensor:
        return self.dequantize(self.quantize(k))


# the reference's backward-compatibility name
SMAQWeightedRotationQuantizer = RotationAdapter
