"""Spectral shaping of the query covariance into the SMAQ metric (host side, torch).

Mirrors smaq/ssf.py:8-29 (gauravsaini/smaq): with ``(lambda, V) = eigh(Sigma_q)`` the shaped
spectrum is ``s = exp(log(log1p(c * max(lambda, 0))) - mean)`` (volume-normalised so
``log det E = 0``), ``E = V diag(sqrt s) V^T`` and ``E_inv = V diag(1/sqrt s) V^T``.

The eigendecomposition runs once per calibration, so it is evaluated on the CPU in fp32
(LAPACK) whatever device the caller uses; the result is identical to the reference's CPU
evaluation and is then moved to the caller's device by the quantizers.
"""

from __future__ import annotations

import torch


def ssf_log(eigvals: torch.Tensor, c: float = 5.0) -> torch.Tensor:
    """Log-compressed, volume-normalised spectral shaping function (over the last dim)."""
    logs = torch.log(torch.log1p(c * eigvals.clamp(min=0)).clamp(min=1e-8))
    return torch.exp(logs - logs.mean(dim=-1, keepdim=True))


def build_smaq_metric(Sigma_q: torch.Tensor, c: float = 5.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Return ``(E, E_inv)`` for the query covariance ``Sigma_q`` (fp32, on Sigma_q's device).
    A stack ``[..., d, d]`` of covariances (the block-VQ blocks) is done in one call: one host
    transfer and one batched eigendecomposition."""
    dev = Sigma_q.device
    lam, V = torch.linalg.eigh(Sigma_q.detach().to("cpu", torch.float32))
    root = ssf_log(lam, c).sqrt()
    if Sigma_q.dim() == 2:
        E = V @ torch.diag(root) @ V.T
        E_inv = V @ torch.diag(1.0 / root) @ V.T
    else:
        Vt = V.transpose(-2, -1)
        E = (V * root[..., None, :]) @ Vt
        E_inv = (V * (1.0 / root)[..., None, :]) @ Vt
    return E.to(dev), E_inv.to(dev)
