"""Block vector quantizer (API of smaq/block_vq.py, encode on sm_100a).

Keys are split into ``head_dim / block_dim`` blocks; block ``b`` is mapped by its own metric
``E_b`` and assigned the nearest of ``n_centroids`` k-means centroids (distances as torch.cdist
computes them: ``sqrt(clamp(|x|^2 + |c|^2 - 2 x.c, 0))``, first index on ties).  Encoding runs
the ``smaq_quantize_keys_bvq`` CUDA kernel; calibration (``fit``: per-block metric and k-means)
is a one-time torch computation on the caller's device.
"""

from __future__ import annotations

import math
from typing import NamedTuple, Optional

import torch
import torch.nn as nn

from smaq_b200 import ops
from smaq_b200._lib import SMAQ_KEYS_BVQ
from smaq_b200.ssf import build_smaq_metric


class BlockVQQuantized(NamedTuple):
    """Per-block centroid indices ``(..., n_blocks)`` (int64, as the reference returns them)."""

    indices: torch.Tensor
    n_blocks: int
    block_dim: int


def _kmeans(data: torch.Tensor, n_centroids: int, n_iters: int = 20, seed: int = 42) -> torch.Tensor:
    """k-means++ seeding then Lloyd iterations (smaq/block_vq.py:37-79).

    The random draws (one ``randint`` then one ``multinomial`` per further centre, from a
    generator seeded with ``seed`` on the data's device) follow the reference call for call, so
    the same data and seed give the reference's codebook on the same device.
    """
    n, d = data.shape
    gen = torch.Generator(device=data.device).manual_seed(seed)
    if n <= n_centroids:
        out = torch.zeros((n_centroids, d), device=data.device, dtype=data.dtype)
        out[:n] = data
        return out
    chosen = [int(torch.randint(n, (1,), generator=gen, device=data.device).item())]
    while len(chosen) < n_centroids:
        dmin = torch.cdist(data, data[chosen]).min(dim=1).values
        w = dmin.square()
        tot = w.sum()
        if tot > 0:
            w = w / tot
        else:
            w = torch.full((n,), 1.0 / n, device=data.device, dtype=data.dtype)
        chosen.append(int(torch.multinomial(w, 1, generator=gen).item()))
    return _lloyd(data, data[chosen].clone(), n_iters)


def _lloyd(data: torch.Tensor, cent: torch.Tensor, n_iters: int) -> torch.Tensor:
    """Lloyd steps of ``_kmeans``: nearest centre, mean of the assigned points, empty clusters
    keep their centre."""
    ones = torch.ones(data.shape[0], device=data.device)
    for _ in range(n_iters):
        assign = torch.cdist(data, cent).argmin(dim=1)
        sums = torch.zeros_like(cent).index_add_(0, assign, data)
        cnt = torch.zeros(cent.shape[0], device=data.device).index_add_(0, assign, ones)
        hit = cnt > 0
        sums[hit] /= cnt[hit].unsqueeze(1)
        sums[~hit] = cent[~hit]
        cent = sums
    return cent


class SMAQBlockVQ(nn.Module):
    """SMAQ block VQ (constructor and buffers of smaq/block_vq.py:86-149)."""

    def __init__(self, head_dim: int, block_dim: int = 8, n_centroids: int = 256, c: float = 5.0,
                 device: Optional[torch.device] = None, dtype: torch.dtype = torch.float32):
        super().__init__()
        if head_dim % block_dim != 0:
            raise ValueError(f"head_dim={head_dim} must be divisible by block_dim={block_dim}")
        self.head_dim = head_dim
        self.block_dim = block_dim
        self.n_blocks = head_dim // block_dim
        self.n_centroids = n_centroids
        self.c = c
        self._device = torch.device(device) if device is not None else torch.device("cpu")
        self._dtype = dtype
        eye = torch.eye(block_dim, device=self._device, dtype=dtype).expand(self.n_blocks, -1, -1)
        self.register_buffer("E_blocks", eye.clone())
        self.register_buffer("E_inv_blocks", eye.clone())
        z = torch.zeros(self.n_blocks, n_centroids, block_dim, device=self._device, dtype=dtype)
        self.register_buffer("centroids", z.clone())
        self.register_buffer("decoded_centroids", z.clone())
        self._fitted = False
        self._cb16 = (None, None)

    def fp16_codebook(self) -> Optional[torch.Tensor]:
        """The decoded centroids as fp16 when they are exactly fp16-valued (then the decode runs
        the tensor-core kernel), else None.  Recomputed only when the table changed."""
        t = self.decoded_centroids
        key = (t.data_ptr(), t._version, t.device)
        if self._cb16[0] != key:
            self._cb16 = (key, ops.fp16_codebook(t) if t.is_cuda else None)
        return self._cb16[1]

    @property
    def bits_per_dim(self) -> float:
        return math.log2(self.n_centroids) / self.block_dim

    def fit(self, calibration_keys: torch.Tensor, calibration_queries: torch.Tensor, kmeans_iters: int = 20,
            seed: int = 42, kmeans: str = "auto") -> "SMAQBlockVQ":
        """Per block: uncentered query covariance -> metric -> k-means in the shaped space ->
        pre-decoded centroids ``centroid @ E_inv_b^T`` (smaq/block_vq.py:160-210).

        ``kmeans``: "device" runs every block's k-means in one ``smaq_kmeans`` call (no host
        round trip per centre or iteration; its own generator, so a seed gives a codebook of the
        same quality, not the reference's); "reference" runs ``_kmeans`` block by block with the
        reference's torch generator calls (the reference's codebook on the same device); "auto"
        is "device" for CUDA inputs, else "reference"."""
        if kmeans not in ("auto", "device", "reference"):
            raise ValueError(f"kmeans must be auto, device or reference, not {kmeans!r}")
        N = calibration_keys.shape[0]
        bd = self.block_dim
        sig = []
        for b in range(self.n_blocks):
            qb = calibration_queries[:, b * bd:(b + 1) * bd].float()
            sig.append((qb.T @ qb) / N)
        E_all, Ei_all = build_smaq_metric(torch.stack(sig), c=self.c)   # one batched eigh
        Es, Eis = list(E_all), list(Ei_all)
        shaped = [calibration_keys[:, b * bd:(b + 1) * bd].float() @ Es[b].T for b in range(self.n_blocks)]
        on_device = kmeans == "device" or (kmeans == "auto" and calibration_keys.is_cuda)
        if on_device and N >= self.n_centroids:
            cs = list(ops.kmeans(torch.stack(shaped), self.n_centroids, kmeans_iters, seed))
        else:
            cs = [_kmeans(x, self.n_centroids, kmeans_iters, seed + b) for b, x in enumerate(shaped)]
        ds = [c @ Ei.T for c, Ei in zip(cs, Eis)]
        self.E_blocks = torch.stack(Es).to(self._device, self._dtype)
        self.E_inv_blocks = torch.stack(Eis).to(self._device, self._dtype)
        self.centroids = torch.stack(cs).to(self._device, self._dtype)
        self.decoded_centroids = torch.stack(ds).to(self._device, self._dtype)
        self._fitted = True
        return self

    def quantize_u8(self, k: torch.Tensor) -> torch.Tensor:
        """GPU encode returning the compact uint8 indices the store keeps."""
        return ops.quantize_keys_bvq(k, self.E_blocks, self.centroids)

    def quantize(self, k: torch.Tensor) -> BlockVQQuantized:
        idx = self.quantize_u8(k).to(torch.int64)
        return BlockVQQuantized(indices=idx, n_blocks=self.n_blocks, block_dim=self.block_dim)

    def dequantize(self, q: BlockVQQuantized) -> torch.Tensor:
        """Gather of the pre-decoded centroids (pure lookup)."""
        lead = q.indices.shape[:-1]
        idx = q.indices.reshape(-1, self.n_blocks).long()
        parts = [self.decoded_centroids[b][idx[:, b]] for b in range(self.n_blocks)]
        return torch.cat(parts, dim=-1).reshape(*lead, self.head_dim)

    def attention_score(self, query: torch.Tensor, quantized_key: BlockVQQuantized,
                        scale: Optional[float] = None) -> torch.Tensor:
        """``q . k_hat [* scale]`` in the query dtype (smaq/block_vq.py:273-297): one
        ``smaq_key_scores`` launch over per-block score tables, no key reconstruction."""
        return ops.key_scores(query, key_format=SMAQ_KEYS_BVQ, scale=scale, key_idx=quantized_key.indices,
                              decoded_centroids=self.decoded_centroids)

    def logit_mse(self, queries: torch.Tensor, keys: torch.Tensor) -> float:
        """Held-out logit MSE ``E[(q . (k - k_hat))^2]``."""
        k_hat = self.dequantize(self.quantize(keys))
        return (queries.float() * (keys.float() - k_hat.float())).sum(-1).square().mean().item()

    def forward(self, k: torch.Tensor) -> torch.Tensor:
        return self.dequantize(self.quantize(k))
