"""Seeded synthetic KV distributions used by the tests, the golden fixtures and the bench.

No public dataset is involved.  Keys follow ``N(0, U diag(lambda) U^T)`` with
``U`` a seeded random orthogonal matrix and ``lambda_i = i^-1.2``; four seeded
channels are scaled by 8 to model the outlier channels of real key caches.
Values are ``N(0, 1)``.  Queries come from the same spectrum with their own
seeds so the calibrated metric is non-trivial.

Seeds (fixed by convention): keys 0, values 1, calibration queries 2, decode
queries 3, sequence lengths 4, k-means 42.
"""

from __future__ import annotations

import numpy as np

SEED_KEYS, SEED_VALUES, SEED_CAL_Q, SEED_DEC_Q, SEED_LENGTHS, SEED_KMEANS = 0, 1, 2, 3, 4, 42
N_OUTLIERS = 4
OUTLIER_GAIN = 8.0


def spectrum(d: int) -> np.ndarray:
    return np.arange(1, d + 1, dtype=np.float64) ** -1.2


def basis(d: int, seed: int = 1234) -> tuple[np.ndarray, np.ndarray]:
    """Return ``(U, outlier_channels)`` for head dimension ``d``."""
    rng = np.random.default_rng(seed)
    q, r = np.linalg.qr(rng.standard_normal((d, d)))
    q = q * np.sign(np.diag(r))[None, :]
    ch = rng.choice(d, size=N_OUTLIERS, replace=False)
    return q, np.sort(ch)


def spectral_vectors(shape: tuple[int, ...], d: int, seed: int, outliers: bool) -> np.ndarray:
    """``shape + (d,)`` float32 draws from the spectral distribution."""
    U, ch = basis(d)
    rng = np.random.default_rng(seed)
    n = int(np.prod(shape)) if shape else 1
    z = rng.standard_normal((n, d)) * np.sqrt(spectrum(d))[None, :]
    x = z @ U.T
    if outliers:
        x[:, ch] *= OUTLIER_GAIN
    return x.reshape(*shape, d).astype(np.float32)


def keys(shape, d=128, seed=SEED_KEYS):
    return spectral_vectors(tuple(shape), d, seed, outliers=True)


def queries(shape, d=128, seed=SEED_DEC_Q):
    return spectral_vectors(tuple(shape), d, seed, outliers=False)


def calibration_queries(n=512, d=128, seed=SEED_CAL_Q):
    return spectral_vectors((n,), d, seed, outliers=False)


def values(shape, d=128, seed=SEED_VALUES):
    rng = np.random.default_rng(seed)
    return rng.standard_normal(tuple(shape) + (d,)).astype(np.float32)


def seq_lengths(n: int, lo: int, hi: int, seed=SEED_LENGTHS) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=n).astype(np.int64)
