"""The bf16 kernels compute bf16(x / d) as bf16(x * (1/d)) (x, d bf16; 1/d and the product
rounded to fp32).  They rely on a quotient of two bf16 values never sitting on, or within
2^-17 of, a bf16 rounding midpoint.  This checks the claim exhaustively over every finite bf16
x (normal quotients) against every bf16 significand of d at several exponents."""

import numpy as np


def bf16_rne(f32: np.ndarray) -> np.ndarray:
    u = f32.view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return r.astype(np.uint32)


def test_reciprocal_quotient_rounds_like_division():
    xs = (np.arange(0x10000, dtype=np.uint32) << 16).view(np.float32)
    xs = xs[np.isfinite(xs) & (xs != 0)]
    x64 = xs.astype(np.float64)
    bad = 0
    for e in (-20, -3, 0, 1, 7, 30):
        for m in range(128, 256):
            d = np.float32(m * 2.0 ** (e - 7))
            rcp = np.float32(1.0) / d
            prod = (xs * rcp).astype(np.float32)
            exact = (x64 / np.float64(d)).astype(np.float32)   # fp64 quotient -> fp32 (RN)
            keep = np.abs(exact) >= np.float32(2.0 ** -126)     # normal quotients
            bad += int((bf16_rne(prod)[keep] != bf16_rne(exact)[keep]).sum())
    assert bad == 0
