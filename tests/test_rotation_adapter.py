"""RotationAdapter (smaq/weighted_scalar.py) on the CPU: the host-side tables of the port and the
oracle, both against the reference's golden vectors (tests/golden/golden_rotation.npz)."""

import os

import numpy as np
import pytest

from oracle import smaq_oracle as O

GOLDEN_ROT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_rotation.npz")
CASES = ["identity3", "diag4", "rot3", "block2"]


@pytest.fixture(scope="module")
def grot():
    return np.load(GOLDEN_ROT)


def fused(g, tag):
    """E = diag(s) R and E_inv = diag(1/s) R of a golden case (R = identity unless rotated)."""
    R = g["ra_rotation"].astype(np.float64) if bool(g[f"ra_{tag}_rotated"]) else np.eye(128)
    s = g[f"ra_{tag}_coord_scales"].astype(np.float64)
    inv = g[f"ra_{tag}_inv_coord_scales"].astype(np.float64)
    return s[:, None] * R, inv[:, None] * R


def test_metric_scales_match_reference(grot):
    import torch
    from smaq_b200.weighted_scalar import build_block_diagonal_metric_scales, build_rotated_diagonal_metric_scales
    sig = torch.from_numpy(grot["ra_sigma"])
    R = torch.from_numpy(grot["ra_rotation"])
    np.testing.assert_allclose(build_rotated_diagonal_metric_scales(sig, rotation=R).numpy(), grot["ra_scales_rot"],
                               rtol=1e-6)
    np.testing.assert_allclose(build_rotated_diagonal_metric_scales(sig).numpy(), grot["ra_scales_norot"], rtol=1e-6)
    np.testing.assert_allclose(build_block_diagonal_metric_scales(sig, 2).numpy(), grot["ra_scales_block2"], rtol=1e-6)
    np.testing.assert_allclose(build_block_diagonal_metric_scales(sig, 3).numpy(), grot["ra_scales_block3"], rtol=1e-6)


@pytest.mark.parametrize("tag", CASES)
def test_adapter_tables_match_reference(grot, tag):
    """Constructor buffers (scales, midpoint codebook) equal the reference's; no kernel runs."""
    import torch
    from smaq_b200.weighted_scalar import RotationAdapter, build_block_diagonal_metric_scales
    sig = torch.from_numpy(grot["ra_sigma"])
    R = torch.from_numpy(grot["ra_rotation"])
    bits = int(grot[f"ra_{tag}_bits"])
    kw = {"identity3": dict(coord_scales=torch.ones(128)), "diag4": dict(Sigma_q=sig),
          "rot3": dict(Sigma_q=sig, rotation=R),
          "block2": dict(coord_scales=build_block_diagonal_metric_scales(sig, 2))}[tag]
    ad = RotationAdapter(128, bits=bits, device="cpu", **kw)
    for name in ("coord_scales", "inv_coord_scales", "centroids", "decision_boundaries"):
        np.testing.assert_allclose(getattr(ad, name).numpy(), grot[f"ra_{tag}_{name}"], rtol=1e-6, atol=1e-7,
                                   err_msg=name)
    E, E_inv = fused(grot, tag)
    np.testing.assert_allclose(ad.E.numpy(), E, rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(ad.E_inv.numpy(), E_inv, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("tag", CASES)
@pytest.mark.parametrize("dn", ["fp32", "bf16"])
def test_oracle_codes_with_fused_matrix(grot, tag, dn):
    """Codes of k_unit @ (diag(s) R)^T match the reference's (k_unit @ R^T) * s outside the
    fp32 rounding band; norms exact."""
    bits = int(grot[f"ra_{tag}_bits"])
    E, _ = fused(grot, tag)
    r = O.quantize_keys_scalar(grot[f"ra_{dn}_k"], E, grot[f"ra_{tag}_decision_boundaries"], bits, dn)
    ref = O.unpack_indices(grot[f"ra_{tag}_{dn}_indices"], bits, 128)
    assert ((ref != r["codes"]) & ~r["near_boundary"]).sum() == 0
    if dn == "fp32":
        np.testing.assert_allclose(r["norms"], grot[f"ra_{tag}_{dn}_norms"], rtol=1e-6)
    else:
        assert np.array_equal(r["norms"], grot[f"ra_{tag}_{dn}_norms"])


def test_oracle_hybrid_with_diagonal_metric_store(grot):
    """The oracle's hybrid attention over the reference's stored diagonal-metric codes reproduces
    the reference's output."""
    p = "ra_hy_"
    Hq, Hkv, nh, nr = (int(x) for x in grot[p + "meta"])
    R = grot["ra_rotation"].astype(np.float64)
    E_inv = (1.0 / np.maximum(grot[p + "coord_scales"].astype(np.float64), 1e-6))[:, None] * R
    K = O.scalar_score_keys(grot[p + "key_indices"], grot[p + "key_norms"], 4, E_inv, grot[p + "centroids"], 128)
    V = O.dequantize_values(grot[p + "v_data"], grot[p + "v_scales"], grot[p + "v_zeros"], 2, 32)
    out, _, _ = O.hybrid_attention(grot[p + "q"], "bf16", K, V, grot[p + "recent_k"], grot[p + "recent_v"], Hq, Hkv)
    assert O.rel_l2(out, grot[p + "out"]) <= 2e-3


def test_strategy_classes_and_store_dispatch():
    """The scalar strategies share the scalar-key kernels; the store accepts them all."""
    from smaq_b200._lib import SMAQ_KEYS_SCALAR
    from smaq_b200.store import key_format_of
    from smaq_b200.strategies import (IdentityScalarStrategy, SMAQDiagonalMetricStrategy,
                                      SMAQFullMetricScalarStrategy)
    for strat in (IdentityScalarStrategy(128, bits=3, device="cpu"),
                  SMAQDiagonalMetricStrategy(128, bits=4, device="cpu"),
                  SMAQFullMetricScalarStrategy(128, bits=3, device="cpu")):
        assert key_format_of(strat) == SMAQ_KEYS_SCALAR
        qz = strat.quantizer
        for name in ("E", "E_inv", "centroids", "decision_boundaries"):
            assert getattr(qz, name) is not None
    assert SMAQDiagonalMetricStrategy.name == "smaq_diagonal_metric"
    assert IdentityScalarStrategy.name == "identity_scalar"
