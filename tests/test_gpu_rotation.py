"""RotationAdapter and the diagonal-metric strategy on the GPU (scalar-key kernels through the C
ABI), against the reference's golden vectors (tests/golden/golden_rotation.npz)."""

import os

import numpy as np
import pytest

from oracle import smaq_oracle as O
from smaq_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

GOLDEN_ROT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_rotation.npz")
CASES = ["identity3", "diag4", "rot3", "block2"]
DT = {"fp32": "float32", "bf16": "bfloat16"}


@pytest.fixture(scope="module")
def grot():
    return np.load(GOLDEN_ROT)


def tt(a, dn, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(getattr(torch, DT[dn]))


def tn(t):
    import torch
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.cpu().numpy()


def adapter(grot, tag, dev):
    import torch
    from smaq_b200.weighted_scalar import RotationAdapter, build_block_diagonal_metric_scales
    sig = torch.from_numpy(grot["ra_sigma"])
    R = torch.from_numpy(grot["ra_rotation"])
    kw = {"identity3": dict(coord_scales=torch.ones(128)), "diag4": dict(Sigma_q=sig),
          "rot3": dict(Sigma_q=sig, rotation=R),
          "block2": dict(coord_scales=build_block_diagonal_metric_scales(sig, 2))}[tag]
    return RotationAdapter(128, bits=int(grot[f"ra_{tag}_bits"]), device=dev, **kw)


@pytest.mark.parametrize("tag", CASES)
@pytest.mark.parametrize("dn", ["fp32", "bf16"])
def test_adapter_quantize_vs_reference(grot, cuda, tag, dn):
    """Kernel codes equal the reference's outside the fp32 rounding band; norms exact."""
    ad = adapter(grot, tag, cuda)
    bits = ad.bits
    qk = ad.quantize(tt(grot[f"ra_{dn}_k"], dn, cuda))
    got = O.unpack_indices(tn(qk.indices), bits, 128)
    ref = O.unpack_indices(grot[f"ra_{tag}_{dn}_indices"], bits, 128)
    orc = O.quantize_keys_scalar(grot[f"ra_{dn}_k"], tn(ad.E), grot[f"ra_{tag}_decision_boundaries"], bits, dn)
    amb = O.norm_ambiguous(orc["norm64"], dn)
    assert ((got != ref) & ~orc["near_boundary"] & ~amb[..., None]).sum() == 0
    if dn == "fp32":
        np.testing.assert_allclose(tn(qk.norms), grot[f"ra_{tag}_{dn}_norms"], rtol=1e-6)
    else:
        assert ((tn(qk.norms) != grot[f"ra_{tag}_{dn}_norms"]) & ~amb).sum() == 0


@pytest.mark.parametrize("tag", CASES)
@pytest.mark.parametrize("dn", ["fp32", "bf16"])
def test_adapter_scores_vs_reference(grot, cuda, tag, dn):
    """attention_score on the reference's own codes reproduces the reference's scores."""
    import torch
    from smaq_b200.quantizer import SMAQQuantized
    ad = adapter(grot, tag, cuda)
    qk = SMAQQuantized(indices=torch.from_numpy(grot[f"ra_{tag}_{dn}_indices"].astype(np.uint8)).to(cuda),
                       norms=tt(grot[f"ra_{tag}_{dn}_norms"], dn, cuda), bits=ad.bits)
    s = ad.attention_score(tt(grot[f"ra_{dn}_q"], dn, cuda), qk, scale=128 ** -0.5)
    assert O.rel_l2(tn(s), grot[f"ra_{tag}_{dn}_scores"]) <= (1e-5 if dn == "fp32" else 2e-3)
    if dn == "fp32":
        np.testing.assert_allclose(tn(ad.dequantize(qk)), grot[f"ra_{tag}_fp32_dequant"], rtol=1e-4, atol=1e-5)


def test_diagonal_metric_store_hybrid_vs_reference(grot, cuda):
    """CompressedKVStore keyed by SMAQDiagonalMetricStrategy (append kernels, fused decode) gives
    the reference's compute_hybrid_attention output."""
    import torch
    from smaq_b200.score import compute_hybrid_attention
    from smaq_b200.store import CompressedKVStore
    from smaq_b200.strategies import SMAQDiagonalMetricStrategy
    p = "ra_hy_"
    Hq, Hkv, nh, nr = (int(x) for x in grot[p + "meta"])
    strat = SMAQDiagonalMetricStrategy(128, bits=4, Sigma_q=torch.from_numpy(grot["ra_sigma"]),
                                       rotation=torch.from_numpy(grot["ra_rotation"]), device=cuda)
    store = CompressedKVStore(128, Hkv, key_bits=4, device=cuda, key_strategy=strat)
    hk = tt(grot[p + "hist_k"], "bf16", cuda)
    hv = torch.from_numpy(syn.values((nh, Hkv), 128, seed=66)).to(cuda).to(torch.bfloat16)
    store.append_chunk(hk[:70], hv[:70])
    store.append_chunk(hk[70:], hv[70:])
    # the store holds the reference's bytes (codes outside the rounding band, values exactly)
    flat = store.get_flat_cache()
    assert np.array_equal(tn(flat.value_q.data), grot[p + "v_data"])
    assert np.array_equal(tn(flat.value_q.scales), grot[p + "v_scales"])
    out = compute_hybrid_attention(tt(grot[p + "q"], "bf16", cuda), store, tt(grot[p + "recent_k"], "bf16", cuda),
                                   tt(grot[p + "recent_v"], "bf16", cuda), Hq)
    assert O.rel_l2(tn(out), grot[p + "out"]) <= 2e-3


def test_adapter_fit_picks_reference_choice(grot, cuda):
    """RotationAdapter.fit (keys quantized by the kernel) selects the reference's c and rotation
    choice, with the same held-out logit MSEs to 2%."""
    import torch
    from smaq_b200.weighted_scalar import RotationAdapter
    calq = torch.from_numpy(syn.calibration_queries(512, 128)).to(cuda)
    calk = torch.from_numpy(syn.keys((512,), 128, seed=64)).to(cuda)
    _, res = RotationAdapter.fit(128, 3, calq, calk, rotation=torch.from_numpy(grot["ra_rotation"]).to(cuda),
                                 c_values=[1.0, 5.0, 20.0], device=cuda)
    best_c, best_rot = grot["ra_fit_best"]
    assert res["best_c"] == best_c and res["best_use_rotation"] == bool(best_rot)
    np.testing.assert_allclose([r["lmse"] for r in res["all_results"]], grot["ra_fit_lmse"], rtol=2e-2)
