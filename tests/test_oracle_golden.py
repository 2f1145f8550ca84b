"""The CPU oracle against the golden vectors the reference produced (no GPU)."""

import numpy as np
import pytest

from oracle import smaq_oracle as O


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("dn", ["fp32", "bf16", "fp16"])
def test_scalar_keys(golden, bits, dn):
    p = f"sq_b{bits}_{dn}_"
    r = O.quantize_keys_scalar(golden[p + "k"], golden[f"sq_b{bits}_E"], golden[f"sq_b{bits}_boundaries"], bits, dn)
    ref = O.unpack_indices(golden[p + "indices"], bits, 128)
    assert ((ref != r["codes"]) & ~r["near_boundary"]).sum() == 0
    if dn == "fp32":
        np.testing.assert_allclose(r["norms"], golden[p + "norms"], rtol=1e-6)
    else:
        assert np.array_equal(r["norms"], golden[p + "norms"])
    # the pack/unpack restatement round-trips the reference's bytes
    assert np.array_equal(O.pack_indices(ref, bits), golden[p + "indices"])


def test_scalar_codebook_matches_reference(golden):
    for bits in (2, 3, 4):
        c, b = O.scalar_codebook(bits)
        np.testing.assert_allclose(c, golden[f"sq_b{bits}_centroids"], rtol=2e-7, atol=1e-7)
        np.testing.assert_allclose(b, golden[f"sq_b{bits}_boundaries"], rtol=2e-7, atol=1e-7)


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("gs", [32, 64])
@pytest.mark.parametrize("dn", ["fp32", "bf16", "fp16"])
def test_values_bit_exact(golden, bits, gs, dn):
    p = f"vq_b{bits}_g{gs}_{dn}_"
    with np.errstate(invalid="ignore"):
        r = O.quantize_values(golden[p + "v"], bits, gs, dn)
    for k in ("data", "scales", "zeros"):
        assert np.array_equal(r[k], golden[p + k]), k
    dq = O.dequantize_values(golden[p + "data"], golden[p + "scales"], golden[p + "zeros"], bits, gs)
    assert np.array_equal(dq, golden[p + "dequant"])


@pytest.mark.parametrize("dn", ["fp32", "bf16", "fp16"])
def test_bvq(golden, dn):
    r = O.bvq_quantize(golden[f"bvq_{dn}_k"], golden["bvq_E_blocks"], golden["bvq_centroids"])
    ref = golden[f"bvq_{dn}_indices"]
    assert ((r["indices"] != ref) & ~r["near_tie"]).sum() == 0
    dq = O.bvq_dequantize(ref, golden["bvq_decoded_centroids"])
    np.testing.assert_array_equal(dq.astype(np.float32), golden[f"bvq_{dn}_dequant"])


HY = {"cfg0": ("scalar4", 4, "fp32"), "s3_bf16_gqa7": ("scalar3", 3, "bf16"), "s4_hist15": ("scalar4", 4, "bf16"),
      "s4_hist16": ("scalar4", 4, "bf16"), "s4_histonly": ("scalar4", 4, "bf16"),
      "s4_recentonly": ("scalar4", 4, "bf16"), "s4_empty": ("scalar4", 4, "bf16"),
      "bvq_bf16": ("bvq", 0, "bf16"), "bvq_fp32": ("bvq", 0, "fp32")}


@pytest.mark.parametrize("tag", list(HY))
def test_hybrid_attention(golden, tag):
    kind, bits, qd = HY[tag]
    p = f"hy_{tag}_"
    Hq, Hkv, nh, nr = (int(x) for x in golden[p + "meta"])
    K = V = None
    if nh:
        if kind == "bvq":
            K = O.bvq_dequantize(golden[p + "key_indices"], golden["bvq_decoded_centroids"])
        else:
            K = O.scalar_score_keys(golden[p + "key_indices"], golden[p + "key_norms"], bits,
                                    golden[f"hy_{kind}_E_inv"], golden[f"sq_b{bits}_centroids"], 128)
        V = O.dequantize_values(golden[p + "v_data"], golden[p + "v_scales"], golden[p + "v_zeros"], 2, 32)
    rk = golden[p + "recent_k"] if nr else None
    rv = golden[p + "recent_v"] if nr else None
    out, _, _ = O.hybrid_attention(golden[p + "q"], qd, K, V, rk, rv, Hq, Hkv)
    assert O.rel_l2(out, golden[p + "out"]) <= (1e-5 if qd == "fp32" else 2e-3)


@pytest.mark.parametrize("tag", ["s3_bf16_gqa7", "s4_hist16", "s4_histonly"])
def test_store_roundtrip_from_raw(golden, tag):
    """From the raw history, oracle quantization reproduces the reference's stored bytes."""
    kind, bits, qd = HY[tag]
    p = f"hy_{tag}_"
    hk, hv = golden[p + "hist_k"], golden[p + "hist_v"]        # [N, Hkv, D]
    kt = hk.transpose(1, 0, 2)
    r = O.quantize_keys_scalar(kt, golden[f"hy_{kind}_E"], golden[f"sq_b{bits}_boundaries"], bits, qd)
    ref = O.unpack_indices(golden[p + "key_indices"], bits, 128)
    assert ((ref != r["codes"]) & ~r["near_boundary"]).sum() == 0
    vq = O.quantize_values(hv.transpose(1, 0, 2), 2, 32, qd)
    assert np.array_equal(vq["data"], golden[p + "v_data"])
    assert np.array_equal(vq["scales"], golden[p + "v_scales"])
