"""Parity of the CUDA kernels (through the C-ABI) with the reference's golden vectors and the oracle."""

import numpy as np
import pytest

from oracle import smaq_oracle as O

pytestmark = pytest.mark.gpu

DT = {"fp32": "float32", "bf16": "bfloat16", "fp16": "float16"}


def tt(a, dtype, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(getattr(torch, DT[dtype]))


def tn(t):
    import torch
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.cpu().numpy()


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("gs", [32, 64])
@pytest.mark.parametrize("dn", ["fp32", "bf16", "fp16"])
def test_values_bit_exact_vs_reference(golden, cuda, bits, gs, dn):
    from smaq_b200 import ops
    p = f"vq_b{bits}_g{gs}_{dn}_"
    v = tt(golden[p + "v"], dn, cuda)
    data, scales, zeros = ops.quantize_values(v, bits, gs)
    assert np.array_equal(tn(data), golden[p + "data"])
    assert np.array_equal(tn(scales), golden[p + "scales"])
    assert np.array_equal(tn(zeros), golden[p + "zeros"])


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("dn", ["fp32", "bf16", "fp16"])
def test_scalar_keys_vs_reference(golden, cuda, bits, dn):
    from smaq_b200 import ops
    import torch
    p = f"sq_b{bits}_{dn}_"
    k = tt(golden[p + "k"], dn, cuda)
    E = torch.from_numpy(golden[f"sq_b{bits}_E"]).to(cuda)
    bnd = torch.from_numpy(golden[f"sq_b{bits}_boundaries"]).to(cuda)
    codes, norms = ops.quantize_keys_scalar(k, E, bnd, bits)
    orc = O.quantize_keys_scalar(golden[p + "k"], golden[f"sq_b{bits}_E"], golden[f"sq_b{bits}_boundaries"], bits, dn)
    got = O.unpack_indices(tn(codes), bits, 128)
    ref = O.unpack_indices(golden[p + "indices"], bits, 128)
    amb_tok = O.norm_ambiguous(orc["norm64"], dn)
    mism = (got != ref) & ~orc["near_boundary"] & ~amb_tok[..., None]
    assert mism.sum() == 0, f"{mism.sum()} code mismatches outside the rounding band"
    n_got, n_ref = tn(norms), golden[p + "norms"]
    if dn == "fp32":
        np.testing.assert_allclose(n_got, n_ref, rtol=1e-6, atol=0)
    else:
        bad = (n_got != n_ref) & ~amb_tok
        assert bad.sum() == 0


@pytest.mark.parametrize("dn", ["fp32", "bf16", "fp16"])
def test_bvq_keys_vs_reference(golden, cuda, dn):
    from smaq_b200 import ops
    import torch
    k = tt(golden[f"bvq_{dn}_k"], dn, cuda)
    Eb = torch.from_numpy(golden["bvq_E_blocks"]).to(cuda)
    C = torch.from_numpy(golden["bvq_centroids"]).to(cuda)
    idx = tn(ops.quantize_keys_bvq(k, Eb, C)).astype(np.int64)
    ref = golden[f"bvq_{dn}_indices"]
    orc = O.bvq_quantize(golden[f"bvq_{dn}_k"], golden["bvq_E_blocks"], golden["bvq_centroids"])
    bad = (idx != ref) & ~orc["near_tie"]
    assert bad.sum() == 0


HY = {"cfg0": ("scalar4", 4, "fp32"), "s3_bf16_gqa7": ("scalar3", 3, "bf16"), "s4_hist15": ("scalar4", 4, "bf16"),
      "s4_hist16": ("scalar4", 4, "bf16"), "s4_histonly": ("scalar4", 4, "bf16"),
      "s4_recentonly": ("scalar4", 4, "bf16"), "s4_empty": ("scalar4", 4, "bf16"),
      "bvq_bf16": ("bvq", 0, "bf16"), "bvq_fp32": ("bvq", 0, "fp32")}
RECENT_DT = {"cfg0": "fp16"}


def tol(dn):
    return 1e-5 if dn == "fp32" else 2e-3


@pytest.mark.parametrize("tag", list(HY))
def test_decode_vs_reference_golden(golden, cuda, tag):
    """Decode fed the reference's own quantized cache reproduces compute_hybrid_attention."""
    import torch
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_KEYS_BVQ, SMAQ_KEYS_SCALAR
    kind, bits, qd = HY[tag]
    p = f"hy_{tag}_"
    Hq, Hkv, nh, nr = (int(x) for x in golden[p + "meta"])
    D = 128
    kvd = qd
    rdt = RECENT_DT.get(tag, qd)
    q = tt(golden[p + "q"], qd, cuda)                      # [1, Hq, D]
    if nh:
        kc = torch.from_numpy(golden[p + "key_indices"].astype(np.uint8)).to(cuda).contiguous()
        vd = torch.from_numpy(golden[p + "v_data"].astype(np.uint8)).to(cuda)
        vs = tt(golden[p + "v_scales"], kvd, cuda)
        vz = tt(golden[p + "v_zeros"], kvd, cuda)
    else:
        kc = torch.zeros((Hkv, 1, 64), dtype=torch.uint8, device=cuda)
        vd = torch.zeros((Hkv, 1, 32), dtype=torch.uint8, device=cuda)
        vs = torch.zeros((Hkv, 1, 4), dtype=getattr(torch, DT[kvd]), device=cuda)
        vz = vs.clone()
    page = max(nh, 1)
    hl = torch.tensor([nh], dtype=torch.int32, device=cuda)
    kw = {}
    if kind == "bvq":
        kw.update(key_format=SMAQ_KEYS_BVQ, centroids=torch.from_numpy(golden["bvq_decoded_centroids"]).to(cuda))
    else:
        kn = tt(golden[p + "key_norms"], kvd, cuda) if nh else torch.zeros((Hkv, 1), dtype=vs.dtype, device=cuda)
        kw.update(key_format=SMAQ_KEYS_SCALAR, key_bits=bits, key_norms=kn,
                  E_inv=torch.from_numpy(golden[f"hy_{kind}_E_inv"]).to(cuda),
                  centroids=torch.from_numpy(golden[f"sq_b{bits}_centroids"]).to(cuda))
    if nr:
        rk = tt(golden[p + "recent_k"], rdt, cuda)[None]
        rv = tt(golden[p + "recent_v"], rdt, cuda)[None]
        rl = torch.tensor([nr], dtype=torch.int32, device=cuda)
    else:
        rk = rv = rl = None
    out = ops.decode(q, n_kv_heads=Hkv, key_codes=kc, v_data=vd, v_scales=vs, v_zeros=vz, hist_len=hl,
                     page_size=page, recent_k=rk, recent_v=rv, recent_len=rl, **kw)
    got = tn(out)
    ref = golden[p + "out"]
    assert got.shape == ref.shape
    assert O.rel_l2(got, ref) <= tol(qd), O.rel_l2(got, ref)
