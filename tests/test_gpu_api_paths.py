"""The reference-facing API runs the fast kernels.

``CompressedKVStore`` (smaq/store.py:28-130) keeps bf16 rows in the decode byte order, and
``compute_hybrid_attention`` (smaq/score.py:23-72) then selects the one-launch tensor-core
kernels: block-VQ keys with an fp16-valued codebook, and 3/4-bit SMAQ scalar keys.  Each case
replays a golden store the reference built (same chunks, same tables) and checks the output
against the reference's, the flat-cache bytes against the reference's, and the kernel path.
"""

import numpy as np
import pytest

from oracle import smaq_oracle as O

pytestmark = pytest.mark.gpu
D = 128


def tn(t):
    import torch
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.cpu().numpy()


def tt(a, dev, dtype=None):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dtype or torch.bfloat16)


def _scalar_store(golden, cuda, bits=3, tag="s3_bf16_gqa7"):
    import torch
    from smaq_b200.store import CompressedKVStore
    from smaq_b200.strategies import SMAQFullMetricScalarStrategy
    p = f"hy_{tag}_"
    Hq, Hkv, nh, nr = (int(x) for x in golden[p + "meta"])
    strat = SMAQFullMetricScalarStrategy(D, bits=bits, device=cuda)
    strat.quantizer.E.copy_(torch.from_numpy(golden[f"hy_scalar{bits}_E"]))
    strat.quantizer.E_inv.copy_(torch.from_numpy(golden[f"hy_scalar{bits}_E_inv"]))
    store = CompressedKVStore(D, Hkv, key_bits=bits, device=cuda, key_strategy=strat)
    hk, hv = tt(golden[p + "hist_k"], cuda), tt(golden[p + "hist_v"], cuda)
    h1 = nh // 3                     # the reference's two chunks
    store.append_chunk(hk[:h1], hv[:h1])
    store.append_chunk(hk[h1:], hv[h1:])
    return store, (Hq, Hkv, nh, nr), p


def test_scalar_store_runs_fused_kernel_and_matches_reference(golden, cuda):
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_LAYOUT_DECODE
    from smaq_b200.score import compute_hybrid_attention, hybrid_kernel_path
    store, (Hq, Hkv, nh, nr), p = _scalar_store(golden, cuda)
    assert store.layout == SMAQ_LAYOUT_DECODE
    q, rk, rv = tt(golden[p + "q"], cuda), tt(golden[p + "recent_k"], cuda), tt(golden[p + "recent_v"], cuda)
    assert hybrid_kernel_path(q, store, rk, rv, Hq) == ops.PATH_FUSED_SCALAR
    out = compute_hybrid_attention(q, store, rk, rv, Hq)
    assert O.rel_l2(tn(out), golden[p + "out"]) <= 2e-3
    # the flat cache is the reference's view: its bytes, in its order
    flat = store.get_flat_cache()
    assert np.array_equal(tn(flat.value_q.data), golden[p + "v_data"])
    assert np.array_equal(tn(flat.value_q.scales), golden[p + "v_scales"])
    got = O.unpack_indices(tn(flat.key_q.indices), 3, D)
    ref = O.unpack_indices(golden[p + "key_indices"], 3, D)
    hk = golden[p + "hist_k"].transpose(1, 0, 2)                       # [Hkv, n, D]
    orc = O.quantize_keys_scalar(hk, golden["hy_scalar3_E"], golden["sq_b3_boundaries"], 3, "bf16")
    assert ((got != ref) & ~orc["near_boundary"]).sum() == 0


def test_scalar_store_fp32_query_takes_general_kernel(golden, cuda):
    """An fp32 query on a bf16 decode-layout store runs the general kernel, which reads the
    permuted rows correctly (oracle on the flat cache, fp32 tolerance)."""
    import torch
    from smaq_b200 import ops
    from smaq_b200.score import compute_hybrid_attention, hybrid_kernel_path
    store, (Hq, Hkv, nh, nr), p = _scalar_store(golden, cuda)
    q = tt(golden[p + "q"], cuda, torch.float32)
    rk, rv = tt(golden[p + "recent_k"], cuda), tt(golden[p + "recent_v"], cuda)
    assert hybrid_kernel_path(q, store, rk, rv, Hq) == ops.PATH_GENERAL
    out = compute_hybrid_attention(q, store, rk, rv, Hq)
    flat = store.get_flat_cache()
    qz = store.key_strategy.quantizer
    K = O.scalar_score_keys(tn(flat.key_q.indices), tn(flat.key_q.norms), 3, tn(qz.E_inv), tn(qz.centroids), D)
    V = O.dequantize_values(tn(flat.value_q.data), tn(flat.value_q.scales), tn(flat.value_q.zeros), 2, 32)
    ref, _, _ = O.hybrid_attention(tn(q), "fp32", K, V, tn(rk), tn(rv), Hq, Hkv)
    assert O.rel_l2(tn(out), ref) <= 1e-5


def test_bvq_store_runs_fused_kernel_and_matches_reference(golden, cuda):
    import torch
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_LAYOUT_DECODE
    from smaq_b200.score import compute_hybrid_attention, hybrid_kernel_path
    from smaq_b200.store import CompressedKVStore
    from smaq_b200.strategies import SMAQBlockVQStrategy
    p = "hy_bvq_bf16_store_"
    Hq, Hkv, nh, nr = (int(x) for x in golden[p + "meta"])
    strat = SMAQBlockVQStrategy(D, device=cuda)
    vq = strat.quantizer
    for name in ("E_blocks", "E_inv_blocks", "centroids", "decoded_centroids"):
        setattr(vq, name, torch.from_numpy(golden["bvq_" + name]).to(cuda))
    store = CompressedKVStore(D, Hkv, device=cuda, key_strategy=strat)
    hk, hv = tt(golden[p + "hist_k"], cuda), tt(golden[p + "hist_v"], cuda)
    h1 = nh // 3
    store.append_chunk(hk[:h1], hv[:h1])
    store.append_chunk(hk[h1:], hv[h1:])
    assert store.layout == SMAQ_LAYOUT_DECODE
    q, rk, rv = tt(golden[p + "q"], cuda), tt(golden[p + "recent_k"], cuda), tt(golden[p + "recent_v"], cuda)
    assert vq.fp16_codebook() is not None
    assert hybrid_kernel_path(q, store, rk, rv, Hq) == ops.PATH_FUSED_BVQ
    out = compute_hybrid_attention(q, store, rk, rv, Hq)
    assert O.rel_l2(tn(out), golden[p + "out"]) <= 2e-3
    flat = store.get_flat_cache()
    ref = golden[p + "key_indices"]
    got = tn(flat.key_q.indices)
    # indices equal the reference's except at near-ties of the block distance
    assert (got != ref).mean() < 1e-3
    assert np.array_equal(tn(flat.value_q.data), golden[p + "v_data"])
    # the flat cache holds the bytes the oracle scores: same output from them
    K = O.bvq_dequantize(got.astype(np.int64), golden["bvq_decoded_centroids"])
    V = O.dequantize_values(tn(flat.value_q.data), tn(flat.value_q.scales), tn(flat.value_q.zeros), 2, 32)
    orc, _, _ = O.hybrid_attention(tn(q), "bf16", K, V, tn(rk), tn(rv), Hq, Hkv)
    assert O.rel_l2(tn(out), orc) <= 2e-3
