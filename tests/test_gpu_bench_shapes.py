"""Parity at the benchmarked shapes: every fast kernel is run on one layer of exactly the data
``bench.py`` times (its own builders), and its output is compared with the oracle on a sample of
(sequence, KV head) pairs -- stream partitions over hundreds of segments, 32K-128K token
histories, the 16-token paged store, and the full configs[2] append batch.

Decode parity is isolated from quantize parity: the oracle reads back the rows the GPU wrote
(reference layout restored) and evaluates compute_hybrid_attention (smaq/score.py:23-72) per
pair in fp64; the bound is the north-star tolerance, rel-L2 <= 2e-3 for bf16 outputs.
"""

import numpy as np
import pytest

from oracle import smaq_oracle as O

pytestmark = pytest.mark.gpu
D = 128
TOL_BF16 = 2e-3


def tn(t):
    import torch
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.cpu().numpy()


@pytest.fixture(scope="module")
def codebook(cuda):
    import bench
    return bench.make_codebook(cuda)


def _bvq_pair_ref(L, vq, b, h, G):
    """Oracle output [G, D] of kv head h of sequence b from the GPU-written decode-layout rows."""
    from smaq_b200 import ops
    idx = tn(ops.bvq_to_reference(L["codes"][b, h])).astype(np.int64)            # [T, 16]
    K = O.bvq_dequantize(idx[None], tn(vq.decoded_centroids))                     # [1, T, D]
    V = O.dequantize_values(tn(ops.values_to_reference(L["vdata"][b, h]))[None], tn(L["vs"][b, h])[None],
                            tn(L["vz"][b, h])[None], 2, 32)
    q = tn(L["q"][b:b + 1, h * G:(h + 1) * G])
    ref, _, _ = O.hybrid_attention(q, "bf16", K, V, tn(L["rk"][b, :, h:h + 1]), tn(L["rv"][b, :, h:h + 1]), G, 1)
    return ref[0]


def _decode_one_layer(spec, cuda, vq, head0=0):
    import torch
    import bench
    from smaq_b200 import ops
    spec.layers = 1
    L = bench.build_layers(spec, cuda, vq, seed0=1, head0=head0)[0]
    hl = torch.full((spec.batch,), spec.ctx, dtype=torch.int32, device=cuda)
    rl = torch.full((spec.batch,), spec.window, dtype=torch.int32, device=cuda)
    ws = torch.empty(ops.decode_workspace_bytes(spec.batch, spec.hq, spec.hkv, D), dtype=torch.uint8, device=cuda)
    bench.decode_layer(spec, L, vq, hl, rl, ws, overlap=True)
    torch.cuda.synchronize()
    ops.decode_status(spec.batch, spec.hkv, ws)
    return L


def test_cfg1_layer_matches_oracle(cuda, codebook):
    """16 sequences x 8 KV heads x 32768 tokens + 128 window, G = 4 (one launch)."""
    import bench
    spec = bench.decode_spec("decode", 1)
    L = _decode_one_layer(spec, cuda, codebook)
    G = spec.hq // spec.hkv
    out = tn(L["out"])
    worst = 0.0
    for b in (0, 7, 15):
        for h in (range(spec.hkv) if b != 7 else (3,)):
            ref = _bvq_pair_ref(L, codebook, b, h, G)
            worst = max(worst, O.rel_l2(out[b, h * G:(h + 1) * G], ref))
    print(f"cfg1 worst rel-L2 {worst:.3e}")
    assert worst <= TOL_BF16, worst


def test_cfg4_layer_matches_oracle_and_head_shard(cuda, codebook):
    """4 sequences x 8 KV heads x 131072 tokens, G = 8 (one launch); and the same layer
    as 8-way KV-head sharding builds it on one rank (KV head 5 alone) gives the same rows."""
    import bench
    spec = bench.decode_spec("longctx", 1)
    L = _decode_one_layer(spec, cuda, codebook)
    G = spec.hq // spec.hkv
    out = tn(L["out"])
    worst = 0.0
    for b, h in ((0, 0), (0, 5), (3, 7), (2, 2)):
        ref = _bvq_pair_ref(L, codebook, b, h, G)
        worst = max(worst, O.rel_l2(out[b, h * G:(h + 1) * G], ref))
    print(f"cfg4 worst rel-L2 {worst:.3e}")
    assert worst <= TOL_BF16, worst
    shard = bench.decode_spec("longctx", 8)
    assert (shard.hq, shard.hkv) == (8, 1)
    Ls = _decode_one_layer(shard, cuda, codebook, head0=5)
    # the rank's data is KV head 5 of the full layer
    assert np.array_equal(tn(Ls["codes"][:, 0]), tn(L["codes"][:, 5]))
    got = tn(Ls["out"])
    for b in range(spec.batch):
        ref = _bvq_pair_ref(Ls, codebook, b, 0, G)
        assert O.rel_l2(got[b], ref) <= TOL_BF16
        assert O.rel_l2(got[b], out[b, 5 * G:6 * G]) <= TOL_BF16


def test_cfg3_paged_layer_matches_oracle(cuda):
    """64 sequences of 1K-64K tokens (seed 4) in a shuffled 16-token paged store,
    4-bit scalar keys, G = 7, 64-token window (one launch over 512 segments)."""
    import torch
    import bench
    from smaq_b200 import ops
    layers, quant, lens = bench.build_paged_layers(1, cuda)
    L = layers[0]
    hl = torch.from_numpy(lens.astype(np.int32)).to(cuda)
    rl = torch.full((bench.PG_B,), bench.PG_W, dtype=torch.int32, device=cuda)
    ws = torch.empty(ops.decode_workspace_bytes(bench.PG_B, bench.PG_HQ, bench.PG_HKV, D), dtype=torch.uint8,
                     device=cuda)
    bench.paged_decode(L, quant, hl, rl, ws, overlap=True)
    torch.cuda.synchronize()
    ops.decode_status(bench.PG_B, bench.PG_HKV, ws)
    out = tn(L["out"])
    bt = tn(L["bt"])
    codes_all = tn(ops.scalar_codes_to_reference(L["codes"]))
    vdata_all = tn(ops.values_to_reference(L["vdata"]))
    norms_all, vs_all, vz_all = tn(L["norms"]), tn(L["vs"]), tn(L["vz"])
    Einv, cent = tn(quant.E_inv), tn(quant.centroids)
    order = np.argsort(lens)
    worst = 0.0
    for b in (int(order[0]), int(order[-1]), int(order[len(order) // 2]), 5):
        n = int(lens[b])
        t = np.arange(n)
        pg, off = bt[b, t // bench.PG_PAGE], t % bench.PG_PAGE
        K = O.scalar_score_keys(codes_all[pg, :, off].transpose(1, 0, 2), norms_all[pg, :, off].T, bench.PG_BITS,
                                Einv, cent, D)
        V = O.dequantize_values(vdata_all[pg, :, off].transpose(1, 0, 2), vs_all[pg, :, off].transpose(1, 0, 2),
                                vz_all[pg, :, off].transpose(1, 0, 2), 2, 32)
        ref, _, _ = O.hybrid_attention(tn(L["q"][b:b + 1]), "bf16", K, V, tn(L["rk"][b]), tn(L["rv"][b]),
                                       bench.PG_HQ, bench.PG_HKV)
        worst = max(worst, O.rel_l2(out[b:b + 1], ref))
    print(f"cfg3 worst rel-L2 {worst:.3e}")
    assert worst <= TOL_BF16, worst


def test_cfg2_append_batch_matches_oracle(cuda):
    """8 x 8192 x 8 bf16 token-heads through the tcgen05 key kernel and the value
    kernel in one append.  On 65536 sampled rows: 3-bit codes bit-exact outside the fp32
    rounding band, norms bit-exact outside the bf16 midpoint band, values bit-exact.  Run three
    times: the output must not depend on scheduling."""
    import torch
    import bench
    from smaq_b200 import ops
    k, v, quant, o = bench.append_inputs(cuda)
    rows_total = k.shape[0] * k.shape[1]
    rng = np.random.default_rng(77)
    rows = np.sort(rng.choice(rows_total, size=65536, replace=False))
    ri = torch.from_numpy(rows).to(cuda)
    kr = k.reshape(rows_total, D).index_select(0, ri)
    vr = v.reshape(rows_total, D).index_select(0, ri)
    # decode-layout destination rows of token t, head h: (page t // 8192, head h, t % 8192)
    t, h = rows // bench.AP_H, rows % bench.AP_H
    dst = torch.from_numpy(((t // bench.AP_T) * bench.AP_H + h) * bench.AP_T + t % bench.AP_T).to(cuda)
    orc = O.quantize_keys_scalar(tn(kr), tn(quant.E), tn(quant.decision_boundaries), bench.AP_BITS, "bf16")
    amb = O.norm_ambiguous(orc["norm64"], "bf16")
    ov = O.quantize_values(tn(vr), 2, 32, "bf16")
    for _ in range(3):
        for x in o.values():
            x.zero_()
        bench.append_step(k, v, quant, o)
        torch.cuda.synchronize()
        ops.append_status()
        codes = tn(ops.scalar_codes_to_reference(o["codes"].index_select(0, dst)))
        got = O.unpack_indices(codes, bench.AP_BITS, D)
        mism = (got != orc["codes"]) & ~orc["near_boundary"] & ~amb[..., None]
        assert mism.sum() == 0, f"{mism.sum()} code mismatches outside the band"
        assert ((tn(o["norms"].index_select(0, dst)) != orc["norms"]) & ~amb).sum() == 0
        assert np.array_equal(tn(ops.values_to_reference(o["vd"].index_select(0, dst))), ov["data"])
        assert np.array_equal(tn(o["vs"].index_select(0, dst)), ov["scales"])
        assert np.array_equal(tn(o["vz"].index_select(0, dst)), ov["zeros"])
