"""Generate the golden fixtures by running the REFERENCE implementation on CPU.

Usage::

    python tests/golden/make_golden.py [--reference PATH]

``PATH`` is a checkout of gauravsaini/smaq (the package directory ``smaq/``
must sit directly under it).  The reference is pure Python on PyTorch; it is
imported here, fed the seeded synthetic inputs of ``smaq_b200.synthetic``, and
its outputs are written to ``tests/golden/golden.npz`` and, for the rotation adapter
(smaq/weighted_scalar.py), ``tests/golden/golden_rotation.npz``, and for the exact-key
shadow strategy, ``tests/golden/golden_shadow.npz``.  bf16/fp16 tensors are
stored as float32 arrays holding exactly representable values.  The GPU box
never runs this script; the tests only read the ``.npz`` files it wrote.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from smaq_b200 import synthetic as syn  # noqa: E402


def t2n(t):
    import torch
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.detach().cpu().numpy()


def rotation_goldens(out):
    """RotationAdapter (smaq/weighted_scalar.py) and its strategies: scales, codebooks, codes,
    norms, scores, calibration choice and a hybrid decode through the store."""
    import torch
    from smaq.weighted_scalar import (RotationAdapter, build_block_diagonal_metric_scales,
                                      build_rotated_diagonal_metric_scales)
    from smaq.strategies import SMAQDiagonalMetricStrategy
    from smaq.store import CompressedKVStore
    from smaq.score import compute_hybrid_attention
    D = 128
    cpu = torch.device("cpu")
    calq = torch.from_numpy(syn.calibration_queries(512, D))
    sig = (calq.T @ calq) / calq.shape[0]
    R = torch.linalg.qr(torch.from_numpy(np.random.default_rng(61).standard_normal((D, D)).astype(np.float32)))[0]
    out["ra_sigma"] = t2n(sig)
    out["ra_rotation"] = t2n(R)
    out["ra_scales_rot"] = t2n(build_rotated_diagonal_metric_scales(sig, rotation=R))
    out["ra_scales_norot"] = t2n(build_rotated_diagonal_metric_scales(sig))
    out["ra_scales_block2"] = t2n(build_block_diagonal_metric_scales(sig, block_size=2))
    out["ra_scales_block3"] = t2n(build_block_diagonal_metric_scales(sig, block_size=3))
    DT = {"fp32": torch.float32, "bf16": torch.bfloat16}
    kq = syn.keys((48, 4), D, seed=62).reshape(192, D)
    kq[0] = 0.0
    qq = syn.queries((6,), D, seed=63)
    cases = {
        "identity3": dict(bits=3, coord_scales=torch.ones(D)),
        "diag4": dict(bits=4, Sigma_q=sig),
        "rot3": dict(bits=3, Sigma_q=sig, rotation=R),
        "block2": dict(bits=2, coord_scales=build_block_diagonal_metric_scales(sig, block_size=2)),
    }
    for dn, dt in DT.items():
        out[f"ra_{dn}_k"] = t2n(torch.from_numpy(kq).to(dt))
        out[f"ra_{dn}_q"] = t2n(torch.from_numpy(qq).to(dt))
    for tag, kw in cases.items():
        ad = RotationAdapter(D, device=cpu, **kw)
        p = f"ra_{tag}_"
        for name in ("coord_scales", "inv_coord_scales", "centroids", "decision_boundaries"):
            out[p + name] = t2n(getattr(ad, name))
        out[p + "bits"] = np.array(kw["bits"], np.int64)
        out[p + "rotated"] = np.array("rotation" in kw)
        for dn, dt in DT.items():
            qk = ad.quantize(torch.from_numpy(kq).to(dt))
            out[p + dn + "_indices"] = t2n(qk.indices)
            out[p + dn + "_norms"] = t2n(qk.norms)
            if dn == "fp32":
                out[p + dn + "_dequant"] = t2n(ad.dequantize(qk))
            qt = torch.from_numpy(qq).to(dt)
            out[p + dn + "_scores"] = t2n(ad.attention_score(qt, qk, scale=D ** -0.5))
    # calibration: c and rotation-or-identity by held-out logit MSE
    calk = torch.from_numpy(syn.keys((512,), D, seed=64))
    _, res = RotationAdapter.fit(D, 3, calq, calk, rotation=R, c_values=[1.0, 5.0, 20.0], device=cpu)
    out["ra_fit_best"] = np.array([res["best_c"], float(res["best_use_rotation"])], np.float64)
    out["ra_fit_lmse"] = np.array([r["lmse"] for r in res["all_results"]], np.float64)
    # hybrid decode through a store keyed by the diagonal-metric strategy (bf16, GQA 4)
    strat = SMAQDiagonalMetricStrategy(D, bits=4, Sigma_q=sig, rotation=R, device=cpu)
    Hq, Hkv, nh, nr = 16, 4, 200, 40
    hk = torch.from_numpy(syn.keys((nh, Hkv), D, seed=65)).to(torch.bfloat16)
    hv = torch.from_numpy(syn.values((nh, Hkv), D, seed=66)).to(torch.bfloat16)
    rk = torch.from_numpy(syn.keys((nr, Hkv), D, seed=67)).to(torch.bfloat16)
    rv = torch.from_numpy(syn.values((nr, Hkv), D, seed=68)).to(torch.bfloat16)
    q = torch.from_numpy(syn.queries((1, Hq), D, seed=69)).to(torch.bfloat16)
    store = CompressedKVStore(D, Hkv, key_bits=4, device=cpu, key_strategy=strat)
    store.append_chunk(hk[:70], hv[:70])
    store.append_chunk(hk[70:], hv[70:])
    o = compute_hybrid_attention(q, store, rk, rv, Hq)
    flat = store.get_flat_cache()
    p = "ra_hy_"
    for name, t in (("hist_k", hk), ("recent_k", rk), ("recent_v", rv), ("q", q), ("out", o),
                    ("key_indices", flat.key_q.indices), ("key_norms", flat.key_q.norms),
                    ("v_data", flat.value_q.data), ("v_scales", flat.value_q.scales),
                    ("v_zeros", flat.value_q.zeros), ("coord_scales", strat.quantizer.coord_scales),
                    ("centroids", strat.quantizer.centroids),
                    ("decision_boundaries", strat.quantizer.decision_boundaries)):
        out[p + name] = t2n(t)
    out[p + "meta"] = np.array([Hq, Hkv, nh, nr], np.int64)


def shadow_goldens(out):
    """ExactShadowStrategy (smaq/strategies.py:258-298) through the store and
    compute_hybrid_attention: exact history keys, 2-bit values, bf16 and fp32."""
    import torch
    from smaq.strategies import ExactShadowStrategy
    from smaq.store import CompressedKVStore
    from smaq.score import compute_hybrid_attention
    D = 128
    cpu = torch.device("cpu")
    cases = (("bf16", torch.bfloat16, 28, 4, 300, 64, 700), ("bf16_histonly", torch.bfloat16, 8, 2, 120, 0, 710),
             ("fp32", torch.float32, 8, 2, 150, 10, 720), ("hist15", torch.bfloat16, 8, 2, 15, 20, 730))
    for tag, dt, Hq, Hkv, nh, nr, seed in cases:
        hk = torch.from_numpy(syn.keys((nh, Hkv), D, seed=seed)).to(dt)
        hv = torch.from_numpy(syn.values((nh, Hkv), D, seed=seed + 1)).to(dt)
        rk = torch.from_numpy(syn.keys((nr, Hkv), D, seed=seed + 2)).to(dt) if nr else None
        rv = torch.from_numpy(syn.values((nr, Hkv), D, seed=seed + 3)).to(dt) if nr else None
        q = torch.from_numpy(syn.queries((1, Hq), D, seed=seed + 4)).to(dt)
        store = CompressedKVStore(D, Hkv, device=cpu, key_strategy=ExactShadowStrategy())
        h1 = nh // 3
        store.append_chunk(hk[:h1], hv[:h1])
        store.append_chunk(hk[h1:], hv[h1:])
        o = compute_hybrid_attention(q, store, rk, rv, Hq)
        p = f"sh_{tag}_"
        flat = store.get_flat_cache()
        for name, t in (("hist_k", hk), ("hist_v", hv), ("q", q), ("out", o), ("v_data", flat.value_q.data)):
            out[p + name] = t2n(t)
        if nr:
            out[p + "recent_k"], out[p + "recent_v"] = t2n(rk), t2n(rv)
        out[p + "meta"] = np.array([Hq, Hkv, nh, nr], np.int64)
        out[p + "memory_bytes"] = np.array([store.memory_bytes()], np.int64)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SMAQ_REFERENCE"),
                    help="checkout of gauravsaini/smaq (or set SMAQ_REFERENCE)")
    ap.add_argument("--only", choices=["all", "rotation", "shadow"], default="all",
                    help="rotation: write only golden_rotation.npz; shadow: only golden_shadow.npz")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference PATH (or SMAQ_REFERENCE) is required")
    sys.path.insert(0, args.reference)
    import torch
    if args.only in ("all", "shadow"):
        import smaq  # the reference package
        assert "reference" in smaq.__file__ or args.reference in smaq.__file__, smaq.__file__
        sh = {}
        shadow_goldens(sh)
        path = os.path.join(HERE, "golden_shadow.npz")
        np.savez_compressed(path, **sh)
        print("wrote", path, os.path.getsize(path) // 1024, "KiB,", len(sh), "arrays")
        if args.only == "shadow":
            return
    if args.only in ("all", "rotation"):
        import smaq  # the reference package
        assert "reference" in smaq.__file__ or args.reference in smaq.__file__, smaq.__file__
        rot = {}
        rotation_goldens(rot)
        path = os.path.join(HERE, "golden_rotation.npz")
        np.savez_compressed(path, **rot)
        print("wrote", path, os.path.getsize(path) // 1024, "KiB,", len(rot), "arrays")
        if args.only == "rotation":
            return
    torch.set_num_threads(os.cpu_count() or 1)
    import smaq  # the reference package
    from smaq.quantizer import SMAQQuantizer
    from smaq.kv_cache import quantize_values, dequantize_values
    from smaq.block_vq import SMAQBlockVQ
    from smaq.store import CompressedKVStore
    from smaq.strategies import SMAQBlockVQStrategy, SMAQFullMetricScalarStrategy
    from smaq.score import compute_hybrid_attention
    from smaq.capture import KVCaptureEngine

    assert "reference" in smaq.__file__ or args.reference in smaq.__file__, smaq.__file__
    DT = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}
    D = 128
    calq = syn.calibration_queries(512, D)
    out = {}

    # ---------------- scalar key quantization -------------------------------
    kq = syn.keys((48, 4), D)
    kq[0, 0] = 0.0                          # zero key: y = 0 sits on the middle boundary
    kq[1, 1] = kq[1, 1] * 1e-3              # tiny norm
    for bits in (2, 3, 4):
        quant = SMAQQuantizer(D, bits=bits, device=torch.device("cpu"))
        quant.fit(torch.from_numpy(calq))
        for dn, dt in DT.items():
            kt = torch.from_numpy(kq).to(dt)
            qk = quant.quantize(kt)
            p = f"sq_b{bits}_{dn}_"
            out[p + "k"] = t2n(kt)
            out[p + "indices"] = t2n(qk.indices)
            out[p + "norms"] = t2n(qk.norms)
            deq = quant.dequantize(qk)
            out[p + "dequant"] = t2n(deq)
        out[f"sq_b{bits}_E"] = t2n(quant.E)
        out[f"sq_b{bits}_E_inv"] = t2n(quant.E_inv)
        out[f"sq_b{bits}_centroids"] = t2n(quant.centroids)
        out[f"sq_b{bits}_boundaries"] = t2n(quant.decision_boundaries)

    # ---------------- value codec --------------------------------------------
    vv = syn.values((40, 4), D)
    vv[0, 0, :32] = 0.75                    # constant group -> scale clamps to 1e-10
    vv[0, 1, 32:64] = np.linspace(-1.5, 1.5, 32)  # exact .5 ties for round-half-even
    vv[2, 3, :] *= 1e-12                    # sub-1e-10 ranges
    for bits in (2, 4):
        for gs in (32, 64):
            for dn, dt in DT.items():
                vt = torch.from_numpy(vv).to(dt)
                vq = quantize_values(vt, bits=bits, group_size=gs)
                p = f"vq_b{bits}_g{gs}_{dn}_"
                out[p + "v"] = t2n(vt)
                out[p + "data"] = t2n(vq.data)
                out[p + "scales"] = t2n(vq.scales)
                out[p + "zeros"] = t2n(vq.zeros)
                out[p + "dequant"] = t2n(dequantize_values(vq, gs))

    # ---------------- block VQ ----------------------------------------------
    calk = syn.keys((4096,), D, seed=11)
    vq = SMAQBlockVQ(D, device=torch.device("cpu"))
    vq.fit(torch.from_numpy(calk), torch.from_numpy(syn.calibration_queries(4096, D, seed=12)))
    # the fitted tables as the reference's k-means produced them (before any rounding)
    for name in ("E_blocks", "E_inv_blocks", "centroids", "decoded_centroids"):
        out["bvq_fit_" + name] = t2n(getattr(vq, name)).copy()
    # fp16 codebook: reference buffers rounded to fp16-representable values
    for name in ("E_blocks", "E_inv_blocks", "centroids", "decoded_centroids"):
        getattr(vq, name).copy_(getattr(vq, name).half().float())
    kb = syn.keys((64, 4), D, seed=13)
    for dn, dt in DT.items():
        kt = torch.from_numpy(kb).to(dt)
        q = vq.quantize(kt)
        out[f"bvq_{dn}_k"] = t2n(kt)
        out[f"bvq_{dn}_indices"] = t2n(q.indices)
        out[f"bvq_{dn}_dequant"] = t2n(vq.dequantize(q))
    for name in ("E_blocks", "E_inv_blocks", "centroids", "decoded_centroids"):
        out["bvq_" + name] = t2n(getattr(vq, name))

    # ---------------- hybrid attention through the store ---------------------
    def run_case(tag, key_strategy, Hq, Hkv, n_hist, n_recent, q_dtype, kv_dtype, recent_dtype, seed):
        hk = syn.keys((n_hist, Hkv), D, seed=seed)
        hv = syn.values((n_hist, Hkv), D, seed=seed + 1)
        rk = syn.keys((n_recent, Hkv), D, seed=seed + 2)
        rv = syn.values((n_recent, Hkv), D, seed=seed + 3)
        qq = syn.queries((1, Hq), D, seed=seed + 4)
        store = CompressedKVStore(D, Hkv, key_bits=getattr(key_strategy, "bits", 3),
                                  device=torch.device("cpu"), key_strategy=key_strategy)
        if n_hist:
            # two chunks: exercises the concat path of get_flat_cache
            h1 = n_hist // 3
            kt = torch.from_numpy(hk).to(kv_dtype)
            vt = torch.from_numpy(hv).to(kv_dtype)
            if h1:
                store.append_chunk(kt[:h1], vt[:h1])
            store.append_chunk(kt[h1:], vt[h1:])
        rkt = torch.from_numpy(rk).to(recent_dtype) if n_recent else None
        rvt = torch.from_numpy(rv).to(recent_dtype) if n_recent else None
        qt = torch.from_numpy(qq).to(q_dtype)
        o = compute_hybrid_attention(qt, store, rkt, rvt, Hq)
        p = f"hy_{tag}_"
        if n_hist * Hkv <= 2048:  # raw history only for the small cases (size of the fixture)
            out[p + "hist_k"] = t2n(torch.from_numpy(hk).to(kv_dtype))
            out[p + "hist_v"] = t2n(torch.from_numpy(hv).to(kv_dtype))
        out[p + "recent_k"] = t2n(torch.from_numpy(rk).to(recent_dtype))
        out[p + "recent_v"] = t2n(torch.from_numpy(rv).to(recent_dtype))
        out[p + "q"] = t2n(qt)
        out[p + "out"] = t2n(o)
        out[p + "meta"] = np.array([Hq, Hkv, n_hist, n_recent], np.int64)
        flat = store.get_flat_cache()
        if flat is not None:
            kq_ = flat.key_q
            if hasattr(kq_, "norms"):
                out[p + "key_indices"] = t2n(kq_.indices)
                out[p + "key_norms"] = t2n(kq_.norms)
            else:
                out[p + "key_indices"] = t2n(kq_.indices)
            out[p + "v_data"] = t2n(flat.value_q.data)
            out[p + "v_scales"] = t2n(flat.value_q.scales)
            out[p + "v_zeros"] = t2n(flat.value_q.zeros)

    def scalar_strategy(bits):
        s = SMAQFullMetricScalarStrategy(D, bits=bits, device=torch.device("cpu"))
        s.fit(torch.from_numpy(calq))
        return s

    s4 = scalar_strategy(4)
    out["hy_scalar4_E"] = t2n(s4.quantizer.E)
    out["hy_scalar4_E_inv"] = t2n(s4.quantizer.E_inv)
    # config 0 at full size: fp32, 32/8 heads, 2048 history + 128 fp16 recent
    run_case("cfg0", s4, 32, 8, 2048, 128, torch.float32, torch.float32, torch.float16, 100)
    s3 = scalar_strategy(3)
    out["hy_scalar3_E"] = t2n(s3.quantizer.E)
    out["hy_scalar3_E_inv"] = t2n(s3.quantizer.E_inv)
    run_case("s3_bf16_gqa7", s3, 28, 4, 300, 64, torch.bfloat16, torch.bfloat16, torch.bfloat16, 200)
    run_case("s4_hist15", s4, 8, 2, 15, 20, torch.bfloat16, torch.bfloat16, torch.bfloat16, 300)
    run_case("s4_hist16", s4, 8, 2, 16, 20, torch.bfloat16, torch.bfloat16, torch.bfloat16, 310)
    run_case("s4_histonly", s4, 8, 2, 200, 0, torch.bfloat16, torch.bfloat16, torch.bfloat16, 320)
    run_case("s4_recentonly", s4, 8, 2, 0, 33, torch.bfloat16, torch.bfloat16, torch.bfloat16, 330)
    run_case("s4_empty", s4, 8, 2, 0, 0, torch.bfloat16, torch.bfloat16, torch.bfloat16, 340)
    bstrat = SMAQBlockVQStrategy(D, device=torch.device("cpu"))
    bstrat.quantizer = vq
    run_case("bvq_bf16", bstrat, 32, 8, 400, 128, torch.bfloat16, torch.bfloat16, torch.bfloat16, 400)
    run_case("bvq_fp32", bstrat, 8, 2, 150, 10, torch.float32, torch.float32, torch.float32, 410)
    # bf16 block VQ with the raw history kept (fits the fixture): replayed through the store
    run_case("bvq_bf16_store", bstrat, 16, 4, 300, 64, torch.bfloat16, torch.bfloat16, torch.bfloat16, 420)

    # ---------------- capture engine flush pattern (RingBuffer, F13) ---------
    store = CompressedKVStore(D, 2, key_bits=3, device=torch.device("cpu"))
    eng = KVCaptureEngine(store, ring_capacity=8, device=torch.device("cpu"), dtype=torch.float32)
    kk = torch.from_numpy(syn.keys((40, 2), D, seed=500))
    vvv = torch.from_numpy(syn.values((40, 2), D, seed=501))
    eng.ingest_prefill(kk[:13], vvv[:13], 13)
    trace = [store.num_tokens, eng.ring.size]
    for t in range(13, 40):
        eng.ingest_decode(kk[t:t + 1], vvv[t:t + 1], 1)
        trace += [store.num_tokens, eng.ring.size]
    out["capture_trace"] = np.array(trace, np.int64)
    out["capture_chunks"] = np.array(store._chunk_lengths, np.int64)

    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path) // 1024, "KiB,", len(out), "arrays")


if __name__ == "__main__":
    main()
