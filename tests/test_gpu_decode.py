"""Batched / paged decode and append through slot mappings, checked against the oracle."""

import numpy as np
import pytest

from oracle import smaq_oracle as O
from smaq_b200 import synthetic as syn

pytestmark = pytest.mark.gpu
D = 128


def tn(t):
    import torch
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.cpu().numpy()


def scalar_tables(bits, dev):
    import torch
    from smaq_b200.quantizer import SMAQQuantizer
    qz = SMAQQuantizer(D, bits=bits, device=dev)
    qz.fit(torch.from_numpy(syn.calibration_queries(512, D)).to(dev))
    return qz


def random_codebook(dev, seed=7):
    import torch
    rng = np.random.default_rng(seed)
    Eb = (np.eye(8)[None] + 0.1 * rng.standard_normal((16, 8, 8))).astype(np.float32)
    C = rng.standard_normal((16, 256, 8)).astype(np.float32)
    # fp16-valued decoded codebook (like BASELINE config 1's), so the tensor-core path applies
    dec = (rng.standard_normal((16, 256, 8)) * 0.5).astype(np.float16).astype(np.float32)
    return [torch.from_numpy(x).to(dev) for x in (Eb, C, dec)]


def build_paged(dev, kind, bits, B, Hkv, hist, page_size, dtype, seed):
    """Quantize per-sequence histories into a shuffled paged store via slot mappings."""
    import torch
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_KEYS_BVQ, SMAQ_KEYS_SCALAR
    rng = np.random.default_rng(seed)
    pages_per = [(int(n) + page_size - 1) // page_size for n in hist]
    n_pages = max(1, sum(pages_per))
    perm = rng.permutation(n_pages)
    maxp = max(1, max(pages_per))
    bt = np.zeros((B, maxp), np.int32)
    o = 0
    for b in range(B):
        bt[b, :pages_per[b]] = perm[o:o + pages_per[b]]
        o += pages_per[b]
    P = ops.packed_dim(D, bits) if kind == "scalar" else 16
    tdt = getattr(torch, dtype)
    st = {
        "codes": torch.zeros((n_pages, Hkv, page_size, P), dtype=torch.uint8, device=dev),
        "norms": torch.zeros((n_pages, Hkv, page_size), dtype=tdt, device=dev),
        "vdata": torch.zeros((n_pages, Hkv, page_size, D // 4), dtype=torch.uint8, device=dev),
        "vs": torch.zeros((n_pages, Hkv, page_size, D // 32), dtype=tdt, device=dev),
        "vz": torch.zeros((n_pages, Hkv, page_size, D // 32), dtype=tdt, device=dev),
        "bt": torch.from_numpy(bt).to(dev),
    }
    raw = []
    for b in range(B):
        n = int(hist[b])
        k = torch.from_numpy(syn.keys((n, Hkv), D, seed=seed * 100 + b)).to(dev).to(tdt)
        v = torch.from_numpy(syn.values((n, Hkv), D, seed=seed * 100 + 50 + b)).to(dev).to(tdt)
        t = np.arange(n)
        slots = torch.from_numpy(bt[b, t // page_size].astype(np.int64) * page_size + t % page_size).to(dev)
        raw.append((k, v, slots))
    return st, raw


def run_case(cuda, kind, bits, B, Hkv, G, hist, recent, page_size, dtype, seed, num_ctas=0, layout=0,
             entry="smaq_decode"):
    import torch
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_KEYS_BVQ, SMAQ_KEYS_SCALAR
    tdt = getattr(torch, dtype)
    qd = {"float32": "fp32", "bfloat16": "bf16", "float16": "fp16"}[dtype]
    st, raw = build_paged(cuda, kind, bits, B, Hkv, hist, page_size, dtype, seed)
    if kind == "scalar":
        qz = scalar_tables(bits, cuda)
        E, E_inv, cent, bnd = qz.E, qz.E_inv, qz.centroids, qz.decision_boundaries
    else:
        Eb, C, dec = random_codebook(cuda)
    for b, (k, v, slots) in enumerate(raw):
        if kind == "scalar":
            ops.append(k, v, n_heads=Hkv, slots=slots, page_size=page_size, key_format=SMAQ_KEYS_SCALAR,
                       key_bits=bits, E=E, boundaries=bnd, key_codes=st["codes"], key_norms=st["norms"],
                       v_data=st["vdata"], v_scales=st["vs"], v_zeros=st["vz"], layout=layout)
        else:
            ops.append(k, v, n_heads=Hkv, slots=slots, page_size=page_size, key_format=SMAQ_KEYS_BVQ,
                       E_blocks=Eb, centroids=C, key_codes=st["codes"], v_data=st["vdata"],
                       v_scales=st["vs"], v_zeros=st["vz"], layout=layout)
    W = max(1, int(max(recent)))
    rk = torch.from_numpy(syn.keys((B, W, Hkv), D, seed=seed + 7)).to(cuda).to(tdt)
    rv = torch.from_numpy(syn.values((B, W, Hkv), D, seed=seed + 8)).to(cuda).to(tdt)
    q = torch.from_numpy(syn.queries((B, Hkv * G), D, seed=seed + 9)).to(cuda).to(tdt)
    hl = torch.tensor(hist, dtype=torch.int32, device=cuda)
    rl = torch.tensor(recent, dtype=torch.int32, device=cuda)
    kw = dict(key_format=SMAQ_KEYS_SCALAR, key_bits=bits, E_inv=E_inv, centroids=cent,
              key_norms=st["norms"]) if kind == "scalar" else dict(key_format=SMAQ_KEYS_BVQ, centroids=dec)
    if kind == "bvq" and layout == 1:
        kw["centroids_f16"] = ops.fp16_codebook(dec)
        assert kw["centroids_f16"] is not None
    out = ops.decode(q, n_kv_heads=Hkv, key_codes=st["codes"], v_data=st["vdata"], v_scales=st["vs"],
                     v_zeros=st["vz"], hist_len=hl, page_size=page_size, block_table=st["bt"],
                     recent_k=rk, recent_v=rv, recent_len=rl, num_ctas=num_ctas, layout=layout, entry=entry, **kw)
    got = tn(out)
    # oracle per sequence, from the GPU-written rows (isolates decode from quantize parity)
    codes_t, vdata_t = st["codes"], st["vdata"]
    if layout == 1:
        vdata_t = ops.values_to_reference(vdata_t)
        if kind == "bvq":
            codes_t = ops.bvq_to_reference(codes_t)
        else:
            codes_t = ops.scalar_codes_to_reference(codes_t)
    codes, norms = tn(codes_t), tn(st["norms"])
    vdata, vs, vz = tn(vdata_t), tn(st["vs"]), tn(st["vz"])
    bt = tn(st["bt"])
    worst = 0.0
    for b in range(B):
        n = int(hist[b])
        t = np.arange(n)
        pg = bt[b, t // page_size]
        off = t % page_size
        c_b = codes[pg, :, off].transpose(1, 0, 2)          # [Hkv, n, P]
        if kind == "scalar":
            K = O.scalar_score_keys(c_b, norms[pg, :, off].T, bits, tn(E_inv), tn(cent), D) if n else None
        else:
            K = O.bvq_dequantize(c_b.astype(np.int64), tn(dec)) if n else None
        V = O.dequantize_values(vdata[pg, :, off].transpose(1, 0, 2), vs[pg, :, off].transpose(1, 0, 2),
                                vz[pg, :, off].transpose(1, 0, 2), 2, 32) if n else None
        r = int(recent[b])
        ref, _, _ = O.hybrid_attention(tn(q[b:b + 1]), qd, K, V, tn(rk[b, :r]) if r else None,
                                       tn(rv[b, :r]) if r else None, Hkv * G, Hkv)
        e = O.rel_l2(got[b:b + 1], ref)
        worst = max(worst, e)
    assert worst <= (1e-5 if qd == "fp32" else 2e-3), worst
    return got


@pytest.mark.parametrize("kind,bits", [("scalar", 4), ("scalar", 3), ("scalar", 2), ("bvq", 0)])
def test_paged_decode_bf16(cuda, kind, bits):
    hist = [700, 15, 16, 0, 333, 1]
    recent = [64, 3, 0, 17, 1, 0]
    run_case(cuda, kind, bits, B=6, Hkv=4, G=7, hist=hist, recent=recent, page_size=16, dtype="bfloat16",
             seed=11)


@pytest.mark.parametrize("kind,bits", [("scalar", 4), ("bvq", 0)])
def test_paged_decode_fp32_gqa8(cuda, kind, bits):
    run_case(cuda, kind, bits, B=3, Hkv=2, G=8, hist=[513, 40, 1000], recent=[5, 128, 0], page_size=16,
             dtype="float32", seed=12)


@pytest.mark.parametrize("num_ctas", [1, 3, 29, 2000])
def test_stream_k_partition_invariance(cuda, num_ctas):
    """Any number of CTAs (one slice, many splits, more CTAs than tokens) gives the same answer."""
    a = run_case(cuda, "bvq", 0, B=4, Hkv=2, G=4, hist=[900, 300, 17, 64], recent=[128, 0, 9, 1],
                 page_size=16, dtype="bfloat16", seed=13, num_ctas=num_ctas)
    b = run_case(cuda, "bvq", 0, B=4, Hkv=2, G=4, hist=[900, 300, 17, 64], recent=[128, 0, 9, 1],
                 page_size=16, dtype="bfloat16", seed=13, num_ctas=0)
    assert O.rel_l2(a, b) < 1e-3


@pytest.mark.parametrize("G", [1, 4, 7, 8])
def test_fast_bvq_decode_paged(cuda, G):
    """Block-VQ fast path (decode layout, TMA staging, tensor-core P.V) against the oracle."""
    run_case(cuda, "bvq", 0, B=5, Hkv=2, G=G, hist=[1000, 15, 16, 333, 2048], recent=[64, 3, 0, 128, 1],
             page_size=16, dtype="bfloat16", seed=21, layout=1)


def test_fast_bvq_decode_long_pages(cuda):
    run_case(cuda, "bvq", 0, B=2, Hkv=4, G=4, hist=[5000, 4097], recent=[128, 128], page_size=1024,
             dtype="bfloat16", seed=22, layout=1)


@pytest.mark.parametrize("num_ctas", [1, 7, 300])
def test_fast_bvq_partition_invariance(cuda, num_ctas):
    run_case(cuda, "bvq", 0, B=3, Hkv=2, G=4, hist=[3000, 100, 17], recent=[128, 0, 9], page_size=16,
             dtype="bfloat16", seed=23, num_ctas=num_ctas, layout=1)


def test_decode_layout_bytes_are_permuted_reference_bytes(cuda):
    """Decode-layout rows hold exactly the reference bytes, permuted (bit-exact)."""
    import torch
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_KEYS_BVQ
    Eb, C, _ = random_codebook(cuda)
    k = torch.from_numpy(syn.keys((64, 2), D, seed=31)).to(cuda).to(torch.bfloat16)
    v = torch.from_numpy(syn.values((64, 2), D, seed=32)).to(cuda).to(torch.bfloat16)
    out = {}
    for lay in (0, 1):
        codes = torch.zeros((2, 64, 16), dtype=torch.uint8, device=cuda)
        vd = torch.zeros((2, 64, 32), dtype=torch.uint8, device=cuda)
        vs = torch.zeros((2, 64, 4), dtype=torch.bfloat16, device=cuda)
        vz = torch.zeros_like(vs)
        ops.append(k, v, n_heads=2, page_size=64, key_format=SMAQ_KEYS_BVQ, E_blocks=Eb, centroids=C,
                   key_codes=codes, v_data=vd, v_scales=vs, v_zeros=vz, layout=lay)
        out[lay] = (codes, vd, vs, vz)
    assert torch.equal(ops.bvq_to_reference(out[1][0]), out[0][0])
    assert torch.equal(ops.values_to_reference(out[1][1]), out[0][1])
    assert torch.equal(out[1][2], out[0][2]) and torch.equal(out[1][3], out[0][3])
    ref_idx = ops.quantize_keys_bvq(k, Eb, C).reshape(64, 2, 16).transpose(0, 1)
    assert torch.equal(out[0][0], ref_idx)


@pytest.mark.parametrize("bits", [3, 4])
@pytest.mark.parametrize("G", [1, 4, 7, 8])
def test_fast_scalar_decode_paged(cuda, bits, G):
    """Scalar-key fast path (decode layout, split-fp16 tensor-core scores) against the oracle."""
    run_case(cuda, "scalar", bits, B=5, Hkv=2, G=G, hist=[1000, 15, 16, 333, 2048], recent=[64, 3, 0, 128, 1],
             page_size=16, dtype="bfloat16", seed=41, layout=1)


@pytest.mark.parametrize("num_ctas", [1, 7, 300])
def test_fast_scalar_partition_invariance(cuda, num_ctas):
    run_case(cuda, "scalar", 4, B=3, Hkv=2, G=7, hist=[3000, 100, 17], recent=[64, 0, 9], page_size=16,
             dtype="bfloat16", seed=43, num_ctas=num_ctas, layout=1)


@pytest.mark.parametrize("bits", [3, 4])
def test_scalar_decode_layout_bytes(cuda, bits):
    """Decode-layout scalar code rows (SIMT and tensor-core append kernels) hold the reference
    bytes permuted (bit-exact), norms identical."""
    import torch
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_KEYS_SCALAR
    qz = scalar_tables(bits, cuda)
    for dt, H in ((torch.bfloat16, 2), (torch.float32, 2), (torch.bfloat16, 3)):
        k = torch.from_numpy(syn.keys((256, H), D, seed=51)).to(cuda).to(dt)
        out = {}
        for lay in (0, 1):
            codes = torch.zeros((H, 256, 64), dtype=torch.uint8, device=cuda)
            norms = torch.zeros((H, 256), dtype=dt, device=cuda)
            ops.append(k, None, n_heads=H, page_size=256, key_format=SMAQ_KEYS_SCALAR, key_bits=bits, E=qz.E,
                       boundaries=qz.decision_boundaries, key_codes=codes, key_norms=norms, layout=lay)
            out[lay] = (codes, norms)
        assert torch.equal(ops.scalar_codes_to_reference(out[1][0]), out[0][0])
        assert torch.equal(out[1][1], out[0][1])


@pytest.mark.parametrize("kind", ["bvq", "scalar"])
def test_overlapped_launches_match_plain(cuda, kind):
    """overlap_prior (programmatic dependent launch): back-to-back launches sharing one workspace,
    each right after a kernel that rewrites its queries, give exactly the plain launches' outputs."""
    import torch
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_KEYS_BVQ, SMAQ_KEYS_SCALAR
    B, Hkv, G, page_size = 5, 2, 4, 16
    hist, recent = [1000, 15, 16, 333, 2048], [64, 3, 0, 128, 1]
    bits = 4 if kind == "scalar" else 0
    st, raw = build_paged(cuda, kind, bits, B, Hkv, hist, page_size, "bfloat16", 41)
    if kind == "scalar":
        qz = scalar_tables(bits, cuda)
        for k, v, slots in raw:
            ops.append(k, v, n_heads=Hkv, slots=slots, page_size=page_size, key_format=SMAQ_KEYS_SCALAR,
                       key_bits=bits, E=qz.E, boundaries=qz.decision_boundaries, key_codes=st["codes"],
                       key_norms=st["norms"], v_data=st["vdata"], v_scales=st["vs"], v_zeros=st["vz"], layout=1)
        kw = dict(key_format=SMAQ_KEYS_SCALAR, key_bits=bits, E_inv=qz.E_inv, centroids=qz.centroids,
                  key_norms=st["norms"])
    else:
        Eb, C, dec = random_codebook(cuda)
        for k, v, slots in raw:
            ops.append(k, v, n_heads=Hkv, slots=slots, page_size=page_size, key_format=SMAQ_KEYS_BVQ,
                       E_blocks=Eb, centroids=C, key_codes=st["codes"], v_data=st["vdata"], v_scales=st["vs"],
                       v_zeros=st["vz"], layout=1)
        kw = dict(key_format=SMAQ_KEYS_BVQ, centroids=dec, centroids_f16=ops.fp16_codebook(dec))
    bf = torch.bfloat16
    rk = torch.from_numpy(syn.keys((B, 128, Hkv), D, seed=42)).to(cuda).to(bf)
    rv = torch.from_numpy(syn.values((B, 128, Hkv), D, seed=43)).to(cuda).to(bf)
    hl = torch.tensor(hist, dtype=torch.int32, device=cuda)
    rl = torch.tensor(recent, dtype=torch.int32, device=cuda)
    n = 6
    src = [torch.from_numpy(syn.queries((B, Hkv * G), D, seed=50 + i)).to(cuda).to(bf) for i in range(n)]
    ws = torch.empty(ops.decode_workspace_bytes(B, Hkv * G, Hkv, D), dtype=torch.uint8, device=cuda)

    def run(overlap):
        q = torch.zeros_like(src[0])
        outs = []
        for i in range(n):
            q.copy_(src[i])  # the kernel right before each launch writes its queries
            outs.append(ops.decode(q, n_kv_heads=Hkv, key_codes=st["codes"], v_data=st["vdata"], v_scales=st["vs"],
                                   v_zeros=st["vz"], hist_len=hl, page_size=page_size, block_table=st["bt"],
                                   recent_k=rk, recent_v=rv, recent_len=rl, workspace=ws, layout=1,
                                   overlap_prior=overlap, **kw))
        torch.cuda.synchronize()
        return outs

    plain, over = run(False), run(True)
    for a, b in zip(plain, over):
        assert torch.equal(a, b)
    ops.decode_status(B, Hkv, ws)  # raises if a device wait ran out
