"""Device side of the sequence-split decode (smaq_b200.distributed) on one GPU: each emulated
rank decodes its token range into fp32 partials (smaq_decode with partial_out and hist_total),
the partials are stacked as the all-gather would stack them, and smaq_merge_partials combines
them.  The result must match the unsplit decode, and both must match the oracle."""

import numpy as np
import pytest

from oracle import smaq_oracle as O

pytestmark = pytest.mark.gpu
D = 128


@pytest.mark.parametrize("kind,layout", [("bvq", 1), ("scalar", 0), ("bvq", 0)])
@pytest.mark.parametrize("splits", [2, 3])
def test_split_partials_merge_to_unsplit(cuda, kind, layout, splits):
    import torch
    from smaq_b200 import ops
    from smaq_b200.distributed import make_plan
    from smaq_b200._lib import SMAQ_KEYS_BVQ, SMAQ_KEYS_SCALAR
    from test_gpu_decode import build_paged, random_codebook, scalar_tables, tn
    B, Hkv, G, page = 3, 2, 4, 16
    hist = [700, 40, 9]          # the last one is below the 16-token minimum as a whole
    recent = [33, 0, 12]
    bits = 4
    st, raw = build_paged(cuda, kind, bits, B, Hkv, hist, page, "bfloat16", 91)
    if kind == "scalar":
        qz = scalar_tables(bits, cuda)
        kw = dict(key_format=SMAQ_KEYS_SCALAR, key_bits=bits, E_inv=qz.E_inv, centroids=qz.centroids,
                  key_norms=st["norms"])
        for k, v, slots in raw:
            ops.append(k, v, n_heads=Hkv, slots=slots, page_size=page, key_format=SMAQ_KEYS_SCALAR, key_bits=bits,
                       E=qz.E, boundaries=qz.decision_boundaries, key_codes=st["codes"], key_norms=st["norms"],
                       v_data=st["vdata"], v_scales=st["vs"], v_zeros=st["vz"], layout=layout)
    else:
        Eb, C, dec = random_codebook(cuda)
        kw = dict(key_format=SMAQ_KEYS_BVQ, centroids=dec)
        if layout == 1:
            kw["centroids_f16"] = ops.fp16_codebook(dec)
        for k, v, slots in raw:
            ops.append(k, v, n_heads=Hkv, slots=slots, page_size=page, key_format=SMAQ_KEYS_BVQ, E_blocks=Eb,
                       centroids=C, key_codes=st["codes"], v_data=st["vdata"], v_scales=st["vs"], v_zeros=st["vz"],
                       layout=layout)
    from smaq_b200 import synthetic as syn
    W = max(recent)
    rk = torch.from_numpy(syn.keys((B, W, Hkv), D, seed=5)).to(cuda).to(torch.bfloat16)
    rv = torch.from_numpy(syn.values((B, W, Hkv), D, seed=6)).to(cuda).to(torch.bfloat16)
    q = torch.from_numpy(syn.queries((B, Hkv * G), D, seed=7)).to(cuda).to(torch.bfloat16)
    common = dict(n_kv_heads=Hkv, key_codes=st["codes"], v_data=st["vdata"], v_scales=st["vs"],
                  v_zeros=st["vz"], page_size=page, recent_k=rk, recent_v=rv, layout=layout, **kw)
    full = ops.decode(q, hist_len=torch.tensor(hist, dtype=torch.int32, device=cuda), block_table=st["bt"],
                      recent_len=torch.tensor(recent, dtype=torch.int32, device=cuda), **common)
    plan = make_plan(splits, 1)  # one head group, `splits` sequence splits
    parts = []
    for r in range(splits):
        rng = [plan.token_range(n, r) for n in hist]
        bt = torch.zeros_like(st["bt"])
        for b, (lo, hi) in enumerate(rng):
            npg = (hi - lo + page - 1) // page
            bt[b, :npg] = st["bt"][b, lo // page:lo // page + npg]
        hl = torch.tensor([hi - lo for lo, hi in rng], dtype=torch.int32, device=cuda)
        rl = torch.tensor(recent if plan.holds_recent(r) else [0] * B, dtype=torch.int32, device=cuda)
        part = torch.empty((B, Hkv * G, 2 * D + 2), dtype=torch.float32, device=cuda)
        ops.decode(q, hist_len=hl, hist_total=torch.tensor(hist, dtype=torch.int32, device=cuda), block_table=bt,
                   recent_len=rl, partial_out=part, want_out=False, **common)
        parts.append(part)
    merged = ops.merge_partials(torch.stack(parts, 0), torch.bfloat16)
    assert O.rel_l2(tn(merged), tn(full)) <= 2e-3
