"""smaq_decode_noalloc -- decode for callers that cannot allocate device memory.

Some hosts cannot call cudaMalloc: every byte of device memory is owned by another allocator or
memory pool, or the GPU is reached only through this C ABI.  smaq_decode_noalloc takes its
scratch from a fixed array inside the library instead of a caller workspace.  This test calls
it through the C ABI twice in a row (the second call runs on scratch left over from the first)
and checks both results against smaq_decode with a caller workspace, at the tolerance the
decode tests use.  The file name makes pytest collect it last.
"""

import numpy as np
import pytest

from oracle import smaq_oracle as O
from smaq_b200 import synthetic as syn

pytestmark = pytest.mark.gpu
D = 128


def _case(cuda, fast: bool, B=3, Hkv=2, G=4):
    import torch
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_KEYS_BVQ
    rng = np.random.default_rng(3)
    T, W = 1024, 40
    Eb = torch.from_numpy((np.eye(8)[None] + 0.1 * rng.standard_normal((16, 8, 8))).astype(np.float32)).to(cuda)
    C = torch.from_numpy(rng.standard_normal((16, 256, 8)).astype(np.float32)).to(cuda)
    dec = torch.from_numpy((rng.standard_normal((16, 256, 8)) * 0.5).astype(np.float16).astype(np.float32)).to(cuda)
    layout = 1 if fast else 0
    codes = torch.zeros((B, Hkv, T, 16), dtype=torch.uint8, device=cuda)
    vd = torch.zeros((B, Hkv, T, 32), dtype=torch.uint8, device=cuda)
    vs = torch.zeros((B, Hkv, T, 4), dtype=torch.bfloat16, device=cuda)
    vz = torch.zeros_like(vs)
    for b in range(B):
        k = torch.from_numpy(syn.keys((T, Hkv), D, seed=40 + b)).to(cuda).to(torch.bfloat16)
        v = torch.from_numpy(syn.values((T, Hkv), D, seed=50 + b)).to(cuda).to(torch.bfloat16)
        ops.append(k, v, n_heads=Hkv, slot_offset=b * T, page_size=T, key_format=SMAQ_KEYS_BVQ, E_blocks=Eb,
                   centroids=C, key_codes=codes, v_data=vd, v_scales=vs, v_zeros=vz, layout=layout)
    q = torch.from_numpy(syn.queries((B, Hkv * G), D, seed=60)).to(cuda).to(torch.bfloat16)
    rk = torch.from_numpy(syn.keys((B, W, Hkv), D, seed=61)).to(cuda).to(torch.bfloat16)
    rv = torch.from_numpy(syn.values((B, W, Hkv), D, seed=62)).to(cuda).to(torch.bfloat16)
    kw = dict(n_kv_heads=Hkv, key_format=SMAQ_KEYS_BVQ, centroids=dec, key_codes=codes, v_data=vd, v_scales=vs,
              v_zeros=vz, hist_len=torch.tensor([1000, 17, 600][:B] + [700] * (B - 3), dtype=torch.int32, device=cuda),
              page_size=T, recent_k=rk, recent_v=rv,
              recent_len=torch.tensor([40, 0, 5][:B] + [9] * (B - 3), dtype=torch.int32, device=cuda),
              layout=layout, centroids_f16=ops.fp16_codebook(dec) if fast else None)
    return q, kw


@pytest.mark.parametrize("fast", [True, False])
def test_noalloc_matches_workspace_entry_point_twice(cuda, fast):
    import torch
    from smaq_b200 import ops
    q, kw = _case(cuda, fast)
    ref = ops.decode(q, **kw).float().cpu().numpy()
    for _ in range(2):
        got = ops.decode(q, entry="smaq_decode_noalloc", **kw)
        torch.cuda.synchronize()
        assert O.rel_l2(got.float().cpu().numpy(), ref) <= 2e-3


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda):
    import torch
    from smaq_b200 import _lib, ops
    lib = _lib.load()
    big = 1 << 16  # 65536 sequences x 2 kv heads needs far more than the fixed scratch
    assert ops.decode_workspace_bytes(big, 8, 2, 128) > lib.smaq_decode_noalloc_max_workspace()
    q = torch.zeros((big, 8, 128), dtype=torch.bfloat16, device=cuda)
    _, kw = _case(cuda, True)
    kw["hist_len"] = torch.zeros((big,), dtype=torch.int32, device=cuda)
    kw["recent_len"] = None
    with pytest.raises(RuntimeError, match="scratch"):
        ops.decode(q, entry="smaq_decode_noalloc", **kw)


def test_noalloc_alternating_shapes_and_paths(cuda):
    """Calls of different shapes in a row reuse the scratch at different offsets (plan, pair
    counters, error word, slots); reference-layout rows take the multi-launch general path."""
    import torch
    from smaq_b200 import ops
    for B, Hkv, G, fast in ((3, 2, 4, True), (1, 8, 8, True), (3, 2, 4, True), (2, 2, 8, False),
                            (3, 2, 4, False), (1, 8, 8, True)):
        q, kw = _case(cuda, fast, B=B, Hkv=Hkv, G=G)
        ref = ops.decode(q, **kw).float().cpu().numpy()
        got = ops.decode(q, entry="smaq_decode_noalloc", **kw)
        torch.cuda.synchronize()
        ops.decode_status(B, Hkv)          # the no-allocation scratch's error word
        assert O.rel_l2(got.float().cpu().numpy(), ref) <= 2e-3, (B, Hkv, G, fast)
