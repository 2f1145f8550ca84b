"""Scalar key codes of bf16 keys through the tensor-core (tcgen05) rotation kernel, at sizes
beyond the golden fixture: many tiles, a ragged last tile, paged destination rows, strided
inputs, and head counts that take the SIMT kernel instead.  Checked against the oracle's
restatement of SMAQQuantizer.quantize (smaq/quantizer.py:138-145): codes bit-exact outside
the fp32 rounding band around the decision boundaries, norms bit-exact outside the bf16
rounding-midpoint band."""

import numpy as np
import pytest

from oracle import smaq_oracle as O
from smaq_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

D = 128


def _check(golden, cuda, bits, T, H, seed, strided=False, paged=False):
    import torch
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_KEYS_SCALAR
    k32 = syn.keys((T, H), D, seed=seed)
    kb = torch.from_numpy(k32).to(torch.bfloat16)
    kq = kb.float().numpy()
    if strided:  # [T, H, D] view of a wider [T, H, 2D] buffer
        wide = torch.zeros((T, H, 2 * D), dtype=torch.bfloat16)
        wide[:, :, :D] = kb
        key = wide.to(cuda)[:, :, :D]
    else:
        key = kb.to(cuda)
    E = torch.from_numpy(golden[f"sq_b{bits}_E"]).to(cuda)
    bnd = torch.from_numpy(golden[f"sq_b{bits}_boundaries"]).to(cuda)
    page = 16
    n_pages = (T + page - 1) // page
    pd = D // (4 if bits == 2 else 2)
    codes = torch.zeros((n_pages * H * page, pd), dtype=torch.uint8, device=cuda)
    norms = torch.zeros((n_pages * H * page,), dtype=torch.bfloat16, device=cuda)
    slots = None
    if paged:
        perm = np.random.default_rng(seed).permutation(n_pages)
        s = np.arange(T)
        slots_np = perm[s // page] * page + s % page
        slots = torch.from_numpy(slots_np).to(cuda)
    else:
        slots_np = np.arange(T)
    ops.append(key, None, n_heads=H, slots=slots, page_size=page, key_format=SMAQ_KEYS_SCALAR, key_bits=bits,
               E=E, boundaries=bnd, key_codes=codes, key_norms=norms)
    torch.cuda.synchronize()
    rows = ((slots_np // page)[:, None] * H + np.arange(H)[None]) * page + (slots_np % page)[:, None]  # [T, H]
    got_codes = codes.cpu().numpy()[rows]
    got_norms = norms.float().cpu().numpy()[rows]
    orc = O.quantize_keys_scalar(kq, golden[f"sq_b{bits}_E"], golden[f"sq_b{bits}_boundaries"], bits, "bf16")
    got = O.unpack_indices(got_codes, bits, D)
    amb = O.norm_ambiguous(orc["norm64"], "bf16")
    mism = (got != orc["codes"]) & ~orc["near_boundary"] & ~amb[..., None]
    assert mism.sum() == 0, f"{mism.sum()} code mismatches outside the band ({orc['near_boundary'].sum()} in band)"
    bad = (got_norms != orc["norms"]) & ~amb
    assert bad.sum() == 0, f"{bad.sum()} norm mismatches"


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_tc_keys_many_tiles(golden, cuda, bits):
    _check(golden, cuda, bits, T=4099, H=8, seed=700 + bits)


def test_tc_keys_paged(golden, cuda):
    _check(golden, cuda, 3, T=1000, H=4, seed=710, paged=True)


def test_tc_keys_strided(golden, cuda):
    _check(golden, cuda, 4, T=777, H=2, seed=720, strided=True)


def test_tc_keys_one_head(golden, cuda):
    _check(golden, cuda, 4, T=300, H=1, seed=730)


def test_simt_keys_odd_heads(golden, cuda):
    # 3 heads do not divide a 128-row tile: the SIMT kernel serves them
    _check(golden, cuda, 3, T=500, H=3, seed=740)


def test_tc_keys_reference_fn(golden, cuda):
    """The dense-rows entry point (SMAQQuantizer.quantize) on a larger batch."""
    import torch
    from smaq_b200 import ops
    k32 = syn.keys((2, 5000), D, seed=750)
    kb = torch.from_numpy(k32).to(torch.bfloat16)
    E = torch.from_numpy(golden["sq_b4_E"]).to(cuda)
    bnd = torch.from_numpy(golden["sq_b4_boundaries"]).to(cuda)
    codes, norms = ops.quantize_keys_scalar(kb.to(cuda), E, bnd, 4)
    orc = O.quantize_keys_scalar(kb.float().numpy(), golden["sq_b4_E"], golden["sq_b4_boundaries"], 4, "bf16")
    got = O.unpack_indices(codes.cpu().numpy(), 4, D)
    amb = O.norm_ambiguous(orc["norm64"], "bf16")
    assert ((got != orc["codes"]) & ~orc["near_boundary"] & ~amb[..., None]).sum() == 0
    assert ((norms.float().cpu().numpy() != orc["norms"]) & ~amb).sum() == 0
