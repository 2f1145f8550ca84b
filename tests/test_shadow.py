"""ExactShadowStrategy (smaq/strategies.py:258-298): exact history keys, 2-bit values.

CPU: the strategy's own methods against the reference's behaviour (clone, matmul scores,
flatten / concat / head selection, byte accounting, capability flags).  GPU: stores built from
the reference's golden inputs (tests/golden/golden_shadow.npz, written by make_golden.py from
the reference) give the reference's hybrid output, value bytes and memory accounting."""

import os

import numpy as np
import pytest

from conftest import REPO

SHADOW = os.path.join(REPO, "tests", "golden", "golden_shadow.npz")
D = 128


def test_strategy_methods_cpu():
    import torch
    from smaq_b200.strategies import ExactShadowQuantized, ExactShadowStrategy
    s = ExactShadowStrategy()
    k = torch.randn(1, 3, 7, D)
    q = s.quantize(k)
    assert isinstance(q, ExactShadowQuantized) and torch.equal(q.values, k)
    assert q.values.data_ptr() != k.data_ptr()                     # a copy, as the reference clones
    assert torch.equal(s.dequantize(q), k)
    flat = s.flatten_quantized(q)
    assert flat.values.shape == (3, 7, D)
    cat = s.concat_quantized([flat, flat])
    assert cat.values.shape == (3, 14, D)
    h1 = s.select_head(cat, 1)
    assert h1.values.shape == (14, D)
    qq = torch.randn(4, D)
    sc = s.attention_score(qq, h1, scale=0.125)
    assert torch.allclose(sc, (qq @ h1.values.T) * 0.125, rtol=1e-5, atol=1e-5)
    assert s.memory_bytes(flat) == 3 * 7 * D * 4
    cap = s.capabilities
    assert cap.compressed_history is False and cap.compressed_history_shadow_only is True
    assert cap.strategy_name == "exact_shadow" and cap.quantization_name == "shadow_exact"


@pytest.mark.gpu
@pytest.mark.parametrize("tag", ["bf16", "bf16_histonly", "fp32", "hist15"])
def test_store_and_hybrid_attention_match_reference(cuda, tag):
    import torch
    from oracle import smaq_oracle as O
    from smaq_b200.score import compute_hybrid_attention
    from smaq_b200.store import CompressedKVStore
    from smaq_b200.strategies import ExactShadowStrategy
    g = np.load(SHADOW)
    p = f"sh_{tag}_"
    Hq, Hkv, nh, nr = (int(x) for x in g[p + "meta"])
    dt = torch.float32 if tag == "fp32" else torch.bfloat16

    def tt(name):
        return torch.from_numpy(np.ascontiguousarray(g[p + name])).to(cuda).to(dt)

    store = CompressedKVStore(D, Hkv, device=cuda, key_strategy=ExactShadowStrategy())
    hk, hv = tt("hist_k"), tt("hist_v")
    h1 = nh // 3
    store.append_chunk(hk[:h1], hv[:h1])
    store.append_chunk(hk[h1:], hv[h1:])
    rk = tt("recent_k") if nr else None
    rv = tt("recent_v") if nr else None
    out = compute_hybrid_attention(tt("q"), store, rk, rv, Hq)
    assert out.dtype == dt and out.shape == (1, Hq, D)
    tol = 1e-5 if dt == torch.float32 else 2e-3
    err = O.rel_l2(out.float().cpu().numpy(), g[p + "out"])
    assert err <= tol, err
    flat = store.get_flat_cache()
    assert torch.equal(flat.key_q.values.float().cpu(), torch.from_numpy(g[p + "hist_k"]).transpose(0, 1))
    assert np.array_equal(flat.value_q.data.cpu().numpy(), g[p + "v_data"])
    assert store.memory_bytes() == int(g[p + "memory_bytes"][0])
