"""The vLLM hooks' hybrid decode path on the device: prefill through do_kv_cache_update fills
the compressed store and the exact ring (reference flush rule), and a decode step through the
hooked forward returns compute_hybrid_attention over them."""

import types

import pytest
import torch

from smaq_b200 import synthetic as syn

pytestmark = pytest.mark.gpu
D = 128


def test_hooked_decode_matches_hybrid_attention(cuda):
    from smaq_b200.integration import vllm as iv
    from smaq_b200.score import compute_hybrid_attention
    from test_vllm_hooks import FakeRunner, meta
    r = FakeRunner(n_layers=1, device="cuda")
    im = r.compilation_config.static_forward_context["layer.0"].impl
    im.head_size, im.num_kv_heads, im.num_heads, im.scale = D, 2, 8, D ** -0.5
    states = iv.install_hooks(r, mode=iv.MODE_HYBRID, ring_capacity=64, key_bits=4, initial_layers_count=0)
    st = states["layer.0"]
    n = 300
    k = torch.from_numpy(syn.keys((n, 2), D, seed=61)).to(cuda).to(torch.bfloat16)
    v = torch.from_numpy(syn.values((n, 2), D, seed=62)).to(cuda).to(torch.bfloat16)
    im.do_kv_cache_update(None, k, v, None, torch.arange(n, device=cuda))
    for t in range(5):  # decode-time writes
        kt = torch.from_numpy(syn.keys((1, 2), D, seed=70 + t)).to(cuda).to(torch.bfloat16)
        im.do_kv_cache_update(None, kt, kt, None, torch.arange(1, device=cuda))
    assert st.store.num_tokens + st.engine.ring.size == n + 5 and st.store.num_tokens >= 16
    q = torch.from_numpy(syn.queries((1, 8), D, seed=63)).to(cuda).to(torch.bfloat16)
    out = im.forward(None, q, q[:, :2], q[:, :2], None, meta(1, 1))
    rk, rv = st.engine.ring.peek()
    ref = compute_hybrid_attention(q, st.store, rk, rv, 8, scale=im.scale)
    assert out.shape == (1, 8, D) and torch.isfinite(out.float()).all()
    assert torch.equal(out, ref.to(out.dtype))
    stats = iv.get_stats(r)
    assert stats["layer.0"]["compressed_tokens"] == st.store.num_tokens
