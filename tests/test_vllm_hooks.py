"""Host logic of the vLLM integration (smaq_b200.integration.vllm, smaq_b200.vllm_attn_backend)
on fake model runners, mirroring smaq/integration/vllm.py and smaq/vllm_attn_backend.py.
CPU tests keep every layer's tokens inside the exact ring (no store append, which needs the
device); tests/test_gpu_vllm_hooks.py drives the compressed path on the GPU."""

import types

import pytest
import torch

from smaq_b200 import vllm_attn_backend as vab
from smaq_b200.integration import vllm as iv

D = 64


class FakeImpl:
    def __init__(self, num_kv_heads=2, num_heads=4, head_size=D, separate_update=True):
        self.num_kv_heads = num_kv_heads
        self.num_heads = num_heads
        self.head_size = head_size
        self.scale = head_size ** -0.5
        self.calls = []
        if separate_update:
            self.do_kv_cache_update = types.MethodType(FakeImpl._update, self)

    def _update(self, layer, key, value, kv_cache, slot_mapping):
        self.calls.append(("update", key.shape[0]))

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output=None, output_scale=None,
                output_block_scale=None):
        self.calls.append(("forward", query.shape[0]))
        return torch.full_like(query, 7.0)


class FakeMLA:
    num_kv_heads = 1
    kv_lora_rank = 32

    def __init__(self):
        self.calls = []

    def do_kv_cache_update(self, kv_c_normed, k_pe, kv_cache, slot_mapping, kv_cache_dtype, k_scale):
        self.calls.append("mla_update")

    def forward_mqa(self, q, kv_cache, attn_metadata, layer):
        self.calls.append("mla_forward")
        return q


class FakeAttn:
    def __init__(self, impl):
        self.impl = impl
        self.kv_cache = [torch.zeros(1000, dtype=torch.float16)]


class FakeRunner:
    def __init__(self, n_layers=6, mla=False, device="cpu"):
        impls = [FakeImpl(separate_update=(i % 2 == 0)) for i in range(n_layers)]
        ctx = {f"layer.{i}": FakeAttn(im) for i, im in enumerate(impls)}
        if mla:
            ctx["mla.0"] = FakeAttn(FakeMLA())
        ctx["not_attention"] = object()
        self.compilation_config = types.SimpleNamespace(static_forward_context=ctx)
        self.device = torch.device(device)
        self.kv_caches = [a.kv_cache[0] for a in ctx.values() if hasattr(a, "kv_cache")]


def meta(n, max_q):
    return types.SimpleNamespace(num_actual_tokens=n, max_query_len=max_q)


def test_modes():
    for m in (iv.MODE_OFF, iv.MODE_CAPTURE_ONLY, iv.MODE_HYBRID, iv.MODE_FULL_SMAQ):
        iv.set_mode(m)
        assert iv.get_mode() == m
    with pytest.raises(ValueError):
        iv.set_mode("nope")
    vab.set_mode(vab.MODE_ACTIVE)
    assert vab.get_mode() == vab.MODE_ACTIVE and iv.get_mode() == iv.MODE_HYBRID
    vab.set_mode(vab.MODE_SHADOW)
    assert iv.get_mode() == iv.MODE_CAPTURE_ONLY
    with pytest.raises(ValueError):
        vab.set_mode("hybrid")


def test_install_hooks_layers_and_bits():
    r = FakeRunner(n_layers=6, mla=True)
    states = iv.install_hooks(r, key_bits=3, initial_layers_count=2, ring_capacity=64)
    assert list(states) == [f"layer.{i}" for i in range(6)] + ["mla.0"]
    assert [s.config.key_bits for s in states.values()][:6] == [4, 4, 3, 3, 3, 3]
    assert states["mla.0"].config.backend_kind == "mla" and not states["mla.0"].supports_hybrid
    assert states["layer.0"].config.num_query_heads == 4 and states["layer.0"].config.head_dim == D
    assert r._smaq_layer_states is states
    assert all(s.config.ring_capacity == 64 for s in states.values())


def test_capture_routing_and_passthrough():
    r = FakeRunner(n_layers=2)
    states = iv.install_hooks(r, mode=iv.MODE_CAPTURE_ONLY, ring_capacity=128)
    ctx = r.compilation_config.static_forward_context
    im0, im1 = ctx["layer.0"].impl, ctx["layer.1"].impl   # separate update / capture in forward
    k = torch.randn(10, 2, D)
    q = torch.randn(10, 4, D)
    im0.do_kv_cache_update(None, k, k, None, torch.arange(10))
    assert states["layer.0"].engine.ring.size == 10 and im0.calls == [("update", 10)]
    out = im1.forward(None, q, k, k, None, meta(10, 10))
    assert torch.all(out == 7.0) and states["layer.1"].engine.ring.size == 10
    im1.forward(None, q[:1], k[:1], k[:1], None, meta(1, 1))   # decode: one more token, passthrough
    assert states["layer.1"].engine.ring.size == 11
    iv.set_mode(iv.MODE_OFF)
    im0.do_kv_cache_update(None, k[:1], k[:1], None, torch.arange(1))
    assert states["layer.0"].engine.ring.size == 10           # off: vLLM write only
    iv.set_mode(iv.MODE_CAPTURE_ONLY)


def test_hybrid_without_history_passes_through_or_zeros():
    r = FakeRunner(n_layers=1)
    iv.install_hooks(r, mode=iv.MODE_HYBRID)
    im = r.compilation_config.static_forward_context["layer.0"].impl
    q = torch.randn(1, 4, D)
    assert torch.all(im.forward(None, q, q[:, :2], q[:, :2], None, meta(1, 1)) == 7.0)
    r2 = FakeRunner(n_layers=1)
    iv.install_hooks(r2, mode=iv.MODE_HYBRID, no_alloc=True)
    im2 = r2.compilation_config.static_forward_context["layer.0"].impl
    out = im2.forward(None, q.reshape(1, 4 * D), q[:, :2].reshape(1, 2 * D), q[:, :2].reshape(1, 2 * D), None,
                      meta(1, 1))
    assert out.shape == (1, 4 * D) and torch.all(out == 0)


def test_no_alloc_prefill_is_causal_attention():
    r = FakeRunner(n_layers=1)
    iv.install_hooks(r, mode=iv.MODE_HYBRID, no_alloc=True)
    im = r.compilation_config.static_forward_context["layer.0"].impl
    n = 7
    q, k, v = torch.randn(n, 4, D), torch.randn(n, 2, D), torch.randn(n, 2, D)
    out = im.forward(None, q, k, v, None, meta(n, n))
    kk, vv = k.repeat_interleave(2, 1), v.repeat_interleave(2, 1)
    s = torch.einsum("thd,shd->hts", q, kk) * im.scale
    s = s.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool), 1), float("-inf"))
    ref = torch.einsum("hts,shd->thd", s.softmax(-1), vv)
    assert torch.allclose(out, ref, atol=1e-5)
    buf = torch.zeros(n, 4 * D)
    im.forward(None, q.reshape(n, -1), k.reshape(n, -1), v.reshape(n, -1), None, meta(n, n), output=buf)
    assert torch.allclose(buf.view(n, 4, D), ref, atol=1e-5)


def test_mla_passthrough_and_stats_and_free():
    r = FakeRunner(n_layers=2, mla=True)
    states = vab.install_smaq_hooks(r, mode=vab.MODE_SHADOW, buffer_size=32)
    assert r._smaq_states is states and iv.get_mode() == iv.MODE_CAPTURE_ONLY
    mla = r.compilation_config.static_forward_context["mla.0"].impl
    mla.do_kv_cache_update(None, None, None, None, None, None)
    assert mla.forward_mqa("q", None, None, None) == "q" and mla.calls == ["mla_update", "mla_forward"]
    k = torch.randn(5, 2, D)
    r.compilation_config.static_forward_context["layer.0"].impl.do_kv_cache_update(None, k, k, None, torch.arange(5))
    st = iv.get_stats(r)
    assert st["layer.0"]["buffered_tokens"] == 5 and st["_totals"]["buffered_tokens"] == 5
    assert st["_totals"]["layers"] == 3
    freed = vab.free_kv_cache(r)
    assert freed == 2 * 1000 * 2                           # the two flash layers' caches
    ctx = r.compilation_config.static_forward_context
    assert ctx["layer.0"].kv_cache[0].numel() == 1 and ctx["mla.0"].kv_cache[0].numel() == 1000
    assert iv.free_kv_cache(FakeRunner(n_layers=1)) == 0   # nothing hooked
