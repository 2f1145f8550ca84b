"""Host logic of the vLLM integration (smaq_b200.integration.vllm / paged / vllm_backend and the
legacy smaq_b200.vllm_attn_backend) on fake model runners, CPU only.  The device launches
(``ops.append`` / ``ops.decode``) are replaced by recorders here; tests/test_gpu_vllm_hooks.py
runs the same batched path on the GPU against per-sequence oracle attention."""

import types

import numpy as np
import pytest
import torch

from smaq_b200 import vllm_attn_backend as vab
from smaq_b200.capture import KVCaptureEngine
from smaq_b200.integration import paged
from smaq_b200.integration import vllm as iv

D = 64
BS = 16


class FakeImpl:
    """A flash-attention implementation: vLLM-style cache writes through slots, and a forward
    that returns 7s (so a test sees when the SMAQ path answered instead)."""

    def __init__(self, num_kv_heads=2, num_heads=4, head_size=D, separate_update=True):
        self.num_kv_heads, self.num_heads, self.head_size = num_kv_heads, num_heads, head_size
        self.scale = head_size ** -0.5
        self.calls = []
        if separate_update:
            self.do_kv_cache_update = types.MethodType(FakeImpl._update, self)

    def _update(self, layer, key, value, kv_cache, slot_mapping):
        self.calls.append(("update", slot_mapping.shape[0]))
        if kv_cache is not None and kv_cache.dim() == 5:
            n, bs = slot_mapping.shape[0], kv_cache.shape[2]
            s = slot_mapping.long()
            ok = s >= 0
            kv_cache[0][s[ok] // bs, s[ok] % bs] = key[:n][ok].to(kv_cache.dtype)
            kv_cache[1][s[ok] // bs, s[ok] % bs] = value[:n][ok].to(kv_cache.dtype)

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
    def __init__(self, impl, kv_cache):
        self.impl = impl
        self.kv_cache = [kv_cache]


class FakeRunner:
    def __init__(self, n_layers=6, mla=False, device="cpu", num_blocks=64, impl_kw=None, dtype=torch.float32):
        impls = [FakeImpl(separate_update=(i % 2 == 0), **(impl_kw or {})) for i in range(n_layers)]
        ctx = {}
        for i, im in enumerate(impls):
            cache = torch.zeros(2, num_blocks, BS, im.num_kv_heads, im.head_size, dtype=dtype, device=device)
            ctx[f"layer.{i}"] = FakeAttn(im, cache)
        if mla:
            ctx["mla.0"] = FakeAttn(FakeMLA(), torch.zeros(1000, dtype=torch.float16))
        ctx["not_attention"] = object()
        self.compilation_config = types.SimpleNamespace(static_forward_context=ctx)
        self.device = torch.device(device)
        self.kv_caches = [a.kv_cache[0] for a in ctx.values() if hasattr(a, "kv_cache")]


def meta(n, max_q):
    return types.SimpleNamespace(num_actual_tokens=n, max_query_len=max_q)


class Recorder:
    """Stands in for the device launches of integration.paged."""

    def __init__(self, monkeypatch):
        self.appends, self.decodes = [], []
        monkeypatch.setattr(paged.ops, "append", self._append)
        monkeypatch.setattr(paged.ops, "decode", self._decode)
        monkeypatch.setattr(paged.ops, "decode_workspace_bytes", lambda *a, **k: 256)

    def _append(self, k, v, **kw):
        self.appends.append(dict(k=k.clone(), v=v.clone(), **kw))

    def _decode(self, q, **kw):
        self.decodes.append(dict(q=q.clone(), **kw))
        return torch.zeros_like(q)


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


class _CountingStore:
    """Token counter standing in for the compressed store of the reference's capture engine."""

    def __init__(self, h, d):
        self.num_kv_heads, self.head_dim, self.device, self.num_tokens = h, d, torch.device("cpu"), 0

    def append_chunk(self, k, v):
        self.num_tokens += k.shape[0]

    def reset(self):
        self.num_tokens = 0


def reference_split(n0, n_decode, capacity):
    """(compressed, exact) token counts of the reference's capture engine (capture.py rule)
    after a prompt of n0 tokens and n_decode decode tokens, as the hook's decode sees them."""
    st = _CountingStore(1, 4)
    eng = KVCaptureEngine(st, ring_capacity=capacity, device=torch.device("cpu"), dtype=torch.float32)
    eng.ingest_prefill(torch.zeros(n0, 1, 4), torch.zeros(n0, 1, 4), n0)
    for _ in range(n_decode):
        eng.ingest_decode(torch.zeros(1, 1, 4), torch.zeros(1, 1, 4), 1)
    h, r = st.num_tokens, eng.ring.size
    if h < 16:  # the hook answers from exact attention over every token
        return 0, h + r
    return h, r


@pytest.mark.parametrize("capacity", [8, 64, 128])
def test_window_rule_is_the_reference_ring(capacity):
    for n0 in (1, 5, capacity - 1, capacity, capacity + 1, 3 * capacity + 7):
        for nd in (1, 2, capacity - 1, capacity, capacity + 3, 2 * capacity + 1):
            L = torch.tensor([n0 + nd])
            h, r = paged.split_history(L, torch.tensor([n0]), capacity)
            assert (int(h), int(r)) == reference_split(n0, nd, capacity), (n0, nd)


class Batch:
    """Sequences in shuffled vLLM blocks, driven through a hooked implementation step by step."""

    def __init__(self, prompt_lens, n_decode, num_blocks, seed=0, hkv=2, hq=4, d=D, device="cpu",
                 dtype=torch.float32):
        self.rng = np.random.default_rng(seed)
        self.lens = list(prompt_lens)
        self.hkv, self.hq, self.d, self.device, self.dtype = hkv, hq, d, torch.device(device), dtype
        need = [(n + n_decode + BS - 1) // BS for n in prompt_lens]
        perm = self.rng.permutation(num_blocks)[: sum(need)]
        self.bt = torch.zeros(len(prompt_lens), max(need), dtype=torch.int32)
        o = 0
        for b, k in enumerate(need):
            self.bt[b, :k] = torch.from_numpy(perm[o:o + k].astype(np.int32))
            o += k
        self.bt = self.bt.to(self.device)
        self.k = [torch.empty(0, hkv, d) for _ in prompt_lens]   # every token written, per sequence
        self.v = [torch.empty(0, hkv, d) for _ in prompt_lens]

    def _slots(self, b, pos):
        pos = torch.as_tensor(pos, dtype=torch.int64)
        return self.bt[b].cpu().long()[pos // BS] * BS + pos % BS

    def _tokens(self, n):
        k = torch.from_numpy(self.rng.standard_normal((n, self.hkv, self.d)).astype(np.float32))
        v = torch.from_numpy(self.rng.standard_normal((n, self.hkv, self.d)).astype(np.float32))
        return k, v

    def _step(self, impl, kv_cache, counts, pad=3):
        ks, vs, slots = [], [], []
        for b, n in enumerate(counts):
            k, v = self._tokens(n)
            slots.append(self._slots(b, range(len(self.k[b]), len(self.k[b]) + n)))
            self.k[b], self.v[b] = torch.cat([self.k[b], k]), torch.cat([self.v[b], v])
            ks.append(k)
            vs.append(v)
        N = sum(counts)
        key = torch.cat(ks + [torch.zeros(pad, self.hkv, self.d)])        # padded rows, as vLLM pads
        val = torch.cat(vs + [torch.zeros(pad, self.hkv, self.d)])
        sm = torch.cat(slots + [torch.full((pad,), -1, dtype=torch.int64)])
        dev = lambda t: t.to(self.device)
        key, val = dev(key).to(self.dtype), dev(val).to(self.dtype)
        impl.do_kv_cache_update(None, key, val, kv_cache, dev(sm))
        self.lens = [len(x) for x in self.k]
        qsl = torch.tensor([0] + list(np.cumsum(counts)), dtype=torch.int32)
        md = types.SimpleNamespace(num_actual_tokens=N, max_query_len=max(counts), query_start_loc=dev(qsl),
                                   seq_lens=dev(torch.tensor(self.lens, dtype=torch.int32)), block_table=self.bt,
                                   slot_mapping=dev(sm))
        q = dev(torch.from_numpy(self.rng.standard_normal((N + pad, self.hq, self.d)).astype(np.float32))).to(self.dtype)
        out = impl.forward(None, q, key, val, kv_cache, md)
        return q[:N], out, sm

    def prefill(self, impl, kv_cache):
        return self._step(impl, kv_cache, list(self.lens_prompt()))

    def lens_prompt(self):
        return self.lens

    def decode(self, impl, kv_cache):
        return self._step(impl, kv_cache, [1] * len(self.lens))


def _batched_runner(monkeypatch, capacity=32):
    rec = Recorder(monkeypatch)
    r = FakeRunner(n_layers=1, num_blocks=128)
    states = iv.install_hooks(r, mode=iv.MODE_HYBRID, ring_capacity=capacity, key_bits=3, initial_layers_count=0)
    attn = r.compilation_config.static_forward_context["layer.0"]
    return rec, r, states["layer.0"], attn.impl, attn.kv_cache[0]


def test_batched_path_three_sequences(monkeypatch):
    """Three sequences of distinct prompt lengths in shuffled blocks: one append launch per step
    over all tokens (padding to the scratch page), prefill through vLLM's own attention, and
    one decode launch per decode step with the block table, the reference split per sequence
    and the exact window rows read from vLLM's cache."""
    C = 32
    rec, r, st, im, kv = _batched_runner(monkeypatch, C)
    prompts = [40, 150, 9]
    bt = Batch(prompts, n_decode=40, num_blocks=128, seed=3)
    q, out, sm = bt.prefill(im, kv)
    assert torch.all(out == 7.0)                                  # prefill: vLLM's attention
    assert len(rec.appends) == 1 and rec.decodes == []
    a = rec.appends[0]
    slots = a["slots"]
    assert slots.shape[0] == sum(prompts) + 3 and a["page_size"] == BS
    assert torch.equal(slots[: sum(prompts)], sm[: sum(prompts)])
    assert torch.all(slots[sum(prompts):] // BS == 128)               # padding -> scratch page
    assert torch.equal(st.cache.prompt_len[bt.bt[:, 0].long()], torch.tensor(prompts, dtype=torch.int32))
    for step in range(40):
        q, out, _ = bt.decode(im, kv)
        d = rec.decodes[-1]
        assert len(rec.decodes) == step + 1 and len(rec.appends) == step + 2
        assert torch.equal(d["block_table"], bt.bt) and d["page_size"] == BS
        hist, rl = d["hist_len"], d["recent_len"]
        for b, n0 in enumerate(prompts):
            h_ref, r_ref = reference_split(n0, step + 1, C)
            assert (int(hist[b]), int(rl[b])) == (h_ref, r_ref), (step, b)
            L = bt.lens[b]
            assert torch.equal(d["recent_k"][b, :r_ref], bt.k[b][L - r_ref:L])
            assert torch.equal(d["recent_v"][b, :r_ref], bt.v[b][L - r_ref:L])
        assert torch.equal(d["q"], q) and torch.all(out == 0)       # answered by the decode launch
    assert iv.get_stats(r)["layer.0"]["compressed_tokens"] == sum(prompts) + 3 + 40 * (3 + 3)


def test_capture_only_and_off_pass_through(monkeypatch):
    rec, r, st, im, kv = _batched_runner(monkeypatch)
    iv.set_mode(iv.MODE_CAPTURE_ONLY)
    bt = Batch([20, 30], n_decode=2, num_blocks=128, seed=4)
    bt.prefill(im, kv)
    _, out, _ = bt.decode(im, kv)
    assert torch.all(out == 7.0) and len(rec.appends) == 2 and rec.decodes == []
    iv.set_mode(iv.MODE_OFF)
    _, out, _ = bt.decode(im, kv)
    assert torch.all(out == 7.0) and len(rec.appends) == 2          # off: vLLM's write only
    assert im.calls.count(("update", 2 + 3)) == 2
    iv.set_mode(iv.MODE_HYBRID)


def test_mixed_prefill_decode_step_runs_vllm_attention(monkeypatch):
    rec, r, st, im, kv = _batched_runner(monkeypatch)
    bt = Batch([20, 30], n_decode=4, num_blocks=128, seed=5)
    bt.prefill(im, kv)
    _, out, _ = bt._step(im, kv, [1, 3])                        # one decode row, one chunk row
    assert torch.all(out == 7.0) and rec.decodes == []
    assert int(st.cache.prompt_len[bt.bt[1, 0].long()]) == 33    # the chunk row's new prompt length


def test_no_alloc_prefill_needs_the_gpu_and_empty_decode_is_zero():
    """CPU half: the no-allocation prefill runs on this package's kernel, so CPU tensors raise
    (no fallback); a decode before anything was compressed is zero; vLLM's cache write is
    skipped.  The prefill's numbers are checked on the GPU (tests/test_gpu_causal.py)."""
    r = FakeRunner(n_layers=1)
    iv.install_hooks(r, mode=iv.MODE_HYBRID, no_alloc=True)
    im = r.compilation_config.static_forward_context["layer.0"].impl
    n = 7
    q, k, v = torch.randn(n, 4, D), torch.randn(n, 2, D), torch.randn(n, 2, D)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        im.forward(None, q, k, v, None, meta(n, n))
    dq = torch.randn(1, 4 * D)
    out = im.forward(None, dq, dq[:, : 2 * D], dq[:, : 2 * D], None, meta(1, 1))
    assert out.shape == (1, 4 * D) and torch.all(out == 0)     # nothing compressed yet
    im.do_kv_cache_update(None, k, v, None, torch.arange(n))
    st = r._smaq_layer_states["layer.0"]
    assert st.engine.ring.size == n and im.calls == []          # no_alloc: vLLM's write skipped


def test_mla_passthrough_and_stats_and_free(monkeypatch):
    Recorder(monkeypatch)
    r = FakeRunner(n_layers=2, mla=True)
    states = vab.install_smaq_hooks(r, mode=vab.MODE_SHADOW, buffer_size=32)
    assert r._smaq_states is states and iv.get_mode() == iv.MODE_CAPTURE_ONLY
    mla = r.compilation_config.static_forward_context["mla.0"].impl
    mla.do_kv_cache_update(None, None, None, None, None, None)
    assert mla.forward_mqa("q", None, None, None) == "q" and mla.calls == ["mla_update", "mla_forward"]
    attn0 = r.compilation_config.static_forward_context["layer.0"]
    k = torch.randn(5, 2, D)
    attn0.impl.do_kv_cache_update(None, k, k, attn0.kv_cache[0], torch.arange(5))
    st = iv.get_stats(r)
    assert st["layer.0"]["compressed_tokens"] == 5 and st["_totals"]["compressed_tokens"] == 5
    assert st["layer.0"]["memory_bytes"] == states["layer.0"].cache.device_bytes() > 0
    assert st["_totals"]["layers"] == 3
    cache_bytes = attn0.kv_cache[0].nelement() * 4
    freed = vab.free_kv_cache(r)
    assert freed == 2 * cache_bytes                               # the two flash layers' caches
    ctx = r.compilation_config.static_forward_context
    assert ctx["layer.0"].kv_cache[0].numel() == 1 and ctx["mla.0"].kv_cache[0].numel() == 1000
    assert all(t.numel() == 1 for t in r.kv_caches[:2]) and r.kv_caches[2].numel() == 1000
    assert iv.free_kv_cache(FakeRunner(n_layers=1)) == 0          # nothing hooked


def test_enable_no_alloc_layout_wrapper_takes_vllm_022_arguments(monkeypatch):
    pytest.importorskip("vllm")
    from vllm.v1.executor.abstract import Executor
    from vllm.v1.worker.gpu_model_runner import GPUModelRunner
    seen = []

    def layout(self, kv_caches, kernel_block_sizes):
        seen.append((dict(kv_caches), kernel_block_sizes))

    monkeypatch.setattr(GPUModelRunner, "_update_hybrid_attention_mamba_layout", layout)
    monkeypatch.setattr(GPUModelRunner, "_smaq_layout_patch", False, raising=False)
    monkeypatch.setattr(Executor, "_smaq_patched", False, raising=False)
    monkeypatch.setattr(Executor, "get_kv_cache_specs", lambda self: "specs")
    vab.enable_no_alloc(key_bits=3)
    runner = types.SimpleNamespace(shared_kv_cache_layers={"l1": "l0"})
    GPUModelRunner._update_hybrid_attention_mamba_layout(runner, {"l0": "cache0"}, [16])
    assert seen == [({"l0": "cache0", "l1": "cache0"}, [16])]

    calls = []

    class FakeExecutor:
        def collective_rpc(self, fn):
            calls.append(fn)

    assert Executor.get_kv_cache_specs(FakeExecutor()) == "specs" and len(calls) == 1


def test_backend_registers_as_custom():
    pytest.importorskip("vllm")
    from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl
    from vllm.v1.attention.backends.registry import AttentionBackendEnum
    from smaq_b200.integration import vllm_backend as vb
    try:
        path = vb.register(key_bits=4, ring_capacity=64)
        assert AttentionBackendEnum.CUSTOM.get_path() == path
        cls = AttentionBackendEnum.CUSTOM.get_class()
        assert cls is vb.SmaqAttentionBackend and cls.get_name() == "CUSTOM"
        assert issubclass(cls.get_impl_cls(), FlashAttentionImpl)
        assert iv.get_mode() == iv.MODE_HYBRID
        cfg = vb._layer_config(types.SimpleNamespace(head_size=128, num_kv_heads=8, num_heads=32), 9,
                               torch.device("cpu"))
        assert (cfg.key_bits, cfg.ring_capacity, cfg.num_query_heads) == (4, 64, 32)
    finally:
        AttentionBackendEnum.CUSTOM.clear_override()
        iv.set_mode(iv.MODE_CAPTURE_ONLY)


def test_fp8_cache_is_left_to_vllm(monkeypatch):
    rec = Recorder(monkeypatch)
    r = FakeRunner(n_layers=1, num_blocks=32, dtype=torch.float8_e4m3fn)
    iv.install_hooks(r, mode=iv.MODE_HYBRID, ring_capacity=16, initial_layers_count=0)
    attn = r.compilation_config.static_forward_context["layer.0"]
    im, kv = attn.impl, attn.kv_cache[0]
    bt = Batch([40], n_decode=2, num_blocks=32, seed=6)
    bt.prefill(im, kv)
    _, out, _ = bt.decode(im, kv)
    assert torch.all(out == 7.0) and rec.appends == [] and rec.decodes == []
