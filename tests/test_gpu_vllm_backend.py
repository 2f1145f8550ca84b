"""The registered backend's implementation class with vLLM's own pieces on the device: vLLM's
FlashAttentionImpl constructor and its cache write (reshape_and_cache_flash) under
SmaqAttentionImpl, three sequences in shuffled 16-token blocks, decode steps answered by the SMAQ
paged path and checked against per-sequence oracle attention (smaq/score.py:23-72)."""

import types

import pytest
import torch

from oracle import smaq_oracle as O

pytestmark = pytest.mark.gpu
D = 128


def test_smaq_attention_impl_decodes_a_batch(cuda):
    vb = pytest.importorskip("smaq_b200.integration.vllm_backend")
    if vb.FlashAttentionImpl is None:
        pytest.skip("vLLM is not installed")
    from smaq_b200.integration import vllm as iv
    from test_gpu_vllm_hooks import _oracle
    from test_vllm_hooks import Batch
    C = 32
    vb.register(key_bits=3, ring_capacity=C, initial_layers_count=0)
    try:
        impl = vb.SmaqAttentionImpl(num_heads=8, head_size=D, scale=D ** -0.5, num_kv_heads=2, alibi_slopes=None,
                                    sliding_window=None, kv_cache_dtype="auto")
    except Exception as exc:  # vLLM's constructor needs its compiled ops on this box
        pytest.skip(f"vLLM FlashAttentionImpl unavailable here: {type(exc).__name__}: {exc}")
    layer = types.SimpleNamespace(_k_scale=torch.ones((), device=cuda), _v_scale=torch.ones((), device=cuda),
                                  _k_scale_float=1.0, _v_scale_float=1.0)
    kv = torch.zeros(2, 96, 16, 2, D, dtype=torch.bfloat16, device=cuda)
    prompts = [300, 45, 700]
    bt = Batch(prompts, n_decode=12, num_blocks=96, seed=21, hkv=2, hq=8, d=D, device="cuda", dtype=torch.bfloat16)

    class Runner:  # drives the impl the way vLLM's attention layer does
        def do_kv_cache_update(self, _layer, key, value, kv_cache, slot_mapping):
            impl.do_kv_cache_update(layer, key, value, kv_cache, slot_mapping)

        def forward(self, _layer, query, key, value, kv_cache, md, output=None):
            if md.max_query_len > 1:  # prefill: only the prompt lengths are needed here
                qsl = md.query_start_loc
                impl._smaq_state.cache.note_prompts(md.block_table, md.seq_lens, qsl[1:] - qsl[:-1])
                return None
            out = torch.empty_like(query)
            return impl.forward(layer, query, key, value, kv_cache, md, out)

    try:
        bt.prefill(Runner(), kv)
    except Exception as exc:
        pytest.skip(f"vLLM cache write unavailable here: {type(exc).__name__}: {exc}")
    st = impl._smaq_state
    assert isinstance(st, iv.LayerState) and st.cache is not None
    # vLLM's own write put the exact tokens in its cache
    b, t = 1, 44
    blk, off = int(bt.bt[b, t // 16]), t % 16
    assert torch.equal(kv[0, blk, off].float().cpu(), bt.k[b][t].to(torch.bfloat16).float())
    worst = 0.0
    for step in range(12):
        q, out, _ = bt.decode(Runner(), kv)
        torch.cuda.synchronize()
        qn, on = q.float().cpu().numpy(), out[: len(prompts)].float().cpu().numpy()
        for b, n0 in enumerate(prompts):
            ref = _oracle(st, bt, b, n0, step + 1, qn[b], C)
            worst = max(worst, O.rel_l2(on[b], ref))
    print(f"registered backend decode worst rel-L2 {worst:.3e}")
    assert worst <= 2e-3, worst
    from vllm.v1.attention.backends.registry import AttentionBackendEnum
    AttentionBackendEnum.CUSTOM.clear_override()
    iv.set_mode(iv.MODE_CAPTURE_ONLY)
