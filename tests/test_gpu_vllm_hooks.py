"""The batched vLLM path on the device: three sequences of distinct prompt lengths in shuffled
16-token vLLM blocks go through the hooked ``do_kv_cache_update`` / ``forward`` (one append
launch per step, one paged decode launch per decode step), and every decode output matches the
oracle's per-sequence hybrid attention (smaq/score.py:23-72) over the reference's split: the
compressed history quantized by the oracle, the exact window from the written tokens."""

import numpy as np
import pytest
import torch

from oracle import smaq_oracle as O

pytestmark = pytest.mark.gpu
D = 128


def _oracle(st, bt, b, n0, n_decode, q, capacity):
    from test_vllm_hooks import reference_split
    h, r = reference_split(n0, n_decode, capacity)
    L = bt.lens[b]
    k = bt.k[b].to(torch.bfloat16).float().numpy()
    v = bt.v[b].to(torch.bfloat16).float().numpy()
    qz = st.cache.quantizer
    K = V = None
    if h:
        kq = O.quantize_keys_scalar(k[:h].transpose(1, 0, 2), qz.E.cpu().numpy(),
                                    qz.decision_boundaries.cpu().numpy(), 3, "bf16")
        K = O.scalar_score_keys(kq["indices"], kq["norms"], 3, qz.E_inv.cpu().numpy(), qz.centroids.cpu().numpy(), D)
        vq = O.quantize_values(v[:h].transpose(1, 0, 2), 2, 32, "bf16")
        V = O.dequantize_values(vq["data"], vq["scales"], vq["zeros"], 2, 32)
    ref, _, _ = O.hybrid_attention(q[None], "bf16", K, V, k[L - r:L], v[L - r:L], bt.hq, bt.hkv, scale=D ** -0.5)
    return ref[0]


def test_batched_decode_matches_oracle_per_sequence(cuda):
    from smaq_b200._lib import SMAQ_LAYOUT_DECODE
    from smaq_b200.integration import vllm as iv
    from test_vllm_hooks import Batch, FakeRunner
    C = 32
    r = FakeRunner(n_layers=1, num_blocks=96, device="cuda", dtype=torch.bfloat16,
                   impl_kw=dict(num_kv_heads=2, num_heads=8, head_size=D))
    states = iv.install_hooks(r, mode=iv.MODE_HYBRID, ring_capacity=C, key_bits=3, initial_layers_count=0)
    st = states["layer.0"]
    attn = r.compilation_config.static_forward_context["layer.0"]
    im, kv = attn.impl, attn.kv_cache[0]
    prompts = [300, 45, 700]
    bt = Batch(prompts, n_decode=40, num_blocks=96, seed=11, hkv=2, hq=8, d=D, device="cuda", dtype=torch.bfloat16)
    bt.prefill(im, kv)
    assert st.cache.layout == SMAQ_LAYOUT_DECODE   # bf16, D 128, 3-bit keys: the fused paged kernel
    worst = 0.0
    for step in range(40):
        q, out, _ = bt.decode(im, kv)
        torch.cuda.synchronize()
        qn, on = q.float().cpu().numpy(), out[: len(prompts)].float().cpu().numpy()
        for b, n0 in enumerate(prompts):
            if step % 13 and b != 1:
                continue  # every step for the short prompt (window / history edges), a sample for the rest
            ref = _oracle(st, bt, b, n0, step + 1, qn[b], C)
            worst = max(worst, O.rel_l2(on[b], ref))
    print(f"batched vLLM decode worst rel-L2 {worst:.3e}")
    assert worst <= 2e-3, worst
