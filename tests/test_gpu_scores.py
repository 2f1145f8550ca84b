"""Standalone scores and attend kernels (smaq_key_scores / smaq_attend_values) against fp64
restatements of the reference's eager torch (smaq/quantizer.py:154-184, smaq/block_vq.py:273-297,
smaq/kv_cache.py:94-103, :218-267), and the HF-style SMAQKVCache routed through them."""

import numpy as np
import pytest
import torch

from oracle import smaq_oracle as O

pytestmark = pytest.mark.gpu


def tn(t):
    return t.float().cpu().numpy().astype(np.float64) if t.dtype != torch.int64 else t.cpu().numpy()


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("qdt", [torch.float32, torch.bfloat16])
def test_scalar_key_scores(cuda, bits, D, qdt):
    from smaq_b200.quantizer import SMAQQuantizer
    g = torch.Generator().manual_seed(bits * 100 + D)
    qz = SMAQQuantizer(D, bits=bits, device=cuda)
    qz.fit(torch.randn(512, D, generator=g).to(cuda))
    keys = torch.randn(2, 3, 777, D, generator=g).to(cuda).to(torch.bfloat16)
    kq = qz.quantize(keys)
    for Q in (1, 5, 9):
        q = torch.randn(2, 3, Q, D, generator=g).to(cuda).to(qdt)
        got = qz.attention_score(q, kq, scale=D ** -0.5)
        assert got.shape == (2, 3, Q, 777) and got.dtype == qdt
        y = tn(qz.centroids)[O.unpack_indices(tn(kq.indices).astype(np.uint8), bits, D)]
        qr = tn(q) @ tn(qz.E_inv).T
        ref = np.einsum("abqd,abtd->abqt", qr, y) * tn(kq.norms)[:, :, None, :] * D ** -0.5
        assert rel(tn(got), ref) <= (2e-6 if qdt == torch.float32 else 4e-3)


def test_triton_kernels_entry_point(cuda):
    """smaq.triton_kernels.smaq_attention_scores (smaq/triton_kernels.py:190-208): the reference's
    decode-tile shape (query [n_qh, D], packed keys [N, P], norms [N]) -> unscaled fp32 scores,
    on the CUDA scoring kernel."""
    from smaq_b200.quantizer import SMAQQuantizer
    from smaq_b200.triton_kernels import smaq_attention_scores
    g = torch.Generator().manual_seed(7)
    D, bits = 128, 4
    qz = SMAQQuantizer(D, bits=bits, device=cuda)
    qz.fit(torch.randn(512, D, generator=g).to(cuda))
    kq = qz.quantize(torch.randn(1000, D, generator=g).to(cuda).to(torch.bfloat16))
    q = torch.randn(8, D, generator=g).to(cuda).to(torch.bfloat16)
    got = smaq_attention_scores(qz, q, kq)
    assert got.shape == (8, 1000) and got.dtype == torch.float32
    y = tn(qz.centroids)[O.unpack_indices(tn(kq.indices).astype(np.uint8), bits, D)]
    ref = (tn(q) @ tn(qz.E_inv).T) @ y.T * tn(kq.norms)[None, :]
    assert rel(tn(got), ref) <= 2e-6


@pytest.mark.parametrize("int64", [True, False])
def test_bvq_key_scores(cuda, int64):
    from smaq_b200.block_vq import SMAQBlockVQ
    D = 128
    g = torch.Generator().manual_seed(7)
    vq = SMAQBlockVQ(D, device=cuda)
    vq.fit(torch.randn(4096, D, generator=g).to(cuda), torch.randn(1024, D, generator=g).to(cuda))
    keys = torch.randn(4, 1000, D, generator=g).to(cuda).to(torch.bfloat16)
    kq = vq.quantize(keys)
    if not int64:
        kq = kq._replace(indices=kq.indices.to(torch.uint8))
    q = torch.randn(4, 6, D, generator=g).to(cuda)
    got = vq.attention_score(q, kq, scale=0.1)
    K = O.bvq_dequantize(tn(kq.indices).astype(np.int64), tn(vq.decoded_centroids))
    ref = np.einsum("aqd,atd->aqt", tn(q), K) * 0.1
    assert rel(tn(got), ref) <= 2e-6


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("N", [50, 5000])
@pytest.mark.parametrize("D,gs", [(128, 32), (64, 64)])
def test_attend_values(cuda, bits, N, D, gs):
    from smaq_b200 import ops
    from smaq_b200.kv_cache import quantize_values
    g = torch.Generator().manual_seed(N + bits)
    v = torch.randn(2, 3, N, D, generator=g).to(cuda).to(torch.bfloat16)
    vq = quantize_values(v, bits=bits, group_size=gs)
    for Q in (1, 6):
        w = torch.softmax(torch.randn(2, 3, Q, N, generator=g), -1).to(cuda)
        got = ops.attend_values(w, vq.data, vq.scales, vq.zeros, bits=bits, group_size=gs)
        V = O.dequantize_values(tn(vq.data).astype(np.uint8), tn(vq.scales), tn(vq.zeros), bits, gs)
        ref = np.einsum("abqt,abtd->abqd", tn(w), V)
        assert got.shape == (2, 3, Q, D) and rel(tn(got), ref) <= 2e-6


def test_hf_cache_scores_and_attend(cuda):
    """prefill + appends across the buffer edge: the logits and the attended output equal the
    eager restatement over the cache's own compressed rows and exact buffer."""
    from smaq_b200.kv_cache import SMAQKVCache, dequantize_values
    D, B, H = 128, 2, 4
    g = torch.Generator().manual_seed(3)
    cache = SMAQKVCache(D, buffer_size=64, device=cuda, dtype=torch.bfloat16)
    rnd = lambda *s: torch.randn(*s, generator=g).to(cuda).to(torch.bfloat16)
    cache.prefill(rnd(B, H, 300, D), rnd(B, H, 300, D))
    for n in (1, 5, 70, 1):
        cache.append(rnd(B, H, n, D), rnd(B, H, n, D))
    assert cache.get_seq_length() == 377 and cache.key_buffer.shape[-2] == 64
    kq, vq = cache.key_quantized, cache.value_quantized
    assert kq.indices.shape[-2] == 313 and vq.data.shape[-2] == 313
    q = rnd(B, H, 1, D)
    s = cache.attention_scores(q)
    qz = cache.key_quantizer.quantizer
    y = tn(qz.centroids)[O.unpack_indices(tn(kq.indices).astype(np.uint8), 3, D)]
    hist = np.einsum("abqd,abtd->abqt", tn(q) @ tn(qz.E_inv).T, y) * tn(kq.norms)[:, :, None, :]
    exact = np.einsum("abqd,abtd->abqt", tn(q), tn(cache.key_buffer))
    ref = np.concatenate([hist, exact], -1) * D ** -0.5
    assert s.shape == (B, H, 1, 377) and rel(tn(s), ref) <= 4e-3
    w = torch.softmax(s.float(), -1)
    out = cache.attend(w)
    V = tn(dequantize_values(vq, 32))
    ref = np.einsum("abqt,abtd->abqd", tn(w)[..., :313], V) + np.einsum("abqt,abtd->abqd", tn(w)[..., 313:],
                                                                         tn(cache.value_buffer))
    assert out.dtype == torch.float32 and rel(tn(out), ref) <= 1e-5
    info = cache.memory_bytes()
    assert info["total"] == info["quantized_keys"] + info["quantized_values"] + info["buffer"]
