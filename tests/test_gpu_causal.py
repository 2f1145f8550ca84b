"""No-allocation prefill attention (smaq/integration/vllm.py:133-163 replaced): causal attention of a
chunk over itself on this package's decode kernel (``ops.causal_attention``), against an fp64
restatement with grouped query heads.  Shapes cover the fused tensor-core window (bf16,
2 n Hkv <= 2048), the general kernel (more rows, fp32), one token, and G = 8."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def causal_ref(q, k, v, scale):
    n, Hq, D = q.shape
    G = Hq // k.shape[1]
    qq, kk, vv = q.double(), k.double().repeat_interleave(G, 1), v.double().repeat_interleave(G, 1)
    s = torch.einsum("thd,shd->hts", qq, kk) * scale
    s = s.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool, device=q.device), 1), float("-inf"))
    return torch.einsum("hts,shd->thd", s.softmax(-1), vv)


def rel_l2(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize("n,Hq,Hkv,dtype,path", [
    (37, 28, 4, torch.bfloat16, "fused"),
    (100, 64, 8, torch.bfloat16, "fused"),
    (300, 28, 4, torch.bfloat16, "general"),
    (513, 32, 8, torch.float16, "general"),
    (64, 8, 2, torch.float32, "general"),
    (1, 8, 2, torch.bfloat16, "fused"),
])
def test_causal_attention_matches_fp64(cuda, n, Hq, Hkv, dtype, path):
    from smaq_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(n * 31 + Hq)
    D = 128
    q = torch.randn(n, Hq, D, generator=g).to(cuda, dtype)
    k = torch.randn(n, Hkv, D, generator=g).to(cuda, dtype)
    v = torch.randn(n, Hkv, D, generator=g).to(cuda, dtype)
    scale = 1.0 / math.sqrt(D)
    out = ops.causal_attention(q, k, v, scale)
    torch.cuda.synchronize()
    assert out.shape == q.shape and out.dtype == dtype
    err = rel_l2(out, causal_ref(q, k, v, scale))
    tol = 1e-5 if dtype == torch.float32 else 2e-3
    assert err <= tol, (path, err)


def test_vllm_no_alloc_prefill_uses_it(cuda):
    from smaq_b200.integration import vllm as iv
    D = 128
    q = torch.randn(50, 12, D, device=cuda, dtype=torch.bfloat16)
    kv = torch.randn(50, 2, 2, D, device=cuda, dtype=torch.bfloat16)
    k, v = kv[:, 0], kv[:, 1]                                     # strided views, as vLLM hands them
    out = iv._causal_chunk_attention(q, k, v, 0.1)
    assert rel_l2(out, causal_ref(q, k, v, 0.1)) <= 2e-3
