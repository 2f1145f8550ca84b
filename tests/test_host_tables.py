"""Host-side tables and the capture flush pattern against the reference's own outputs (CPU).

These are the one-time parts of the path that stay in torch: the scalar codebook
(SMAQQuantizer.__init__, smaq/quantizer.py:96-119), the metric fit (SMAQQuantizer.fit,
smaq/quantizer.py:121-129, through build_smaq_metric, smaq/ssf.py:8-29), the block-VQ fit with
its k-means (SMAQBlockVQ.fit / _kmeans, smaq/block_vq.py:37-79, :160-210) and the ring-buffer
flush of KVCaptureEngine (smaq/capture.py:60-91).  The golden arrays were written by
tests/golden/make_golden.py running the reference.
"""

import numpy as np
import pytest
import torch

from smaq_b200 import synthetic as syn

D = 128
CPU = torch.device("cpu")


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_scalar_quantizer_tables_match_reference(golden, bits):
    from smaq_b200.quantizer import SMAQQuantizer
    qz = SMAQQuantizer(D, bits=bits, device=CPU)
    # the codebook is a pure function of the bit width: bit-identical
    assert np.array_equal(qz.centroids.numpy(), golden[f"sq_b{bits}_centroids"])
    assert np.array_equal(qz.decision_boundaries.numpy(), golden[f"sq_b{bits}_boundaries"])
    qz.fit(torch.from_numpy(syn.calibration_queries(512, D)))
    # same torch ops in the same order on the same inputs (eigh included)
    for name in ("E", "E_inv"):
        got, ref = getattr(qz, name).numpy(), golden[f"sq_b{bits}_{name}"]
        np.testing.assert_allclose(got, ref, rtol=0, atol=2e-6 * np.abs(ref).max())


def test_strategy_fit_matches_reference(golden):
    """SMAQFullMetricScalarStrategy.fit (the store's default strategy) gives the reference's E."""
    from smaq_b200.strategies import SMAQFullMetricScalarStrategy
    for bits in (3, 4):
        s = SMAQFullMetricScalarStrategy(D, bits=bits, device=CPU)
        s.fit(torch.from_numpy(syn.calibration_queries(512, D)))
        for name in ("E", "E_inv"):
            got, ref = getattr(s.quantizer, name).numpy(), golden[f"hy_scalar{bits}_{name}"]
            np.testing.assert_allclose(got, ref, rtol=0, atol=2e-6 * np.abs(ref).max())


def test_block_vq_fit_matches_reference(golden):
    """Per-block metric, k-means++ seeding (same RNG calls) and 20 Lloyd steps: the reference's
    codebook on the same CPU inputs."""
    from smaq_b200.block_vq import SMAQBlockVQ
    calk = syn.keys((4096,), D, seed=11)
    vq = SMAQBlockVQ(D, device=CPU)
    vq.fit(torch.from_numpy(calk), torch.from_numpy(syn.calibration_queries(4096, D, seed=12)))
    for name in ("E_blocks", "E_inv_blocks", "centroids", "decoded_centroids"):
        got, ref = getattr(vq, name).numpy(), golden["bvq_fit_" + name]
        np.testing.assert_allclose(got, ref, rtol=0, atol=1e-5 * max(1.0, np.abs(ref).max()), err_msg=name)
    # after rounding to fp16 values the tables the GPU tests use are exactly the golden ones
    for name in ("E_blocks", "centroids", "decoded_centroids"):
        assert np.array_equal(getattr(vq, name).half().float().numpy(), golden["bvq_" + name]), name


class _CountingStore:
    """Stands in for the compressed store: records the chunk lengths handed to it."""

    def __init__(self, num_kv_heads, head_dim):
        self.num_kv_heads, self.head_dim, self.device = num_kv_heads, head_dim, CPU
        self.chunks = []

    @property
    def num_tokens(self):
        return sum(self.chunks)

    def append_chunk(self, k, v):
        assert k.shape == v.shape and k.shape[1:] == (self.num_kv_heads, self.head_dim)
        self.chunks.append(k.shape[0])

    def reset(self):
        self.chunks.clear()


def test_capture_flush_trace_matches_reference(golden):
    """Replays the golden capture run: prefill 13 tokens into an 8-slot ring, then 27 decode
    tokens; the store size and ring size after every step, and the flushed chunk lengths, equal
    the reference's (whole-ring flush when a token arrives at a full ring)."""
    from smaq_b200.capture import KVCaptureEngine
    store = _CountingStore(2, D)
    eng = KVCaptureEngine(store, ring_capacity=8, device=CPU, dtype=torch.float32)
    kk = torch.from_numpy(syn.keys((40, 2), D, seed=500))
    vv = torch.from_numpy(syn.values((40, 2), D, seed=501))
    eng.ingest_prefill(kk[:13], vv[:13], 13)
    trace = [store.num_tokens, eng.ring.size]
    for t in range(13, 40):
        eng.ingest_decode(kk[t:t + 1], vv[t:t + 1], 1)
        trace += [store.num_tokens, eng.ring.size]
    assert trace == golden["capture_trace"].tolist()
    assert store.chunks == golden["capture_chunks"].tolist()
    # the exact window keeps the most recent tokens, in order
    k_win, _ = eng.ring.peek()
    n = eng.ring.size
    assert torch.equal(k_win, kk[40 - n:40])
