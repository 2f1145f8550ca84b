"""Device k-means (smaq_kmeans) for block-VQ calibration against the torch restatement of the
reference's _kmeans (smaq/block_vq.py:37-79): the same Lloyd result from the same seeds, the
same distortion from its own k-means++ draws, determinism, and SMAQBlockVQ.fit end to end."""

import pytest
import torch

from smaq_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _data(cuda, nb=4, n=8192, d=8, seed=5):
    g = torch.Generator().manual_seed(seed)
    # clustered points: 64 centres, anisotropic noise
    centres = torch.randn(nb, 64, d, generator=g) * 3
    pick = torch.randint(0, 64, (nb, n), generator=g)
    x = centres.gather(1, pick[..., None].expand(nb, n, d)) + torch.randn(nb, n, d, generator=g) * 0.7
    return x.to(cuda)


def _distortion(x, c):
    return float(torch.cdist(x, c).min(dim=1).values.square().mean())


def test_seeding_picks_distinct_data_points_and_is_deterministic(cuda):
    from smaq_b200 import ops
    x = _data(cuda)
    c0 = ops.kmeans(x, 256, n_iters=0, seed=3)
    assert torch.equal(c0, ops.kmeans(x, 256, n_iters=0, seed=3))
    assert not torch.equal(c0, ops.kmeans(x, 256, n_iters=0, seed=4))
    for b in range(x.shape[0]):
        d = (c0[b][:, None, :] - x[b][None, :, :]).abs().amax(-1).min(dim=1).values
        assert float(d.max()) == 0.0                               # every centre is a data point
        assert torch.unique(c0[b], dim=0).shape[0] == 256          # k-means++ never repeats one


def test_lloyd_matches_torch_from_the_same_seeds(cuda):
    from smaq_b200 import ops
    from smaq_b200.block_vq import _lloyd
    x = _data(cuda)
    c0 = ops.kmeans(x, 256, n_iters=0, seed=9)
    got = ops.kmeans(x, 256, n_iters=20, seed=9)
    for b in range(x.shape[0]):
        ref = _lloyd(x[b], c0[b].clone(), 20)
        # float summation order differs (torch adds with atomics); a near-tie may move a point
        close = (got[b] - ref).abs().max(dim=1).values <= 1e-3
        assert float(close.float().mean()) >= 0.97
        assert abs(_distortion(x[b], got[b]) / _distortion(x[b], ref) - 1) <= 2e-3


def test_distortion_matches_reference_kmeans(cuda):
    from smaq_b200 import ops
    from smaq_b200.block_vq import _kmeans
    x = _data(cuda, nb=2)
    got = ops.kmeans(x, 256, n_iters=20, seed=42)
    for b in range(2):
        ref = _kmeans(x[b], 256, 20, 42 + b)
        assert _distortion(x[b], got[b]) <= 1.03 * _distortion(x[b], ref)


def test_block_vq_fit_device_vs_reference(cuda):
    from smaq_b200.block_vq import SMAQBlockVQ
    D = 128
    k = torch.from_numpy(syn.keys((8192,), D, seed=31)).to(cuda)
    q = torch.from_numpy(syn.calibration_queries(2048, D, seed=32)).to(cuda)
    held_k = torch.from_numpy(syn.keys((2048,), D, seed=33)).to(cuda)
    held_q = torch.from_numpy(syn.calibration_queries(2048, D, seed=34)).to(cuda)
    dev = SMAQBlockVQ(D, device=cuda).fit(k, q)                    # auto: device k-means
    ref = SMAQBlockVQ(D, device=cuda).fit(k, q, kmeans="reference")
    assert torch.equal(dev.E_blocks, ref.E_blocks)
    assert dev.logit_mse(held_q, held_k) <= 1.05 * ref.logit_mse(held_q, held_k)
