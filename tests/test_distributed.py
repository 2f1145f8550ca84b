"""Host logic of the multi-GPU decode path (smaq_b200.distributed) on CPU: gloo ranks, the
oracle as the per-rank compute and as the combine, checked against the unsplit reference
attention.  The device kernels of the same path are covered by tests/test_gpu_sharded.py."""

import os

import numpy as np
import pytest

from oracle import smaq_oracle as O
from smaq_b200 import synthetic as syn
from smaq_b200.distributed import ShardPlan, make_plan

D = 128


def test_make_plan_prefers_heads():
    assert make_plan(8, 8) == ShardPlan(8, 8, 8, 1)
    assert make_plan(8, 4) == ShardPlan(8, 4, 4, 2)
    assert make_plan(2, 8) == ShardPlan(2, 8, 2, 1)
    assert make_plan(4, 2) == ShardPlan(4, 2, 2, 2)
    assert make_plan(6, 4) == ShardPlan(6, 4, 2, 3)
    with pytest.raises(ValueError):
        make_plan(0, 4)


@pytest.mark.parametrize("world,n_kv", [(2, 1), (4, 2), (8, 4), (3, 3), (6, 4)])
@pytest.mark.parametrize("n", [0, 5, 16, 40, 1000, 4097])
def test_ranges_cover_every_token_once(world, n_kv, n):
    plan = make_plan(world, n_kv)
    for hg in range(plan.head_groups):
        seen = np.zeros(n, np.int64)
        for sp in range(plan.seq_splits):
            r = hg * plan.seq_splits + sp
            lo, hi = plan.token_range(n, r)
            assert 0 <= lo <= hi <= n
            if sp < plan.seq_splits - 1 and hi < n:
                assert hi % 16 == 0
            seen[lo:hi] += 1
        assert (seen == 1).all()
    heads = sorted(h for r in range(world) if plan.coords(r)[1] == 0 for h in plan.kv_heads(r))
    assert heads == list(range(n_kv))
    assert sum(plan.holds_recent(r) for r in range(world)) == plan.head_groups


def _case(seed, n_hist, n_recent, Hkv, G):
    K = syn.keys((n_hist, Hkv), D, seed=seed).transpose(1, 0, 2)
    V = syn.values((n_hist, Hkv), D, seed=seed + 1).transpose(1, 0, 2)
    rk = syn.keys((n_recent, Hkv), D, seed=seed + 2)
    rv = syn.values((n_recent, Hkv), D, seed=seed + 3)
    q = syn.queries((1, Hkv * G), D, seed=seed + 4)
    return q, K, V, rk, rv


def _worker(rank, world, port, Hkv, G, cases, q_dtype, result_path):
    import torch
    import torch.distributed as dist
    from smaq_b200 import distributed as sd
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = sd.make_plan(world, Hkv)
        groups = sd.split_groups(plan)
        worst = 0.0
        for seed, n_hist, n_recent in cases:
            q, K, V, rk, rv = _case(seed, n_hist, n_recent, Hkv, G)
            kv = plan.kv_heads(rank)
            qh = plan.q_heads(rank, Hkv * G)
            lo, hi = plan.token_range(n_hist, rank)
            rec = plan.holds_recent(rank)

            def decode_fn(partial):
                part = O.partial_attention(q[0, qh.start:qh.stop], K[kv.start:kv.stop, lo:hi],
                                           V[kv.start:kv.stop, lo:hi],
                                           rk[:, kv.start:kv.stop] if rec else None,
                                           rv[:, kv.start:kv.stop] if rec else None,
                                           len(qh), len(kv), hist_total=n_hist)
                if partial:
                    return torch.from_numpy(part[None].astype(np.float32))
                return torch.from_numpy(O.merge_partials(part[None, None], q_dtype)[0])

            def merge_fn(parts, out_dtype):
                return torch.from_numpy(O.merge_partials(parts.numpy(), q_dtype))

            got = sd.sharded_decode(plan, rank, groups, decode_fn, torch.float32, merge_fn).numpy().reshape(len(qh), D)
            ref, _, _ = O.hybrid_attention(q, q_dtype, K if n_hist else None, V if n_hist else None,
                                           rk if n_recent else None, rv if n_recent else None, Hkv * G, Hkv)
            worst = max(worst, O.rel_l2(got, ref[0, qh.start:qh.stop]))
        with open(f"{result_path}.{rank}", "w") as fh:
            fh.write(repr(worst))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,Hkv,G", [(2, 1, 4), (4, 2, 4), (2, 2, 7)])
def test_sharded_decode_matches_reference_gloo(tmp_path, world, Hkv, G):
    import torch.multiprocessing as mp
    cases = [(11, 300, 17), (12, 40, 0), (13, 10, 9), (14, 0, 5), (15, 33, 64)]
    port = 29500 + (os.getpid() % 1000) + world * 7 + G
    res = str(tmp_path / "worst")
    mp.start_processes(_worker, args=(world, port, Hkv, G, cases, "bf16", res), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        w = float(open(f"{res}.{r}").read())
        assert w <= 2e-3, (r, w)


def _failure_worker(rank, world, port, mode, result_path):
    """Rank 1 fails on the host before the partials exchange (``exit``: the process ends;
    ``stall``: it stays alive but never joins); rank 0 must get a PeerFailure within the
    split group's timeout instead of waiting forever."""
    import time
    import torch
    import torch.distributed as dist
    from smaq_b200 import distributed as sd
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    plan = sd.make_plan(world, 1)
    groups = sd.split_groups(plan, timeout=3.0)
    if rank == 1:
        if mode == "exit":
            os._exit(0)
        time.sleep(20.0)
        os._exit(0)
    t0 = time.monotonic()
    outcome = "completed"
    try:
        sd.sharded_decode(plan, rank, groups, lambda partial: torch.zeros((1, 4, 2 * D + 2)), torch.float32,
                          lambda parts, dt: parts[0, :, :, :D])
    except sd.PeerFailure as e:
        outcome = "PeerFailure:" + str(e).splitlines()[0][:200]
    with open(result_path, "w") as fh:
        fh.write(f"{time.monotonic() - t0:.3f}\n{outcome}\n")
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_peer_failure_is_detected_gloo(tmp_path, mode):
    import torch.multiprocessing as mp
    port = 31000 + (os.getpid() % 1000) + (0 if mode == "exit" else 3)
    res = str(tmp_path / "outcome")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_failure_worker, args=(r, 2, port, mode, res)) for r in range(2)]
    for p in procs:
        p.start()
    procs[0].join(60)
    alive = procs[0].is_alive()
    for p in procs:
        if p.is_alive():
            p.kill()
        p.join(5)
    assert not alive, "rank 0 hung in the exchange"
    elapsed, outcome = open(res).read().splitlines()
    assert outcome.startswith("PeerFailure:"), outcome
    assert "ranks [0, 1]" in outcome
    assert float(elapsed) < 30.0
