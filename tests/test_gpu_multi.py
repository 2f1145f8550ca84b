"""Sequence-split decode across real GPUs over NCCL (smaq_b200.distributed.sharded_decode): each
rank decodes its token range into partials, the partials are all-gathered (torch process group,
or the library's own communicator, smaq_comm_*) and merged, and the result must match the
single-GPU decode of the whole history.  Needs >= 2 GPUs (skipped
otherwise); every rank runs in its own process."""

import os

import numpy as np
import pytest

from oracle import smaq_oracle as O

pytestmark = pytest.mark.gpu
D = 128


def _worker(rank, world, port, result_path, native=False):
    import torch
    import torch.distributed as dist
    from smaq_b200 import distributed as sd, ops, synthetic as syn
    from smaq_b200._lib import SMAQ_KEYS_BVQ, SMAQ_LAYOUT_DECODE
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        B, Hkv, G, page = 2, 1, 4, 16
        hist, recent = [3000, 40], [64, 5]
        rng = np.random.default_rng(3)
        C = torch.from_numpy(rng.standard_normal((16, 256, 8)).astype(np.float32)).to(dev)
        Eb = torch.from_numpy((np.eye(8)[None] + 0.1 * rng.standard_normal((16, 8, 8))).astype(np.float32)).to(dev)
        dec = torch.from_numpy((rng.standard_normal((16, 256, 8)) * 0.5).astype(np.float16).astype(np.float32)).to(dev)
        plan = sd.make_plan(world, Hkv)
        groups = sd.native_split_comms(plan, rank, timeout=30.0) if native else sd.split_groups(plan)
        # every rank builds the whole store (same seeds) and attends only to its range
        pages = [(n + page - 1) // page for n in hist]
        st = {k: torch.zeros((sum(pages), Hkv, page, w), dtype=torch.uint8, device=dev) for k, w in
              (("codes", 16), ("vd", 32))}
        vs = torch.zeros((sum(pages), Hkv, page, 4), dtype=torch.bfloat16, device=dev)
        vz = torch.zeros_like(vs)
        bt = torch.zeros((B, max(pages)), dtype=torch.int32, device=dev)
        o = 0
        for b, n in enumerate(hist):
            bt[b, :pages[b]] = torch.arange(o, o + pages[b], dtype=torch.int32)
            k = torch.from_numpy(syn.keys((n, Hkv), D, seed=10 + b)).to(dev).to(torch.bfloat16)
            v = torch.from_numpy(syn.values((n, Hkv), D, seed=20 + b)).to(dev).to(torch.bfloat16)
            t = torch.arange(n, device=dev)
            ops.append(k, v, n_heads=Hkv, slots=(o * page + t).to(torch.int64), page_size=page,
                       key_format=SMAQ_KEYS_BVQ, E_blocks=Eb, centroids=C, key_codes=st["codes"], v_data=st["vd"],
                       v_scales=vs, v_zeros=vz, layout=SMAQ_LAYOUT_DECODE)
            o += pages[b]
        rk = torch.from_numpy(syn.keys((B, max(recent), Hkv), D, seed=30)).to(dev).to(torch.bfloat16)
        rv = torch.from_numpy(syn.values((B, max(recent), Hkv), D, seed=31)).to(dev).to(torch.bfloat16)
        q = torch.from_numpy(syn.queries((B, Hkv * G), D, seed=32)).to(dev).to(torch.bfloat16)
        common = dict(n_kv_heads=Hkv, key_format=SMAQ_KEYS_BVQ, centroids=dec, centroids_f16=ops.fp16_codebook(dec),
                      key_codes=st["codes"], v_data=st["vd"], v_scales=vs, v_zeros=vz, page_size=page,
                      recent_k=rk, recent_v=rv, layout=SMAQ_LAYOUT_DECODE)
        full = ops.decode(q, hist_len=torch.tensor(hist, dtype=torch.int32, device=dev), block_table=bt,
                          recent_len=torch.tensor(recent, dtype=torch.int32, device=dev), **common)

        def decode_fn(partial):
            rngs = [plan.token_range(n, rank) for n in hist]
            btl = torch.zeros_like(bt)
            for b, (lo, hi) in enumerate(rngs):
                npg = (hi - lo + page - 1) // page
                btl[b, :npg] = bt[b, lo // page:lo // page + npg]
            rl = recent if plan.holds_recent(rank) else [0] * B
            part = torch.empty((B, Hkv * G, 2 * D + 2), dtype=torch.float32, device=dev)
            ops.decode(q, hist_len=torch.tensor([hi - lo for lo, hi in rngs], dtype=torch.int32, device=dev),
                       hist_total=torch.tensor(hist, dtype=torch.int32, device=dev), block_table=btl,
                       recent_len=torch.tensor(rl, dtype=torch.int32, device=dev), partial_out=part, want_out=False,
                       **common)
            return part

        got = sd.sharded_decode(plan, rank, groups, decode_fn, torch.bfloat16)
        torch.cuda.synchronize()
        err = O.rel_l2(got.float().cpu().numpy(), full.float().cpu().numpy())
        with open(f"{result_path}.{rank}", "w") as fh:
            fh.write(repr(err))
        for g in groups:
            if isinstance(g, sd.SplitComm):
                g.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("native", [False, True], ids=["torch_group", "smaq_comm"])
def test_sequence_split_over_nccl(tmp_path, native):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    from smaq_b200 import build
    build.build()
    world = 2
    res = str(tmp_path / "err")
    mp.start_processes(_worker, args=(world, 29700 + os.getpid() % 200 + 300 * native, res, native), nprocs=world,
                       join=True,
                       start_method="spawn")
    for r in range(world):
        assert float(open(f"{res}.{r}").read()) <= 2e-3
