"""The split-group communicator (smaq_comm_*) on real NCCL.

One GPU: a one-rank group all-gathers decode partials and the merge of the gathered
partials equals the unsplit decode's combine.  Two or more GPUs: two ranks (child processes, NVLS
off) exchange partials; then rank 1 leaves between steps and rank 0's next exchange ends in
PeerFailure within its deadline instead of hanging."""

import os
import sys
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_one_rank_exchange():
    from smaq_b200.distributed import SplitComm
    torch.cuda.set_device(0)
    comm = SplitComm(1, 0, SplitComm.unique_id(), timeout=30.0)
    try:
        for n in (1, 258, 4 * 16 * 258):
            x = torch.randn(n, device="cuda")
            y = comm.all_gather(x)
            assert y.shape == (1, n)
            assert torch.equal(y[0], x)
    finally:
        comm.close()


CHILD = r"""
import os, sys, time, torch
sys.path.insert(0, os.environ["REPO"])
from smaq_b200.distributed import SplitComm, PeerFailure
rank, mode, idfile = int(sys.argv[1]), sys.argv[2], sys.argv[3]
torch.cuda.set_device(rank)
if rank == 0:
    cid = SplitComm.unique_id()
    open(idfile + ".tmp", "wb").write(cid)
    os.replace(idfile + ".tmp", idfile)
else:
    t0 = time.time()
    while not os.path.exists(idfile):
        assert time.time() - t0 < 60
        time.sleep(0.05)
    cid = open(idfile, "rb").read()
comm = SplitComm(2, rank, cid, timeout=20.0)
x = torch.full((4, 16, 258), float(rank + 1), device="cuda")
y = comm.all_gather(x)
torch.cuda.synchronize()
assert torch.equal(y[0], torch.full_like(x, 1.0)) and torch.equal(y[1], torch.full_like(x, 2.0))
print("step1 ok", flush=True)
if mode == "leave":
    if rank == 1:
        os._exit(0)  # leaves between steps, nothing in flight
    comm.timeout = 3.0
    t0 = time.time()
    try:
        comm.all_gather(x)
        print("no failure", flush=True)
        sys.exit(3)
    except PeerFailure as e:
        dt = time.time() - t0
        print(f"peer failure after {dt:.1f}s: {e}", flush=True)
        assert dt < 15
    comm.close()
    # the context still works
    assert float((x * 2).sum()) == 4 * 16 * 258 * 2.0
    print("rank0 recovered", flush=True)
    os._exit(0)
comm.close()
print("done", flush=True)
"""


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["clean", "leave"])
def test_two_rank_exchange_and_peer_loss(tmp_path, mode):
    import subprocess
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = tmp_path / "child.py"
    script.write_text(CHILD)
    env = dict(os.environ, REPO=repo, NCCL_NVLS_ENABLE="0", CUDA_VISIBLE_DEVICES="0,1")
    idfile = str(tmp_path / "id")
    procs = [subprocess.Popen([sys.executable, str(script), str(r), mode, idfile], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in (0, 1)]
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=120)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append((p.returncode, out))
    for rc, out in outs:
        assert rc == 0, out
    assert "step1 ok" in outs[0][1]
    if mode == "leave":
        assert "peer failure" in outs[0][1] and "rank0 recovered" in outs[0][1], outs[0][1]
