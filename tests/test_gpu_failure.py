"""Failure detection on the device without a device fault: a kernel whose mbarrier wait can never
complete runs out of its poll bound, records the error and returns; the host reads the status
and the context stays usable for the real kernels afterwards.  The host-side half (a peer rank
that dies or stalls before the partials exchange) is covered with gloo ranks in
tests/test_distributed.py."""

import pytest

from test_gpu_decode import run_case

pytestmark = pytest.mark.gpu


def test_bounded_wait_returns_error_status(cuda):
    import torch
    from smaq_b200 import _lib, ops
    for limit in (1, 64, 4096):
        assert ops.selftest_wait_timeout(limit) == 5
        assert b"ran out" in _lib.load().smaq_last_error()
    torch.cuda.synchronize()  # the context is still healthy


def test_kernels_run_and_report_ok_after_a_timeout(cuda):
    from smaq_b200 import ops
    assert ops.selftest_wait_timeout(256) == 5
    # block-VQ fused path and scalar fused path through the no-allocation entry point, whose
    # error word smaq_decode_status reads back
    run_case(cuda, "bvq", 0, B=3, Hkv=2, G=4, hist=[900, 17, 0], recent=[128, 9, 1], page_size=16,
             dtype="bfloat16", seed=31, layout=1, entry="smaq_decode_noalloc")
    ops.decode_status(3, 2)
    run_case(cuda, "scalar", 4, B=2, Hkv=2, G=4, hist=[500, 40], recent=[64, 3], page_size=16,
             dtype="bfloat16", seed=32, layout=1, entry="smaq_decode_noalloc")
    ops.decode_status(2, 2)
    ops.append_status()


def test_decode_status_rejects_bad_sizes(cuda):
    from smaq_b200 import ops
    with pytest.raises(RuntimeError, match="INVALID"):
        ops.decode_status(0, 2)
