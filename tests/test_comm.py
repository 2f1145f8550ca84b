"""The split-group communicator's failure handling (smaq_comm_*), driven on the host through a
test double of the NCCL calls: a peer that never arrives, a remote error during the exchange, a
finalize that never completes.  Nothing here touches a GPU; the real NCCL path is covered by
tests/test_gpu_comm.py."""

import ctypes
import time

import pytest

from smaq_b200 import _lib
from smaq_b200.distributed import PeerFailure, SplitComm

IN_PROGRESS, REMOTE_ERROR = 7, 6


class FakeNccl:
    """Records calls; ``state`` is what ncclCommGetAsyncError reports, ``gather_result`` what
    ncclAllGather returns, ``finalize_state`` the state after ncclCommFinalize."""

    def __init__(self, state=0, gather_result=0, finalize_state=0):
        self.state, self.gather_result, self.finalize_state = state, gather_result, finalize_state
        self.calls = []
        self._handle = ctypes.c_int(0)

        def unique_id(buf):
            ctypes.memset(buf, 7, _lib.COMM_ID_BYTES)
            return 0

        def init_rank(handle, n, id_, rank):
            self.calls.append(("init", n, rank))
            handle[0] = ctypes.addressof(self._handle)
            return IN_PROGRESS

        def async_error(h):
            self.calls.append("poll")
            return self.state

        def all_gather(send, recv, nbytes, h, stream):
            self.calls.append(("all_gather", nbytes))
            return self.gather_result

        def abort_comm(h):
            self.calls.append("abort")
            return 0

        def finalize(h):
            self.calls.append("finalize")
            self.state = self.finalize_state
            return IN_PROGRESS

        def destroy(h):
            self.calls.append("destroy")
            return 0

        self.table = _lib.CommBackend(_lib.CommUniqueId(unique_id), _lib.CommInitRank(init_rank),
                                      _lib.CommHandleCall(async_error), _lib.CommAllGather(all_gather),
                                      _lib.CommHandleCall(abort_comm), _lib.CommHandleCall(finalize),
                                      _lib.CommHandleCall(destroy))

    def count(self, name):
        return sum(1 for c in self.calls if c == name or (isinstance(c, tuple) and c[0] == name))


@pytest.fixture
def lib():
    lib = _lib.load()
    yield lib
    assert lib.smaq_comm_set_backend(None) == 0


def install(lib, fake):
    assert lib.smaq_comm_set_backend(ctypes.byref(fake.table)) == 0


def init(lib, timeout=2.0, n=2, rank=0):
    h = ctypes.c_void_p()
    st = lib.smaq_comm_init(ctypes.byref(h), n, rank, b"\x07" * _lib.COMM_ID_BYTES, timeout)
    return st, h


def test_incomplete_backend_table_is_rejected(lib):
    t = _lib.CommBackend()
    assert lib.smaq_comm_set_backend(ctypes.byref(t)) == 1
    assert b"every call" in lib.smaq_last_error()


def test_init_of_a_missing_peer_times_out_and_aborts(lib):
    fake = FakeNccl(state=IN_PROGRESS)  # the other rank never joins: init stays in progress
    install(lib, fake)
    t0 = time.monotonic()
    st, h = init(lib, timeout=0.3)
    dt = time.monotonic() - t0
    assert st == _lib.SMAQ_ERR_TIMEOUT, lib.smaq_last_error()
    assert not h.value
    assert 0.3 <= dt < 3.0
    assert fake.count("abort") == 1
    assert b"no progress" in lib.smaq_last_error()


def test_bad_rank_is_invalid(lib):
    install(lib, FakeNccl())
    st, _ = init(lib, n=2, rank=2)
    assert st == 1


def test_remote_error_during_the_exchange_aborts(lib):
    fake = FakeNccl()
    install(lib, fake)
    st, h = init(lib)
    assert st == 0, lib.smaq_last_error()
    fake.gather_result, fake.state = IN_PROGRESS, REMOTE_ERROR  # enqueued, then the peer fails
    st = lib.smaq_comm_allgather(h, 16, 32, 16, None, 2.0)
    assert st == _lib.SMAQ_ERR_PEER
    assert fake.count("abort") == 1
    # every later call fails fast; destroy frees without finalize / destroy on the aborted handle
    assert lib.smaq_comm_wait(h, None, 2.0) == _lib.SMAQ_ERR_PEER
    assert b"aborted" in lib.smaq_last_error()
    assert lib.smaq_comm_destroy(h, 1.0) == 0
    assert fake.count("finalize") == 0 and fake.count("destroy") == 0
    assert fake.count("abort") == 1


def test_enqueue_that_never_settles_times_out(lib):
    fake = FakeNccl()
    install(lib, fake)
    st, h = init(lib)
    assert st == 0
    fake.gather_result, fake.state = IN_PROGRESS, IN_PROGRESS
    t0 = time.monotonic()
    assert lib.smaq_comm_allgather(h, 16, 32, 16, None, 0.2) == _lib.SMAQ_ERR_TIMEOUT
    assert 0.2 <= time.monotonic() - t0 < 3.0
    assert fake.count("abort") == 1
    assert lib.smaq_comm_destroy(h, 1.0) == 0


def test_wait_reports_a_peer_error_before_touching_the_device(lib):
    fake = FakeNccl()
    install(lib, fake)
    st, h = init(lib)
    assert st == 0
    assert lib.smaq_comm_allgather(h, 16, 32, 16, None, 1.0) == 0
    fake.state = REMOTE_ERROR
    assert lib.smaq_comm_status(h) == _lib.SMAQ_ERR_PEER
    assert fake.count("abort") == 1
    assert lib.smaq_comm_destroy(h, 1.0) == 0


def test_finalize_that_never_completes_is_aborted(lib):
    fake = FakeNccl(finalize_state=IN_PROGRESS)
    install(lib, fake)
    st, h = init(lib)
    assert st == 0
    assert lib.smaq_comm_destroy(h, 0.2) == _lib.SMAQ_ERR_TIMEOUT
    assert fake.count("abort") == 1 and fake.count("destroy") == 0


def test_clean_lifecycle(lib):
    fake = FakeNccl()
    install(lib, fake)
    st, h = init(lib)
    assert st == 0
    assert lib.smaq_comm_allgather(h, 16, 32, 16, None, 1.0) == 0
    assert lib.smaq_comm_status(h) == 0
    assert lib.smaq_comm_destroy(h, 1.0) == 0
    assert fake.count("finalize") == 1 and fake.count("destroy") == 1 and fake.count("abort") == 0


def test_split_comm_raises_peer_failure(lib):
    fake = FakeNccl(state=IN_PROGRESS)
    install(lib, fake)
    assert len(SplitComm.unique_id()) == _lib.COMM_ID_BYTES
    with pytest.raises(PeerFailure, match="init"):
        SplitComm(2, 1, SplitComm.unique_id(), timeout=0.2)
