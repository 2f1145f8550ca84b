"""Multi-GPU sharding of hybrid decode attention: one process per GPU, torch.distributed.

The reference runs on one device and has no multi-GPU path; this module adds one for long
contexts.  Units of work are (sequence, KV head) pairs, which are independent.

* KV heads are split into ``head_groups`` contiguous ranges, one range per group of ranks.
  Query heads follow their KV head (GQA), so a head group needs no communication: its output
  rows are its own query heads.
* When there are more ranks than KV heads can be split over (``world > head_groups``), each
  head group's history is further split into ``seq_splits`` contiguous token ranges.  Every
  rank of the split group attends to its own range and writes the decode partials
  ``(acc_hist[D], acc_recent[D], m, l)`` (``smaq_decode`` with ``partial_out``).  The exact
  recent window is attended by the last split only.  The partials are all-gathered inside the
  split group (NCCL over NVLink on GPUs) and merged with ``smaq_merge_partials``, which
  applies the log-sum-exp combine and the reference's per-part rounding.  The minimum-history
  rule of ``compute_hybrid_attention`` (smaq/score.py:37) looks at the whole sequence, which
  the kernel receives as ``hist_total``.

Rank ``r`` of a plan sits at head group ``r // seq_splits`` and split ``r % seq_splits``.

Failure handling: the exchange is the only point where a rank waits on another.  Give
``split_groups`` a ``timeout``; a peer that died or never reaches the exchange then ends the
all-gather with an error, which ``sharded_decode`` re-raises as ``PeerFailure`` naming the
split group, between decode steps and with no kernel of this rank in flight.
``native_split_comms`` gives the same groups on the library's own communicator
(``SplitComm``, ``smaq_comm_*``): non-blocking NCCL, host-side deadlines on every step, and
``ncclCommAbort`` when one runs out.
"""

from __future__ import annotations

import ctypes
import datetime
import math
from dataclasses import dataclass
from typing import Callable, Optional, Sequence

import torch

PARTIAL_EXTRA = 2  # (m, l) after acc_hist[D] and acc_recent[D]


class PeerFailure(RuntimeError):
    """A rank of this rank's split group failed to join the partials exchange."""


@dataclass(frozen=True)
class ShardPlan:
    world: int
    n_kv_heads: int
    head_groups: int
    seq_splits: int

    def coords(self, rank: int) -> tuple[int, int]:
        if not 0 <= rank < self.world:
            raise ValueError(f"rank {rank} outside world {self.world}")
        return rank // self.seq_splits, rank % self.seq_splits

    def kv_heads(self, rank: int) -> range:
        """KV heads owned by ``rank``'s head group."""
        hg, _ = self.coords(rank)
        per = self.n_kv_heads // self.head_groups
        return range(hg * per, (hg + 1) * per)

    def q_heads(self, rank: int, n_q_heads: int) -> range:
        G = n_q_heads // self.n_kv_heads
        kv = self.kv_heads(rank)
        return range(kv.start * G, kv.stop * G)

    def token_range(self, n_tokens: int, rank: int, align: int = 16) -> tuple[int, int]:
        """History tokens ``[lo, hi)`` of a sequence of ``n_tokens`` attended by ``rank``.  Split
        boundaries are multiples of ``align`` (the store's page granularity), so every range
        but the last holds whole pages; ranges are contiguous and cover every token once."""
        _, sp = self.coords(rank)
        if self.seq_splits == 1:
            return 0, n_tokens
        units = (n_tokens + align - 1) // align
        lo = min(n_tokens, (units * sp // self.seq_splits) * align)
        hi = min(n_tokens, (units * (sp + 1) // self.seq_splits) * align)
        return lo, hi

    def holds_recent(self, rank: int) -> bool:
        return self.coords(rank)[1] == self.seq_splits - 1

    def split_peers(self, rank: int) -> list[int]:
        hg, _ = self.coords(rank)
        return [hg * self.seq_splits + s for s in range(self.seq_splits)]


def make_plan(world: int, n_kv_heads: int) -> ShardPlan:
    """Split by KV head as far as the head count allows, then by sequence."""
    if world < 1 or n_kv_heads < 1:
        raise ValueError("world and n_kv_heads must be >= 1")
    hg = math.gcd(world, n_kv_heads)
    return ShardPlan(world, n_kv_heads, hg, world // hg)


def split_groups(plan: ShardPlan, backend: Optional[str] = None, timeout: Optional[float] = None):
    """One process group per head group, over its sequence-split ranks (``None`` entries when
    there is no split).  Every rank must call this, in the same order.  ``timeout`` (seconds)
    bounds each exchange: a peer that does not arrive within it fails the collective."""
    import torch.distributed as dist
    kw = {} if timeout is None else {"timeout": datetime.timedelta(seconds=timeout)}
    groups = []
    for hg in range(plan.head_groups):
        ranks = [hg * plan.seq_splits + s for s in range(plan.seq_splits)]
        groups.append(dist.new_group(ranks, backend=backend, **kw) if plan.seq_splits > 1 else None)
    return groups


class SplitComm:
    """The library's own exchange for one split group (``smaq_comm_*``): an NCCL communicator in
    non-blocking mode whose every step has a deadline.  A missing or failed peer raises
    ``PeerFailure`` within ``timeout`` seconds and leaves the communicator aborted, instead of
    blocking the host inside NCCL.  The current CUDA device at construction is the
    communicator's device."""

    def __init__(self, n_ranks: int, rank: int, comm_id: bytes, timeout: float = 60.0):
        from . import _lib
        self._lib = _lib.load()
        if len(comm_id) != _lib.COMM_ID_BYTES:
            raise ValueError(f"comm_id must be {_lib.COMM_ID_BYTES} bytes")
        self.n_ranks, self.rank, self.timeout = n_ranks, rank, float(timeout)
        self._h = ctypes.c_void_p()
        self._check(self._lib.smaq_comm_init(ctypes.byref(self._h), n_ranks, rank, comm_id, self.timeout),
                    "init")

    @staticmethod
    def unique_id() -> bytes:
        """A fresh communicator id; rank 0 of the split group makes it and shares it."""
        from . import _lib
        lib = _lib.load()
        buf = ctypes.create_string_buffer(_lib.COMM_ID_BYTES)
        st = lib.smaq_comm_unique_id(buf)
        if st != 0:
            raise RuntimeError(f"smaq_comm_unique_id: {lib.smaq_last_error().decode()}")
        return buf.raw

    def _check(self, st: int, what: str) -> None:
        if st == 0:
            return
        from . import _lib
        msg = self._lib.smaq_last_error().decode()
        if st in (_lib.SMAQ_ERR_TIMEOUT, _lib.SMAQ_ERR_PEER):
            raise PeerFailure(f"split-group {what} (rank {self.rank} of {self.n_ranks}): {msg}")
        raise RuntimeError(f"smaq_comm {what}: {_lib.STATUS.get(st, st)}: {msg}")

    def all_gather(self, partial: torch.Tensor) -> torch.Tensor:
        """``[...]`` on every rank -> ``[n_ranks, ...]``, on the current stream; returns after the
        exchange completed (or raises ``PeerFailure``)."""
        part = partial.contiguous()
        out = torch.empty((self.n_ranks,) + tuple(part.shape), dtype=part.dtype, device=part.device)
        stream = torch.cuda.current_stream(part.device).cuda_stream
        nbytes = part.numel() * part.element_size()
        self._check(self._lib.smaq_comm_allgather(self._h, part.data_ptr(), out.data_ptr(), nbytes, stream,
                                                  self.timeout), "all-gather")
        self._check(self._lib.smaq_comm_wait(self._h, stream, self.timeout), "wait")
        return out

    def abort(self) -> None:
        if self._h:
            self._lib.smaq_comm_abort(self._h)

    def close(self) -> None:
        if self._h:
            h, self._h = self._h, ctypes.c_void_p()
            self._lib.smaq_comm_destroy(h, self.timeout)


def native_split_comms(plan: ShardPlan, rank: int, timeout: float = 60.0) -> list:
    """``split_groups`` built on ``SplitComm``: every rank calls it (same order); the ids travel
    over the default process group.  Entries are ``None`` without sequence splits, and only this
    rank's head group gets a communicator."""
    import torch.distributed as dist
    if plan.seq_splits == 1:
        return [None] * plan.head_groups
    ids = [SplitComm.unique_id() for _ in range(plan.head_groups)] if rank == 0 else [None] * plan.head_groups
    dist.broadcast_object_list(ids, src=0)
    hg, sp = plan.coords(rank)
    groups: list = [None] * plan.head_groups
    groups[hg] = SplitComm(plan.seq_splits, sp, ids[hg], timeout=timeout)
    return groups


def gather_partials(partial: torch.Tensor, group, world_size: int) -> torch.Tensor:
    """All-gather ``[B, Hq_local, 2D+2]`` fp32 partials over ``group`` -> ``[R, B, Hq_local, 2D+2]``.
    ``group`` is a torch process group or a ``SplitComm``."""
    if isinstance(group, SplitComm):
        return group.all_gather(partial)
    import torch.distributed as dist
    parts = [torch.empty_like(partial) for _ in range(world_size)]
    dist.all_gather(parts, partial.contiguous(), group=group)
    return torch.stack(parts, 0)


def combine(partials: torch.Tensor, out_dtype: torch.dtype,
            merge_fn: Optional[Callable[[torch.Tensor, torch.dtype], torch.Tensor]] = None) -> torch.Tensor:
    """Log-sum-exp combine of gathered partials (``smaq_merge_partials`` on the device)."""
    if merge_fn is None:
        from . import ops
        merge_fn = ops.merge_partials
    return merge_fn(partials, out_dtype)


def sharded_decode(plan: ShardPlan, rank: int, groups: Sequence, decode_fn: Callable[..., torch.Tensor],
                   out_dtype: torch.dtype, merge_fn=None) -> torch.Tensor:
    """Run this rank's share of a decode step and return the output rows of its query heads.

    ``decode_fn(partial: bool)`` runs the local decode (this rank's KV heads, token range and,
    on the last split, the recent window) and returns the ``[B, Hq_local, D]`` output, or, with
    ``partial=True``, the ``[B, Hq_local, 2D+2]`` fp32 partials.  With one split per head group
    nothing is exchanged."""
    hg, _ = plan.coords(rank)
    if plan.seq_splits == 1:
        return decode_fn(partial=False)
    part = decode_fn(partial=True)
    try:
        gathered = gather_partials(part, groups[hg], plan.seq_splits)
    except PeerFailure:
        raise
    except Exception as e:  # the backend's timeout / closed-connection error
        raise PeerFailure(f"rank {rank}: partials exchange with ranks {plan.split_peers(rank)} failed: {e}") from e
    return combine(gathered, out_dtype, merge_fn)
