"""Exact recent-token ring buffer and the capture engine (API of smaq/capture.py).

Behaviour kept from the reference (smaq/capture.py:60-91): the ring is not a sliding window.
When it is full and another token arrives, all ``capacity`` buffered tokens are handed back
as overflow (and flushed to the compressed store by the engine) and writing restarts at
position 0, so the exact window holds between 1 and ``capacity`` tokens.
"""

from __future__ import annotations

from typing import TYPE_CHECKING, Optional

import torch

if TYPE_CHECKING:
    from smaq_b200.store import CompressedKVStore


class RingBuffer:
    """Fixed-capacity buffer of exact ``[capacity, Hkv, D]`` keys and values."""

    __slots__ = ("capacity", "num_kv_heads", "head_dim", "device", "dtype", "_k", "_v", "_pos", "_total_written")

    def __init__(self, capacity: int, num_kv_heads: int, head_dim: int, device: torch.device,
                 dtype: torch.dtype = torch.bfloat16):
        self.capacity = capacity
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.device = device
        self.dtype = dtype
        self._k = torch.zeros(capacity, num_kv_heads, head_dim, device=device, dtype=dtype)
        self._v = torch.zeros(capacity, num_kv_heads, head_dim, device=device, dtype=dtype)
        self._pos = 0
        self._total_written = 0

    @property
    def size(self) -> int:
        return self._pos

    @property
    def total_written(self) -> int:
        return self._total_written

    def write(self, key: torch.Tensor, value: torch.Tensor, num_tokens: int
              ) -> Optional[tuple[torch.Tensor, torch.Tensor]]:
        """Append ``num_tokens`` tokens; returns the flushed tokens when the ring was full."""
        spill_k, spill_v = [], []
        src = 0
        while src < num_tokens:
            if self._pos >= self.capacity:
                spill_k.append(self._k[: self._pos].clone())
                spill_v.append(self._v[: self._pos].clone())
                self._pos = 0
            n = min(num_tokens - src, self.capacity - self._pos)
            self._k[self._pos:self._pos + n] = key[src:src + n]
            self._v[self._pos:self._pos + n] = value[src:src + n]
            self._pos += n
            src += n
        self._total_written += num_tokens
        if not spill_k:
            return None
        return torch.cat(spill_k, dim=0), torch.cat(spill_v, dim=0)

    def drain(self) -> Optional[tuple[torch.Tensor, torch.Tensor]]:
        if self._pos == 0:
            return None
        out = self._k[: self._pos].clone(), self._v[: self._pos].clone()
        self._pos = 0
        return out

    def peek(self) -> Optional[tuple[torch.Tensor, torch.Tensor]]:
        if self._pos == 0:
            return None
        return self._k[: self._pos], self._v[: self._pos]

    def reset(self):
        self._pos = 0
        self._total_written = 0


class KVCaptureEngine:
    """Routes prefill and decode tokens into the ring buffer and the compressed store."""

    def __init__(self, store: "CompressedKVStore", ring_capacity: int = 128, device: torch.device | None = None,
                 dtype: torch.dtype = torch.bfloat16):
        self.store = store
        self.ring = RingBuffer(capacity=ring_capacity, num_kv_heads=store.num_kv_heads, head_dim=store.head_dim,
                               device=device or store.device, dtype=dtype)
        self._prefill_done = False

    @property
    def total_compressed_tokens(self) -> int:
        return self.store.num_tokens

    @property
    def total_buffered_tokens(self) -> int:
        return self.ring.size

    @property
    def total_tokens(self) -> int:
        return self.total_compressed_tokens + self.total_buffered_tokens

    def ingest_prefill(self, key: torch.Tensor, value: torch.Tensor, num_tokens: int):
        """All but the last ``capacity`` tokens go to the store; the tail stays exact."""
        cap = self.ring.capacity
        if num_tokens <= cap:
            self.ring.write(key[:num_tokens], value[:num_tokens], num_tokens)
        else:
            cut = num_tokens - cap
            self.store.append_chunk(key[:cut], value[:cut])
            self.ring.write(key[cut:num_tokens], value[cut:num_tokens], cap)
        self._prefill_done = True

    def ingest_prefill_from_paged_cache(self, kv_cache_tensor: torch.Tensor, num_tokens: int,
                                        block_table: torch.Tensor, block_size: int):
        """Gather a prefill from a vLLM ``[2, num_blocks, block_size, Hkv, D]`` paged cache."""
        nblk = (num_tokens + block_size - 1) // block_size
        blocks = block_table[:nblk].to(torch.long)
        k = kv_cache_tensor[0].index_select(0, blocks).reshape(-1, *kv_cache_tensor.shape[-2:])[:num_tokens]
        v = kv_cache_tensor[1].index_select(0, blocks).reshape(-1, *kv_cache_tensor.shape[-2:])[:num_tokens]
        self.ingest_prefill(k, v, num_tokens)

    def ingest_decode(self, key: torch.Tensor, value: torch.Tensor, num_tokens: int):
        spill = self.ring.write(key[:num_tokens], value[:num_tokens], num_tokens)
        if spill is not None:
            self.store.append_chunk(*spill)

    def flush(self):
        data = self.ring.drain()
        if data is not None:
            self.store.append_chunk(*data)

    def reset(self):
        self.ring.reset()
        self.store.reset()
        self._prefill_done = False
