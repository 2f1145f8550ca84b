"""Batched SMAQ decode over a serving engine's paged KV cache.

A ``PagedCompressedCache`` holds the compressed rows of one attention layer in pages that mirror
the engine's exact cache: block ``p`` of the engine's ``[2, num_blocks, block_size, Hkv, D]``
cache and page ``p`` here hold the same tokens.  Every K/V write the engine makes (a flat slot
``block * block_size + offset`` per token) is quantized into the same slot here, all tokens of a
step in one ``smaq_append`` launch.  A decode step of ``B`` sequences is one ``smaq_decode``
launch that follows the engine's block table through the compressed pages for the history and
reads the exact window from the engine's own cache.

Which tokens are history and which are the exact window follows the reference's ring rule
(smaq/capture.py:60-91, driven by smaq/integration/vllm.py): after a prompt of ``n0`` tokens the
ring holds ``min(n0, C)`` exact tokens; every later token extends it, or, when it is full,
flushes all ``C`` to the compressed store and restarts at one.  Quantization is per token, so
quantizing every token on arrival and choosing the split at read time gives the reference's rows
for the history part.  A sequence whose history would be shorter than ``MIN_HISTORY_FOR_SMAQ``
is answered from exact tokens only, as the reference's hook falls back to the engine's own
attention there (smaq/integration/vllm.py:221-240).

The prompt length ``n0`` of a sequence is recorded, on the device, under the sequence's first
block when a prefill step writes it (``note_prompts``), and looked up the same way at decode, so
nothing here syncs with the host.
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import ops
from .._lib import SMAQ_KEYS_SCALAR, SMAQ_LAYOUT_DECODE, SMAQ_LAYOUT_REFERENCE
from ..score import MIN_HISTORY_FOR_SMAQ
from ..strategies import SMAQFullMetricScalarStrategy


def reference_window_len(seq_lens: torch.Tensor, prompt_lens: torch.Tensor, capacity: int) -> torch.Tensor:
    """Exact-window length of each sequence under the reference's ring rule (module docstring).
    ``seq_lens`` count every token written so far, the current decode token included."""
    n0 = prompt_lens.to(torch.int64).clamp(min=1)
    L = torch.maximum(seq_lens.to(torch.int64), n0)
    r0 = n0.clamp(max=capacity)
    return torch.where(L > n0, (r0 - 1 + (L - n0)) % capacity + 1, r0)


def split_history(seq_lens: torch.Tensor, prompt_lens: torch.Tensor, capacity: int,
                  min_history: int = MIN_HISTORY_FOR_SMAQ) -> tuple[torch.Tensor, torch.Tensor]:
    """(history length, window length) per sequence; a history shorter than ``min_history``
    joins the window (at most ``capacity + min_history - 1`` exact tokens)."""
    L = seq_lens.to(torch.int64)
    r = torch.minimum(reference_window_len(L, prompt_lens, capacity), L)
    h = L - r
    short = h < min_history
    return torch.where(short, torch.zeros_like(h), h), torch.where(short, L, r)


def gather_window(kv_cache: torch.Tensor, block_table: torch.Tensor, start: torch.Tensor, length: torch.Tensor,
                  width: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Exact keys and values ``[B, width, Hkv, D]`` of tokens ``start .. start + length`` of each
    sequence, read from an engine cache ``[2, num_blocks, block_size, Hkv, D]`` through its block
    table.  Positions past ``length`` repeat the last token (the decode kernel ignores them)."""
    bs = kv_cache.shape[2]
    j = torch.arange(width, device=block_table.device, dtype=torch.int64)
    last = (start + length - 1).clamp(min=0)
    pos = torch.minimum(start[:, None] + j[None, :], last[:, None])
    blocks = block_table.to(torch.int64).gather(1, pos // bs)
    offs = pos % bs
    return kv_cache[0][blocks, offs], kv_cache[1][blocks, offs]


class PagedCompressedCache:
    """Compressed rows of one attention layer, paged like the engine's KV cache (module
    docstring).  Keys: SMAQ scalar codes (smaq/quantizer.py) with the layer's metric; values:
    ``value_bits`` codes in groups of ``group_size`` (smaq/kv_cache.py).  Page ``num_blocks`` is
    scratch: padding tokens (slot < 0) are written there."""

    def __init__(self, num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int, *,
                 key_bits: int = 3, value_bits: int = 2, group_size: int = 32, capacity: int = 128,
                 Sigma_q: Optional[torch.Tensor] = None, dtype: torch.dtype = torch.bfloat16,
                 device: torch.device | str = "cuda"):
        self.num_blocks, self.block_size = num_blocks, block_size
        self.num_kv_heads, self.head_dim = num_kv_heads, head_dim
        self.key_bits, self.value_bits, self.group_size = key_bits, value_bits, min(group_size, head_dim)
        self.capacity = capacity
        self.dtype = dtype
        self.device = torch.device(device)
        self.strategy = SMAQFullMetricScalarStrategy(dim=head_dim, Sigma_q=Sigma_q, bits=key_bits, device=self.device,
                                                     dtype=torch.float32)
        fast = (dtype == torch.bfloat16 and head_dim == 128 and value_bits == 2 and self.group_size == 32
                and key_bits in (3, 4) and block_size % 16 == 0)
        self.layout = SMAQ_LAYOUT_DECODE if fast else SMAQ_LAYOUT_REFERENCE
        P, H, bs, D = num_blocks + 1, num_kv_heads, block_size, head_dim
        dev = self.device
        self.codes = torch.zeros((P, H, bs, ops.packed_dim(D, key_bits)), dtype=torch.uint8, device=dev)
        self.norms = torch.zeros((P, H, bs), dtype=dtype, device=dev)
        self.v_data = torch.zeros((P, H, bs, D * value_bits // 8), dtype=torch.uint8, device=dev)
        self.v_scales = torch.zeros((P, H, bs, D // self.group_size), dtype=dtype, device=dev)
        self.v_zeros = torch.zeros_like(self.v_scales)
        # prompt length of the sequence whose first block is p (entry num_blocks: scratch)
        self.prompt_len = torch.zeros(P, dtype=torch.int32, device=dev)
        self._workspace: Optional[torch.Tensor] = None

    @property
    def quantizer(self):
        return self.strategy.quantizer

    def device_bytes(self) -> int:
        return sum(t.nelement() * t.element_size() for t in (self.codes, self.norms, self.v_data, self.v_scales,
                                                              self.v_zeros))

    # ------------------------------------------------------------------ writes
    def write(self, key: torch.Tensor, value: torch.Tensor, slot_mapping: torch.Tensor) -> None:
        """Quantize the step's ``[N, Hkv, D]`` keys and values into their slots (one launch).
        ``key``/``value`` may hold more rows than ``slot_mapping`` (engine padding)."""
        n = slot_mapping.shape[0]
        if n == 0:
            return
        slots = slot_mapping.to(torch.int64)
        pad = self.num_blocks * self.block_size + torch.arange(n, device=slots.device) % self.block_size
        slots = torch.where(slots >= 0, slots, pad)
        k, v = key[:n], value[:n]
        if k.dim() == 2:
            k = k.view(n, self.num_kv_heads, self.head_dim)
            v = v.view(n, self.num_kv_heads, self.head_dim)
        k, v = k.to(self.dtype), v.to(self.dtype)
        qz = self.quantizer
        ops.append(k, v, n_heads=self.num_kv_heads, slots=slots, page_size=self.block_size,
                   key_format=SMAQ_KEYS_SCALAR, key_bits=self.key_bits, E=qz.E, boundaries=qz.decision_boundaries,
                   key_codes=self.codes, key_norms=self.norms, value_bits=self.value_bits, group_size=self.group_size,
                   v_data=self.v_data, v_scales=self.v_scales, v_zeros=self.v_zeros, layout=self.layout)

    def note_prompts(self, block_table: torch.Tensor, seq_lens: torch.Tensor, query_lens: torch.Tensor) -> None:
        """Record the prompt length of every sequence of a step that writes more than one token
        (a prefill or a prefill chunk: the last chunk leaves the full prompt length)."""
        first = block_table[:, 0].to(torch.int64)
        idx = torch.where(query_lens > 1, first, torch.full_like(first, self.num_blocks))
        self.prompt_len.index_put_((idx,), seq_lens.to(torch.int32))

    # ------------------------------------------------------------------ decode
    def decode(self, q: torch.Tensor, kv_cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor,
               scale: Optional[float] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One decode token for each of ``B`` sequences: ``q [B, Hq, D]`` -> ``[B, Hq, D]`` in the
        query dtype.  ``seq_lens`` include the current token (already written)."""
        B = q.shape[0]
        bt = block_table[:B]
        L = seq_lens[:B].to(torch.int64)
        n0 = self.prompt_len[bt[:, 0].to(torch.int64)]
        hist, r = split_history(L, n0, self.capacity)
        width = self.capacity + MIN_HISTORY_FOR_SMAQ - 1
        rk, rv = gather_window(kv_cache, bt, hist, r, width)
        if rk.dtype != q.dtype:
            rk, rv = rk.to(q.dtype), rv.to(q.dtype)
        need = ops.decode_workspace_bytes(B, q.shape[1], self.num_kv_heads, self.head_dim)
        if self._workspace is None or self._workspace.numel() < need:
            self._workspace = torch.empty((max(need, 256),), dtype=torch.uint8, device=q.device)
        qz = self.quantizer
        return ops.decode(q, n_kv_heads=self.num_kv_heads, key_format=SMAQ_KEYS_SCALAR, key_bits=self.key_bits,
                          E_inv=qz.E_inv, centroids=qz.centroids, key_codes=self.codes, key_norms=self.norms,
                          v_data=self.v_data, v_scales=self.v_scales, v_zeros=self.v_zeros,
                          value_bits=self.value_bits, group_size=self.group_size, hist_len=hist,
                          page_size=self.block_size, block_table=bt, recent_k=rk, recent_v=rv, recent_len=r,
                          scale=scale, min_history=MIN_HISTORY_FOR_SMAQ, out=out, workspace=self._workspace,
                          layout=self.layout)
