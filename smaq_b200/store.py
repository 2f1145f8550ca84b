"""Compressed KV store (API of smaq/store.py), preallocated on the device.

The reference keeps a Python list of per-chunk tensors and re-concatenates all of them after
every append.  Here each stream lives in one capacity-doubling device buffer laid out as
store rows ``[Hkv, capacity, row]`` (one page of ``capacity`` tokens per head, see
include/smaq_b200.h), and ``append_chunk`` quantizes straight into rows ``n .. n+T`` with one
``smaq_append`` launch.  Block-VQ indices are kept as uint8 (the reference keeps int64).

Rows use ``SMAQ_LAYOUT_DECODE`` (the reference's bytes permuted inside each row, see
include/smaq_b200.h) whenever the format has a fast decode kernel: bf16 keys/values, head_dim
128, 2-bit values in groups of 32, and 3/4-bit scalar keys or 8-dim block-VQ keys.  Other
formats keep the reference byte order.  ``get_flat_cache`` always returns the reference's
logical view: ``SMAQQuantized`` / ``BlockVQQuantized`` plus ``ValueQuantized`` with
``[Hkv, N, ...]`` shapes in the reference byte order (block-VQ indices as int64).
"""

from __future__ import annotations

from typing import Any, NamedTuple, Optional

import torch

from smaq_b200 import ops
from smaq_b200._lib import SMAQ_KEYS_BVQ, SMAQ_KEYS_SCALAR, SMAQ_LAYOUT_DECODE, SMAQ_LAYOUT_REFERENCE
from smaq_b200.block_vq import BlockVQQuantized
from smaq_b200.calibration import IdentityCalibrationProvider
from smaq_b200.core import CacheCapabilities, CalibrationProvider
from smaq_b200.kv_cache import ValueQuantized
from smaq_b200.quantizer import SMAQQuantized
from smaq_b200.strategies import (ExactShadowQuantized, ExactShadowStrategy, IdentityScalarStrategy,
                                  SMAQBlockVQStrategy, SMAQFullMetricScalarStrategy)

# Exact (unquantized) history keys: ExactShadowStrategy.  Host-side tag only; no kernel key format.
KEYS_SHADOW = -1


class FlatCache(NamedTuple):
    """Flattened history view: key codes, value codes and the token count."""

    key_q: Any
    value_q: ValueQuantized
    num_tokens: int


def key_format_of(strategy) -> int:
    if isinstance(strategy, IdentityScalarStrategy):
        return SMAQ_KEYS_SCALAR
    if isinstance(strategy, SMAQBlockVQStrategy):
        return SMAQ_KEYS_BVQ
    if isinstance(strategy, ExactShadowStrategy):
        return KEYS_SHADOW
    raise NotImplementedError(
        f"key strategy {type(strategy).__name__} has no sm_100a kernel (supported: the scalar strategies "
        "IdentityScalarStrategy / SMAQFullMetricScalarStrategy / SMAQDiagonalMetricStrategy, "
        "SMAQBlockVQStrategy, and ExactShadowStrategy)")


class CompressedKVStore:
    """Chunked SMAQ KV store for one layer of one sequence (smaq/store.py:28-130)."""

    def __init__(self, head_dim: int, num_kv_heads: int, Sigma_q: torch.Tensor | None = None, key_bits: int = 3,
                 value_bits: int = 2, value_group_size: int = 32, device: torch.device | None = None,
                 layer_idx: int = 0, key_strategy: Any | None = None,
                 calibration_provider: CalibrationProvider | None = None, initial_capacity: int = 256):
        self.head_dim = head_dim
        self.num_kv_heads = num_kv_heads
        self.key_bits = key_bits
        self.value_bits = value_bits
        self.value_group_size = min(value_group_size, head_dim)
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda" if torch.cuda.is_available() else "cpu")
        self.layer_idx = layer_idx
        self.calibration_provider = calibration_provider or IdentityCalibrationProvider()
        sigma = Sigma_q if Sigma_q is not None else self.calibration_provider.get_sigma_q(
            layer_idx, head_dim, device=self.device)
        self.key_strategy = key_strategy or SMAQFullMetricScalarStrategy(
            dim=head_dim, Sigma_q=sigma, bits=key_bits, device=self.device, dtype=torch.float32)
        self.quantizer = self.key_strategy
        self.key_format = key_format_of(self.key_strategy)
        self._initial_capacity = max(16, initial_capacity)
        self._chunk_lengths: list[int] = []
        self._n = 0
        self._cap = 0
        self._dtype: Optional[torch.dtype] = None
        self._buf: dict[str, torch.Tensor] = {}
        self._flat: Optional[FlatCache] = None
        self.layout = SMAQ_LAYOUT_REFERENCE

    # ------------------------------------------------------------------ bookkeeping
    @property
    def capabilities(self) -> CacheCapabilities:
        return self.key_strategy.capabilities

    @property
    def num_tokens(self) -> int:
        return self._n

    @property
    def num_chunks(self) -> int:
        return len(self._chunk_lengths)

    @property
    def capacity(self) -> int:
        return self._cap

    @property
    def dtype(self) -> Optional[torch.dtype]:
        return self._dtype

    def _key_row_bytes(self) -> int:
        if self.key_format == SMAQ_KEYS_SCALAR:
            return ops.packed_dim(self.head_dim, self.key_strategy.bits)
        return self.key_strategy.quantizer.n_blocks

    def _alloc(self, cap: int, dtype: torch.dtype) -> dict[str, torch.Tensor]:
        H, D, dev = self.num_kv_heads, self.head_dim, self.device
        ng = D // self.value_group_size
        keys = (torch.empty((H, cap, D), dtype=dtype, device=dev) if self.key_format == KEYS_SHADOW else
                torch.empty((H, cap, self._key_row_bytes()), dtype=torch.uint8, device=dev))
        b = {
            "codes": keys,
            "vdata": torch.empty((H, cap, D * self.value_bits // 8), dtype=torch.uint8, device=dev),
            "vscales": torch.empty((H, cap, ng), dtype=dtype, device=dev),
            "vzeros": torch.empty((H, cap, ng), dtype=dtype, device=dev),
        }
        if self.key_format == SMAQ_KEYS_SCALAR:
            b["norms"] = torch.empty((H, cap), dtype=dtype, device=dev)
        return b

    def _decode_layout_ok(self, dtype: torch.dtype) -> bool:
        """True when the rows can use the fast decode kernels' byte order."""
        if self.key_format == KEYS_SHADOW:
            return False
        if dtype != torch.bfloat16 or self.head_dim != 128 or self.value_bits != 2 or self.value_group_size != 32:
            return False
        if self.key_format == SMAQ_KEYS_SCALAR:
            return self.key_strategy.bits in (3, 4)
        return self.key_strategy.quantizer.block_dim == 8

    def _reserve(self, n_new: int, dtype: torch.dtype):
        if self._dtype is None:
            self._dtype = dtype
            self.layout = SMAQ_LAYOUT_DECODE if self._decode_layout_ok(dtype) else SMAQ_LAYOUT_REFERENCE
        need = self._n + n_new
        if need <= self._cap:
            return
        cap = max(need, 2 * self._cap, self._initial_capacity)
        cap = (cap + 15) // 16 * 16   # decode-layout pages hold a multiple of 16 rows
        nb = self._alloc(cap, self._dtype)
        if self._n:
            for k, t in self._buf.items():
                nb[k][:, : self._n].copy_(t[:, : self._n])
        self._buf = nb
        self._cap = cap

    # ------------------------------------------------------------------ API
    def append_chunk(self, key: torch.Tensor, value: torch.Tensor):
        """Quantize a ``[T, Hkv, D]`` chunk of keys and values into the store (one kernel pass)."""
        ops._cuda(key, value)
        T = key.shape[0]
        self._reserve(T, key.dtype)
        if key.dtype != self._dtype:
            key = key.to(self._dtype)
        if value.dtype != self._dtype:
            value = value.to(self._dtype)
        if T:
            strat = self.key_strategy
            kw = {}
            if self.key_format == KEYS_SHADOW:
                # keys kept as given; the value half of the append kernel quantizes the values
                self._buf["codes"][:, self._n: self._n + T].copy_(key.transpose(0, 1))
                key = None
            elif self.key_format == SMAQ_KEYS_SCALAR:
                qz = strat.quantizer
                kw = dict(key_format=SMAQ_KEYS_SCALAR, key_bits=strat.bits, E=qz.E, boundaries=qz.decision_boundaries,
                          key_norms=self._buf["norms"])
            else:
                qz = strat.quantizer
                kw = dict(key_format=SMAQ_KEYS_BVQ, E_blocks=qz.E_blocks, centroids=qz.centroids)
            ops.append(key, value, n_heads=self.num_kv_heads, slot_offset=self._n, page_size=self._cap,
                       key_codes=self._buf["codes"], value_bits=self.value_bits, group_size=self.value_group_size,
                       v_data=self._buf["vdata"], v_scales=self._buf["vscales"], v_zeros=self._buf["vzeros"],
                       layout=self.layout, **kw)
        self._n += T
        self._chunk_lengths.append(T)
        self._flat = None

    def kernel_view(self) -> dict:
        """Raw device rows for the decode kernel: streams shaped ``[1, Hkv, capacity, ...]``."""
        return {k: v.unsqueeze(0) for k, v in self._buf.items()} | {"page_size": self._cap, "n": self._n,
                                                                      "layout": self.layout}

    def get_flat_cache(self) -> Optional[FlatCache]:
        if self._n == 0:
            return None
        if self._flat is not None:
            return self._flat
        n, b = self._n, self._buf
        dec = self.layout == SMAQ_LAYOUT_DECODE
        codes, vdata = b["codes"][:, :n], b["vdata"][:, :n]
        if self.key_format == KEYS_SHADOW:
            kq = ExactShadowQuantized(values=codes)
        elif self.key_format == SMAQ_KEYS_SCALAR:
            if dec:
                codes = ops.scalar_codes_to_reference(codes)
            kq = SMAQQuantized(indices=codes, norms=b["norms"][:, :n], bits=self.key_strategy.bits)
        else:
            qz = self.key_strategy.quantizer
            if dec:
                codes = ops.bvq_to_reference(codes)
            kq = BlockVQQuantized(indices=codes.to(torch.int64), n_blocks=qz.n_blocks, block_dim=qz.block_dim)
        if dec:
            vdata = ops.values_to_reference(vdata)
        vq = ValueQuantized(data=vdata, scales=b["vscales"][:, :n], zeros=b["vzeros"][:, :n], bits=self.value_bits)
        self._flat = FlatCache(key_q=kq, value_q=vq, num_tokens=n)
        return self._flat

    def memory_bytes(self) -> int:
        """Byte count with the reference's accounting (norms/scales at 2 B, VQ indices as int64)."""
        if self._n == 0:
            return 0
        n, H = self._n, self.num_kv_heads
        ng = self.head_dim // self.value_group_size
        if self.key_format == KEYS_SHADOW:
            keys = H * n * self.head_dim * self._buf["codes"].element_size()
        elif self.key_format == SMAQ_KEYS_SCALAR:
            keys = H * n * self._key_row_bytes() + 2 * H * n
        else:
            keys = H * n * self._key_row_bytes() * 8
        values = H * n * (self.head_dim * self.value_bits // 8) + 4 * H * n * ng
        return keys + values

    def device_bytes(self) -> int:
        """Bytes actually held on the device (allocated capacity)."""
        return sum(t.nelement() * t.element_size() for t in self._buf.values())

    def reset(self):
        self._chunk_lengths.clear()
        self._n = 0
        self._flat = None
