"""Value codec and the HF-style SMAQ KV cache (API of smaq/kv_cache.py).

``quantize_values`` runs the ``smaq_quantize_values`` CUDA kernel: per group of
``group_size`` elements ``scale = clamp((max - min) / (2^bits - 1), 1e-10)``,
``zero = min``, ``code = round_half_even((v - zero) / scale)`` clamped to the code range, with
every step rounded to the value dtype exactly as torch does for bf16/fp16 tensors
(smaq/kv_cache.py:50-91).  2-bit codes pack ``v0 | v1<<2 | v2<<4 | v3<<6``; 4-bit codes pack
``v0 | v1<<4``.
"""

from __future__ import annotations

import math
from typing import Any, NamedTuple, Optional

import torch

from smaq_b200 import ops
from smaq_b200.calibration import IdentityCalibrationProvider
from smaq_b200.core import CacheCapabilities, CalibrationProvider
from smaq_b200.strategies import SMAQFullMetricScalarStrategy


class ValueQuantized(NamedTuple):
    """Packed value codes plus per-group scales and zeros (value dtype)."""

    data: torch.Tensor
    scales: torch.Tensor
    zeros: torch.Tensor
    bits: int = 2


def unpack_values(vq: ValueQuantized) -> torch.Tensor:
    """Packed bytes -> one uint8 code per element (smaq/kv_cache.py:29-47)."""
    bits = vq.bits if len(vq) > 3 else 2
    d = vq.data
    if bits == 2:
        parts = [(d >> s) & 0x03 for s in (0, 2, 4, 6)]
    elif bits == 4:
        parts = [d & 0x0F, (d >> 4) & 0x0F]
    else:
        return d
    return torch.stack(parts, dim=-1).reshape(*d.shape[:-1], d.shape[-1] * len(parts))


def quantize_values(v: torch.Tensor, bits: int = 2, group_size: int = 32) -> ValueQuantized:
    """Group-asymmetric value quantization on the GPU."""
    d = v.shape[-1]
    if d % group_size != 0:
        raise ValueError(f"head_dim {d} must be divisible by group_size {group_size}")
    if bits == 2 and d % 4 != 0:
        raise ValueError(f"head_dim {d} must be divisible by 4 for 2-bit packing")
    if bits == 4 and d % 2 != 0:
        raise ValueError(f"head_dim {d} must be divisible by 2 for 4-bit packing")
    if bits not in (2, 4):
        raise ValueError(f"value bits {bits} not supported (2 or 4)")
    data, scales, zeros = ops.quantize_values(v, bits, group_size)
    return ValueQuantized(data=data, scales=scales, zeros=zeros, bits=bits)


def dequantize_values(vq: ValueQuantized, group_size: int = 32) -> torch.Tensor:
    """``code * scale + zero`` in fp32 (a reconstruction helper; the decode kernel fuses it)."""
    q = unpack_values(vq).float()
    d = q.shape[-1]
    q = q.reshape(*q.shape[:-1], d // group_size, group_size)
    out = q * vq.scales.unsqueeze(-1) + vq.zeros.unsqueeze(-1)
    return out.reshape(*q.shape[:-2], d)


class SMAQKVCache:
    """HF-style cache: compressed history plus an exact recent buffer (smaq/kv_cache.py:106-290).

    Tensors are ``[..., T, D]``.  Keys go through the strategy's GPU quantizer; values through
    ``quantize_values``.  ``attention_scores`` returns the concatenated ``[history || buffer]``
    logits, ``attend`` applies caller-computed weights.
    """

    def __init__(self, head_dim: int, Sigma_q: torch.Tensor | None = None, key_bits: int = 3,
                 value_bits: int = 2, value_group_size: int = 32, buffer_size: int = 128,
                 device: torch.device | None = None, dtype: torch.dtype = torch.float16, layer_idx: int = 0,
                 key_strategy: Any | None = None, calibration_provider: CalibrationProvider | None = None):
        self.head_dim = head_dim
        self.key_bits = key_bits
        self.value_bits = value_bits
        self.value_group_size = value_group_size
        self.buffer_size = buffer_size
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda" if torch.cuda.is_available() else "cpu")
        self.dtype = dtype
        self.layer_idx = layer_idx
        self.calibration_provider = calibration_provider or IdentityCalibrationProvider()
        sigma = Sigma_q if Sigma_q is not None else self.calibration_provider.get_sigma_q(
            layer_idx, head_dim, device=self.device)
        self.key_quantizer = key_strategy or SMAQFullMetricScalarStrategy(
            dim=head_dim, Sigma_q=sigma, bits=key_bits, device=self.device, dtype=torch.float32)
        self.seq_len = 0
        self.key_quantized: Optional[Any] = None
        self.value_quantized: Optional[ValueQuantized] = None
        self.key_buffer: Optional[torch.Tensor] = None
        self.value_buffer: Optional[torch.Tensor] = None

    @property
    def capabilities(self) -> CacheCapabilities:
        return self.key_quantizer.capabilities

    def _compress(self, k: torch.Tensor, v: torch.Tensor):
        return (self.key_quantizer.quantize(k),
                quantize_values(v, bits=self.value_bits, group_size=self.value_group_size))

    def prefill(self, keys: torch.Tensor, values: torch.Tensor):
        n = keys.shape[-2]
        self.seq_len = n
        if n <= self.buffer_size:
            self.key_buffer, self.value_buffer = keys, values
            return
        cut = n - self.buffer_size
        self.key_buffer, self.value_buffer = keys[..., cut:, :], values[..., cut:, :]
        self.key_quantized, self.value_quantized = self._compress(keys[..., :cut, :], values[..., :cut, :])

    def append(self, key: torch.Tensor, value: torch.Tensor):
        self.seq_len += key.shape[-2]
        if self.key_buffer is None:
            self.key_buffer, self.value_buffer = key, value
        else:
            self.key_buffer = torch.cat([self.key_buffer, key], dim=-2)
            self.value_buffer = torch.cat([self.value_buffer, value], dim=-2)
        if self.key_buffer.shape[-2] > self.buffer_size:
            self._flush_buffer()

    def _flush_buffer(self):
        cut = self.key_buffer.shape[-2] - self.buffer_size
        kq, vq = self._compress(self.key_buffer[..., :cut, :], self.value_buffer[..., :cut, :])
        self.key_buffer = self.key_buffer[..., cut:, :]
        self.value_buffer = self.value_buffer[..., cut:, :]
        if self.key_quantized is None:
            self.key_quantized, self.value_quantized = kq, vq
            return
        self.key_quantized = self.key_quantizer.concat_quantized([self.key_quantized, kq])
        old = self.value_quantized
        self.value_quantized = ValueQuantized(
            data=torch.cat([old.data, vq.data], dim=-2), scales=torch.cat([old.scales, vq.scales], dim=-2),
            zeros=torch.cat([old.zeros, vq.zeros], dim=-2), bits=self.value_bits)

    def attention_scores(self, query: torch.Tensor, scale: float | None = None) -> torch.Tensor:
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        parts = []
        if self.key_quantized is not None:
            if getattr(self.key_quantizer, "supports_kernel", False):
                parts.append(self.key_quantizer.attention_score(query, self.key_quantized, scale=scale,
                                                                use_kernel=True))
            else:
                parts.append(self.key_quantizer.attention_score(query, self.key_quantized, scale=scale))
        if self.key_buffer is not None:
            parts.append(torch.matmul(query, self.key_buffer.transpose(-2, -1)) * scale)
        if not parts:
            return torch.empty((*query.shape[:-1], 0), device=query.device, dtype=query.dtype)
        return torch.cat(parts, dim=-1)

    def attend(self, attn_weights: torch.Tensor) -> torch.Tensor:
        outs = []
        col = 0
        if self.value_quantized is not None:
            nq = self.value_quantized.data.shape[-2]
            v = dequantize_values(self.value_quantized, self.value_group_size)
            outs.append(torch.matmul(attn_weights[..., col:col + nq], v))
            col += nq
        if self.value_buffer is not None:
            nb = self.value_buffer.shape[-2]
            outs.append(torch.matmul(attn_weights[..., col:col + nb], self.value_buffer))
        if not outs:
            return torch.zeros(*attn_weights.shape[:-1], self.head_dim, device=attn_weights.device,
                               dtype=attn_weights.dtype)
        return sum(outs)

    def memory_bytes(self) -> dict[str, int]:
        info = {"quantized_keys": 0, "quantized_values": 0, "buffer": 0, "total": 0}
        if self.key_quantized is not None:
            info["quantized_keys"] += self.key_quantizer.memory_bytes(self.key_quantized)
        if self.value_quantized is not None:
            vq = self.value_quantized
            info["quantized_values"] += vq.data.nelement() + 2 * vq.scales.nelement() + 2 * vq.zeros.nelement()
        for buf in (self.key_buffer, self.value_buffer):
            if buf is not None:
                info["buffer"] += buf.nelement() * 2
        info["total"] = info["quantized_keys"] + info["quantized_values"] + info["buffer"]
        return info

    def get_seq_length(self) -> int:
        return self.seq_len
