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


class _GrowingRows:
    """Compressed history of an HF-style cache: every tensor field of a quantized-keys or
    ``ValueQuantized`` tuple kept in one buffer per field that grows by doubling along the token
    axis (axis ``len(lead)``), so an append writes only the new rows and the kernels read the
    first ``n`` rows of each buffer in place."""

    def __init__(self):
        self.n = 0
        self._buf: dict[str, torch.Tensor] = {}
        self._proto = None
        self._axis = 0

    def append(self, q: NamedTuple, axis: int) -> None:
        fields = q._asdict()
        m = next(v for v in fields.values() if isinstance(v, torch.Tensor)).shape[axis]
        need = self.n + m
        cap = next(iter(self._buf.values())).shape[axis] if self._buf else 0
        if need > cap:
            new_cap = max(need, 2 * cap, 64)
            for k, v in fields.items():
                if not isinstance(v, torch.Tensor):
                    continue
                shape = list(v.shape)
                shape[axis] = new_cap
                nb = torch.empty(shape, dtype=v.dtype, device=v.device)
                if self.n:
                    nb.narrow(axis, 0, self.n).copy_(self._buf[k].narrow(axis, 0, self.n))
                self._buf[k] = nb
        for k, v in fields.items():
            if isinstance(v, torch.Tensor):
                self._buf[k].narrow(axis, self.n, m).copy_(v)
        self._proto, self._axis = q, axis
        self.n = need

    def view(self):
        """The history as the tuple type it was appended as (views of the first n rows)."""
        if self._proto is None:
            return None
        f = {k: (self._buf[k].narrow(self._axis, 0, self.n) if isinstance(v, torch.Tensor) else v)
             for k, v in self._proto._asdict().items()}
        return type(self._proto)(**f)


class SMAQKVCache:
    """HF-style cache, tensors ``[..., T, D]`` (API of smaq/kv_cache.py:106-290): compressed
    history plus an exact buffer of the last ``buffer_size`` tokens.  A prefill longer than the
    buffer compresses all but its last ``buffer_size`` tokens; an append that overfills the
    buffer compresses the oldest overflow (smaq/kv_cache.py:150-216).  Keys go through the
    strategy's GPU quantizer, values through ``quantize_values``; the history is kept in
    growing device buffers (``_GrowingRows``).  ``attention_scores`` returns the
    ``[history || buffer]`` logits -- the history part one ``smaq_key_scores`` launch -- and
    ``attend`` applies caller-computed weights, the history part one ``smaq_attend_values``
    launch with the dequantization fused."""

    def __init__(self, head_dim: int, Sigma_q: torch.Tensor | None = None, key_bits: int = 3,
                 value_bits: int = 2, value_group_size: int = 32, buffer_size: int = 128,
                 device: torch.device | None = None, dtype: torch.dtype = torch.float16, layer_idx: int = 0,
                 key_strategy: Any | None = None, calibration_provider: CalibrationProvider | None = None):
        self.head_dim = head_dim
        self.key_bits, self.value_bits, self.value_group_size = key_bits, value_bits, value_group_size
        self.buffer_size = buffer_size
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda" if torch.cuda.is_available() else "cpu")
        self.dtype = dtype
        self.layer_idx = layer_idx
        self.calibration_provider = calibration_provider or IdentityCalibrationProvider()
        if key_strategy is None:
            sigma = Sigma_q if Sigma_q is not None else self.calibration_provider.get_sigma_q(
                layer_idx, head_dim, device=self.device)
            key_strategy = SMAQFullMetricScalarStrategy(dim=head_dim, Sigma_q=sigma, bits=key_bits,
                                                        device=self.device, dtype=torch.float32)
        self.key_quantizer = key_strategy
        self.seq_len = 0
        self._keys = _GrowingRows()
        self._values = _GrowingRows()
        self.key_buffer: Optional[torch.Tensor] = None
        self.value_buffer: Optional[torch.Tensor] = None

    @property
    def capabilities(self) -> CacheCapabilities:
        return self.key_quantizer.capabilities

    @property
    def key_quantized(self):
        return self._keys.view()

    @property
    def value_quantized(self) -> Optional[ValueQuantized]:
        return self._values.view()

    def _compress(self, k: torch.Tensor, v: torch.Tensor) -> None:
        axis = k.dim() - 2
        self._keys.append(self.key_quantizer.quantize(k), axis)
        self._values.append(quantize_values(v, bits=self.value_bits, group_size=self.value_group_size), axis)

    def _keep_last(self, keys: torch.Tensor, values: torch.Tensor) -> None:
        """Buffer the last buffer_size tokens of keys/values, compressing the rest."""
        cut = keys.shape[-2] - self.buffer_size
        if cut > 0:
            self._compress(keys[..., :cut, :], values[..., :cut, :])
            keys, values = keys[..., cut:, :], values[..., cut:, :]
        self.key_buffer, self.value_buffer = keys, values

    def prefill(self, keys: torch.Tensor, values: torch.Tensor):
        self.seq_len = keys.shape[-2]
        self._keys, self._values = _GrowingRows(), _GrowingRows()
        self._keep_last(keys, values)

    def append(self, key: torch.Tensor, value: torch.Tensor):
        self.seq_len += key.shape[-2]
        if self.key_buffer is not None:
            key = torch.cat([self.key_buffer, key], dim=-2)
            value = torch.cat([self.value_buffer, value], dim=-2)
        self._keep_last(key, value)

    def attention_scores(self, query: torch.Tensor, scale: float | None = None) -> torch.Tensor:
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        parts = []
        kq = self.key_quantized
        if kq is not None:
            parts.append(self.key_quantizer.attention_score(query, kq, scale=scale))
        if self.key_buffer is not None:
            parts.append(torch.matmul(query, self.key_buffer.transpose(-2, -1)) * scale)
        if not parts:
            return torch.empty((*query.shape[:-1], 0), device=query.device, dtype=query.dtype)
        return torch.cat(parts, dim=-1)

    def attend(self, attn_weights: torch.Tensor) -> torch.Tensor:
        out = None
        n_hist = self._values.n
        vq = self.value_quantized
        if vq is not None:
            out = ops.attend_values(attn_weights[..., :n_hist], vq.data, vq.scales, vq.zeros, bits=vq.bits,
                                    group_size=self.value_group_size, head_dim=self.head_dim)
        if self.value_buffer is not None:
            nb = self.value_buffer.shape[-2]
            part = torch.matmul(attn_weights[..., n_hist:n_hist + nb], self.value_buffer.to(attn_weights.dtype))
            out = part if out is None else out + part
        if out is None:
            return torch.zeros(*attn_weights.shape[:-1], self.head_dim, device=attn_weights.device,
                               dtype=attn_weights.dtype)
        return out

    def memory_bytes(self) -> dict[str, int]:
        """Bytes with the reference's accounting (smaq/kv_cache.py:269-285)."""
        info = {"quantized_keys": 0, "quantized_values": 0, "buffer": 0}
        kq, vq = self.key_quantized, self.value_quantized
        if kq is not None:
            info["quantized_keys"] = self.key_quantizer.memory_bytes(kq)
        if vq is not None:
            info["quantized_values"] = vq.data.nelement() + 2 * (vq.scales.nelement() + vq.zeros.nelement())
        info["buffer"] = sum(2 * b.nelement() for b in (self.key_buffer, self.value_buffer) if b is not None)
        info["total"] = sum(info.values())
        return info

    def get_seq_length(self) -> int:
        return self.seq_len
