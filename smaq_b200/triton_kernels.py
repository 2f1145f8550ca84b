"""``smaq.triton_kernels`` entry point (smaq/triton_kernels.py:190-208), kept by name only.

The reference scores a decode query tile against scalar-coded keys with a Triton kernel and
falls back to torch.  Here the same public function runs this package's CUDA scoring kernel
(``smaq_key_scores``: query rotated once, codes unpacked and centroids gathered in registers,
no reconstructed keys); there is no Triton and no fallback.
"""

from __future__ import annotations

import torch

from smaq_b200 import ops
from smaq_b200._lib import SMAQ_KEYS_SCALAR
from smaq_b200.quantizer import SMAQQuantized


def smaq_attention_scores(quantizer, query: torch.Tensor, quantized_key: SMAQQuantized) -> torch.Tensor:
    """``(query @ E_inv^T) . centroids[codes] * norm`` in fp32, ``[..., Q, N]`` (unscaled, as the
    reference returns it).  ``quantizer`` is an ``SMAQQuantizer`` or a ``RotationAdapter``."""
    return ops.key_scores(query.float(), key_format=SMAQ_KEYS_SCALAR, scale=None, key_codes=quantized_key.indices,
                          key_norms=quantized_key.norms, key_bits=quantized_key.bits, E_inv=quantizer.E_inv,
                          centroids=quantizer.centroids)
