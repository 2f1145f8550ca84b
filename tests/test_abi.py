"""The C-ABI library loads and exports every symbol include/smaq_b200.h declares (no GPU calls)."""

import os
import re

from conftest import REPO


def declared_symbols():
    src = open(os.path.join(REPO, "include", "smaq_b200.h")).read()
    return sorted(set(re.findall(r"\b(smaq_[a-z_]+)\s*\(", src)))


def test_library_exports_header_symbols():
    from smaq_b200 import _lib, build
    build.build()
    lib = _lib.load()
    decl = declared_symbols()
    assert decl, "no declarations found"
    missing = [s for s in decl if not hasattr(lib, s)]
    assert not missing, missing
    assert set(decl) == set(_lib.EXPORTS)
    assert lib.smaq_abi_version() == 2


def test_struct_mirrors_match_the_library():
    import ctypes
    from smaq_b200 import _lib
    lib = _lib.load()  # also raises on a mismatch
    assert lib.smaq_args_size(0) == ctypes.sizeof(_lib.AppendArgs)
    assert lib.smaq_args_size(1) == ctypes.sizeof(_lib.DecodeArgs)
    assert lib.smaq_args_size(2) == ctypes.sizeof(_lib.ScoresArgs)
    assert lib.smaq_args_size(3) == ctypes.sizeof(_lib.AttendArgs)
    assert lib.smaq_args_size(4) == 0


def test_invalid_arguments_are_reported_without_a_gpu():
    """Argument validation runs on the host and fails with a message, before any CUDA call."""
    import ctypes
    from smaq_b200 import _lib
    lib = _lib.load()
    a = _lib.AppendArgs()
    a.n_tokens, a.n_heads, a.head_dim, a.page_size = 4, 1, 128, 4
    a.dtype = 7
    st = lib.smaq_append(ctypes.byref(a), None)
    assert st == 1
    assert b"dtype" in lib.smaq_last_error()
    d = _lib.DecodeArgs()
    d.batch, d.n_q_heads, d.n_kv_heads, d.head_dim = 1, 6, 4, 128
    assert lib.smaq_decode(ctypes.byref(d), None) == 1
    assert b"head counts" in lib.smaq_last_error()
    assert lib.smaq_decode_workspace_size(2, 32, 8, 128, 100) > 0


def test_cpu_tensors_raise():
    import pytest
    import torch
    from smaq_b200 import ops
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.quantize_values(torch.zeros(4, 128))


def test_status_calls_validate_without_a_gpu():
    from smaq_b200 import _lib
    lib = _lib.load()
    assert lib.smaq_decode_status(None, 0, 2, None) == 1
    assert b"bad sizes" in lib.smaq_last_error()


def test_kernel_path_query_without_a_gpu():
    """smaq_decode_kernel_path picks the fused kernels for their formats and the general path
    otherwise; it validates like smaq_decode and launches nothing."""
    from smaq_b200 import _lib, ops
    lib = _lib.load()
    d = _lib.DecodeArgs()
    d.q, d.q_dtype, d.batch, d.n_q_heads, d.n_kv_heads, d.head_dim = 4096, _lib.SMAQ_BF16, 2, 32, 8, 128
    d.key_codes, d.v_data, d.v_scales, d.v_zeros, d.hist_len, d.out = 4096, 8192, 12288, 16384, 20480, 24576
    d.value_bits, d.group_size, d.page_size, d.kv_dtype = 2, 32, 1024, _lib.SMAQ_BF16
    d.key_format, d.block_dim, d.n_centroids, d.centroids = _lib.SMAQ_KEYS_BVQ, 8, 256, 28672
    d.layout = _lib.SMAQ_LAYOUT_DECODE
    assert lib.smaq_decode_kernel_path(d) == ops.PATH_GENERAL      # no fp16 codebook given
    d.centroids_f16 = 32768
    assert lib.smaq_decode_kernel_path(d) == ops.PATH_FUSED_BVQ
    d.layout = _lib.SMAQ_LAYOUT_REFERENCE
    assert lib.smaq_decode_kernel_path(d) == ops.PATH_GENERAL
    d.layout = _lib.SMAQ_LAYOUT_DECODE
    d.key_format, d.key_bits, d.E_inv, d.key_norms = _lib.SMAQ_KEYS_SCALAR, 4, 36864, 40960
    assert lib.smaq_decode_kernel_path(d) == ops.PATH_FUSED_SCALAR
    d.q_dtype = _lib.SMAQ_F32
    assert lib.smaq_decode_kernel_path(d) == ops.PATH_GENERAL
    d.n_q_heads = 33
    assert lib.smaq_decode_kernel_path(d) == -1                     # invalid head counts
