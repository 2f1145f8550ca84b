"""ctypes binding of ``libsmaq_b200.so`` (declared in ``include/smaq_b200.h``).

The library is loaded from the package directory.  If it is missing the import of any
compute entry point raises: there is no CPU or pure-torch fallback for the hot path.
"""

from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsmaq_b200.so")

SMAQ_F32, SMAQ_BF16, SMAQ_F16 = 0, 1, 2
SMAQ_KEYS_NONE, SMAQ_KEYS_SCALAR, SMAQ_KEYS_BVQ = 0, 1, 2
SMAQ_LAYOUT_REFERENCE, SMAQ_LAYOUT_DECODE = 0, 1
STATUS = {0: "OK", 1: "INVALID", 2: "UNSUPPORTED", 3: "CUDA", 4: "WORKSPACE", 5: "DEVICE", 6: "TIMEOUT", 7: "PEER"}
SMAQ_ERR_TIMEOUT, SMAQ_ERR_PEER = 6, 7
COMM_ID_BYTES = 128

# every symbol include/smaq_b200.h declares (checked by the CPU test suite)
EXPORTS = (
    "smaq_abi_version", "smaq_args_size", "smaq_last_error", "smaq_append", "smaq_quantize_keys_scalar",
    "smaq_quantize_values", "smaq_quantize_keys_bvq", "smaq_decode_workspace_size", "smaq_decode",
    "smaq_decode_kernel_path",
    "smaq_merge_partials", "smaq_decode_noalloc", "smaq_decode_noalloc_max_workspace",
    "smaq_decode_status", "smaq_append_status", "smaq_selftest_wait_timeout",
    "smaq_key_scores", "smaq_attend_workspace_size", "smaq_attend_values", "smaq_kmeans_workspace_size",
    "smaq_kmeans", "smaq_comm_set_backend", "smaq_comm_unique_id", "smaq_comm_init", "smaq_comm_allgather",
    "smaq_comm_wait", "smaq_comm_status", "smaq_comm_abort", "smaq_comm_destroy",
)

vp = C.c_void_p
i64 = C.c_int64
i32 = C.c_int


CommUniqueId = C.CFUNCTYPE(i32, vp)
CommInitRank = C.CFUNCTYPE(i32, C.POINTER(vp), i32, vp, i32)
CommHandleCall = C.CFUNCTYPE(i32, vp)
CommAllGather = C.CFUNCTYPE(i32, vp, vp, C.c_size_t, vp, vp)


class CommBackend(C.Structure):
    """Mirror of smaq_comm_backend: NCCL calls returning ncclResult_t values."""
    _fields_ = [
        ("unique_id", CommUniqueId), ("init_rank", CommInitRank), ("async_error", CommHandleCall),
        ("all_gather", CommAllGather), ("abort_comm", CommHandleCall), ("finalize", CommHandleCall),
        ("destroy", CommHandleCall),
    ]


class AppendArgs(C.Structure):
    _fields_ = [
        ("k", vp), ("v", vp), ("dtype", i32), ("n_tokens", i64), ("n_heads", i32), ("head_dim", i32),
        ("k_stride_t", i64), ("k_stride_h", i64), ("v_stride_t", i64), ("v_stride_h", i64),
        ("slots", vp), ("slot_offset", i64), ("page_size", i64),
        ("key_format", i32), ("key_bits", i32), ("E", vp), ("boundaries", vp), ("E_blocks", vp),
        ("centroids", vp), ("block_dim", i32), ("n_centroids", i32), ("key_codes", vp), ("key_norms", vp),
        ("value_bits", i32), ("group_size", i32), ("v_data", vp), ("v_scales", vp), ("v_zeros", vp),
        ("layout", i32),
    ]


class DecodeArgs(C.Structure):
    _fields_ = [
        ("q", vp), ("q_dtype", i32), ("q_stride_b", i64), ("q_stride_h", i64),
        ("batch", i32), ("n_q_heads", i32), ("n_kv_heads", i32), ("head_dim", i32), ("scale", C.c_float),
        ("key_format", i32), ("key_bits", i32), ("E_inv", vp), ("centroids", vp), ("block_dim", i32),
        ("n_centroids", i32), ("key_codes", vp), ("key_norms", vp), ("kv_dtype", i32),
        ("v_data", vp), ("v_scales", vp), ("v_zeros", vp), ("value_bits", i32), ("group_size", i32),
        ("block_table", vp), ("bt_stride", i64), ("page_size", i64), ("hist_len", vp), ("hist_total", vp),
        ("min_history", i32), ("recent_k", vp), ("recent_v", vp), ("recent_dtype", i32),
        ("r_stride_b", i64), ("r_stride_t", i64), ("r_stride_h", i64), ("recent_len", vp),
        ("out", vp), ("o_stride_b", i64), ("o_stride_h", i64), ("partial_out", vp),
        ("workspace", vp), ("workspace_bytes", C.c_size_t), ("num_ctas", i32), ("layout", i32),
        ("centroids_f16", vp), ("overlap_prior", i32),
    ]


class ScoresArgs(C.Structure):
    _fields_ = [
        ("q", vp), ("q_dtype", i32), ("q_stride_g", i64), ("q_stride_q", i64), ("n_groups", i64),
        ("n_queries", i32), ("n_tokens", i64), ("head_dim", i32), ("key_format", i32),
        ("key_codes", vp), ("codes_stride_g", i64), ("key_norms", vp), ("norms_dtype", i32),
        ("norms_stride_g", i64), ("key_bits", i32), ("E_inv", vp), ("centroids", vp),
        ("key_idx", vp), ("idx_is_int64", i32), ("idx_stride_g", i64), ("block_dim", i32),
        ("n_centroids", i32), ("decoded_centroids", vp), ("scale", C.c_float),
        ("out", vp), ("out_dtype", i32), ("out_stride_g", i64), ("out_stride_q", i64), ("q_rotated", i32),
    ]


class AttendArgs(C.Structure):
    _fields_ = [
        ("w", vp), ("w_dtype", i32), ("w_stride_g", i64), ("w_stride_q", i64), ("n_groups", i64),
        ("n_queries", i32), ("n_tokens", i64), ("head_dim", i32), ("v_data", vp), ("data_stride_g", i64),
        ("v_scales", vp), ("v_zeros", vp), ("sz_dtype", i32), ("sz_stride_g", i64), ("value_bits", i32),
        ("group_size", i32), ("out", vp), ("out_dtype", i32), ("out_stride_g", i64), ("out_stride_q", i64),
        ("workspace", vp), ("workspace_bytes", C.c_size_t),
    ]


_lib = None


def load() -> C.CDLL:
    """Load the CUDA library; raises if it was not built (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    path = LIB_PATH
    if not os.path.exists(path):
        raise RuntimeError(
            f"smaq_b200 CUDA library not found at {path}; build it with "
            "`python -m smaq_b200.build` (there is no CPU fallback)")
    lib = C.CDLL(path)
    lib.smaq_abi_version.restype = i32
    lib.smaq_args_size.argtypes = [i32]
    lib.smaq_args_size.restype = C.c_size_t
    for which, mirror in ((0, AppendArgs), (1, DecodeArgs), (2, ScoresArgs), (3, AttendArgs)):
        if lib.smaq_args_size(which) != C.sizeof(mirror):
            raise RuntimeError(f"{path}: {mirror.__name__} is {C.sizeof(mirror)} bytes here but "
                               f"{lib.smaq_args_size(which)} in the library (stale build or ABI mismatch)")
    lib.smaq_last_error.restype = C.c_char_p
    lib.smaq_append.argtypes = [C.POINTER(AppendArgs), vp]
    lib.smaq_append.restype = i32
    lib.smaq_quantize_keys_scalar.argtypes = [vp, i32, i64, i32, vp, vp, i32, vp, vp, vp]
    lib.smaq_quantize_keys_scalar.restype = i32
    lib.smaq_quantize_values.argtypes = [vp, i32, i64, i32, i32, i32, vp, vp, vp, vp]
    lib.smaq_quantize_values.restype = i32
    lib.smaq_quantize_keys_bvq.argtypes = [vp, i32, i64, i32, vp, vp, i32, i32, vp, vp]
    lib.smaq_quantize_keys_bvq.restype = i32
    lib.smaq_decode_workspace_size.argtypes = [i32, i32, i32, i32, i32]
    lib.smaq_decode_workspace_size.restype = C.c_size_t
    lib.smaq_decode.argtypes = [C.POINTER(DecodeArgs), vp]
    lib.smaq_decode.restype = i32
    lib.smaq_decode_kernel_path.argtypes = [C.POINTER(DecodeArgs)]
    lib.smaq_decode_kernel_path.restype = i32
    lib.smaq_merge_partials.argtypes = [vp, i32, i32, i32, i32, vp, i32, i64, i64, vp]
    lib.smaq_merge_partials.restype = i32
    lib.smaq_decode_noalloc.argtypes = [C.POINTER(DecodeArgs), vp]
    lib.smaq_decode_noalloc.restype = i32
    lib.smaq_decode_noalloc_max_workspace.restype = C.c_size_t
    lib.smaq_decode_status.argtypes = [vp, i32, i32, vp]
    lib.smaq_decode_status.restype = i32
    lib.smaq_append_status.argtypes = [vp]
    lib.smaq_append_status.restype = i32
    lib.smaq_selftest_wait_timeout.argtypes = [C.c_uint, vp]
    lib.smaq_selftest_wait_timeout.restype = i32
    lib.smaq_key_scores.argtypes = [C.POINTER(ScoresArgs), vp]
    lib.smaq_key_scores.restype = i32
    lib.smaq_attend_workspace_size.argtypes = [i64, i32, i64, i32]
    lib.smaq_attend_workspace_size.restype = C.c_size_t
    lib.smaq_attend_values.argtypes = [C.POINTER(AttendArgs), vp]
    lib.smaq_attend_values.restype = i32
    lib.smaq_comm_set_backend.argtypes = [vp]
    lib.smaq_comm_set_backend.restype = i32
    lib.smaq_comm_unique_id.argtypes = [vp]
    lib.smaq_comm_unique_id.restype = i32
    lib.smaq_comm_init.argtypes = [C.POINTER(vp), i32, i32, vp, C.c_double]
    lib.smaq_comm_init.restype = i32
    lib.smaq_comm_allgather.argtypes = [vp, vp, vp, C.c_size_t, vp, C.c_double]
    lib.smaq_comm_allgather.restype = i32
    lib.smaq_comm_wait.argtypes = [vp, vp, C.c_double]
    lib.smaq_comm_wait.restype = i32
    lib.smaq_comm_status.argtypes = [vp]
    lib.smaq_comm_status.restype = i32
    lib.smaq_comm_abort.argtypes = [vp]
    lib.smaq_comm_abort.restype = i32
    lib.smaq_comm_destroy.argtypes = [vp, C.c_double]
    lib.smaq_comm_destroy.restype = i32
    lib.smaq_kmeans_workspace_size.argtypes = [i32, i64]
    lib.smaq_kmeans_workspace_size.restype = C.c_size_t
    lib.smaq_kmeans.argtypes = [vp, i32, i64, i32, i32, i32, C.c_uint64, vp, vp, C.c_size_t, vp]
    lib.smaq_kmeans.restype = i32
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().smaq_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed ({STATUS.get(status, status)}): {msg}")
