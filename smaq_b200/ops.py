"""Torch-facing wrappers of the C-ABI kernels.

Every function here takes CUDA tensors, enqueues the kernel on
``torch.cuda.current_stream()`` and returns freshly allocated outputs (or writes
into caller buffers).  CPU tensors raise ``RuntimeError``: the hot path has no
CPU implementation.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from smaq_b200 import _lib
from smaq_b200._lib import (SMAQ_BF16, SMAQ_F16, SMAQ_F32, SMAQ_KEYS_BVQ, SMAQ_KEYS_SCALAR,
                           SMAQ_LAYOUT_DECODE, SMAQ_LAYOUT_REFERENCE)

_DT = {torch.float32: SMAQ_F32, torch.bfloat16: SMAQ_BF16, torch.float16: SMAQ_F16}

MIN_HISTORY = 16
PATH_GENERAL, PATH_FUSED_BVQ, PATH_FUSED_SCALAR = 0, 1, 2   # smaq_decode_kernel_path


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}; expected float32, bfloat16 or float16") from None


def _cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "smaq_b200 kernels need CUDA tensors (there is no CPU fallback); got a tensor on "
                f"{t.device}")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def packed_dim(dim: int, bits: int) -> int:
    vpb = max(1, 8 // bits)
    return (dim + vpb - 1) // vpb


def _rows(x: torch.Tensor) -> torch.Tensor:
    """Contiguous ``[n_rows, D]`` view of ``(..., D)``."""
    return x.reshape(-1, x.shape[-1]).contiguous()


# --------------------------------------------------------------------- quantize
def quantize_keys_scalar(k: torch.Tensor, E: torch.Tensor, boundaries: torch.Tensor, bits: int):
    """``(..., D)`` keys -> (packed codes ``(..., ceil(D / (8//bits)))`` uint8, norms ``(...)``)."""
    _cuda(k, E, boundaries)
    lib = _lib.load()
    D = k.shape[-1]
    kr = _rows(k)
    n = kr.shape[0]
    codes = torch.empty((n, packed_dim(D, bits)), dtype=torch.uint8, device=k.device)
    norms = torch.empty((n,), dtype=k.dtype, device=k.device)
    Ef = E.to(torch.float32).contiguous()
    bf = boundaries.to(torch.float32).contiguous()
    _lib.check(lib.smaq_quantize_keys_scalar(kr.data_ptr(), dtype_code(k.dtype), n, D, Ef.data_ptr(),
                                             bf.data_ptr(), bits, codes.data_ptr(), norms.data_ptr(),
                                             _stream()), "smaq_quantize_keys_scalar")
    return codes.reshape(*k.shape[:-1], -1), norms.reshape(k.shape[:-1])


def quantize_values(v: torch.Tensor, bits: int = 2, group_size: int = 32):
    """``(..., D)`` values -> (data uint8 ``(..., D*bits/8)``, scales, zeros ``(..., D/group)``)."""
    _cuda(v)
    lib = _lib.load()
    D = v.shape[-1]
    vr = _rows(v)
    n = vr.shape[0]
    data = torch.empty((n, D * bits // 8), dtype=torch.uint8, device=v.device)
    scales = torch.empty((n, D // group_size), dtype=v.dtype, device=v.device)
    zeros = torch.empty_like(scales)
    _lib.check(lib.smaq_quantize_values(vr.data_ptr(), dtype_code(v.dtype), n, D, bits, group_size,
                                        data.data_ptr(), scales.data_ptr(), zeros.data_ptr(), _stream()),
               "smaq_quantize_values")
    lead = v.shape[:-1]
    return data.reshape(*lead, -1), scales.reshape(*lead, -1), zeros.reshape(*lead, -1)


def quantize_keys_bvq(k: torch.Tensor, E_blocks: torch.Tensor, centroids: torch.Tensor) -> torch.Tensor:
    """``(..., D)`` keys -> uint8 block indices ``(..., D / block_dim)``."""
    _cuda(k, E_blocks, centroids)
    lib = _lib.load()
    D = k.shape[-1]
    nb, nc, bd = centroids.shape
    kr = _rows(k)
    n = kr.shape[0]
    idx = torch.empty((n, nb), dtype=torch.uint8, device=k.device)
    Eb = E_blocks.to(torch.float32).contiguous()
    cf = centroids.to(torch.float32).contiguous()
    _lib.check(lib.smaq_quantize_keys_bvq(kr.data_ptr(), dtype_code(k.dtype), n, D, Eb.data_ptr(),
                                          cf.data_ptr(), bd, nc, idx.data_ptr(), _stream()),
               "smaq_quantize_keys_bvq")
    return idx.reshape(*k.shape[:-1], nb)


def append(key: Optional[torch.Tensor], value: Optional[torch.Tensor], *, n_heads: int, slot_offset: int = 0,
           slots: Optional[torch.Tensor] = None, page_size: int, key_format: int = SMAQ_KEYS_SCALAR,
           key_bits: int = 3, E: Optional[torch.Tensor] = None, boundaries: Optional[torch.Tensor] = None,
           E_blocks: Optional[torch.Tensor] = None, centroids: Optional[torch.Tensor] = None,
           key_codes: Optional[torch.Tensor] = None, key_norms: Optional[torch.Tensor] = None,
           value_bits: int = 2, group_size: int = 32, v_data: Optional[torch.Tensor] = None,
           v_scales: Optional[torch.Tensor] = None, v_zeros: Optional[torch.Tensor] = None,
           layout: int = SMAQ_LAYOUT_REFERENCE) -> None:
    """Quantize a ``[T, H, D]`` chunk of keys and/or values into store rows (see include/smaq_b200.h)."""
    _cuda(key, value, slots, E, boundaries, E_blocks, centroids, key_codes, key_norms, v_data)
    lib = _lib.load()
    ref = key if key is not None else value
    if ref is None:
        return
    a = _lib.AppendArgs()
    a.dtype = dtype_code(ref.dtype)
    a.n_tokens = ref.shape[0]
    a.n_heads = n_heads
    a.head_dim = ref.shape[-1]
    keep = []
    if key is not None:
        if key.stride(-1) != 1:
            key = key.contiguous()
        keep.append(key)
        a.k = key.data_ptr()
        a.k_stride_t, a.k_stride_h = key.stride(0), key.stride(1)
        a.key_format = key_format
        a.key_bits = key_bits
        a.key_codes = _ptr(key_codes)
        if key_format == SMAQ_KEYS_SCALAR:
            Ef = E.to(torch.float32).contiguous()
            bf = boundaries.to(torch.float32).contiguous()
            keep += [Ef, bf]
            a.E, a.boundaries = Ef.data_ptr(), bf.data_ptr()
            a.key_norms = _ptr(key_norms)
        else:
            Eb = E_blocks.to(torch.float32).contiguous()
            cf = centroids.to(torch.float32).contiguous()
            keep += [Eb, cf]
            a.E_blocks, a.centroids = Eb.data_ptr(), cf.data_ptr()
            a.block_dim = centroids.shape[2]
            a.n_centroids = centroids.shape[1]
    if value is not None:
        if value.stride(-1) != 1:
            value = value.contiguous()
        keep.append(value)
        a.v = value.data_ptr()
        a.v_stride_t, a.v_stride_h = value.stride(0), value.stride(1)
        a.value_bits = value_bits
        a.group_size = group_size
        a.v_data, a.v_scales, a.v_zeros = _ptr(v_data), _ptr(v_scales), _ptr(v_zeros)
    if slots is not None:
        slots = slots.to(torch.int64).contiguous()
        keep.append(slots)
        a.slots = slots.data_ptr()
    a.slot_offset = slot_offset
    a.page_size = page_size
    a.layout = layout
    _lib.check(lib.smaq_append(a, _stream()), "smaq_append")


# --------------------------------------------------------------------- standalone scores / attend
def _packed_rows(t: torch.Tensor) -> torch.Tensor:
    """``t`` with packed rows (last dim contiguous, rows back to back within a group); a group
    stride may be anything (a capacity buffer sliced along its token dim keeps its storage)."""
    if t.stride(-1) == 1 and (t.dim() < 2 or t.shape[-2] <= 1 or t.stride(-2) == t.shape[-1]):
        return t
    return t.contiguous()


def _groups(lead: torch.Size, *ts: torch.Tensor, tail: tuple[int, ...]) -> list[torch.Tensor]:
    """Each tensor broadcast to ``lead + its own trailing dims`` and flattened to ``[G, ...]``."""
    out = []
    for t, k in zip(ts, tail):
        t = t.expand(*lead, *t.shape[t.dim() - k:])
        out.append(t.reshape(-1, *t.shape[len(lead):]))
    return out


def key_scores(query: torch.Tensor, *, key_format: int, scale: Optional[float] = None,
               key_codes: Optional[torch.Tensor] = None, key_norms: Optional[torch.Tensor] = None, key_bits: int = 3,
               E_inv: Optional[torch.Tensor] = None, centroids: Optional[torch.Tensor] = None,
               key_idx: Optional[torch.Tensor] = None, decoded_centroids: Optional[torch.Tensor] = None
               ) -> torch.Tensor:
    """``scale * q . k_hat`` of ``query [..., Q, D]`` against compressed keys (reference layout):
    scalar ``key_codes [..., N, ceil(D/(8/bits))]`` + ``key_norms [..., N]``, or block-VQ
    ``key_idx [..., N, D/bd]`` (uint8 or int64).  Leading dims broadcast.  Returns ``[..., Q, N]`` in
    the query dtype (smaq_key_scores)."""
    _cuda(query, key_codes, key_idx)
    lib = _lib.load()
    D = query.shape[-1]
    keys = key_codes if key_format == SMAQ_KEYS_SCALAR else key_idx
    lead = torch.broadcast_shapes(query.shape[:-2], keys.shape[:-2])
    N = keys.shape[-2]
    (q,) = _groups(lead, query, tail=(2,))
    q = q if q.stride(-1) == 1 else q.contiguous()
    G, Q = q.shape[0], q.shape[1]
    out = torch.empty((G, Q, N), dtype=query.dtype, device=query.device)
    a = _lib.ScoresArgs()
    a.q, a.q_dtype, a.q_stride_g, a.q_stride_q = q.data_ptr(), dtype_code(q.dtype), q.stride(0), q.stride(1)
    a.n_groups, a.n_queries, a.n_tokens, a.head_dim = G, Q, N, D
    a.key_format = key_format
    a.scale = float(1.0 if scale is None else scale)
    keep = [q]
    if key_format == SMAQ_KEYS_SCALAR:
        # rotate the few query rows once (a small fp32 GEMM) instead of in every CTA
        qr = torch.matmul(q.float(), E_inv.to(q.device, torch.float32).T).contiguous()
        keep.append(qr)
        a.q, a.q_dtype, a.q_stride_g, a.q_stride_q = qr.data_ptr(), SMAQ_F32, qr.stride(0), qr.stride(1)
        a.q_rotated = 1
        codes, norms = _groups(lead, key_codes, key_norms, tail=(2, 1))
        codes, norms = _packed_rows(codes), (norms if norms.stride(-1) == 1 else norms.contiguous())
        Ei = E_inv.to(torch.float32).contiguous()
        cf = centroids.to(torch.float32).contiguous()
        keep += [codes, norms, Ei, cf]
        a.key_codes, a.codes_stride_g = codes.data_ptr(), codes.stride(0)
        a.key_norms, a.norms_dtype, a.norms_stride_g = norms.data_ptr(), dtype_code(norms.dtype), norms.stride(0)
        a.key_bits, a.E_inv, a.centroids = key_bits, Ei.data_ptr(), cf.data_ptr()
    else:
        (idx,) = _groups(lead, key_idx, tail=(2,))
        idx = _packed_rows(idx)
        if idx.dtype not in (torch.uint8, torch.int64):
            idx = idx.to(torch.int64)
        dc = decoded_centroids.to(torch.float32).contiguous()
        keep += [idx, dc]
        a.key_idx, a.idx_is_int64, a.idx_stride_g = idx.data_ptr(), int(idx.dtype == torch.int64), idx.stride(0)
        a.block_dim, a.n_centroids, a.decoded_centroids = dc.shape[2], dc.shape[1], dc.data_ptr()
    a.out, a.out_dtype, a.out_stride_g, a.out_stride_q = out.data_ptr(), dtype_code(out.dtype), out.stride(0), \
        out.stride(1)
    _lib.check(lib.smaq_key_scores(a, _stream()), "smaq_key_scores")
    return out.reshape(*lead, Q, N)


def attend_values(weights: torch.Tensor, v_data: torch.Tensor, v_scales: torch.Tensor, v_zeros: torch.Tensor, *,
                  bits: int = 2, group_size: int = 32, head_dim: Optional[int] = None,
                  out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """``weights [..., Q, N]`` applied to compressed values ``v_data [..., N, D*bits/8]`` with
    ``v_scales / v_zeros [..., N, D/group_size]`` (reference layout): ``[..., Q, D]`` in the
    weights dtype (smaq_attend_values, dequantization fused)."""
    _cuda(weights, v_data)
    lib = _lib.load()
    D = head_dim or v_data.shape[-1] * 8 // bits
    lead = torch.broadcast_shapes(weights.shape[:-2], v_data.shape[:-2])
    w, = _groups(lead, weights, tail=(2,))
    w = w if w.stride(-1) == 1 else w.contiguous()
    data, sc, zs = (_packed_rows(t) for t in _groups(lead, v_data, v_scales, v_zeros, tail=(2, 2, 2)))
    if zs.dtype != sc.dtype:
        zs = zs.to(sc.dtype)
    G, Q, N = w.shape
    out = torch.empty((G, Q, D), dtype=out_dtype or weights.dtype, device=weights.device)
    ws_bytes = int(lib.smaq_attend_workspace_size(G, Q, N, D))
    ws = torch.empty((max(ws_bytes, 16),), dtype=torch.uint8, device=weights.device)
    a = _lib.AttendArgs()
    a.w, a.w_dtype, a.w_stride_g, a.w_stride_q = w.data_ptr(), dtype_code(w.dtype), w.stride(0), w.stride(1)
    a.n_groups, a.n_queries, a.n_tokens, a.head_dim = G, Q, N, D
    a.v_data, a.data_stride_g = data.data_ptr(), data.stride(0)
    a.v_scales, a.v_zeros, a.sz_dtype, a.sz_stride_g = sc.data_ptr(), zs.data_ptr(), dtype_code(sc.dtype), sc.stride(0)
    a.value_bits, a.group_size = bits, group_size
    a.out, a.out_dtype, a.out_stride_g, a.out_stride_q = out.data_ptr(), dtype_code(out.dtype), out.stride(0), \
        out.stride(1)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.smaq_attend_values(a, _stream()), "smaq_attend_values")
    return out.reshape(*lead, Q, D)


# --------------------------------------------------------------------- calibration
def kmeans(data: torch.Tensor, n_centroids: int, n_iters: int = 20, seed: int = 42) -> torch.Tensor:
    """k-means++ + Lloyd on the device for ``data [n_blocks, n_points, dim]`` (fp32, dim <= 16):
    ``[n_blocks, n_centroids, dim]`` centroids, one ``smaq_kmeans`` call, no host round trips
    inside."""
    _cuda(data)
    lib = _lib.load()
    x = data.to(torch.float32).contiguous()
    nb, n, d = x.shape
    cent = torch.empty((nb, n_centroids, d), dtype=torch.float32, device=x.device)
    ws = torch.empty((int(lib.smaq_kmeans_workspace_size(nb, n)),), dtype=torch.uint8, device=x.device)
    _lib.check(lib.smaq_kmeans(x.data_ptr(), nb, n, d, n_centroids, n_iters, seed & (2 ** 64 - 1), cent.data_ptr(),
                               ws.data_ptr(), ws.numel(), _stream()), "smaq_kmeans")
    return cent


# --------------------------------------------------------------------- decode
def decode_workspace_bytes(batch: int, n_q_heads: int, n_kv_heads: int, head_dim: int, num_ctas: int = 0) -> int:
    return int(_lib.load().smaq_decode_workspace_size(batch, n_q_heads, n_kv_heads, head_dim, num_ctas))


def decode(q: torch.Tensor, *, n_kv_heads: int, key_format: int, key_codes: torch.Tensor,
           v_data: torch.Tensor, v_scales: torch.Tensor, v_zeros: torch.Tensor, hist_len: torch.Tensor,
           page_size: int, key_bits: int = 4, E_inv: Optional[torch.Tensor] = None,
           centroids: Optional[torch.Tensor] = None, key_norms: Optional[torch.Tensor] = None,
           value_bits: int = 2, group_size: int = 32, block_table: Optional[torch.Tensor] = None,
           hist_total: Optional[torch.Tensor] = None, recent_k: Optional[torch.Tensor] = None,
           recent_v: Optional[torch.Tensor] = None, recent_len: Optional[torch.Tensor] = None,
           scale: Optional[float] = None, min_history: int = MIN_HISTORY, out: Optional[torch.Tensor] = None,
           partial_out: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None,
           num_ctas: int = 0, want_out: bool = True, layout: int = SMAQ_LAYOUT_REFERENCE,
           centroids_f16: Optional[torch.Tensor] = None, entry: str = "smaq_decode",
           overlap_prior: bool = False, query_path: bool = False):
    """Batched hybrid decode attention.

    ``q``: ``[B, Hq, D]``.  History streams are store rows ``[pages, Hkv, page_size, ...]``;
    ``recent_k/v``: ``[B, W, Hkv, D]`` (stride 0 on B allowed).  Returns ``out [B, Hq, D]`` in
    the query dtype (reference rounding), and/or fills ``partial_out [B, Hq, 2D+2]``.
    ``overlap_prior``: overlap the launch with the end of the previous kernel on the stream
    (programmatic dependent launch); only when that kernel writes none of the history rows,
    block table, lengths or codebooks (``smaq_decode_args.overlap_prior``).
    ``query_path``: launch nothing and return the kernel path these arguments select
    (``PATH_FUSED_BVQ``, ``PATH_FUSED_SCALAR`` or ``PATH_GENERAL``, smaq_decode_kernel_path).
    """
    _cuda(q, key_codes, v_data, hist_len, recent_k, block_table)
    lib = _lib.load()
    B, Hq, D = q.shape
    if q.stride(-1) != 1:
        q = q.contiguous()
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None and want_out and not query_path:
        out = torch.empty((B, Hq, D), dtype=q.dtype, device=q.device)
    keep = [q]
    a = _lib.DecodeArgs()
    a.q, a.q_dtype, a.q_stride_b, a.q_stride_h = q.data_ptr(), dtype_code(q.dtype), q.stride(0), q.stride(1)
    a.batch, a.n_q_heads, a.n_kv_heads, a.head_dim = B, Hq, n_kv_heads, D
    a.scale = float(scale)
    a.key_format = key_format
    a.key_bits = key_bits
    if key_format == SMAQ_KEYS_SCALAR:
        Ei = E_inv.to(torch.float32).contiguous()
        cf = centroids.to(torch.float32).contiguous()
        keep += [Ei, cf]
        a.E_inv, a.centroids = Ei.data_ptr(), cf.data_ptr()
        a.key_norms = key_norms.data_ptr()
        a.kv_dtype = dtype_code(key_norms.dtype)
    else:
        cf = centroids.to(torch.float32).contiguous()
        keep.append(cf)
        a.centroids = cf.data_ptr()
        a.block_dim = centroids.shape[2]
        a.n_centroids = centroids.shape[1]
        a.kv_dtype = dtype_code(v_scales.dtype)
    a.key_codes = key_codes.data_ptr()
    a.v_data, a.v_scales, a.v_zeros = v_data.data_ptr(), v_scales.data_ptr(), v_zeros.data_ptr()
    a.value_bits, a.group_size = value_bits, group_size
    if block_table is not None:
        bt = block_table.to(torch.int32)
        if bt.stride(-1) != 1:
            bt = bt.contiguous()
        keep.append(bt)
        a.block_table, a.bt_stride = bt.data_ptr(), bt.stride(0)
    a.page_size = page_size
    hl = hist_len.to(torch.int32).contiguous()
    keep.append(hl)
    a.hist_len = hl.data_ptr()
    if hist_total is not None:
        ht = hist_total.to(torch.int32).contiguous()
        keep.append(ht)
        a.hist_total = ht.data_ptr()
    a.min_history = min_history
    if recent_k is not None and recent_len is not None:
        if recent_k.stride(-1) != 1 or recent_v.stride(-1) != 1 or recent_k.stride() != recent_v.stride():
            recent_k, recent_v = recent_k.contiguous(), recent_v.contiguous()
        rl = recent_len.to(torch.int32).contiguous()
        keep += [recent_k, recent_v, rl]
        a.recent_k, a.recent_v = recent_k.data_ptr(), recent_v.data_ptr()
        a.recent_dtype = dtype_code(recent_k.dtype)
        a.r_stride_b, a.r_stride_t, a.r_stride_h = recent_k.stride(0), recent_k.stride(1), recent_k.stride(2)
        a.recent_len = rl.data_ptr()
    if out is not None:
        a.out, a.o_stride_b, a.o_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    if partial_out is not None:
        a.partial_out = partial_out.data_ptr()
    if entry != "smaq_decode_noalloc" and not query_path:
        need = decode_workspace_bytes(B, Hq, n_kv_heads, D, num_ctas)
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty((max(need, 256),), dtype=torch.uint8, device=q.device)
        keep.append(workspace)
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    a.num_ctas = num_ctas
    a.layout = layout
    a.overlap_prior = 1 if overlap_prior else 0
    if centroids_f16 is not None:
        c16 = centroids_f16.to(torch.float16).contiguous()
        keep.append(c16)
        a.centroids_f16 = c16.data_ptr()
    if query_path:
        if out is None and partial_out is None:
            a.out = 1  # any non-null output: only the kernel choice is asked for
        st = lib.smaq_decode_kernel_path(a)
        if st < 0:
            _lib.check(-st, "smaq_decode_kernel_path")
        return st
    if entry == "smaq_decode_noalloc":
        # fixed scratch inside the library: no workspace is passed (see include/smaq_b200.h)
        a.workspace, a.workspace_bytes = None, 0
        _lib.check(lib.smaq_decode_noalloc(a, _stream()), "smaq_decode_noalloc")
        return out
    _lib.check(lib.smaq_decode(a, _stream()), "smaq_decode")
    return out


_EMPTY_STORES: dict = {}


def _empty_store(device: torch.device, n_kv_heads: int, head_dim: int, dtype: torch.dtype) -> dict:
    """One 16-row page of 4-bit scalar-key store rows (decode layout) that no decode reads: the
    history streams of a window-only decode must still be valid pointers."""
    key = (device, n_kv_heads, head_dim, dtype)
    st = _EMPTY_STORES.get(key)
    if st is None:
        H, D = n_kv_heads, head_dim
        st = dict(codes=torch.zeros((1, H, 16, packed_dim(D, 4)), dtype=torch.uint8, device=device),
                  norms=torch.zeros((1, H, 16), dtype=dtype, device=device),
                  vdata=torch.zeros((1, H, 16, D // 4), dtype=torch.uint8, device=device),
                  vsz=torch.zeros((1, H, 16, max(1, D // 32)), dtype=dtype, device=device),
                  E_inv=torch.eye(D, dtype=torch.float32, device=device),
                  centroids=torch.zeros(16, dtype=torch.float32, device=device))
        _EMPTY_STORES[key] = st
    return st


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None) -> torch.Tensor:
    """Causal attention of a chunk over itself: ``q [n, Hq, D]``, ``k / v [n, Hkv, D]`` ->
    ``[n, Hq, D]`` in the query dtype; query head ``h`` reads KV head ``h // (Hq / Hkv)``.

    Runs as one ``smaq_decode`` over ``n`` window-only rows: row ``i`` is query token ``i`` with
    an exact window of the chunk's first ``i + 1`` tokens.  The window is the chunk itself for
    every row (batch stride 0), so K and V are neither expanded per query head nor copied per
    row; the rows of one KV head are re-read from L2 (``n^2 / 2`` row reads per head).  bf16 /
    fp16 inputs with head_dim 128 and at most 8 query heads per KV head take the tensor-core
    window of the fused scalar-key kernel while ``2 n Hkv <= 2048``, other shapes the general
    kernel."""
    _cuda(q, k, v)
    n, Hq, D = q.shape
    Hkv = k.shape[1]
    if n == 0:
        return torch.empty_like(q)
    k = k if k.stride(-1) == 1 and k.is_contiguous() else k.contiguous()
    v = v if v.is_contiguous() else v.contiguous()
    if v.dtype != k.dtype:
        v = v.to(k.dtype)
    st = _empty_store(q.device, Hkv, D, k.dtype if k.dtype != torch.float32 else torch.bfloat16)
    rows = torch.arange(1, n + 1, dtype=torch.int32, device=q.device)
    zero = torch.zeros(n, dtype=torch.int32, device=q.device)
    return decode(q, n_kv_heads=Hkv, key_format=SMAQ_KEYS_SCALAR, key_bits=4, E_inv=st["E_inv"],
                  centroids=st["centroids"], key_norms=st["norms"], key_codes=st["codes"], v_data=st["vdata"],
                  v_scales=st["vsz"], v_zeros=st["vsz"], hist_len=zero, page_size=16,
                  block_table=torch.zeros((n, 1), dtype=torch.int32, device=q.device),
                  recent_k=k.unsqueeze(0).expand(n, n, Hkv, D), recent_v=v.unsqueeze(0).expand(n, n, Hkv, D),
                  recent_len=rows, scale=scale, layout=SMAQ_LAYOUT_DECODE)


def merge_partials(partials: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
    """``[R, B, Hq, 2D+2]`` fp32 partials -> ``[B, Hq, D]`` output."""
    _cuda(partials)
    lib = _lib.load()
    R, B, Hq, W = partials.shape
    D = (W - 2) // 2
    p = partials.contiguous()
    out = torch.empty((B, Hq, D), dtype=out_dtype, device=partials.device)
    _lib.check(lib.smaq_merge_partials(p.data_ptr(), R, B, Hq, D, out.data_ptr(), dtype_code(out_dtype),
                                       out.stride(0), out.stride(1), _stream()), "smaq_merge_partials")
    return out


# --------------------------------------------------------------------- failure detection
def decode_status(batch: int, n_kv_heads: int, workspace: Optional[torch.Tensor] = None) -> None:
    """Raise if a bounded device wait of the last ``decode`` that used ``workspace`` (``None``:
    the no-allocation scratch) ran out.  Synchronises the current stream."""
    lib = _lib.load()
    _lib.check(lib.smaq_decode_status(None if workspace is None else workspace.data_ptr(), batch, n_kv_heads,
                                      _stream()), "smaq_decode_status")


def append_status() -> None:
    """Raise if a bounded device wait of the key kernel ran out since the last check (clears it)."""
    _lib.check(_lib.load().smaq_append_status(_stream()), "smaq_append_status")


def selftest_wait_timeout(spin_limit: int = 1 << 12) -> int:
    """Run a kernel whose mbarrier wait can never complete with a ``spin_limit`` poll bound;
    returns the library status (``5`` = SMAQ_ERR_DEVICE when the timeout path works)."""
    return int(_lib.load().smaq_selftest_wait_timeout(spin_limit, _stream()))


# --------------------------------------------------------------------- decode-layout byte order
# (SMAQ_LAYOUT_DECODE, include/smaq_b200.h): same bits as the reference, permuted inside rows.
_VPERM = [4 * (k % 8) + k // 8 for k in range(32)]          # reference byte k lives at _VPERM[k]


def values_to_reference(data: torch.Tensor) -> torch.Tensor:
    """Decode-layout 2-bit value rows ``(..., 32)`` -> reference byte order."""
    return data[..., _VPERM]


def bvq_to_reference(idx: torch.Tensor) -> torch.Tensor:
    """Decode-layout block-VQ rows ``(..., 16)`` -> reference block order."""
    b = torch.arange(16, device=idx.device)
    pos = 2 * (4 * (b // 8) + b % 4) + (b // 4) % 2
    return idx[..., pos]


_SPERM = [16 * (k % 4) + k // 4 for k in range(64)]         # 3/4-bit scalar code byte k at _SPERM[k]


def scalar_codes_to_reference(codes: torch.Tensor) -> torch.Tensor:
    """Decode-layout 3/4-bit scalar key code rows ``(..., 64)`` -> reference byte order."""
    return codes[..., _SPERM]


def fp16_codebook(decoded_centroids: torch.Tensor) -> Optional[torch.Tensor]:
    """fp16 copy of a decoded codebook if it is exactly fp16-valued (enables the tensor-core
    decode kernel), else None."""
    c16 = decoded_centroids.to(torch.float16)
    return c16 if torch.equal(c16.to(decoded_centroids.dtype), decoded_centroids) else None
