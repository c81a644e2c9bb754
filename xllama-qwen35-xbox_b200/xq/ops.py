"""Op-level wrappers: torch tensors in, one C-ABI call each, torch tensors out.

Layouts follow ggml: a torch tensor's shape is ggml's ne reversed and its byte
strides are nb reversed, so any strided view (e.g. a permuted KV-cache view) is
passed through unchanged.  Quantized / F16 KV caches travel as raw uint8
tensors whose last dim holds the bytes of one row of D elements
(rows of D/32 blocks: Q8_0 = 34 bytes/block, Q4_0 = 18 bytes/block).
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import F16, F32, I32, I64, FaParams, Q4_0, Q8_0, Tensor, check, lib

_BLOCK_BYTES = {F16: 2, Q8_0: 34, Q4_0: 18, F32: 4}
_BLOCK_ELEMS = {F16: 1, Q8_0: 32, Q4_0: 32, F32: 1}
_ws_cache: dict = {}


def row_bytes(ggml_type: int, n: int) -> int:
    return n // _BLOCK_ELEMS[ggml_type] * _BLOCK_BYTES[ggml_type]


def _stream(stream):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _dense(t: torch.Tensor) -> Tensor:
    """float32 / float16 torch tensor (<= 4 dims) -> ggml view."""
    assert t.is_cuda or t.is_pinned(), "device or pinned host tensor expected"
    ty = {torch.float32: F32, torch.float16: F16}[t.dtype]
    shape = [1] * (4 - t.dim()) + list(t.shape)
    strides = [0] * (4 - t.dim()) + list(t.stride())
    es = t.element_size()
    x = Tensor()
    x.type, x.data = ty, t.data_ptr()
    for i in range(4):
        x.ne[i] = shape[3 - i]
        x.nb[i] = strides[3 - i] * es
    # size-1 dims: keep ggml's dense convention so broadcasting code is happy
    for i in range(1, 4):
        if x.ne[i] == 1 and x.nb[i] == 0:
            x.nb[i] = x.nb[i - 1] * x.ne[i - 1]
    return x


def _kv(raw: torch.Tensor, ggml_type: int, D: int) -> Tensor:
    """uint8 (n_seq, n_kv, n_head_kv, row_bytes) cache view -> ggml [D, n_kv, n_head_kv, n_seq]."""
    assert raw.is_cuda and raw.dtype == torch.uint8 and raw.dim() == 4
    n_seq, n_kv, n_hkv, rb = raw.shape
    if rb != row_bytes(ggml_type, D) or raw.stride(3) != 1:
        raise ValueError("KV rows must be contiguous rows of D elements")
    x = Tensor()
    x.type, x.data = ggml_type, raw.data_ptr()
    x.ne[0], x.ne[1], x.ne[2], x.ne[3] = D, n_kv, n_hkv, n_seq
    x.nb[0] = _BLOCK_BYTES[ggml_type]
    x.nb[1], x.nb[2], x.nb[3] = raw.stride(1), raw.stride(2), raw.stride(0)
    return x


def _workspace(nbytes: int, device) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    if device.type != "cuda":  # host (pinned) inputs: the workspace is on the GPU
        device = torch.device("cuda", torch.cuda.current_device())
    key = (device.index if device.index is not None else torch.cuda.current_device())
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf


def _fa_params(q, k, v, k_type, v_type, mask, sinks, dst, scale, max_bias, softcap, n_splits):
    p = FaParams()
    D = q.shape[-1]
    p.q = _dense(q)
    p.k = _kv(k, k_type, D)
    p.v = _kv(v, v_type, D)
    if mask is not None:
        assert mask.dtype == torch.float16
        p.mask = _dense(mask)
    p.sinks = sinks.data_ptr() if sinks is not None else None
    p.dst = dst.data_ptr()
    p.scale, p.max_bias, p.softcap = scale, max_bias, softcap
    p.n_splits = n_splits
    return p


def flash_attn_ext(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_type: int,
                   v_type: int | None = None, mask: torch.Tensor | None = None,
                   sinks: torch.Tensor | None = None, scale: float = 1.0, max_bias: float = 0.0,
                   softcap: float = 0.0, n_splits: int = 0, out: torch.Tensor | None = None,
                   stream=None) -> torch.Tensor:
    """GGML_OP_FLASH_ATTN_EXT.  q float32 (n_seq, n_head, n_q, D); k/v raw
    uint8 caches (n_seq_kv, n_kv, n_head_kv, row_bytes); mask float16
    (m3, m2, >=n_q, n_kv) or None.  Returns float32 (n_seq, n_q, n_head, D).
    q and `out` may be pinned host tensors: q is then copied to the GPU by a
    kernel of the library and the result written straight into `out`."""
    v_type = k_type if v_type is None else v_type
    n_seq, n_head, n_q, D = q.shape
    dst = out if out is not None else torch.empty((n_seq, n_q, n_head, D), dtype=torch.float32,
                                                  device=q.device, pin_memory=not q.is_cuda)
    p = _fa_params(q, k, v, k_type, v_type, mask, sinks, dst, scale, max_bias, softcap, n_splits)
    L = lib()
    nbytes = L.xq_flash_attn_ext_workspace(C.byref(p))
    ws = _workspace(nbytes, q.device)
    check(L.xq_flash_attn_ext(C.byref(p), ws.data_ptr() if ws is not None else None,
                              ws.numel() if ws is not None else 0, _stream(stream)))
    return dst


def flash_attn_ext_plan(q, k, v, k_type, v_type=None, mask=None, n_splits=0):
    """(kernel, n_splits, rows_per_split) xq_flash_attn_ext plans for these
    tensors: kernel 0 CUDA-core decode, 1 warp-MMA decode, 2 tensor-core
    prefill (n_splits = rows_per_split = 0)."""
    v_type = k_type if v_type is None else v_type
    dst = torch.empty(1, device=q.device if q.is_cuda else "cuda")
    p = _fa_params(q, k, v, k_type, v_type, mask, None, dst, 1.0, 0.0, 0.0, n_splits)
    kern, ns, rows = C.c_int32(), C.c_int64(), C.c_int64()
    check(lib().xq_flash_attn_ext_plan(C.byref(p), C.byref(kern), C.byref(ns), C.byref(rows)))
    return kern.value, ns.value, rows.value


def flash_attn_ext_workspace(q, k, v, k_type, v_type=None, mask=None, n_splits=0) -> int:
    v_type = k_type if v_type is None else v_type
    dst = torch.empty(1, device=q.device)
    p = _fa_params(q, k, v, k_type, v_type, mask, None, dst, 1.0, 0.0, 0.0, n_splits)
    return int(lib().xq_flash_attn_ext_workspace(C.byref(p)))


def fa_partials(q, k, v, k_type, rows_per_split: int, split_begin: int, split_end: int,
                mask=None, scale=1.0, max_bias=0.0, softcap=0.0, out=None, stream=None):
    """Partial records (acc[D], max, denom) of global KV splits
    [split_begin, split_end): float32 (split_end - split_begin, n_rows, D + 2)."""
    n_seq, n_head, n_q, D = q.shape
    n_rows = n_seq * n_q * n_head
    part = out if out is not None else torch.empty(
        (split_end - split_begin, n_rows, D + 2), dtype=torch.float32, device=q.device)
    dummy = torch.empty(1, device=q.device)
    p = _fa_params(q, k, v, k_type, k_type, mask, None, dummy, scale, max_bias, softcap, 0)
    check(lib().xq_fa_partials(C.byref(p), rows_per_split, split_begin, split_end,
                               part.data_ptr(), _stream(stream)))
    return part


def lse_merge(partials: torch.Tensor, out=None, lse=None, want_lse=True, stream=None):
    """partials float32 (n_splits, n_rows, D + 2) -> (out (n_rows, D), lse (n_rows,))."""
    n_splits, n_rows, d2 = partials.shape
    assert partials.is_contiguous()
    D = d2 - 2
    o = out if out is not None else torch.empty((n_rows, D), dtype=torch.float32,
                                                device=partials.device)
    lz = lse if lse is not None else (torch.empty((n_rows,), dtype=torch.float32,
                                                  device=partials.device) if want_lse else None)
    check(lib().xq_lse_merge(partials.data_ptr(), n_splits, n_rows, D, o.data_ptr(),
                             lz.data_ptr() if lz is not None else None, _stream(stream)))
    return o, lz


def lse_merge_records(partials: torch.Tensor, splits_per_group: int, out=None, stream=None):
    """partials float32 (n_groups * splits_per_group, n_rows, D + 2) -> one
    record per (group, row): float32 (n_groups, n_rows, D + 2) = (O, lse, 1)."""
    n_splits, n_rows, d2 = partials.shape
    assert partials.is_contiguous() and n_splits % splits_per_group == 0
    n_groups = n_splits // splits_per_group
    rec = out if out is not None else torch.empty((n_groups, n_rows, d2), dtype=torch.float32,
                                                  device=partials.device)
    check(lib().xq_lse_merge_records(partials.data_ptr(), n_groups, splits_per_group, n_rows,
                                     d2 - 2, rec.data_ptr(), _stream(stream)))
    return rec


def _rows_view(t: torch.Tensor, ggml_type: int, elems: int) -> Tensor:
    """(n_seq, n_rows, n_head_kv, last) tensor -> ggml [elems, n_rows, n_head_kv, n_seq]
    (the KV-cache view convention of _kv), rows contiguous."""
    assert t.is_cuda and t.dim() == 4 and t.stride(3) == 1
    es = t.element_size()
    x = Tensor()
    x.type, x.data = ggml_type, t.data_ptr()
    x.ne[0], x.ne[1], x.ne[2], x.ne[3] = elems, t.shape[1], t.shape[2], t.shape[0]
    x.nb[0] = _BLOCK_BYTES[ggml_type] if ggml_type in _BLOCK_BYTES else es
    x.nb[1], x.nb[2], x.nb[3] = t.stride(1) * es, t.stride(2) * es, t.stride(0) * es
    return x


def set_rows(cache: torch.Tensor, src: torch.Tensor, idx: torch.Tensor, ggml_type: int,
             stream=None) -> torch.Tensor:
    """GGML_OP_SET_ROWS (the KV-cache write), in place.  cache: uint8 (n_seq,
    n_rows, n_head_kv, row_bytes) for F16/Q8_0/Q4_0 or float32 (n_seq, n_rows,
    n_head_kv, D) for F32; src float32 (n_seq, n_tok, n_head_kv, D); idx int32
    or int64 (n_tok,) or (i2, i1, n_tok) with n_head_kv % i1 == 0 and
    n_seq % i2 == 0.  Row (s, t, h) of src lands in cache row
    idx[s % i2, h % i1, t] of (s, h)."""
    D = src.shape[-1]
    dst = _rows_view(cache, ggml_type, D)
    s = _rows_view(src, F32, D)
    ix = idx.reshape((1, 1) + tuple(idx.shape)) if idx.dim() == 1 else idx
    assert ix.dim() == 3 and ix.is_cuda and ix.stride(2) == 1
    it = Tensor()
    it.type = {torch.int32: I32, torch.int64: I64}[ix.dtype]
    it.data = ix.data_ptr()
    es = ix.element_size()
    it.ne[0], it.ne[1], it.ne[2], it.ne[3] = ix.shape[2], ix.shape[1], ix.shape[0], 1
    it.nb[0], it.nb[1], it.nb[2] = es, ix.stride(1) * es, ix.stride(0) * es
    it.nb[3] = it.nb[2] * ix.shape[0]
    check(lib().xq_set_rows(C.byref(s), C.byref(it), C.byref(dst), _stream(stream)))
    return cache


def split_k(active: int, mode: int) -> int:
    return int(lib().xq_split_k(active, mode))


def attend_range_workspace(storage, n_tokens, active, n_head, n_head_kv, head_dim, mode) -> int:
    return int(lib().xq_attend_range_workspace(storage, n_tokens, active, n_head, n_head_kv,
                                               head_dim, mode))


def attend_range(storage: int, k: torch.Tensor, v: torch.Tensor, q: torch.Tensor,
                 positions: torch.Tensor, n_head_kv: int, origin: int, active: int,
                 kq_scale: float, split_mode: int = 0, stream=None):
    """RKVA RANGE_ATTN.  k/v uint8 [capacity][n_head_kv][row_bytes] (contiguous);
    q float32 (n_tokens, n_head, D); positions int32 (n_tokens,).  Returns
    (out (n_tokens, n_head, D), lse (n_tokens, n_head))."""
    n_tokens, n_head, D = q.shape
    assert q.is_contiguous() and positions.dtype == torch.int32 and positions.is_cuda
    out = torch.empty((n_tokens, n_head, D), dtype=torch.float32, device=q.device)
    lse = torch.empty((n_tokens, n_head), dtype=torch.float32, device=q.device)
    nbytes = attend_range_workspace(storage, n_tokens, active, n_head, n_head_kv, D, split_mode)
    ws = _workspace(nbytes, q.device)
    check(lib().xq_attend_range(storage, k.data_ptr() if active else None,
                                v.data_ptr() if active else None, n_head, n_head_kv, D, origin,
                                active, n_tokens, positions.data_ptr(), q.data_ptr(), kq_scale,
                                split_mode, out.data_ptr(), lse.data_ptr(),
                                ws.data_ptr() if ws is not None else None,
                                ws.numel() if ws is not None else 0, _stream(stream)))
    return out, lse


def attend_range_kvarn4(k_plane: torch.Tensor, v_plane: torch.Tensor, q: torch.Tensor,
                        positions: torch.Tensor, n_head_kv: int, origin: int, capacity: int,
                        precision_tail: int, active: int, kq_scale: float, stream=None,
                        out=None, lse=None):
    """RKVA range attention over native KVarN4 planes (uint8, 16-byte aligned,
    layout in include/xq_b200.h); q float32 (n_tokens, n_head, 256) on the
    device or in pinned host memory, positions int32 (n_tokens,) on the
    device; out / lse, when given, may be pinned host tensors too.  Returns
    (out, lse)."""
    from ._lib import Kvarn4Desc
    n_tokens, n_head, D = q.shape
    assert D == 256 and q.is_contiguous() and positions.dtype == torch.int32
    dev = k_plane.device
    desc = Kvarn4Desc(origin, capacity, precision_tail, n_head_kv)
    if out is None:
        out = torch.empty((n_tokens, n_head, D), dtype=torch.float32, device=dev)
    if lse is None:
        lse = torch.empty((n_tokens, n_head), dtype=torch.float32, device=dev)
    nbytes = lib().xq_attend_range_kvarn4_workspace(C.byref(desc), n_head, active, n_tokens)
    ws = _workspace(nbytes, dev)
    check(lib().xq_attend_range_kvarn4(C.byref(desc), k_plane.data_ptr(), v_plane.data_ptr(),
                                       n_head, active, n_tokens, positions.data_ptr(),
                                       q.data_ptr(), kq_scale, out.data_ptr(), lse.data_ptr(),
                                       ws.data_ptr() if ws is not None else None,
                                       ws.numel() if ws is not None else 0, _stream(stream)))
    return out, lse


def gated_delta_net(q, k, v, g, beta, state, slots: int = 1, out=None, stream=None,
                    chunked: bool = True, head_begin: int | None = None,
                    n_head_total: int | None = None):
    """GGML_OP_GATED_DELTA_NET.  q, k (n_seq_qk, T, H_k, S); v (n_seq, T, H, S);
    g, beta (n_seq, T, H, 1); state (n_seq, H, S, S).  Returns
    (dst_flat, y (n_seq, T, H, S), snapshots (K, n_seq, H, S, S)).
    chunked: long sequences take the tensor-core chunked form
    (xq_gated_delta_net_ws, TF32 products); False keeps the per-token FP32
    recurrence (xq_gated_delta_net) at every length.
    head_begin / n_head_total: v, g, beta, state hold value heads
    [head_begin, head_begin + H) of an op with n_head_total value heads (the
    op sharded by value head, xq_gated_delta_net_heads); q, k stay whole."""
    n_seq, T, H, S = v.shape
    n_y = S * H * T * n_seq
    n_snap = slots * S * S * H * n_seq
    dst = out if out is not None else torch.empty(n_y + n_snap, dtype=torch.float32,
                                                  device=v.device)
    ts = [_dense(t) for t in (q, k, v, g, beta, state)]
    refs = [C.byref(t) for t in ts]
    if head_begin is not None:
        nbytes = lib().xq_gated_delta_net_workspace(refs[2], slots)
        ws = _workspace(nbytes, v.device)
        check(lib().xq_gated_delta_net_heads(*refs, dst.data_ptr(), slots, head_begin,
                                             n_head_total if n_head_total is not None else H,
                                             ws.data_ptr() if ws is not None else None,
                                             ws.numel() if ws is not None else 0,
                                             _stream(stream)))
    elif chunked:
        nbytes = lib().xq_gated_delta_net_workspace(refs[2], slots)
        ws = _workspace(nbytes, v.device)
        check(lib().xq_gated_delta_net_ws(*refs, dst.data_ptr(), slots,
                                          ws.data_ptr() if ws is not None else None,
                                          ws.numel() if ws is not None else 0, _stream(stream)))
    else:
        check(lib().xq_gated_delta_net(*refs, dst.data_ptr(), slots, _stream(stream)))
    return dst, dst[:n_y].view(n_seq, T, H, S), dst[n_y:].view(slots, n_seq, H, S, S)


def dequantize_rows(ggml_type: int, raw: torch.Tensor, n_per_row: int, stream=None):
    rows = raw.reshape(-1, raw.shape[-1])
    out = torch.empty((rows.shape[0], n_per_row), dtype=torch.float32, device=raw.device)
    check(lib().xq_dequantize_rows(ggml_type, rows.data_ptr(), rows.stride(0), out.data_ptr(),
                                   out.stride(0) * 4, rows.shape[0], n_per_row, _stream(stream)))
    return out.reshape(raw.shape[:-1] + (n_per_row,))


def quantize_rows(ggml_type: int, x: torch.Tensor, stream=None):
    n = x.shape[-1]
    rows = x.reshape(-1, n).contiguous()
    rb = row_bytes(ggml_type, n)
    out = torch.empty((rows.shape[0], rb), dtype=torch.uint8, device=x.device)
    check(lib().xq_quantize_rows(ggml_type, rows.data_ptr(), rows.stride(0) * 4, out.data_ptr(),
                                 rb, rows.shape[0], n, _stream(stream)))
    return out.reshape(x.shape[:-1] + (rb,))
