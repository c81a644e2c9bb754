"""CPU oracle for the attention hot path -- TEST INFRASTRUCTURE ONLY.

ctypes wrapper over oracle/xq_ref.c (a C restatement of the reference's ggml-cpu
FLASH_ATTN_EXT / GATED_DELTA_NET arithmetic, RKVA range attention and LSE
merge; xq_ref.h lists the reference file:line each part follows) plus numpy
helpers.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
--impl reference legs import this package, and only as the checker or the CPU
baseline.  The product (the CUDA library behind include/xq_b200.h) never loads
it and has no CPU fallback.

Array conventions: numpy shapes are ggml's ne reversed (C order), and byte
strides map nb[i] = array.strides[3 - i], so any strided numpy view is a valid
ggml tensor view.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "libxq_ref.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libxq_gdn_ref.so")

F32, F16, Q4_0, Q8_0 = 0, 1, 2, 8
TYPE_NAMES = {F32: "f32", F16: "f16", Q4_0: "q4_0", Q8_0: "q8_0"}
FA_NATIVE, FA_SCALAR, FA_POLICY4 = 0, 1, 4


class Tensor(C.Structure):
    _fields_ = [("type", C.c_int), ("data", C.c_void_p), ("ne", C.c_int64 * 4),
                ("nb", C.c_size_t * 4)]


class FaArgs(C.Structure):
    _fields_ = [("q", Tensor), ("k", Tensor), ("v", Tensor), ("mask", Tensor),
                ("sinks", C.c_void_p), ("dst", C.c_void_p), ("scale", C.c_float),
                ("max_bias", C.c_float), ("softcap", C.c_float), ("policy", C.c_int),
                ("no_split_kv", C.c_int), ("nth", C.c_int), ("n_workers", C.c_int)]


class RangeArgs(C.Structure):
    _fields_ = [("storage", C.c_int), ("k", C.c_void_p), ("v", C.c_void_p),
                ("q", C.c_void_p), ("positions", C.c_void_p), ("n_tokens", C.c_uint32),
                ("active", C.c_uint32), ("origin", C.c_uint32), ("n_head", C.c_uint32),
                ("n_head_kv", C.c_uint32), ("head_dim", C.c_uint32), ("split_k", C.c_uint32),
                ("kq_scale", C.c_float), ("out", C.c_void_p), ("lse", C.c_void_p)]


class GdnArgs(C.Structure):
    _fields_ = [("q", Tensor), ("k", Tensor), ("v", Tensor), ("g", Tensor), ("beta", Tensor),
                ("state", Tensor), ("dst", C.c_void_p), ("slots", C.c_int),
                ("n_workers", C.c_int), ("lanes8", C.c_int), ("head_begin", C.c_int64),
                ("n_head_total", C.c_int64)]


_lib = None


def build() -> str:
    """Compile oracle/build/libxq_ref.so (gcc) if missing or stale."""
    src = [os.path.join(HERE, f) for f in ("xq_ref.c", "xq_ref.h")]
    if (not os.path.exists(LIB_PATH)
            or max(os.path.getmtime(s) for s in src) > os.path.getmtime(LIB_PATH)):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB_PATH)
        L.xqr_fp32_to_fp16.restype = C.c_uint16
        L.xqr_fp32_to_fp16.argtypes = [C.c_float]
        L.xqr_fp16_to_fp32.restype = C.c_float
        L.xqr_fp16_to_fp32.argtypes = [C.c_uint16]
        L.xqr_row_size.restype = C.c_size_t
        L.xqr_row_size.argtypes = [C.c_int, C.c_int64]
        for fn in ("xqr_quantize_q8_0", "xqr_quantize_q4_0", "xqr_quantize_q8_0_x86",
                   "xqr_quantize_f16"):
            getattr(L, fn).argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
            getattr(L, fn).restype = None
        L.xqr_dequantize.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int64]
        L.xqr_dequantize.restype = None
        L.xqr_flash_attn_ext.argtypes = [C.POINTER(FaArgs)]
        L.xqr_flash_attn_ext.restype = C.c_int
        L.xqr_flash_attn_f64.argtypes = [C.POINTER(FaArgs), C.c_void_p]
        L.xqr_flash_attn_f64.restype = C.c_int
        L.xqr_range_attn.argtypes = [C.POINTER(RangeArgs)]
        L.xqr_range_attn.restype = C.c_int
        L.xqr_lse_merge.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p,
                                    C.c_void_p]
        L.xqr_lse_merge.restype = None
        L.xqr_split_k.argtypes = [C.c_uint32, C.c_uint32]
        L.xqr_split_k.restype = C.c_uint32
        L.xqr_gated_delta_net.argtypes = [C.POINTER(GdnArgs)]
        L.xqr_gated_delta_net.restype = C.c_int
        L.xqr_std_uniform.argtypes = [C.c_uint32, C.c_float, C.c_float, C.c_int64, C.c_void_p]
        L.xqr_std_uniform.restype = None
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ----------------------------------------------------------------------------
# codecs

def row_size(ggml_type: int, n: int) -> int:
    return int(lib().xqr_row_size(ggml_type, n))


def quantize(ggml_type: int, x: np.ndarray, variant: str = "ref") -> np.ndarray:
    """Quantize float32 rows (last dim multiple of 32) to raw ggml bytes.

    Returns uint8 with the last dim replaced by the row's byte size."""
    x = np.ascontiguousarray(x, np.float32)
    n = x.shape[-1]
    rows = x.size // n
    rb = row_size(ggml_type, n)
    out = np.empty(x.shape[:-1] + (rb,), np.uint8)
    fn = {F16: "xqr_quantize_f16", Q4_0: "xqr_quantize_q4_0",
          Q8_0: "xqr_quantize_q8_0_x86" if variant == "x86" else "xqr_quantize_q8_0"}[ggml_type]
    getattr(lib(), fn)(_ptr(x), _ptr(out), rows * n)
    return out


def dequantize(ggml_type: int, raw: np.ndarray, n: int) -> np.ndarray:
    """Raw rows (last dim = row bytes of n elements) -> float32 (..., n)."""
    raw = np.ascontiguousarray(raw, np.uint8)
    rb = row_size(ggml_type, n)
    rows = raw.size // rb
    out = np.empty(raw.shape[:-1] + (n,), np.float32)
    lib().xqr_dequantize(ggml_type, _ptr(raw), _ptr(out), rows * n)
    return out


def fp16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    return np.array([lib().xqr_fp32_to_fp16(float(v)) for v in x.ravel()], np.uint16).reshape(
        x.shape)


# ----------------------------------------------------------------------------
# ggml tensor views

def kv_tensor(raw: np.ndarray, ggml_type: int, D: int) -> Tensor:
    """K or V cache in llama.cpp / RKVA layout: raw uint8 (n_seq, n_kv,
    n_head_kv, row_bytes) -> ggml view ne = [D, n_kv, n_head_kv, n_seq]."""
    assert raw.ndim == 4 and raw.dtype == np.uint8
    n_seq, n_kv, n_hkv, rb = raw.shape
    assert rb == row_size(ggml_type, D)
    t = Tensor()
    t.type = ggml_type
    t.data = raw.ctypes.data
    t.ne[0], t.ne[1], t.ne[2], t.ne[3] = D, n_kv, n_hkv, n_seq
    s = raw.strides
    t.nb[0] = {F32: 4, F16: 2, Q8_0: 34, Q4_0: 18}[ggml_type]
    t.nb[1], t.nb[2], t.nb[3] = s[1], s[2], s[0]
    return t


def dense_tensor(arr: np.ndarray) -> Tensor:
    """float32 / float16 numpy array (<= 4 dims) -> ggml tensor, nb from strides."""
    assert arr.dtype in (np.float32, np.float16)
    ty = F32 if arr.dtype == np.float32 else F16
    a4 = arr.reshape((1,) * (4 - arr.ndim) + arr.shape) if arr.ndim < 4 else arr
    t = Tensor()
    t.type = ty
    t.data = arr.ctypes.data
    for i in range(4):
        t.ne[i] = a4.shape[3 - i]
        t.nb[i] = a4.strides[3 - i]
    return t


# ----------------------------------------------------------------------------
# FLASH_ATTN_EXT

def flash_attn_ext(q, k_raw, v_raw, k_type, v_type, mask=None, sinks=None, scale=1.0,
                   max_bias=0.0, softcap=0.0, policy=FA_NATIVE, no_split_kv=False, nth=1,
                   n_workers=None, f64=False):
    """ggml-cpu FLASH_ATTN_EXT restated.

    q: float32 (n_seq, n_head, n_q, DK) (any strides);
    k_raw/v_raw: uint8 (n_seq_kv, n_kv, n_head_kv, row_bytes) cache layout;
    mask: float16 (m3, m2, n_q_pad, n_kv) or None.
    Returns dst float32 (n_seq, n_q, n_head, DV) [and lse (n_seq, n_q, n_head)
    when f64]."""
    n_seq, n_head, n_q, DK = q.shape
    DV_raw = v_raw.shape[-1]
    DV = DV_raw // {F32: 4, F16: 2}.get(v_type, 1) if v_type in (F32, F16) else (
        DV_raw // (34 if v_type == Q8_0 else 18) * 32)
    a = FaArgs()
    a.q = dense_tensor(q)
    a.k = kv_tensor(k_raw, k_type, DK)
    a.v = kv_tensor(v_raw, v_type, DV)
    if mask is not None:
        assert mask.dtype == np.float16
        a.mask = dense_tensor(mask)
    else:
        a.mask = Tensor()
    a.sinks = _ptr(sinks) if sinks is not None else None
    dst = np.zeros((n_seq, n_q, n_head, DV), np.float32)
    a.dst = dst.ctypes.data
    a.scale, a.max_bias, a.softcap = scale, max_bias, softcap
    a.policy, a.no_split_kv, a.nth = policy, int(no_split_kv), nth
    a.n_workers = n_workers or os.cpu_count() or 1
    if f64:
        lse = np.zeros((n_seq, n_q, n_head), np.float32)
        rc = lib().xqr_flash_attn_f64(C.byref(a), lse.ctypes.data_as(C.c_void_p))
        if rc:
            raise ValueError(f"xqr_flash_attn_f64 rejected the shapes ({rc})")
        return dst, lse
    rc = lib().xqr_flash_attn_ext(C.byref(a))
    if rc:
        raise ValueError(f"xqr_flash_attn_ext rejected the shapes ({rc})")
    return dst


# ----------------------------------------------------------------------------
# RKVA range attention / merge / policy

def split_k(active: int, mode: int) -> int:
    return int(lib().xqr_split_k(active, mode))


def range_attn(storage, k_raw, v_raw, q, positions, active, origin, n_head, n_head_kv,
               head_dim, kq_scale, split=0):
    q = np.ascontiguousarray(q, np.float32)
    positions = np.ascontiguousarray(positions, np.int32)
    n_tokens = positions.size
    out = np.zeros((n_tokens, n_head, head_dim), np.float32)
    lse = np.zeros((n_tokens, n_head), np.float32)
    k_raw = np.ascontiguousarray(k_raw, np.uint8)
    v_raw = np.ascontiguousarray(v_raw, np.uint8)
    a = RangeArgs(storage, k_raw.ctypes.data, v_raw.ctypes.data, q.ctypes.data,
                  positions.ctypes.data, n_tokens, active, origin, n_head, n_head_kv, head_dim,
                  split, kq_scale, out.ctypes.data, lse.ctypes.data)
    rc = lib().xqr_range_attn(C.byref(a))
    if rc:
        raise ValueError(f"xqr_range_attn rejected the shapes ({rc})")
    return out, lse


def lse_merge(partials: np.ndarray):
    """partials float32 (n_splits, n_rows, D+2) = (acc[D], max, denom)."""
    partials = np.ascontiguousarray(partials, np.float32)
    n_splits, n_rows, d2 = partials.shape
    D = d2 - 2
    out = np.zeros((n_rows, D), np.float32)
    lse = np.zeros((n_rows,), np.float32)
    lib().xqr_lse_merge(_ptr(partials), n_splits, n_rows, D, _ptr(out), _ptr(lse))
    return out, lse


def set_rows(cache: np.ndarray, src: np.ndarray, idx: np.ndarray, ty: int) -> np.ndarray:
    """ggml GGML_OP_SET_ROWS restated (ggml-cpu.c:1957-1959 dispatches it to
    ggml_compute_forward_set_rows, one task): row t of src plane (s, h) is
    converted by the destination type's from_float and stored as row
    idx[s % i2, h % i1, t] of cache plane (s, h).  The converters are this
    oracle's reference quantizers (gguf-pinned).  cache: (n_seq, n_rows,
    n_head_kv, row_bytes) uint8, or float32 (.., D) for F32; src float32
    (n_seq, n_tok, n_head_kv, D); idx (n_tok,) or (i2, i1, n_tok).  Returns
    the updated copy; rows with an index outside [0, n_rows) are skipped."""
    out = cache.copy()
    n_seq, n_tok, n_hkv, _ = src.shape
    ix = idx.reshape(1, 1, -1) if idx.ndim == 1 else idx
    rows = src.astype(np.float32) if ty == F32 else quantize(ty, np.ascontiguousarray(src))
    for s_ in range(n_seq):
        for h in range(n_hkv):
            for t in range(n_tok):
                r = int(ix[s_ % ix.shape[0], h % ix.shape[1], t])
                if 0 <= r < cache.shape[1]:
                    out[s_, r, h] = rows[s_, t, h]
    return out


# ----------------------------------------------------------------------------
# GATED_DELTA_NET

def gated_delta_net(q, k, v, g, beta, state, slots=1, lanes8=False, n_workers=None,
                    head_begin=0, n_head_total=0):
    """q, k: (n_seq_qk, T, H_k, S) ; v: (n_seq, T, H, S) ; g, beta: (n_seq, T, H, 1);
    state: (n_seq, H, S, S) [col][i].  Returns (dst_flat, y, snapshots) with
    y (n_seq, T, H, S) and snapshots (K, n_seq, H, S, S).  head_begin /
    n_head_total: v, g, beta, state hold value heads [head_begin, head_begin +
    H) of an op with n_head_total heads (0: the whole op)."""
    n_seq, T, H, S = v.shape
    a = GdnArgs()
    a.q, a.k, a.v = dense_tensor(q), dense_tensor(k), dense_tensor(v)
    a.g, a.beta, a.state = dense_tensor(g), dense_tensor(beta), dense_tensor(state)
    n_y = S * H * T * n_seq
    n_snap = slots * S * S * H * n_seq
    dst = np.zeros(n_y + n_snap, np.float32)
    a.dst = dst.ctypes.data
    a.slots = slots
    a.n_workers = n_workers or os.cpu_count() or 1
    a.lanes8 = int(lanes8)
    a.head_begin, a.n_head_total = head_begin, n_head_total
    rc = lib().xqr_gated_delta_net(C.byref(a))
    if rc:
        raise ValueError(f"xqr_gated_delta_net rejected the shapes ({rc})")
    return dst, dst[:n_y].reshape(n_seq, T, H, S), dst[n_y:].reshape(slots, n_seq, H, S, S)


def std_uniform(seed: int, lo: float, hi: float, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().xqr_std_uniform(seed, lo, hi, n, _ptr(out))
    return out


def gdn_selftest_inputs(tokens: int, pad: int = 0):
    """Inputs of the reference GDN selftest (src/bridge/ggml_d3d12.cpp:222-258):
    std::mt19937(1701 + j), uniform(-0.05, 0.05), g = -0.3 - |u|, beta = u + 0.5,
    Q/K/V head rows padded by pad / pad+2 / pad+4 floats (1e30 sentinels).
    Returns strided numpy views (q, k, v, g, beta, state) in the layouts
    gated_delta_net() takes, plus the padded backing buffers."""
    shapes = [(128, 16), (128, 16), (128, 32), (1, 32), (1, 32)]
    views, backing = [], []
    for j, (ne0, ne1) in enumerate(shapes):
        row = ne0 + (pad + 2 * j if pad and j < 3 else 0)
        buf = np.full((1, tokens, ne1, row), 1e30, np.float32)
        u = std_uniform(1701 + j, -0.05, 0.05, tokens * ne1 * ne0).reshape(tokens, ne1, ne0)
        if j == 3:
            u = np.float32(-0.3) - np.abs(u)
        if j == 4:
            u = u + np.float32(0.5)
        buf[0, :, :, :ne0] = u
        backing.append(buf)
        views.append(buf[:, :, :, :ne0])
    st = std_uniform(1706, -0.05, 0.05, 32 * 128 * 128).reshape(1, 32, 128, 128)
    backing.append(st)
    views.append(st)
    return views, backing


def ref_gdn_lib():
    """The reference's own GDN host mirror compiled by oracle/build_ref.sh
    (only present where the reference checkout is)."""
    if not os.path.exists(REF_LIB_PATH):
        return None
    L = C.CDLL(REF_LIB_PATH)
    L.xq_gdn_ref_run.argtypes = [C.c_int, C.c_int, C.c_int] + [C.c_void_p] * 7
    L.xq_gdn_ref_run.restype = C.c_int
    L.xq_gdn_ref_input_floats.argtypes = [C.c_int, C.c_int, C.c_int]
    L.xq_gdn_ref_input_floats.restype = C.c_long
    L.xq_std_uniform.argtypes = [C.c_uint, C.c_float, C.c_float, C.c_int, C.c_void_p]
    L.xq_std_uniform.restype = None
    return L
