"""ctypes binding of libxq_b200.so (include/xq_b200.h).

The library is the product: there is no CPU or PyTorch fallback.  Loading fails
loudly when the shared object is missing or was built for another ABI.
"""
from __future__ import annotations

import ctypes as C
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libxq_b200.so")

XQ_OK, XQ_ERR_INVALID, XQ_ERR_UNSUPPORTED, XQ_ERR_CUDA, XQ_ERR_WORKSPACE = range(5)
F32, F16, Q4_0, Q8_0 = 0, 1, 2, 8
I32, I64 = 26, 27

# Every symbol include/xq_b200.h declares (checked by the CPU test suite).
EXPORTS = (
    "xq_flash_attn_ext_workspace", "xq_flash_attn_ext", "xq_fa_partials", "xq_lse_merge",
    "xq_lse_merge_records",
    "xq_attend_range_workspace", "xq_attend_range", "xq_split_k", "xq_gated_delta_net",
    "xq_gated_delta_net_workspace", "xq_gated_delta_net_ws",
    "xq_attend_range_kvarn4_workspace", "xq_attend_range_kvarn4",
    "xq_dequantize_rows", "xq_quantize_rows", "xq_version", "xq_last_error",
    "xq_flash_attn_ext_noalloc", "xq_set_rows", "xq_gated_delta_net_heads",
    "xq_shard_exchange_bytes", "xq_shard_exchange_alloc", "xq_shard_exchange_free",
    "xq_shard_exchange_error",
    "xq_ipc_export", "xq_ipc_open", "xq_ipc_close", "xq_fa_shard_workspace", "xq_fa_shard_push",
    "xq_fa_shard_finish", "xq_flash_attn_ext_plan",
)
SHARD_MAX_RANKS = 16


class XqError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"xq error {code}: {msg}")
        self.code = code


class Tensor(C.Structure):
    _fields_ = [("type", C.c_int32), ("reserved", C.c_int32), ("data", C.c_void_p),
                ("ne", C.c_int64 * 4), ("nb", C.c_uint64 * 4)]


class Kvarn4Desc(C.Structure):
    _fields_ = [("origin", C.c_int32), ("capacity", C.c_int32), ("precision_tail", C.c_int32),
                ("n_head_kv", C.c_int32)]


class IpcHandle(C.Structure):
    _fields_ = [("bytes", C.c_ubyte * 64)]


class ShardPlan(C.Structure):
    _fields_ = [("rows_per_split", C.c_int64), ("splits_per_group", C.c_int64),
                ("n_groups", C.c_int64), ("rank", C.c_int32), ("world", C.c_int32),
                ("step", C.c_uint32), ("reserved", C.c_int32),
                ("exchange", C.c_void_p * 16)]


class FaParams(C.Structure):
    _fields_ = [("q", Tensor), ("k", Tensor), ("v", Tensor), ("mask", Tensor),
                ("sinks", C.c_void_p), ("dst", C.c_void_p), ("scale", C.c_float),
                ("max_bias", C.c_float), ("softcap", C.c_float), ("n_splits", C.c_int32)]


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python xllama-qwen35-xbox_b200/build.py` "
            "(there is no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    vp, sz, i32, u32, i64, u64 = C.c_void_p, C.c_size_t, C.c_int32, C.c_uint32, C.c_int64, C.c_uint64
    P = C.POINTER
    sig = {
        "xq_flash_attn_ext_workspace": (sz, [P(FaParams)]),
        "xq_flash_attn_ext_plan": (C.c_int, [P(FaParams), P(i32), P(i64), P(i64)]),
        "xq_flash_attn_ext": (C.c_int, [P(FaParams), vp, sz, vp]),
        "xq_fa_partials": (C.c_int, [P(FaParams), i64, i64, i64, vp, vp]),
        "xq_lse_merge": (C.c_int, [vp, i64, i64, i64, vp, vp, vp]),
        "xq_lse_merge_records": (C.c_int, [vp, i64, i64, i64, i64, vp, vp]),
        "xq_attend_range_workspace": (sz, [i32, u32, u32, u32, u32, u32, u32]),
        "xq_attend_range": (C.c_int, [i32, vp, vp, u32, u32, u32, u32, u32, u32, vp, vp, C.c_float,
                                      u32, vp, vp, vp, sz, vp]),
        "xq_split_k": (u32, [u32, u32]),
        "xq_gated_delta_net": (C.c_int, [P(Tensor)] * 6 + [vp, i32, vp]),
        "xq_gated_delta_net_workspace": (sz, [P(Tensor), i32]),
        "xq_attend_range_kvarn4_workspace": (sz, [P(Kvarn4Desc), u32, u32, u32]),
        "xq_attend_range_kvarn4": (C.c_int, [P(Kvarn4Desc), vp, vp, u32, u32, u32, vp, vp,
                                             C.c_float, vp, vp, vp, sz, vp]),
        "xq_gated_delta_net_ws": (C.c_int, [P(Tensor)] * 6 + [vp, i32, vp, sz, vp]),
        "xq_gated_delta_net_heads": (C.c_int, [P(Tensor)] * 6 + [vp, i32, i64, i64, vp, sz, vp]),
        "xq_dequantize_rows": (C.c_int, [i32, vp, u64, vp, u64, i64, i64, vp]),
        "xq_quantize_rows": (C.c_int, [i32, vp, u64, vp, u64, i64, i64, vp]),
        "xq_flash_attn_ext_noalloc": (C.c_int, [P(FaParams), vp]),
        "xq_set_rows": (C.c_int, [P(Tensor), P(Tensor), P(Tensor), vp]),
        "xq_shard_exchange_bytes": (sz, [i64, i64, i64]),
        "xq_shard_exchange_alloc": (C.c_int, [sz, P(vp)]),
        "xq_shard_exchange_free": (C.c_int, [vp]),
        "xq_shard_exchange_error": (C.c_int, [vp, i64, i64, i64, vp, P(i32)]),
        "xq_ipc_export": (C.c_int, [vp, P(IpcHandle)]),
        "xq_ipc_open": (C.c_int, [P(IpcHandle), P(vp)]),
        "xq_ipc_close": (C.c_int, [vp]),
        "xq_fa_shard_workspace": (sz, [P(FaParams), P(ShardPlan)]),
        "xq_fa_shard_push": (C.c_int, [P(FaParams), P(ShardPlan), vp, sz, vp]),
        "xq_fa_shard_finish": (C.c_int, [P(ShardPlan), i64, i64, vp, i32, vp, vp, vp]),
        "xq_version": (C.c_char_p, []),
        "xq_last_error": (C.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype, fn.argtypes = res, args
    _lib = L
    return L


def check(rc: int):
    if rc != XQ_OK:
        raise XqError(rc, lib().xq_last_error().decode(errors="replace"))
