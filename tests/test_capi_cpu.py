"""C ABI checks that need no GPU: the library loads, exports every function
include/xq_b200.h declares, and its host-only logic (split policy, argument
contracts that fail before any launch) behaves like the reference."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from conftest import REPO, golden

HEADER = os.path.join(REPO, "include", "xq_b200.h")


def _lib():
    import xq._lib as L
    if not os.path.exists(L.LIB_PATH):
        import importlib.util
        spec = importlib.util.spec_from_file_location(
            "xq_build", os.path.join(REPO, "xllama-qwen35-xbox_b200", "build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    return L.lib()


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(xq_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = _lib()
    names = declared_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(L, n), f"{n} declared in xq_b200.h but not exported"
    import xq._lib as XL
    assert sorted(XL.EXPORTS) == names


def test_version_string():
    assert _lib().xq_version().startswith(b"xq_b200")


def test_split_policy_matches_reference():
    L = _lib()
    g = golden("split_policy.npz")
    for a, row in zip(g["active"], g["split_k"]):
        assert [int(L.xq_split_k(int(a), m)) for m in range(4)] == list(row)


def test_contract_errors_before_launch():
    """Bad shapes are refused on the host with a message, before any launch."""
    import xq._lib as XL
    L = _lib()
    p = XL.FaParams()
    p.q.type = XL.F32
    p.q.nb[0] = 4
    p.k.type = p.v.type = XL.F32  # F32 KV: not claimed
    assert L.xq_flash_attn_ext(C.byref(p), None, 0, None) == XL.XQ_ERR_UNSUPPORTED
    assert b"K/V types" in L.xq_last_error()
    assert L.xq_lse_merge(None, 1, 1, 256, None, None, None) == XL.XQ_ERR_INVALID
    t = XL.Tensor()
    assert L.xq_gated_delta_net(*[C.byref(t)] * 6, None, 1, None) == XL.XQ_ERR_INVALID
    assert L.xq_gated_delta_net_ws(*[C.byref(t)] * 6, None, 1, None, 0, None) == \
        XL.XQ_ERR_INVALID
    # SET_ROWS: ggml_set_rows' shape rules and types, checked before any launch
    src, idx, dst = XL.Tensor(), XL.Tensor(), XL.Tensor()
    src.type, src.nb[0], idx.type, dst.type = XL.F32, 4, XL.I64, XL.Q8_0
    for t_, ne in ((src, (256, 5, 2, 1)), (idx, (5, 1, 1, 1)), (dst, (256, 64, 2, 1))):
        t_.data = 0x1000
        for i in range(4):
            t_.ne[i] = ne[i]
    dst.ne[0] = 128  # row lengths differ
    assert L.xq_set_rows(C.byref(src), C.byref(idx), C.byref(dst), None) == XL.XQ_ERR_INVALID
    assert b"set_rows" in L.xq_last_error()
    dst.ne[0] = 256
    idx.type = XL.F32  # float indices
    assert L.xq_set_rows(C.byref(src), C.byref(idx), C.byref(dst), None) == XL.XQ_ERR_UNSUPPORTED
    idx.type, idx.ne[1] = XL.I32, 3  # 2 heads not a multiple of 3
    assert L.xq_set_rows(C.byref(src), C.byref(idx), C.byref(dst), None) == XL.XQ_ERR_INVALID


def test_gdn_chunked_workspace_sizes():
    """Workspace of the chunked GATED_DELTA_NET: [T''; M] (32 KiB) and factors
    (1 KiB) per (chunk, head, sequence), an error word, and the handed-off
    state when the last tokens run per token; none below two chunks."""
    import xq._lib as XL
    L = _lib()
    v = XL.Tensor()
    v.type = XL.F32

    def ws(T, H, n_seq, slots):
        v.ne[0], v.ne[1], v.ne[2], v.ne[3] = 128, H, T, n_seq
        return L.xq_gated_delta_net_workspace(C.byref(v), slots)

    unit = 32768 + 1024
    assert ws(4096, 32, 1, 1) == 64 * 32 * unit + 256
    assert ws(200, 32, 2, 1) == 4 * 32 * 2 * unit + 256          # last chunk padded
    assert ws(300, 32, 1, 5) == 4 * 32 * unit + 256 + 32 * 65536  # 44 tokens per token
    assert ws(64, 32, 1, 1) == 0 and ws(100, 32, 1, 64) == 0
    assert ws(4096, 32, 1, 0) == 0  # slots outside [1, 64]


def test_kvarn4_workspace_and_contract():
    """KVarN4 split plan (no GPU: 148 SMs assumed): body splits of whole
    128-row groups over rows [0, active - tail), about two CTAs per SM counting
    one tail split; argument contracts fail before any launch."""
    import xq._lib as XL
    L = _lib()

    def ws(origin, cap, tail, n_kv, n_head, active, n_tok=1):
        d = XL.Kvarn4Desc(origin, cap, tail, n_kv)
        return L.xq_attend_range_kvarn4_workspace(C.byref(d), n_head, active, n_tok)

    def size(splits, n_tok=1):
        # split partials, then (256-byte aligned) room to stage a host q
        return (splits * n_tok * 24 * 258 * 4 + 255) // 256 * 256 + n_tok * 24 * 256 * 4

    # 255 body groups: 73 splits wanted -> 4 groups each -> 64 body splits + tail
    assert ws(102400, 32768, 128, 4, 24, 32768) == size(65)
    assert ws(102400, 32768, 0, 4, 24, 32768) == size(64)      # no tail split
    assert ws(0, 640, 128, 4, 24, 100) == size(1)              # everything in the tail
    assert ws(0, 640, 128, 4, 24, 0) == size(1)                # empty: one split
    assert ws(0, 640, 0, 4, 24, 520, n_tok=3) == size(5, 3)    # one group per split
    assert ws(0, 640, -1, 4, 24, 520) == 0

    d = XL.Kvarn4Desc(0, 1024, 128, 4)
    fake = C.c_void_p(4096)

    def call(desc, n_head=24, active=1000, kp=fake, ws_bytes=1 << 30):
        return L.xq_attend_range_kvarn4(C.byref(desc), kp, fake, n_head, active, 1, fake, fake,
                                        0.0625, fake, fake, fake, ws_bytes, None)

    assert call(XL.Kvarn4Desc(64, 1024, 128, 4)) == XL.XQ_ERR_INVALID   # origin % 128
    assert call(XL.Kvarn4Desc(0, 1024, 64, 4)) == XL.XQ_ERR_INVALID     # tail not 0 / 128
    assert call(d, n_head=40) == XL.XQ_ERR_INVALID                      # 10 q heads per kv head
    assert call(d, active=2000) == XL.XQ_ERR_INVALID                    # active > capacity
    assert call(d, kp=C.c_void_p(4100)) == XL.XQ_ERR_INVALID            # plane not 16-byte aligned
    assert call(d, ws_bytes=100) == XL.XQ_ERR_WORKSPACE
    assert b"workspace" in L.xq_last_error()
