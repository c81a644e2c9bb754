"""GPU tests of xq_flash_attn_ext_noalloc, the entry point for callers that
cannot allocate device memory: a host whose device memory a graph allocator
planned ahead (ggml hands a backend only the tensors it planned), or a thread
that must not call cudaMalloc because cudaMalloc can synchronize the device
and stall every other stream.  It keeps its split partials in the library's
fixed static scratch instead of a caller workspace, and must give the results
of xq_flash_attn_ext bit for bit, call after call, although every call finds
the previous call's leftovers in the shared scratch.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test; it also passes alone.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _noalloc(q, k, v, ty, scale, out, n_splits=0, sinks=None):
    from xq import _lib
    from xq.ops import _fa_params, _stream
    p = _fa_params(q, k, v, ty, ty, None, sinks, out, scale, 0.0, 0.0, n_splits)
    return _lib.lib().xq_flash_attn_ext_noalloc(C.byref(p), _stream(None))


def _case(seed, ty, D, H, Hkv, n_kv, dev):
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.normal(0, 1, (1, H, 1, D)).astype(np.float32)).to(dev)
    k = torch.from_numpy(oracle.quantize(
        ty, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))).to(dev)
    v = torch.from_numpy(oracle.quantize(
        ty, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))).to(dev)
    return q, k, v


CASES = [  # (type, D, heads, kv heads, kv rows, n_splits, sinks)
    (oracle.Q8_0, 256, 16, 2, 32768, 0, False),   # config 2 shape, automatic plan
    (oracle.F16, 128, 16, 4, 4096, 0, False),     # config 1 shape
    (oracle.Q8_0, 256, 16, 2, 8192, 0, True),     # attention sinks join the merge
    (oracle.Q4_0, 256, 16, 2, 2048, 1, False),    # one split: direct output, no scratch
    (oracle.Q8_0, 128, 8, 2, 3000, 7, True),      # ragged last split, sinks
]


def test_noalloc_matches_workspace_entry_on_consecutive_calls():
    import xq
    from xq import _lib
    dev = torch.device("cuda")
    # calls in a row, each finding the previous call's leftovers in the scratch;
    # the whole list runs twice
    for rep in range(2):
        for call, (ty, D, H, Hkv, n_kv, ns, use_sinks) in enumerate(CASES):
            q, k, v = _case(100 + call, ty, D, H, Hkv, n_kv, dev)
            sinks = (torch.linspace(-1.0, 1.5, H, device=dev) if use_sinks else None)
            want = xq.flash_attn_ext(q, k, v, ty, sinks=sinks, scale=D ** -0.5, n_splits=ns)
            got = torch.full_like(want, float("nan"))
            rc = _noalloc(q, k, v, ty, D ** -0.5, got, n_splits=ns, sinks=sinks)
            assert rc == 0, _lib.lib().xq_last_error()
            torch.cuda.synchronize()
            g, w = got.cpu().numpy(), want.cpu().numpy()
            # the same kernels with the same split plan: identical bits
            np.testing.assert_array_equal(g, w, err_msg=f"rep {rep} case {call}")
            np.testing.assert_allclose(g, w, rtol=1e-2, atol=2e-3)


def test_noalloc_against_the_oracle():
    from xq import _lib
    dev = torch.device("cuda")
    ty, D, H, Hkv, n_kv = oracle.Q8_0, 256, 16, 2, 4096
    q, k, v = _case(7, ty, D, H, Hkv, n_kv, dev)
    got = torch.empty((1, 1, H, D), device=dev)
    assert _noalloc(q, k, v, ty, 1 / 16, got) == 0, _lib.lib().xq_last_error()
    want = oracle.flash_attn_ext(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), ty, ty,
                                 scale=1 / 16)
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-2, atol=2e-3)


def test_noalloc_pinned_host_q_and_dst():
    from xq import _lib
    dev = torch.device("cuda")
    ty, D, H, Hkv, n_kv = oracle.Q8_0, 256, 16, 2, 8192
    q, k, v = _case(11, ty, D, H, Hkv, n_kv, dev)
    want = torch.empty((1, 1, H, D), device=dev)
    assert _noalloc(q, k, v, ty, 1 / 16, want) == 0, _lib.lib().xq_last_error()
    q_host = q.cpu().pin_memory()
    o_host = torch.full((1, 1, H, D), float("nan"), pin_memory=True)
    for _ in range(2):
        assert _noalloc(q_host, k, v, ty, 1 / 16, o_host) == 0, _lib.lib().xq_last_error()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(o_host.numpy(), want.cpu().numpy())


def test_noalloc_rejects_pageable_host_memory_before_launching():
    from xq import _lib
    from xq.ops import _dense, _kv, _stream
    dev = torch.device("cuda")
    ty, D, H, Hkv, n_kv = oracle.Q8_0, 256, 16, 2, 1024
    q, k, v = _case(3, ty, D, H, Hkv, n_kv, dev)
    out = torch.empty((1, 1, H, D), device=dev)
    q_pageable = np.ascontiguousarray(q.cpu().numpy())
    o_pageable = np.zeros((1, 1, H, D), np.float32)
    L = _lib.lib()
    for qp, op in ((q_pageable.ctypes.data, out.data_ptr()),
                   (q.data_ptr(), o_pageable.ctypes.data)):
        p = _lib.FaParams()
        p.q = _dense(q)
        p.q.data = qp
        p.k, p.v = _kv(k, ty, D), _kv(v, ty, D)
        p.dst, p.scale = op, 1 / 16
        assert L.xq_flash_attn_ext_noalloc(C.byref(p), _stream(None)) == _lib.XQ_ERR_INVALID
        assert b"pageable" in L.xq_last_error()
    torch.cuda.synchronize()
    assert not o_pageable.any()


def test_noalloc_allocates_no_device_memory():
    from xq import _lib
    dev = torch.device("cuda")
    ty, D, H, Hkv, n_kv = oracle.Q8_0, 256, 16, 2, 32768
    q, k, v = _case(5, ty, D, H, Hkv, n_kv, dev)
    out = torch.empty((1, 1, H, D), device=dev)
    # the first call may load the kernels' modules; later calls must leave the
    # device's free memory and torch's allocator untouched
    assert _noalloc(q, k, v, ty, 1 / 16, out) == 0, _lib.lib().xq_last_error()
    torch.cuda.synchronize()
    free0, alloc0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
    for _ in range(3):
        assert _noalloc(q, k, v, ty, 1 / 16, out) == 0, _lib.lib().xq_last_error()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_allocated() == alloc0


def test_noalloc_rejects_plans_beyond_the_static_scratch():
    from xq import _lib
    dev = torch.device("cuda")
    D, H, Hkv, n_kv = 256, 16, 2, 65536
    q = torch.zeros((8, H, 1, D), device=dev)
    k = torch.zeros((8, n_kv, Hkv, 272), dtype=torch.uint8, device=dev)
    out = torch.empty((8, 1, H, D), device=dev)
    # 1024 splits x 128 rows x 258 floats = 135 MB > the static scratch
    rc = _noalloc(q, k, k, oracle.Q8_0, 1.0 / 16, out, n_splits=1024)
    assert rc == _lib.XQ_ERR_WORKSPACE
    assert b"static scratch" in _lib.lib().xq_last_error()
