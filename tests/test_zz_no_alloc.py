"""GPU test of xq_flash_attn_ext_noalloc, the entry point for callers that
cannot allocate device memory (a host whose memory a graph allocator planned
ahead, or a thread that must not call cudaMalloc because it can synchronize
the device).  It uses the library's fixed static scratch instead of a caller
workspace, and must give the results of xq_flash_attn_ext, call after call.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test; it also passes alone.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _noalloc(q, k, v, ty, scale, out, n_splits=0):
    import xq
    from xq import _lib
    from xq.ops import _fa_params, _stream
    p = _fa_params(q, k, v, ty, ty, None, None, out, scale, 0.0, 0.0, n_splits)
    return _lib.lib().xq_flash_attn_ext_noalloc(C.byref(p), _stream(None))


def test_noalloc_matches_workspace_entry_on_consecutive_calls():
    import xq
    from xq import _lib
    dev = torch.device("cuda")
    # three calls in a row: each one finds the previous call's leftovers in the
    # shared scratch
    for call, (ty, D, H, Hkv, n_kv) in enumerate([(oracle.Q8_0, 256, 16, 2, 32768),
                                                   (oracle.F16, 128, 16, 4, 4096),
                                                   (oracle.Q8_0, 256, 16, 2, 8192)]):
        rng = np.random.default_rng(100 + call)
        q = torch.from_numpy(rng.normal(0, 1, (1, H, 1, D)).astype(np.float32)).to(dev)
        k = torch.from_numpy(oracle.quantize(
            ty, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))).to(dev)
        v = torch.from_numpy(oracle.quantize(
            ty, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))).to(dev)
        want = xq.flash_attn_ext(q, k, v, ty, scale=D ** -0.5)
        got = torch.full_like(want, float("nan"))
        rc = _noalloc(q, k, v, ty, D ** -0.5, got)
        assert rc == 0, _lib.lib().xq_last_error()
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=1e-2, atol=2e-3)


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
