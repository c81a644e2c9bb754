"""B200: a ggml graph through the XQ_B200 backend's vtables.

Registry -> device -> backend and buffer type, tensors placed in a backend
buffer with set_tensor, graph_compute + synchronize, get_tensor; results
checked against the CPU oracle.  ggml itself is the mock of
tests/ggml_mock/ggml_mock.c (layouts of ggml_abi_mirror.h)."""
import ctypes as C

import numpy as np
import pytest

import ggml_harness as gh
import oracle
from ggml_harness import F32, Q8_0, Backend, Buf, Buft, Dev, Reg, Tensor, tensor

pytestmark = pytest.mark.gpu

class Session:
    """Backend + one device buffer carved into tensors."""

    def __init__(self, nbytes):
        mock, be = gh.libs()
        assert be.ggml_xq_b200_register()
        self.mock = mock
        regp = be.ggml_backend_xq_b200_reg()
        reg = Reg.from_address(regp)
        assert reg.iface.get_name(regp) == b"XQ_B200"
        assert reg.iface.get_device_count(regp) >= 1
        self.devp = reg.iface.get_device(regp, 0)
        self.dev = Dev.from_address(self.devp)
        self.bep = self.dev.iface.init_backend(self.devp, None)
        self.be = Backend.from_address(self.bep)
        buftp = self.dev.iface.get_buffer_type(self.devp)
        assert self.dev.iface.supports_buft(self.devp, buftp)
        buft = Buft.from_address(buftp)
        self.bufp = buft.iface.alloc_buffer(buftp, nbytes)
        self.buf = Buf.from_address(self.bufp)
        self.base = self.buf.iface.get_base(self.bufp)
        self.off = 0
        self.keep = []

    def place(self, t, host=None):
        self.off = (self.off + 255) // 256 * 256
        t.data = self.base + self.off
        t.buffer = self.bufp
        n = host.nbytes if host is not None else 0
        if host is not None:
            host = np.ascontiguousarray(host)
            self.keep.append(host)
            self.buf.iface.set_tensor(self.bufp, C.byref(t), host.ctypes.data, 0, host.nbytes)
        self.off += max(n, 256)
        return t

    def alloc(self, t, nbytes):
        self.off = (self.off + 255) // 256 * 256
        t.data = self.base + self.off
        t.buffer = self.bufp
        self.off += nbytes
        return t

    def compute(self, nodes):
        arr = (C.POINTER(Tensor) * len(nodes))(*[C.pointer(n) for n in nodes])
        g = gh.Graph(len(nodes), arr)
        for n in nodes:
            assert self.dev.iface.supports_op(self.devp, C.byref(n))
        st = self.be.iface.graph_compute(self.bep, C.byref(g))
        self.be.iface.synchronize(self.bep)
        return st

    def get(self, t, shape, dtype=np.float32):
        out = np.empty(shape, dtype)
        self.buf.iface.get_tensor(self.bufp, C.byref(t), out.ctypes.data, 0, out.nbytes)
        return out

    def close(self):
        self.mock.xq_mock_buffer_free(C.c_void_p(self.bufp))
        self.be.iface.free(self.bep)


def test_flash_attn_and_gdn_through_graph_compute():
    rng = np.random.default_rng(31)
    s = Session(256 << 20)
    try:
        # FLASH_ATTN_EXT: BASELINE config 2 shape at kv 8192, Q8_0 cache layout
        D, H, Hkv, n_kv = 256, 16, 2, 8192
        qh = rng.normal(0, 1, (1, H, 1, D)).astype(np.float32)
        kh = oracle.quantize(Q8_0, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))
        vh = oracle.quantize(Q8_0, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))
        q = s.place(tensor(F32, (D, 1, H, 1)), qh)
        k = s.place(tensor(Q8_0, (D, n_kv, Hkv, 1), nb=(34, Hkv * 272, 272, n_kv * Hkv * 272)),
                    kh)
        v = s.place(tensor(Q8_0, (D, n_kv, Hkv, 1), nb=(34, Hkv * 272, 272, n_kv * Hkv * 272)),
                    vh)
        out = gh.fa_node(q, k, v, scale=1 / 16)
        s.alloc(out, H * D * 4)
        # GATED_DELTA_NET: 32 v-heads / 16 k-heads, 4 tokens, 2 sequences, 3 slots
        S_, Hv, Hk, T, NS, K = 128, 32, 16, 4, 2, 3
        ins = [rng.normal(0, 0.1, (NS, T, Hk, S_)).astype(np.float32),
               rng.normal(0, 0.1, (NS, T, Hk, S_)).astype(np.float32),
               rng.normal(0, 1, (NS, T, Hv, S_)).astype(np.float32),
               -np.abs(rng.normal(0, 1, (NS, T, Hv, 1))).astype(np.float32),
               rng.uniform(0, 1, (NS, T, Hv, 1)).astype(np.float32),
               rng.normal(0, 0.1, (NS, Hv, S_, S_)).astype(np.float32)]
        ts = [s.place(tensor(F32, tuple(reversed(x.shape))), x) for x in ins]
        gout = gh.gdn_node(*ts, slots=K)
        n_dst = S_ * Hv * (T * NS + K * S_ * NS)
        s.alloc(gout, n_dst * 4)
        assert s.compute([out, gout]) == 0
        got = s.get(out, (1, 1, H, D))
        want = oracle.flash_attn_ext(qh, kh, vh, Q8_0, Q8_0, scale=1 / 16)
        np.testing.assert_allclose(got, want, rtol=1e-2, atol=2e-3)
        gd = s.get(gout, (n_dst,))
        wd, _, _ = oracle.gated_delta_net(*ins, slots=K)
        np.testing.assert_allclose(gd, wd, rtol=1e-2, atol=2e-3)
    finally:
        s.close()


def test_unclaimed_node_fails_without_fallback():
    s = Session(1 << 20)
    try:
        bad = tensor(F32, (4, 4, 1, 1), op=gh.OP_MUL_MAT)
        bad.flags = gh.FLAG_COMPUTE
        assert not s.dev.iface.supports_op(s.devp, C.byref(bad))
        arr = (C.POINTER(Tensor) * 1)(C.pointer(bad))
        assert s.be.iface.graph_compute(s.bep, C.byref(gh.Graph(1, arr))) != 0
    finally:
        s.close()


def test_set_rows_through_graph_compute():
    """The KV-cache write node: F32 rows quantized into a Q8_0 cache view at
    I64 indices, then read back bit-identical to the oracle."""
    rng = np.random.default_rng(41)
    s = Session(64 << 20)
    try:
        D, rows, Hkv, n_tok = 256, 512, 2, 7
        ch = oracle.quantize(Q8_0, rng.normal(0, 1, (1, rows, Hkv, D)).astype(np.float32))
        xh = rng.normal(0, 1, (1, n_tok, Hkv, D)).astype(np.float32)
        ih = rng.choice(rows, n_tok, replace=False).astype(np.int64)
        cache = s.place(tensor(Q8_0, (D, rows, Hkv, 1), nb=(34, Hkv * 272, 272, rows * Hkv * 272)),
                        ch)
        src = s.place(tensor(F32, (D, n_tok, Hkv, 1), nb=(4, Hkv * D * 4, D * 4, n_tok * Hkv * D * 4)),
                      xh)
        idx = s.place(tensor(gh.I64, (n_tok, 1, 1, 1)), ih)
        node = gh.set_rows_node(cache, src, idx)
        assert s.compute([node]) == 0
        got = s.get(cache, ch.shape, np.uint8)
        assert np.array_equal(got, oracle.set_rows(ch, xh, ih, Q8_0))
    finally:
        s.close()


def rows_2d(host, off, size, n, stride_tensor, stride_data, dst):
    """ggml's row-loop definition of set_tensor_2d over a byte image."""
    for i in range(n):
        o = off + i * stride_tensor
        dst[o:o + size] = host[i * stride_data:i * stride_data + size]


def test_strided_2d_copies_buffer_and_backend():
    """The fork's set/get_tensor_2d (buffer) and set/get_tensor_2d_async
    (backend) slots against ggml's row-by-row definition: pitched strides
    (one 2-D copy) and overlapping tensor rows (row order decides)."""
    rng = np.random.default_rng(7)
    s = Session(1 << 20)
    try:
        nbytes = 96 * 1024
        t = s.alloc(tensor(F32, (nbytes // 4, 1, 1, 1)), nbytes)
        host_t = rng.integers(0, 256, nbytes, dtype=np.uint8)
        s.buf.iface.set_tensor(s.bufp, C.byref(t), host_t.ctypes.data, 0, nbytes)
        cases = [(40, 1000, 64, 1024, 1500),   # pitched on both sides
                 (8, 700, 50, 512, 700),       # overlapping tensor rows
                 (0, 256, 33, 2048, 0)]        # one host row broadcast
        for off, size, n, st, sd in cases:
            src = rng.integers(0, 256, max(sd * (n - 1) + size, size), dtype=np.uint8)
            want = host_t.copy()
            rows_2d(src, off, size, n, st, sd, want)
            s.buf.iface.set_tensor_2d(s.bufp, C.byref(t), src.ctypes.data, off, size, n, st, sd)
            assert np.array_equal(s.get(t, (nbytes,), np.uint8), want)
            hs = max(sd, size)  # host pitch of the read back
            back = np.zeros(hs * (n - 1) + size + 64, np.uint8)
            s.buf.iface.get_tensor_2d(s.bufp, C.byref(t), back.ctypes.data, off, size, n, st, hs)
            for i in range(n):
                d = i * hs
                assert np.array_equal(back[d:d + size], want[off + i * st:off + i * st + size])
            # the backend's async pair on its stream
            s.buf.iface.set_tensor(s.bufp, C.byref(t), host_t.ctypes.data, 0, nbytes)
            s.be.iface.set_2d_async(s.bep, C.byref(t), src.ctypes.data, off, size, n, st, sd)
            back2 = np.zeros_like(back)
            s.be.iface.get_2d_async(s.bep, C.byref(t), back2.ctypes.data, off, size, n, st, hs)
            s.be.iface.synchronize(s.bep)
            assert np.array_equal(back2, back)
            assert np.array_equal(s.get(t, (nbytes,), np.uint8), want)
            host_t = want
    finally:
        s.close()


def test_host_buffer_type_events_and_cross_backend_copy():
    """Pinned host buffer type (the device's host type and its one extra
    buffer type), device events recorded and waited on by backends, and
    cpy_tensor_async between two backends of the device."""
    rng = np.random.default_rng(9)
    s = Session(1 << 20)
    try:
        hbp = s.dev.iface.get_host_buffer_type(s.devp)
        hb = Buft.from_address(hbp)
        assert hb.iface.get_name(hbp) == b"XQ_B200_Host" and hb.iface.is_host(hbp)
        regp = gh.libs()[1].ggml_backend_xq_b200_reg()
        fp = Reg.from_address(regp).iface.get_proc_address(regp, b"ggml_backend_dev_get_extra_bufts")
        extra = C.CFUNCTYPE(C.POINTER(C.c_void_p), C.c_void_p)(fp)(s.devp)
        assert extra[0] == hbp and not extra[1]
        assert not s.dev.iface.supports_buft(s.devp, hbp)
        hbufp = hb.iface.alloc_buffer(hbp, 1 << 16)
        assert hbufp
        hbuf = Buf.from_address(hbufp)
        pinned = tensor(F32, (4096, 1, 1, 1), data=hbuf.iface.get_base(hbufp))
        pinned.buffer = hbufp
        x = rng.normal(0, 1, 4096).astype(np.float32)
        hbuf.iface.set_tensor(hbufp, C.byref(pinned), x.ctypes.data, 0, x.nbytes)

        # pinned -> device on backend 1, event, backend 2 waits then copies on
        a = s.alloc(tensor(F32, (4096, 1, 1, 1)), x.nbytes)
        b = s.alloc(tensor(F32, (4096, 1, 1, 1)), x.nbytes)
        be2p = s.dev.iface.init_backend(s.devp, None)
        be2 = Backend.from_address(be2p)
        ev = s.dev.iface.event_new(s.devp)
        assert ev
        try:
            s.be.iface.set_tensor_async(s.bep, C.byref(a), pinned.data, 0, x.nbytes)
            s.be.iface.event_record(s.bep, ev)
            be2.iface.event_wait(be2p, ev)
            assert be2.iface.cpy_tensor_async(s.bep, be2p, C.byref(a), C.byref(b))
            out = np.zeros(4096, np.float32)
            be2.iface.get_tensor_async(be2p, C.byref(b), out.ctypes.data, 0, out.nbytes)
            be2.iface.synchronize(be2p)
            s.dev.iface.event_synchronize(s.devp, ev)
            assert np.array_equal(out, x)
            # a host-buffer source is not this backend's to copy
            assert not be2.iface.cpy_tensor_async(s.bep, be2p, C.byref(pinned), C.byref(b))
            back = np.zeros(4096, np.float32)
            hbuf.iface.get_tensor(hbufp, C.byref(pinned), back.ctypes.data, 0, back.nbytes)
            assert np.array_equal(back, x)
        finally:
            s.dev.iface.event_free(s.devp, ev)
            be2.iface.free(be2p)
            s.mock.xq_mock_buffer_free(C.c_void_p(hbufp))
    finally:
        s.close()


def test_per_op_gpu_timing():
    """A backend created with XQ_GGML_TIMING=1 keeps per-op GPU time (CUDA
    events around every node, read at synchronize); a backend without it
    answers false."""
    import os
    _, be = gh.libs()
    be.ggml_xq_b200_backend_op_time.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_uint64),
                                                C.POINTER(C.c_double), C.POINTER(C.c_uint64)]
    be.ggml_xq_b200_backend_op_time.restype = C.c_bool
    rng = np.random.default_rng(3)
    os.environ["XQ_GGML_TIMING"] = "1"
    try:
        s = Session(64 << 20)
    finally:
        del os.environ["XQ_GGML_TIMING"]
    plain = Session(1 << 20)
    try:
        D, H, Hkv, n_kv = 128, 8, 2, 2048
        qh = rng.normal(0, 1, (1, H, 1, D)).astype(np.float32)
        kh = oracle.quantize(gh.F16, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))
        vh = oracle.quantize(gh.F16, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))
        nb = (2, Hkv * 2 * D, 2 * D, n_kv * Hkv * 2 * D)
        q = s.place(tensor(F32, (D, 1, H, 1)), qh)
        k = s.place(tensor(gh.F16, (D, n_kv, Hkv, 1), nb=nb), kh)
        v = s.place(tensor(gh.F16, (D, n_kv, Hkv, 1), nb=nb), vh)
        out = gh.fa_node(q, k, v, scale=D ** -0.5)
        s.alloc(out, H * D * 4)
        for _ in range(3):
            assert s.compute([out]) == 0
        nodes, ms, untimed = C.c_uint64(), C.c_double(), C.c_uint64()
        assert be.ggml_xq_b200_backend_op_time(s.bep, 0, C.byref(nodes), C.byref(ms),
                                               C.byref(untimed))
        assert nodes.value == 3 and untimed.value == 0 and 0.0 < ms.value < 1000.0
        assert be.ggml_xq_b200_backend_op_time(s.bep, 1, C.byref(nodes), C.byref(ms),
                                               C.byref(untimed))
        assert nodes.value == 0 and ms.value == 0.0
        assert not be.ggml_xq_b200_backend_op_time(s.bep, 3, None, None, None)
        assert not be.ggml_xq_b200_backend_op_time(plain.bep, 0, None, None, None)
        np.testing.assert_allclose(
            s.get(out, (1, 1, H, D)),
            oracle.flash_attn_ext(qh, kh, vh, gh.F16, gh.F16, scale=D ** -0.5),
            rtol=1e-2, atol=2e-3)
    finally:
        plain.close()
        s.close()
