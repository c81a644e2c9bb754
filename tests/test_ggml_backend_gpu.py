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
from ggml_harness import F32, Q8_0, Tensor, tensor

pytestmark = pytest.mark.gpu

FN = C.CFUNCTYPE
VP = C.c_void_p


class RegI(C.Structure):
    _fields_ = [("get_name", FN(C.c_char_p, VP)), ("get_device_count", FN(C.c_size_t, VP)),
                ("get_device", FN(VP, VP, C.c_size_t)), ("get_proc_address", VP)]


class Reg(C.Structure):
    _fields_ = [("api_version", C.c_int), ("iface", RegI), ("context", VP)]


class DevI(C.Structure):
    _fields_ = [("get_name", FN(C.c_char_p, VP)), ("get_description", FN(C.c_char_p, VP)),
                ("get_memory", VP), ("get_type", VP), ("get_props", VP),
                ("init_backend", FN(VP, VP, C.c_char_p)), ("get_buffer_type", FN(VP, VP)),
                ("get_host_buffer_type", VP), ("buffer_from_host_ptr", VP),
                ("supports_op", FN(C.c_bool, VP, C.POINTER(Tensor))),
                ("supports_buft", FN(C.c_bool, VP, VP)), ("offload_op", VP), ("event_new", VP),
                ("event_free", VP), ("event_synchronize", VP)]


class Dev(C.Structure):
    _fields_ = [("iface", DevI), ("reg", VP), ("context", VP)]


class BuftI(C.Structure):
    _fields_ = [("get_name", FN(C.c_char_p, VP)), ("alloc_buffer", FN(VP, VP, C.c_size_t)),
                ("get_alignment", FN(C.c_size_t, VP)), ("get_max_size", VP),
                ("get_alloc_size", VP), ("is_host", VP)]


class Buft(C.Structure):
    _fields_ = [("iface", BuftI), ("device", VP), ("context", VP)]


class BufI(C.Structure):
    _fields_ = [("free_buffer", VP), ("get_base", FN(VP, VP)), ("init_tensor", VP),
                ("memset_tensor", VP),
                ("set_tensor", FN(None, VP, C.POINTER(Tensor), VP, C.c_size_t, C.c_size_t)),
                ("get_tensor", FN(None, VP, C.POINTER(Tensor), VP, C.c_size_t, C.c_size_t)),
                ("set_tensor_2d", VP), ("get_tensor_2d", VP), ("cpy_tensor", VP),
                ("clear", FN(None, VP, C.c_uint8)), ("reset", VP)]


class Buf(C.Structure):
    _fields_ = [("iface", BufI), ("buft", VP), ("context", VP), ("size", C.c_size_t),
                ("usage", C.c_int)]


class BackendI(C.Structure):
    _fields_ = [("get_name", FN(C.c_char_p, VP)), ("free", FN(None, VP)),
                ("set_tensor_async", VP), ("get_tensor_async", VP), ("set_2d_async", VP),
                ("get_2d_async", VP), ("cpy_tensor_async", VP), ("synchronize", FN(None, VP)),
                ("plan_create", VP), ("plan_free", VP), ("plan_update", VP),
                ("plan_compute", VP), ("graph_compute", FN(C.c_int, VP, C.POINTER(gh.Graph))),
                ("event_record", VP), ("event_wait", VP), ("graph_optimize", VP)]


class Backend(C.Structure):
    _fields_ = [("guid", VP), ("iface", BackendI), ("device", VP), ("context", VP)]


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
