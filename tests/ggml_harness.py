"""ctypes view of the XQ_B200 ggml backend over the mock ggml of
tests/ggml_mock/ggml_mock.c (layouts of ggml_abi_mirror.h).  Test
infrastructure: builds libggml_mock.so on first use, then loads it globally
so the backend's ggml symbols resolve, then loads libxq_ggml_b200.so."""
import ctypes as C
import os
import subprocess

from conftest import PKG, REPO

MOCK_SRC = os.path.join(REPO, "tests", "ggml_mock", "ggml_mock.c")
MOCK_LIB = os.path.join(REPO, "tests", "ggml_mock", "libggml_mock.so")
BACKEND_LIB = os.path.join(PKG, "lib", "libxq_ggml_b200.so")

# placeholder op ids of ggml_abi_mirror.h
OP_NONE, OP_RESHAPE, OP_VIEW, OP_PERMUTE, OP_TRANSPOSE = 0, 36, 37, 38, 39
OP_FLASH_ATTN_EXT, OP_GATED_DELTA_NET, OP_MUL_MAT, OP_SET_ROWS = 72, 84, 29, 41
F32, F16, Q4_0, Q8_0, I32, I64 = 0, 1, 2, 8, 26, 27
FLAG_COMPUTE = 16


class Tensor(C.Structure):
    pass


Tensor._fields_ = [("type", C.c_int), ("buffer", C.c_void_p), ("ne", C.c_int64 * 4),
                   ("nb", C.c_size_t * 4), ("op", C.c_int), ("op_params", C.c_int32 * 16),
                   ("flags", C.c_int32), ("src", C.POINTER(Tensor) * 10),
                   ("view_src", C.c_void_p), ("view_offs", C.c_size_t), ("data", C.c_void_p),
                   ("name", C.c_char * 64), ("extra", C.c_void_p), ("padding", C.c_char * 8)]


class Graph(C.Structure):
    _fields_ = [("n_nodes", C.c_int), ("nodes", C.POINTER(C.POINTER(Tensor)))]


# vtables of ggml_abi_mirror.h (slots the tests call are typed)
FN = C.CFUNCTYPE
VP = C.c_void_p
# (buffer or backend, tensor, data, offset, size): set/get_tensor[_async]
COPY = FN(None, VP, C.POINTER(Tensor), VP, C.c_size_t, C.c_size_t)
# (..., offset, size, n_copies, stride_tensor, stride_data): the fork's 2-D slots
COPY_2D = FN(None, VP, C.POINTER(Tensor), VP, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t,
             C.c_size_t)


class RegI(C.Structure):
    _fields_ = [("get_name", FN(C.c_char_p, VP)), ("get_device_count", FN(C.c_size_t, VP)),
                ("get_device", FN(VP, VP, C.c_size_t)),
                ("get_proc_address", FN(VP, VP, C.c_char_p))]


class Reg(C.Structure):
    _fields_ = [("api_version", C.c_int), ("iface", RegI), ("context", VP)]


class DevI(C.Structure):
    _fields_ = [("get_name", FN(C.c_char_p, VP)), ("get_description", FN(C.c_char_p, VP)),
                ("get_memory", VP), ("get_type", VP), ("get_props", VP),
                ("init_backend", FN(VP, VP, C.c_char_p)), ("get_buffer_type", FN(VP, VP)),
                ("get_host_buffer_type", FN(VP, VP)), ("buffer_from_host_ptr", VP),
                ("supports_op", FN(C.c_bool, VP, C.POINTER(Tensor))),
                ("supports_buft", FN(C.c_bool, VP, VP)), ("offload_op", VP),
                ("event_new", FN(VP, VP)), ("event_free", FN(None, VP, VP)),
                ("event_synchronize", FN(None, VP, VP))]


class Dev(C.Structure):
    _fields_ = [("iface", DevI), ("reg", VP), ("context", VP)]


class BuftI(C.Structure):
    _fields_ = [("get_name", FN(C.c_char_p, VP)), ("alloc_buffer", FN(VP, VP, C.c_size_t)),
                ("get_alignment", FN(C.c_size_t, VP)), ("get_max_size", VP),
                ("get_alloc_size", VP), ("is_host", FN(C.c_bool, VP))]


class Buft(C.Structure):
    _fields_ = [("iface", BuftI), ("device", VP), ("context", VP)]


class BufI(C.Structure):
    _fields_ = [("free_buffer", VP), ("get_base", FN(VP, VP)), ("init_tensor", VP),
                ("memset_tensor", VP),
                ("set_tensor", COPY), ("get_tensor", COPY), ("set_tensor_2d", COPY_2D), ("get_tensor_2d", COPY_2D),
                ("cpy_tensor", FN(C.c_bool, VP, C.POINTER(Tensor), C.POINTER(Tensor))),
                ("clear", FN(None, VP, C.c_uint8)), ("reset", VP)]


class Buf(C.Structure):
    _fields_ = [("iface", BufI), ("buft", VP), ("context", VP), ("size", C.c_size_t),
                ("usage", C.c_int)]


class BackendI(C.Structure):
    _fields_ = [("get_name", FN(C.c_char_p, VP)), ("free", FN(None, VP)),
                ("set_tensor_async", COPY), ("get_tensor_async", COPY), ("set_2d_async", COPY_2D),
                ("get_2d_async", COPY_2D),
                ("cpy_tensor_async", FN(C.c_bool, VP, VP, C.POINTER(Tensor), C.POINTER(Tensor))),
                ("synchronize", FN(None, VP)),
                ("plan_create", VP), ("plan_free", VP), ("plan_update", VP),
                ("plan_compute", VP), ("graph_compute", FN(C.c_int, VP, C.POINTER(Graph))),
                ("event_record", FN(None, VP, VP)), ("event_wait", FN(None, VP, VP)),
                ("graph_optimize", VP)]


class Backend(C.Structure):
    _fields_ = [("guid", VP), ("iface", BackendI), ("device", VP), ("context", VP)]


_libs = None


def libs():
    global _libs
    if _libs is None:
        if (not os.path.exists(MOCK_LIB)
                or os.path.getmtime(MOCK_SRC) > os.path.getmtime(MOCK_LIB)):
            subprocess.run(["gcc", "-O2", "-fPIC", "-shared", "-I",
                            os.path.join(PKG, "ggml"), MOCK_SRC, "-o", MOCK_LIB], check=True)
        mock = C.CDLL(MOCK_LIB, mode=C.RTLD_GLOBAL)
        if not os.path.exists(BACKEND_LIB):
            import importlib.util
            spec = importlib.util.spec_from_file_location("xq_build", os.path.join(PKG, "build.py"))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            mod.build()
        be = C.CDLL(BACKEND_LIB)
        be.ggml_xq_b200_supports_op.argtypes = [C.POINTER(Tensor)]
        be.ggml_xq_b200_supports_op.restype = C.c_bool
        be.ggml_backend_xq_b200_reg.restype = C.c_void_p
        be.ggml_xq_b200_register.restype = C.c_bool
        mock.xq_mock_registered.restype = C.c_int
        _libs = (mock, be)
    return _libs


BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_0: (32, 18), I32: (1, 4), I64: (1, 8)}


def tensor(ty, ne, nb=None, data=None, op=OP_NONE, srcs=(), op_params=()):
    t = Tensor()
    t.type = ty
    for i in range(4):
        t.ne[i] = ne[i] if i < len(ne) else 1
    if nb is None:
        blk, bs = BLOCK[ty]
        nb = [bs, bs * (t.ne[0] // blk)]
        for i in range(2, 4):
            nb.append(nb[-1] * t.ne[i - 1])
    for i in range(4):
        t.nb[i] = nb[i]
    t.op = op
    for i, p in enumerate(op_params):
        t.op_params[i] = p
    for i, s in enumerate(srcs):
        if s is not None:
            t.src[i] = C.pointer(s)
    t.data = data
    return t


def f32_bits(x):
    import struct
    return struct.unpack("<i", struct.pack("<f", x))[0]


def fa_node(q, k, v, mask=None, sinks=None, scale=1.0, max_bias=0.0, softcap=0.0, dst_data=None):
    D, n_q, H, S = (q.ne[i] for i in range(4))
    out = tensor(F32, (D, H, n_q, S), data=dst_data, op=OP_FLASH_ATTN_EXT,
                 srcs=(q, k, v, mask, sinks),
                 op_params=(f32_bits(scale), f32_bits(max_bias), f32_bits(softcap)))
    out.flags = FLAG_COMPUTE
    return out


def set_rows_node(cache, rows, idx):
    """ggml_set_rows(cache, rows, idx): a view of `cache` whose op writes rows."""
    out = tensor(cache.type, tuple(cache.ne), nb=tuple(cache.nb), data=cache.data,
                 op=OP_SET_ROWS, srcs=(rows, idx))
    out.flags = FLAG_COMPUTE
    return out


def gdn_node(q, k, v, g, beta, state, slots=1, gate_mode=0, dst_data=None):
    S, H, T, NS = (v.ne[i] for i in range(4))
    out = tensor(F32, (S * H, T * NS + slots * S * NS, 1, 1), data=dst_data,
                 op=OP_GATED_DELTA_NET, srcs=(q, k, v, g, beta, state),
                 op_params=(slots, gate_mode))
    out.flags = FLAG_COMPUTE
    return out
