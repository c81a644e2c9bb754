"""The XQ_B200 ggml backend's supports_op contract (host logic, no GPU).

Mirrors how the reference gates its D3D12 GATED_DELTA_NET
(src/bridge/ggml_d3d12.cpp:77-109, widened to any n_seq and T) and keeps
FLASH_ATTN_EXT to what the kernels take; everything else is refused so the
scheduler leaves it on its current backend."""
import ggml_harness as gh
from ggml_harness import F16, F32, I32, I64, Q4_0, Q8_0, tensor


def fa(D=256, H=16, Hkv=2, n_kv=4096, n_q=1, S=1, kt=Q8_0, vt=None, mask=False, mt=F16,
       sinks=False):
    q = tensor(F32, (D, n_q, H, S))
    k = tensor(kt, (D, n_kv, Hkv, S))
    v = tensor(kt if vt is None else vt, (D, n_kv, Hkv, S))
    m = tensor(mt, (n_kv, max(n_q, 1), 1, 1)) if mask else None
    sk = tensor(F32, (H, 1, 1, 1)) if sinks else None
    return gh.fa_node(q, k, v, m, sk, scale=D ** -0.5)


def gdn(S=128, H=32, Hk=16, T=1, NS=8, slots=1, gate_mode=0, g_dim=1):
    q = tensor(F32, (S, Hk, T, NS))
    k = tensor(F32, (S, Hk, T, NS))
    v = tensor(F32, (S, H, T, NS))
    g = tensor(F32, (g_dim, H, T, NS))
    b = tensor(F32, (1, H, T, NS))
    st = tensor(F32, (S, S, H, NS))
    return gh.gdn_node(q, k, v, g, b, st, slots=slots, gate_mode=gate_mode)


def supported(t):
    return gh.libs()[1].ggml_xq_b200_supports_op(t)


def test_flash_attn_claims():
    for kt in (F16, Q8_0, Q4_0):
        assert supported(fa(kt=kt))
        assert supported(fa(kt=kt, D=128, H=16, Hkv=4))
    assert supported(fa(kt=F16, n_q=8192, H=24, Hkv=4, n_kv=8192, mask=True))
    assert supported(fa(sinks=True, mask=True, n_q=3))
    assert supported(fa(S=8, n_kv=262144, H=24, Hkv=4))


def test_flash_attn_refusals():
    assert not supported(fa(kt=F32))                 # F32 KV: not claimed
    assert not supported(fa(kt=Q8_0, vt=F16))         # mixed K/V types
    assert not supported(fa(D=96))                    # head size
    assert not supported(fa(mask=True, mt=F32))       # mask must be F16
    assert not supported(fa(H=12, Hkv=8))             # GQA must divide


def test_gdn_claims_and_refusals():
    assert supported(gdn())                          # C3 decode, batch 8
    assert supported(gdn(T=4096, NS=1))              # C3 chunked prefill shape
    assert supported(gdn(T=64, NS=1, slots=5))       # the reference contract
    assert not supported(gdn(S=64))                  # head size 128 only
    assert not supported(gdn(gate_mode=1))           # gates not yet activated
    assert not supported(gdn(g_dim=128))             # per-dim gates
    assert not supported(gdn(slots=0))
    assert not supported(gdn(H=24, Hk=16))           # H % H_k


def set_rows(ct=Q8_0, D=256, rows=4096, Hkv=2, n_tok=1, it=I64, i1=1, st=F32):
    cache = tensor(ct, (D, rows, Hkv, 1))
    src = tensor(st, (D, n_tok, Hkv, 1))
    idx = tensor(it, (n_tok, i1, 1, 1))
    return gh.set_rows_node(cache, src, idx)


def test_set_rows_claims_and_refusals():
    for ct in (F32, F16, Q8_0, Q4_0):
        assert supported(set_rows(ct=ct))              # KV-cache append
    assert supported(set_rows(n_tok=512, it=I32, i1=2))  # prefill, per-head indices
    assert supported(set_rows(D=512, Hkv=1))           # llama.cpp's 2D cache rows
    assert not supported(set_rows(st=F16))             # rows must be F32
    assert not supported(set_rows(it=F32))             # indices I32 / I64 only
    assert not supported(set_rows(i1=3))               # heads % i1
    assert not supported(set_rows(ct=Q8_0, D=80))      # whole 32-element blocks


def test_view_ops_and_others():
    for op in (gh.OP_NONE, gh.OP_RESHAPE, gh.OP_VIEW, gh.OP_PERMUTE, gh.OP_TRANSPOSE):
        assert supported(tensor(F32, (4, 4, 1, 1), op=op))
    assert not supported(tensor(F32, (4, 4, 1, 1), op=gh.OP_MUL_MAT))


def test_registry_without_gpu_registers_nothing():
    import ctypes as C
    mock, be = gh.libs()
    reg = be.ggml_backend_xq_b200_reg()
    assert reg
    import torch
    if not torch.cuda.is_available():
        assert not be.ggml_xq_b200_register()
        assert mock.xq_mock_registered() == 0


def test_proc_address_answers_extra_bufts():
    """get_proc_address answers "ggml_backend_dev_get_extra_bufts" (as the
    reference's registry does) with a null-terminated list holding the pinned
    host buffer type; other names answer null."""
    import ctypes as C
    _, be = gh.libs()
    regp = be.ggml_backend_xq_b200_reg()
    reg = gh.Reg.from_address(regp)
    assert reg.iface.get_proc_address(regp, b"ggml_backend_set_n_threads") is None
    fp = reg.iface.get_proc_address(regp, b"ggml_backend_dev_get_extra_bufts")
    assert fp
    lst = C.CFUNCTYPE(C.POINTER(C.c_void_p), C.c_void_p)(fp)(None)
    assert lst[0] and not lst[1]
    buft = gh.Buft.from_address(lst[0])
    assert buft.iface.get_name(lst[0]) == b"XQ_B200_Host"
    assert buft.iface.is_host(lst[0])
    assert buft.iface.get_alignment(lst[0]) == 64
