"""B200 parity: FLASH_ATTN_EXT decode / short multi-query through the C ABI.

Each case runs libxq_b200.so (via the xq host package) and the CPU oracle (the
ggml-cpu restatement in oracle/) on the same seeded inputs.  Tolerance is the
north-star bound |gpu - cpu| <= 2e-3 + 1e-2 * |cpu| (fp32 accumulation on the
GPU vs ggml-cpu's order, Q8_0-quantized q and fp16 value accumulator).
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def _xq():
    import xq
    return xq


def make_case(seed, ty, D, n_head, n_hkv, n_kv, n_q=1, n_seq=1, n_seq_kv=None, mask=None):
    rng = np.random.default_rng(seed)
    n_seq_kv = n_seq if n_seq_kv is None else n_seq_kv
    q = rng.normal(0, 1, (n_seq, n_head, n_q, D)).astype(np.float32)
    kf = rng.normal(0, 1, (n_seq_kv, n_kv, n_hkv, D)).astype(np.float32)
    vf = rng.normal(0, 1, (n_seq_kv, n_kv, n_hkv, D)).astype(np.float32)
    k = oracle.quantize(ty, kf)
    v = oracle.quantize(ty, vf)
    m = None
    if mask == "random":
        m = np.zeros((1, 1, max(n_q, 1), n_kv), np.float16)
        m[rng.random(m.shape) < 0.3] = -np.inf
    elif mask == "causal":
        m = np.zeros((1, 1, n_q, n_kv), np.float16)
        for i in range(n_q):
            m[0, 0, i, n_kv - n_q + i + 1:] = -np.inf
    return q, k, v, m


def run_both(q, k, v, m, ty, scale, n_splits=0, sinks=None, softcap=0.0, max_bias=0.0,
             nth=8):
    xq = _xq()
    dev = torch.device("cuda")
    tq = torch.from_numpy(q).to(dev)
    tk = torch.from_numpy(k).to(dev)
    tv = torch.from_numpy(v).to(dev)
    tm = torch.from_numpy(m).to(dev) if m is not None else None
    ts = torch.from_numpy(sinks).to(dev) if sinks is not None else None
    got = xq.flash_attn_ext(tq, tk, tv, ty, mask=tm, sinks=ts, scale=scale, n_splits=n_splits,
                            softcap=softcap, max_bias=max_bias)
    torch.cuda.synchronize()
    want = oracle.flash_attn_ext(q, k, v, ty, ty, mask=m, sinks=sinks, scale=scale,
                                 softcap=softcap, max_bias=max_bias, nth=nth)
    return got.cpu().numpy(), want


@pytest.mark.parametrize("ty", [oracle.F16, oracle.Q8_0, oracle.Q4_0])
@pytest.mark.parametrize("D,n_head,n_hkv,n_kv", [(128, 16, 4, 4096), (256, 16, 2, 4096),
                                                 (256, 24, 4, 1000), (64, 8, 8, 777)])
def test_decode_parity(ty, D, n_head, n_hkv, n_kv):
    q, k, v, m = make_case(D + n_kv + ty, ty, D, n_head, n_hkv, n_kv)
    got, want = run_both(q, k, v, m, ty, D ** -0.5)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


def test_c1_config_f16_split_kv():
    """16 Q / 4 KV heads, D=128, kv 4096, F16, seed 0."""
    q, k, v, m = make_case(0, oracle.F16, 128, 16, 4, 4096)
    for nth in (1, 6, 8):  # ggml split-KV result depends on the thread count
        got, want = run_both(q, k, v, m, oracle.F16, 128 ** -0.5, nth=nth)
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("ty", [oracle.Q8_0, oracle.Q4_0])
def test_c2_config_full_size(ty):
    """BASELINE config 2 at full size: 16 Q / 2 KV heads, D=256, kv 32768."""
    q, k, v, m = make_case(0, ty, 256, 16, 2, 32768)
    got, want = run_both(q, k, v, m, ty, 1.0 / 16)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    # ggml quantizes q to Q8_0 before the K dot; both sides do, so both sit
    # the same distance from exact float64 attention on unquantized q
    ref64, _ = oracle.flash_attn_ext(q, k, v, ty, ty, scale=1.0 / 16, f64=True)
    assert np.abs(got - ref64).max() <= 1.5 * np.abs(want - ref64).max() + 1e-5


@pytest.mark.parametrize("n_splits", [1, 2, 7, 64, 0])
def test_split_count_invariance(n_splits):
    q, k, v, m = make_case(3, oracle.Q8_0, 256, 16, 2, 3000)
    got, want = run_both(q, k, v, m, oracle.Q8_0, 1.0 / 16, n_splits=n_splits)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("ty", [oracle.F16, oracle.Q8_0])
@pytest.mark.parametrize("n_q,n_seq", [(2, 1), (5, 1), (3, 3), (9, 2)])
def test_multi_query_and_sequences(ty, n_q, n_seq):
    q, k, v, m = make_case(11 * n_q + n_seq, ty, 256, 24, 4, 900, n_q=n_q, n_seq=n_seq,
                           mask="causal")
    got, want = run_both(q, k, v, m, ty, 1.0 / 16)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("ty", [oracle.F16, oracle.Q8_0, oracle.Q4_0])
@pytest.mark.parametrize("D,n_head,n_hkv,n_q", [(128, 16, 2, 3), (256, 16, 2, 4),
                                                (128, 12, 2, 5), (256, 32, 4, 7)])
def test_two_block_ctas(ty, D, n_head, n_hkv, n_q):
    """More than 16 (query, head) rows per KV head: each CTA serves two 8-row
    blocks from every K/V group it loads -- full pairs (32 rows), a pair whose
    second block is empty (24 rows) or partly filled (30 rows: 16 + 14)."""
    q, k, v, m = make_case(D + 7 * n_q + ty, ty, D, n_head, n_hkv, 1700, n_q=n_q,
                           mask="causal")
    for n_splits in (1, 0):
        got, want = run_both(q, k, v, m, ty, D ** -0.5, n_splits=n_splits)
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL, err_msg=str(n_splits))


@pytest.mark.parametrize("ty", [oracle.F16, oracle.Q4_0])
def test_two_block_ctas_softcap_alibi_sinks(ty):
    """Per-row ALiBi slopes, sinks and the mask row of each (query, head) row
    inside a two-block CTA (20 heads over 2 KV heads, 3 queries: 30 rows)."""
    q, k, v, m = make_case(13, ty, 128, 20, 2, 1200, n_q=3, mask="random")
    sinks = np.random.default_rng(2).normal(0, 1, 20).astype(np.float32)
    for kw in ({"softcap": 30.0}, {"max_bias": 8.0}, {"sinks": sinks}):
        for n_splits in (1, 0):
            got, want = run_both(q, k, v, m, ty, 0.3, n_splits=n_splits, **kw)
            np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL, err_msg=str(kw))


def test_kv_sequence_broadcast():
    q, k, v, m = make_case(5, oracle.Q8_0, 128, 8, 2, 600, n_seq=4, n_seq_kv=2)
    got, want = run_both(q, k, v, m, oracle.Q8_0, 128 ** -0.5)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


def test_mask_softcap_alibi_sinks():
    q, k, v, m = make_case(7, oracle.F16, 128, 8, 2, 1500, n_q=2, mask="random")
    sinks = np.random.default_rng(1).normal(0, 1, 8).astype(np.float32)
    for kw in ({"softcap": 30.0}, {"max_bias": 8.0}, {"sinks": sinks}, {}):
        for n_splits in (1, 0):
            got, want = run_both(q, k, v, m, oracle.F16, 0.3, n_splits=n_splits, **kw)
            np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL, err_msg=str(kw))


def test_fully_masked_rows_are_zero():
    q, k, v, _ = make_case(9, oracle.Q4_0, 128, 4, 4, 300)
    m = np.full((1, 1, 1, 300), -np.inf, np.float16)
    got, want = run_both(q, k, v, m, oracle.Q4_0, 0.1, n_splits=3)
    assert np.all(got == 0) and np.all(want == 0)


def test_strided_q_view_and_canaries():
    """q as a permuted view of [n_q][n_head][D] (ggml's permute of the Q
    projection); the destination is surrounded by canaries that must survive."""
    xq = _xq()
    rng = np.random.default_rng(21)
    D, H, Hkv, n_kv = 256, 16, 2, 2048
    qbuf = rng.normal(0, 1, (1, 1, H, D)).astype(np.float32)  # [seq][q][head][D]
    q = np.ascontiguousarray(qbuf)
    kf = rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32)
    k = oracle.quantize(oracle.Q8_0, kf)
    v = oracle.quantize(oracle.Q8_0, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))
    tq = torch.from_numpy(q).cuda().permute(0, 2, 1, 3)  # (n_seq, n_head, n_q, D) view
    canary = torch.full((H * D + 2048,), 1e30, dtype=torch.float32, device="cuda")
    out = canary[1024:1024 + H * D].view(1, 1, H, D)
    tk, tv = torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()
    before_k = tk.clone()
    xq.flash_attn_ext(tq, tk, tv, oracle.Q8_0, scale=1 / 16, out=out)
    torch.cuda.synchronize()
    want = oracle.flash_attn_ext(np.ascontiguousarray(q.transpose(0, 2, 1, 3)), k, v,
                                 oracle.Q8_0, oracle.Q8_0, scale=1 / 16)
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=RTOL, atol=ATOL)
    c = canary.cpu().numpy()
    assert np.all(c[:1024] == np.float32(1e30)) and np.all(c[1024 + H * D:] == np.float32(1e30))
    assert torch.equal(before_k, tk)


def test_unsupported_types_fail_loudly():
    xq = _xq()
    q = torch.zeros((1, 4, 1, 96), device="cuda")
    k = torch.zeros((1, 64, 4, 192), dtype=torch.uint8, device="cuda")
    with pytest.raises(xq.XqError):
        xq.flash_attn_ext(q, k, k, oracle.F16)


@pytest.mark.parametrize("ty,D,H,Hkv,n_kv,n_q", [(oracle.Q8_0, 256, 16, 2, 32768, 1),
                                                  (oracle.F16, 128, 16, 4, 4096, 1),
                                                  (oracle.Q4_0, 256, 24, 4, 3000, 3)])
def test_pinned_host_q_and_out(ty, D, H, Hkv, n_kv, n_q):
    """q and the output may live in pinned host memory: the library copies q
    to the GPU with a kernel and writes the result in place; the output is
    the same as with device buffers."""
    xq = _xq()
    rng = np.random.default_rng(77)
    qn = rng.normal(0, 1, (1, H, n_q, D)).astype(np.float32)
    k = torch.from_numpy(oracle.quantize(ty, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))).cuda()
    v = torch.from_numpy(oracle.quantize(ty, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))).cuda()
    want = xq.flash_attn_ext(torch.from_numpy(qn).cuda(), k, v, ty, scale=D ** -0.5).cpu()
    q_host = torch.from_numpy(qn).pin_memory()
    out_host = torch.full((1, n_q, H, D), float("nan"), dtype=torch.float32).pin_memory()
    for _ in range(2):
        xq.flash_attn_ext(q_host, k, v, ty, scale=D ** -0.5, out=out_host)
        torch.cuda.synchronize()
        assert torch.equal(out_host, want)
    with pytest.raises(Exception):
        xq.flash_attn_ext(torch.from_numpy(qn), k, v, ty, scale=D ** -0.5)  # pageable q


def _ws_call(q, k, v, ty, scale, out, ws, n_splits=0, sinks=None):
    import ctypes as C

    from xq import _lib
    from xq.ops import _fa_params, _stream
    p = _fa_params(q, k, v, ty, ty, None, sinks, out, scale, 0.0, 0.0, n_splits)
    rc = _lib.lib().xq_flash_attn_ext(C.byref(p), ws.data_ptr(), ws.numel(), _stream(None))
    assert rc == 0, _lib.lib().xq_last_error()


@pytest.mark.parametrize("ty,D,H,Hkv,n_kv,n_splits", [
    (oracle.Q8_0, 256, 16, 2, 32768, 0), (oracle.F16, 128, 16, 4, 4096, 0),
    (oracle.Q4_0, 256, 16, 2, 9000, 37), (oracle.Q8_0, 128, 8, 1, 5000, 3)])
def test_any_workspace_contents_graph_replays_and_the_split_records(ty, D, H, Hkv, n_kv,
                                                                     n_splits):
    """xq_flash_attn_ext with a caller workspace of any contents (random
    bytes, then the previous call's leftovers) and under CUDA-graph replays
    gives the same bits every time; the result equals the split records
    (xq_fa_partials) merged by xq_lse_merge within fp32 rounding, and the
    oracle within the north-star tolerance."""
    xq = _xq()
    q, k, v, _ = make_case(31 + n_kv, ty, D, H, Hkv, n_kv)
    dev = torch.device("cuda")
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    scale = D ** -0.5
    nbytes = xq.flash_attn_ext_workspace(tq, tk, tv, ty, n_splits=n_splits)
    ws = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device=dev)
    outs = []
    for _ in range(3):
        o = torch.full((1, 1, H, D), float("nan"), device=dev)
        _ws_call(tq, tk, tv, ty, scale, o, ws, n_splits)
        outs.append(o)
    ws.random_(0, 256)
    o = torch.empty((1, 1, H, D), device=dev)
    _ws_call(tq, tk, tv, ty, scale, o, ws, n_splits)
    outs.append(o)
    og = torch.empty((1, 1, H, D), device=dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        _ws_call(tq, tk, tv, ty, scale, og, ws, n_splits)
    for _ in range(3):
        og.zero_()
        g.replay()
        torch.cuda.synchronize()
        outs.append(og.clone())
    del g
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    # the same split records through the separate merge kernel
    kern, nsp, rows = xq.flash_attn_ext_plan(tq, tk, tv, ty, n_splits=n_splits)
    assert kern == 1 and nsp >= 1
    part = xq.fa_partials(tq, tk, tv, ty, rows, 0, nsp, scale=scale)
    two, _ = xq.lse_merge(part, want_lse=False)
    torch.cuda.synchronize()
    # the same plan, the same kernels: the same bits
    assert torch.equal(outs[0].view(H, D), two)
    want = oracle.flash_attn_ext(q, k, v, ty, ty, scale=scale, nth=8)
    np.testing.assert_allclose(outs[0].cpu().numpy(), want, rtol=RTOL, atol=ATOL)


def test_a_non_finite_value_poisons_its_rows_through_the_merge():
    """A NaN block scale in one V row of KV head 0 (config 2, 148 splits): the
    merge poisons every q head of that KV head (ggml-cpu's result is NaN there
    too) and leaves KV head 1's heads finite."""
    xq = _xq()
    ty, D, H, Hkv, n_kv = oracle.Q8_0, 256, 16, 2, 32768
    q, k, v, _ = make_case(5, ty, D, H, Hkv, n_kv)
    v = v.copy()
    v[0, 20000, 0, 0:2] = np.frombuffer(np.float16(np.nan).tobytes(), np.uint8)
    dev = torch.device("cuda")
    got = xq.flash_attn_ext(*(torch.from_numpy(x).to(dev) for x in (q, k, v)), ty, scale=1 / 16)
    got = got.cpu().numpy()
    assert np.all(np.isnan(got[0, 0, :8])) and np.all(np.isfinite(got[0, 0, 8:]))
