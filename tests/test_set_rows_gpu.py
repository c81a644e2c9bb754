"""B200 parity: GGML_OP_SET_ROWS (the KV-cache write) through the C ABI.

F32 rows are quantized on the GPU and scattered to the cache rows named by
I32/I64 indices, with ggml's broadcast of the index tensor over heads and
sequences.  The result must be bit-identical to the oracle (ggml's reference
quantizers, pinned against gguf), and every row not named must keep its old
bytes.
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _xq():
    import xq
    return xq


def _cache(rng, ty, n_seq, n_rows, n_hkv, D):
    if ty == oracle.F32:
        return rng.normal(0, 1, (n_seq, n_rows, n_hkv, D)).astype(np.float32)
    return oracle.quantize(ty, rng.normal(0, 1, (n_seq, n_rows, n_hkv, D)).astype(np.float32))


@pytest.mark.parametrize("ty", [oracle.F16, oracle.Q8_0, oracle.Q4_0, oracle.F32])
@pytest.mark.parametrize("itype", [np.int64, np.int32])
def test_set_rows_decode_append(ty, itype):
    """One decode step's K rows for 2 KV heads land at scattered positions."""
    xq = _xq()
    rng = np.random.default_rng(ty * 10 + (itype == np.int32))
    n_seq, n_rows, n_hkv, D, n_tok = 1, 96, 2, 256, 5
    cache = _cache(rng, ty, n_seq, n_rows, n_hkv, D)
    src = rng.normal(0, 1.5, (n_seq, n_tok, n_hkv, D)).astype(np.float32)
    idx = rng.choice(n_rows, n_tok, replace=False).astype(itype)
    want = oracle.set_rows(cache, src, idx, ty)
    got = xq.set_rows(torch.from_numpy(cache).cuda(), torch.from_numpy(src).cuda(),
                      torch.from_numpy(idx).cuda(), ty).cpu().numpy()
    assert np.array_equal(got.view(np.uint8), want.view(np.uint8))


@pytest.mark.parametrize("ty", [oracle.Q8_0, oracle.Q4_0])
def test_set_rows_prefill_broadcast_and_row_layout(ty):
    """A prefill batch written with an index tensor broadcast over heads
    (i1 = 1) and per sequence (i2 = n_seq), plus llama.cpp's 2D cache layout
    (one row = all KV heads of a token); an out-of-range index skips its row."""
    xq = _xq()
    rng = np.random.default_rng(21 + ty)
    n_seq, n_rows, n_hkv, D, n_tok = 2, 300, 4, 128, 70
    cache = _cache(rng, ty, n_seq, n_rows, n_hkv, D)
    src = rng.normal(0, 1, (n_seq, n_tok, n_hkv, D)).astype(np.float32)
    idx = np.stack([rng.choice(n_rows, n_tok, replace=False) for _ in range(n_seq)])
    idx = idx.reshape(n_seq, 1, n_tok).astype(np.int64)
    idx[1, 0, 3] = n_rows + 5  # skipped
    want = oracle.set_rows(cache, src, idx, ty)
    got = xq.set_rows(torch.from_numpy(cache).cuda(), torch.from_numpy(src).cuda(),
                      torch.from_numpy(idx).cuda(), ty).cpu().numpy()
    assert np.array_equal(got, want)
    # llama.cpp layout: cache [n_embd_k_gqa = n_hkv * D, kv_size]
    cache2 = _cache(rng, ty, 1, n_rows, 1, n_hkv * D)
    src2 = src[:1].reshape(1, n_tok, 1, n_hkv * D).copy()
    idx2 = np.arange(40, 40 + n_tok, dtype=np.int32)
    want2 = oracle.set_rows(cache2, src2, idx2, ty)
    got2 = xq.set_rows(torch.from_numpy(cache2).cuda(), torch.from_numpy(src2).cuda(),
                       torch.from_numpy(idx2).cuda(), ty).cpu().numpy()
    assert np.array_equal(got2, want2)


def test_set_rows_then_decode_reads_the_new_rows():
    """Quantize-on-append followed by flash-attn decode over the cache equals
    decoding the oracle-quantized cache."""
    xq = _xq()
    rng = np.random.default_rng(5)
    D, H, Hkv, n_kv = 256, 16, 2, 4096
    kc = oracle.quantize(oracle.Q8_0, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))
    vc = oracle.quantize(oracle.Q8_0, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))
    knew = rng.normal(0, 1, (1, 1, Hkv, D)).astype(np.float32)
    vnew = rng.normal(0, 1, (1, 1, Hkv, D)).astype(np.float32)
    pos = np.array([n_kv - 1], np.int64)
    kd, vd = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    xq.set_rows(kd, torch.from_numpy(knew).cuda(), torch.from_numpy(pos).cuda(), oracle.Q8_0)
    xq.set_rows(vd, torch.from_numpy(vnew).cuda(), torch.from_numpy(pos).cuda(), oracle.Q8_0)
    q = rng.normal(0, 1, (1, H, 1, D)).astype(np.float32)
    got = xq.flash_attn_ext(torch.from_numpy(q).cuda(), kd, vd, oracle.Q8_0, scale=1 / 16)
    k2 = oracle.set_rows(kc, knew, pos, oracle.Q8_0)
    v2 = oracle.set_rows(vc, vnew, pos, oracle.Q8_0)
    want = oracle.flash_attn_ext(q, k2, v2, oracle.Q8_0, oracle.Q8_0, scale=1 / 16)
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-2, atol=2e-3)


@pytest.mark.parametrize("ty", [oracle.F16, oracle.Q8_0, oracle.Q4_0, oracle.F32])
@pytest.mark.parametrize("width", [256, 768, 1024, 4096, 4352])
def test_set_rows_row_widths_and_edge_blocks(ty, width):
    """Row widths through the warp-per-row kernel (1, 6, 8 and 32 float4
    units per lane) and past its 4096-element limit (the per-block kernel),
    with an all-zero block, a block whose largest magnitude appears twice with
    both signs (Q4_0 keeps the first), tiny and large magnitudes, and a row
    whose index is negative (left untouched)."""
    xq = _xq()
    rng = np.random.default_rng(1000 + width + ty)
    n_rows, n_tok = 64, 9
    cache = _cache(rng, ty, 1, n_rows, 1, width)
    src = rng.normal(0, 1, (1, n_tok, 1, width)).astype(np.float32)
    src[0, 0, 0, 32:64] = 0.0
    src[0, 1, 0, 0:32] = rng.normal(0, 1, 32).astype(np.float32)
    src[0, 1, 0, 5], src[0, 1, 0, 20] = 3.0, -3.0
    src[0, 2, 0, :32] *= 1e-30
    src[0, 3, 0, 64:96] *= 1e6
    idx = rng.choice(n_rows, n_tok, replace=False).astype(np.int64)
    idx[4] = -1
    want = oracle.set_rows(cache, src, idx, ty)
    got = xq.set_rows(torch.from_numpy(cache).cuda(), torch.from_numpy(src).cuda(),
                      torch.from_numpy(idx).cuda(), ty).cpu().numpy()
    assert np.array_equal(got.view(np.uint8), want.view(np.uint8))


@pytest.mark.parametrize("ty", [oracle.F16, oracle.Q8_0, oracle.Q4_0, oracle.F32])
@pytest.mark.parametrize("D", [256, 512])
def test_set_rows_per_head_indices_several_rows_per_warp(ty, D):
    """Per-head, per-sequence index tensors (i1 = n_head_kv, i2 = n_seq) with
    rows of 256 and 512 elements, where the row kernel takes four or two rows
    per warp; row counts that leave the last warp partly empty, and two
    skipped rows."""
    xq = _xq()
    rng = np.random.default_rng(77 + D + ty)
    n_seq, n_rows, n_hkv, n_tok = 2, 50, 4, 7
    cache = _cache(rng, ty, n_seq, n_rows, n_hkv, D)
    src = rng.normal(0, 1, (n_seq, n_tok, n_hkv, D)).astype(np.float32)
    idx = np.stack([np.stack([rng.choice(n_rows, n_tok, replace=False) for _ in range(n_hkv)])
                    for _ in range(n_seq)]).astype(np.int32)
    idx[0, 1, 2] = -3
    idx[1, 3, 6] = n_rows
    want = oracle.set_rows(cache, src, idx, ty)
    got = xq.set_rows(torch.from_numpy(cache).cuda(), torch.from_numpy(src).cuda(),
                      torch.from_numpy(idx).cuda(), ty).cpu().numpy()
    assert np.array_equal(got.view(np.uint8), want.view(np.uint8))
