"""B200 parity: tensor-core prefill (FLASH_ATTN_EXT with many queries, F16 K/V).

The GPU rounds q to f16 and accumulates in fp32 (TMEM); the oracle is ggml-cpu's
scalar one_chunk path (q -> f16, F16 dot, fp16 value accumulator).  Tolerance
|gpu - cpu| <= 2e-3 + 1e-2 |cpu|.  The full BASELINE config 4 (8192 tokens,
24 Q / 4 KV heads, D=256, causal) is checked on sampled query rows.
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def causal_mask(n_q, n_kv):
    m = np.zeros((1, 1, n_q, n_kv), np.float16)
    for i in range(n_q):
        m[0, 0, i, n_kv - n_q + i + 1:] = -np.inf
    return m


def run(q, k, v, m, scale):
    import xq
    dev = torch.device("cuda")
    out = xq.flash_attn_ext(torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev),
                            torch.from_numpy(v).to(dev), oracle.F16,
                            mask=torch.from_numpy(m).to(dev) if m is not None else None,
                            scale=scale)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("D,H,Hkv,n_q,n_kv,mask", [
    (128, 4, 1, 128, 128, "causal"), (256, 2, 1, 128, 128, "causal"),
    (256, 6, 2, 200, 200, "causal"), (128, 8, 2, 256, 384, "causal"),
    (256, 4, 4, 130, 130, "none"), (128, 4, 2, 192, 320, "random"),
    (256, 24, 4, 256, 256, "causal")])
def test_prefill_parity(D, H, Hkv, n_q, n_kv, mask):
    rng = np.random.default_rng(D + H + n_q + n_kv)
    q = rng.normal(0, 1, (1, H, n_q, D)).astype(np.float32)
    k = oracle.quantize(oracle.F16, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))
    v = oracle.quantize(oracle.F16, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))
    if mask == "causal":
        m = causal_mask(n_q, n_kv)
    elif mask == "random":
        m = np.zeros((1, 1, n_q, n_kv), np.float16)
        m[rng.random(m.shape) < 0.4] = -np.inf
        m[0, 0, 5, :] = -np.inf   # one fully masked row -> zeros
    else:
        m = None
    scale = D ** -0.5
    got = run(q, k, v, m, scale)
    want = oracle.flash_attn_ext(q, k, v, oracle.F16, oracle.F16, mask=m, scale=scale,
                                 policy=oracle.FA_SCALAR)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    if mask == "random":
        assert np.all(got[0, 5] == 0)


def test_prefill_strided_q_and_sequences():
    """q as ggml's permuted view of [n_seq][n_q][n_head][D]; two sequences."""
    import xq
    rng = np.random.default_rng(3)
    D, H, Hkv, n_q, n_kv, S = 128, 4, 2, 160, 160, 2
    qb = rng.normal(0, 1, (S, n_q, H, D)).astype(np.float32)
    k = oracle.quantize(oracle.F16, rng.normal(0, 1, (S, n_kv, Hkv, D)).astype(np.float32))
    v = oracle.quantize(oracle.F16, rng.normal(0, 1, (S, n_kv, Hkv, D)).astype(np.float32))
    m = causal_mask(n_q, n_kv)
    tq = torch.from_numpy(qb).cuda().permute(0, 2, 1, 3)
    got = xq.flash_attn_ext(tq, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(),
                            oracle.F16, mask=torch.from_numpy(m).cuda(), scale=D ** -0.5)
    want = oracle.flash_attn_ext(np.ascontiguousarray(qb.transpose(0, 2, 1, 3)), k, v,
                                 oracle.F16, oracle.F16, mask=m, scale=D ** -0.5,
                                 policy=oracle.FA_SCALAR)
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=RTOL, atol=ATOL)


def test_c4_config_sampled_rows():
    """BASELINE config 4 at full size: 8192 tokens, 24 Q / 4 KV heads, D=256,
    causal; 12 query rows (spread over every query tile position) vs the oracle."""
    import xq
    N, H, Hkv, D = 8192, 24, 4, 256
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    q = torch.randn((1, H, N, D), generator=g, device="cuda")
    kf = torch.randn((1, N, Hkv, D), generator=g, device="cuda")
    vf = torch.randn((1, N, Hkv, D), generator=g, device="cuda")
    k = xq.quantize_rows(oracle.F16, kf)
    v = xq.quantize_rows(oracle.F16, vf)
    mask = torch.zeros((1, 1, N, N), dtype=torch.float16, device="cuda")
    mask.masked_fill_(torch.triu(torch.ones(N, N, dtype=torch.bool, device="cuda"), 1)[None, None],
                      float("-inf"))
    out = xq.flash_attn_ext(q, k, v, oracle.F16, mask=mask, scale=1 / 16)
    torch.cuda.synchronize()
    rows = np.array([0, 1, 127, 128, 255, 1000, 4095, 4096, 6001, 8063, 8190, 8191])
    qs = q[:, :, rows, :].cpu().numpy()
    ms = mask[:, :, rows, :].cpu().numpy()
    want = oracle.flash_attn_ext(np.ascontiguousarray(qs), k.cpu().numpy(), v.cpu().numpy(),
                                 oracle.F16, oracle.F16, mask=ms, scale=1 / 16,
                                 policy=oracle.FA_SCALAR)
    got = out[:, rows].cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


def _quant_prefill_case(seed, ty, H, Hkv, D, n_q, n_kv, n_seq=1):
    rng = np.random.default_rng(seed)
    q = rng.normal(0, 1, (n_seq, H, n_q, D)).astype(np.float32)
    k = oracle.quantize(ty, rng.normal(0, 1, (n_seq, n_kv, Hkv, D)).astype(np.float32))
    v = oracle.quantize(ty, rng.normal(0, 1, (n_seq, n_kv, Hkv, D)).astype(np.float32))
    return q, k, v, causal_mask(n_q, n_kv)


@pytest.mark.parametrize("ty", [oracle.Q8_0, oracle.Q4_0])
@pytest.mark.parametrize("n_q,n_kv", [(64, 2048), (512, 1024), (200, 700)])
def test_quantized_kv_prefill_parity(ty, n_q, n_kv):
    """A prompt chunk over a Q8_0 / Q4_0 cache -- the reference's product
    configuration (a quantized KV cache forces flash attention on; prompts go
    in as n_batch-token chunks) -- with the BASELINE config-4 head shape (24 Q
    / 4 KV heads, D=256), causal over the tail of the cache.  ggml-cpu takes
    these through one_chunk whatever the query count (its tiled path needs
    F16/F32 K/V): q quantized to Q8_0, integer block dots, V dequantized to
    f32.  Ragged last query and key tiles in the (200, 700) case."""
    import xq
    q, k, v, m = _quant_prefill_case(1000 + n_q + ty, ty, 24, 4, 256, n_q, n_kv)
    dev = torch.device("cuda")
    got = xq.flash_attn_ext(torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev),
                            torch.from_numpy(v).to(dev), ty, mask=torch.from_numpy(m).to(dev),
                            scale=1 / 16)
    torch.cuda.synchronize()
    want = oracle.flash_attn_ext(q, k, v, ty, ty, mask=m, scale=1 / 16)
    got = got.cpu().numpy()
    assert np.all(np.isfinite(got))
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("ty", [oracle.Q8_0, oracle.Q4_0])
def test_quantized_kv_prefill_two_sequences_no_mask(ty):
    """Two sequences with their own caches, no mask, D=128, GQA 4."""
    import xq
    q, k, v, _ = _quant_prefill_case(77 + ty, ty, 8, 2, 128, 130, 300, n_seq=2)
    dev = torch.device("cuda")
    got = xq.flash_attn_ext(torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev),
                            torch.from_numpy(v).to(dev), ty, scale=128 ** -0.5)
    torch.cuda.synchronize()
    want = oracle.flash_attn_ext(q, k, v, ty, ty, scale=128 ** -0.5)
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=RTOL, atol=ATOL)
