"""The CPU oracle pinned against the reference's own fixtures (no GPU).

Golden files come from tests/golden/make_golden.py: gguf 0.19.0 codecs, the
reference's numpy models of its RKVA decode kernels and LSE reducer, and the
reference's compiled GDN host mirror (src/bridge/ggml_d3d12.cpp:113-158).
"""
import numpy as np
import pytest

import oracle
from conftest import golden


def test_fp16_conversion_matches_numpy_rne():
    g = golden("codecs.npz")
    assert np.array_equal(oracle.fp16_bits(g["f16_in"]), g["f16_bits"])


@pytest.mark.parametrize("ty,key", [(oracle.Q8_0, "q8"), (oracle.Q4_0, "q4")])
def test_block_codecs_bit_exact_vs_gguf(ty, key):
    g = golden("codecs.npz")
    raw = oracle.quantize(ty, g["x"])
    assert np.array_equal(raw, g[key]), "quantizer differs from gguf/ggml reference"
    deq = oracle.dequantize(ty, g[key], g["x"].shape[-1])
    assert np.array_equal(deq.view(np.uint32), g[key + "_deq"].astype(np.float32).view(np.uint32))


def test_split_policy_matches_reference_model():
    g = golden("split_policy.npz")
    for a, row in zip(g["active"], g["split_k"]):
        assert [oracle.split_k(int(a), m) for m in range(4)] == list(row)


@pytest.mark.parametrize("name,storage", [("f16", oracle.F16), ("q8_0", oracle.Q8_0),
                                          ("q4_0", oracle.Q4_0)])
def test_range_attention_vs_reference_models(name, storage):
    g = golden(f"range_{name}.npz")
    H, Hkv, D = (int(x) for x in g["shape"])
    cases = sorted({k.split("_")[0] for k in g.files if k.startswith("c")})
    for c in cases:
        active, pos, origin, limit, sk = (int(x) for x in g[c + "_meta"])
        out, lse = oracle.range_attn(storage, g[c + "_k"], g[c + "_v"], g[c + "_q"],
                                     np.array([pos], np.int32), active, origin, H, Hkv, D,
                                     1.0 / 16.0, split=sk)
        out = out[0]
        lse = lse[0]
        ref_o, ref_l = g[c + "_oref"], g[c + "_lref"]
        assert np.array_equal(np.isneginf(lse), np.isneginf(ref_l))
        # float32 restatement of the same kernel + reducer; only the order of
        # the float32 dot-product sums differs from the numpy model
        scale = max(1.0, float(np.abs(ref_o).max()))
        np.testing.assert_allclose(out, ref_o, rtol=1e-4, atol=1e-5 * scale)
        fin = ~np.isneginf(ref_l)
        np.testing.assert_allclose(lse[fin], ref_l[fin], rtol=1e-5, atol=1e-4)
        # and against the float64 oracle
        np.testing.assert_allclose(out, g[c + "_o64"], rtol=1e-4, atol=2e-5 * scale)


def test_lse_merge_poison_and_empty_semantics():
    g = golden("reduce.npz")
    names = sorted({k.rsplit("_", 1)[0] for k in g.files if k.endswith("_partials")})
    for n in names:
        out, lse = oracle.lse_merge(g[n + "_partials"])
        ro, rl = g[n + "_out"], g[n + "_lse"]
        assert np.array_equal(np.isnan(out), np.isnan(ro)), n
        assert np.array_equal(np.isnan(lse), np.isnan(rl)), n
        fin = ~np.isnan(ro)
        np.testing.assert_allclose(out[fin], ro[fin], rtol=1e-6, atol=1e-7, err_msg=n)
        fl = ~np.isnan(rl)
        np.testing.assert_allclose(lse[fl], rl[fl], rtol=1e-6, atol=1e-6, err_msg=n)


def test_std_mt19937_restatement_matches_libstdcxx():
    g = golden("gdn_selftest.npz")
    for j in range(6):
        mine = oracle.std_uniform(1701 + j, -0.05, 0.05, 64)
        assert np.array_equal(mine.view(np.uint32), g["std_uniform_1701_1706"][j].view(np.uint32))


@pytest.mark.parametrize("T,K,pad", [(5, 5, 0), (1, 5, 0), (2, 5, 0), (3, 5, 0), (4, 5, 0),
                                     (64, 5, 0), (5, 1, 0), (1, 1, 0), (64, 1, 0), (3, 5, 3),
                                     (4, 5, 3)])
def test_gdn_oracle_vs_reference_host_mirror(T, K, pad):
    g = golden("gdn_selftest.npz")
    key = f"T{T}_K{K}_p{pad}"
    views, _ = oracle.gdn_selftest_inputs(T, pad)
    for lanes8 in (True, False):
        _, y, snaps = oracle.gated_delta_net(*views, slots=K, lanes8=lanes8, n_workers=4)
        y = y[0]
        written = min(T, K)
        s = snaps[:written, 0].reshape(written, 32, -1)
        if lanes8:  # same eight-lane order as the reference mirror: bit-exact
            assert np.array_equal(y[:min(T, 5)].view(np.uint32), g[key + "_y_head"].view(np.uint32))
            assert np.array_equal(s.reshape(written, -1)[:, g["snap_sample_idx"]].view(np.uint32),
                                  g[key + "_snap_sample"].view(np.uint32))
        ref_max = np.abs(g[key + "_y_head"]).max()
        rel = np.abs(y[:min(T, 5)] - g[key + "_y_head"]).max() / ref_max
        assert rel <= 1e-4  # the reference selftest's own bound
        np.testing.assert_allclose(y.astype(np.float64).sum(axis=2), g[key + "_y_sum"],
                                   rtol=1e-4, atol=1e-6)
        np.testing.assert_allclose(s.astype(np.float64).sum(axis=2), g[key + "_snap_sum"],
                                   rtol=1e-4, atol=1e-4)
        np.testing.assert_allclose((s.astype(np.float64) ** 2).sum(axis=2), g[key + "_snap_sq"],
                                   rtol=1e-5)


def test_fa_oracle_modes_agree_with_float64():
    rng = np.random.default_rng(0)
    D, H, Hkv, n_kv = 128, 16, 4, 1024
    q = rng.normal(0, 1, (1, H, 1, D)).astype(np.float32)
    kf = rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32)
    vf = rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32)
    for ty in (oracle.F16, oracle.Q8_0, oracle.Q4_0):
        k, v = oracle.quantize(ty, kf), oracle.quantize(ty, vf)
        ref, _ = oracle.flash_attn_ext(q, k, v, ty, ty, scale=D ** -0.5, f64=True)
        for policy, nosplit, nth in ((oracle.FA_NATIVE, False, 8), (oracle.FA_NATIVE, True, 1),
                                     (oracle.FA_POLICY4, True, 1)):
            got = oracle.flash_attn_ext(q, k, v, ty, ty, scale=D ** -0.5, policy=policy,
                                        no_split_kv=nosplit, nth=nth)
            np.testing.assert_allclose(got, ref, rtol=1e-2, atol=2e-3)
