"""B200 parity: RKVA range attention, split partials + LSE merge, block codecs.

Golden files are the reference's own numpy models (range_*.npz, reduce.npz)
and gguf 0.19.0 codecs (codecs.npz); see tests/golden/make_golden.py.
"""
import numpy as np
import pytest
import torch

import oracle
from conftest import golden

pytestmark = pytest.mark.gpu


def _xq():
    import xq
    return xq


@pytest.mark.parametrize("name,storage", [("f16", oracle.F16), ("q8_0", oracle.Q8_0),
                                          ("q4_0", oracle.Q4_0)])
@pytest.mark.parametrize("mode", [0, 1, 2, 3, 4])
def test_attend_range_vs_reference_models(name, storage, mode):
    xq = _xq()
    g = golden(f"range_{name}.npz")
    H, Hkv, D = (int(x) for x in g["shape"])
    cases = sorted({k.split("_")[0] for k in g.files if k.startswith("c")})
    for c in cases:
        active, pos, origin, limit, _ = (int(x) for x in g[c + "_meta"])
        k = torch.from_numpy(g[c + "_k"]).cuda()
        v = torch.from_numpy(g[c + "_v"]).cuda()
        q = torch.from_numpy(g[c + "_q"]).cuda().view(1, H, D)
        p = torch.tensor([pos], dtype=torch.int32, device="cuda")
        out, lse = xq.attend_range(storage, k, v, q, p, Hkv, origin, active, 1.0 / 16, mode)
        out, lse = out.cpu().numpy()[0], lse.cpu().numpy()[0]
        ref_o, ref_l = g[c + "_o64"], g[c + "_l64"]
        assert np.array_equal(np.isneginf(lse), np.isneginf(ref_l)), c
        scale = max(1.0, float(np.abs(ref_o).max()))
        np.testing.assert_allclose(out, ref_o, rtol=1e-4, atol=2e-5 * scale, err_msg=c)
        fin = ~np.isneginf(ref_l)
        np.testing.assert_allclose(lse[fin], ref_l[fin], rtol=1e-5, atol=1e-4, err_msg=c)
        if limit == 0:
            assert np.all(out == 0)


def test_attend_range_multi_token_causal():
    xq = _xq()
    rng = np.random.default_rng(4)
    H, Hkv, D, active, origin = 24, 4, 256, 700, 5000
    kf = rng.normal(0, 1, (active, Hkv, D)).astype(np.float32)
    vf = rng.normal(0, 1, (active, Hkv, D)).astype(np.float32)
    k, v = oracle.quantize(oracle.Q8_0, kf), oracle.quantize(oracle.Q8_0, vf)
    q = rng.normal(0, 1, (6, H, D)).astype(np.float32)
    pos = np.array([origin - 3, origin, origin + 17, origin + 350, origin + 699, origin + 5000],
                   np.int32)
    ro, rl = oracle.range_attn(oracle.Q8_0, k, v, q, pos, active, origin, H, Hkv, D, 1 / 16,
                               split=3)
    for mode in (0, 2, 4):
        out, lse = xq.attend_range(oracle.Q8_0, torch.from_numpy(k).cuda(),
                                   torch.from_numpy(v).cuda(), torch.from_numpy(q).cuda(),
                                   torch.from_numpy(pos).cuda(), Hkv, origin, active, 1 / 16, mode)
        out, lse = out.cpu().numpy(), lse.cpu().numpy()
        np.testing.assert_allclose(out, ro, rtol=1e-3, atol=1e-5)
        assert np.array_equal(np.isneginf(lse), np.isneginf(rl))
        fin = ~np.isneginf(rl)
        np.testing.assert_allclose(lse[fin], rl[fin], rtol=1e-5, atol=1e-4)


def test_lse_merge_golden_semantics():
    xq = _xq()
    g = golden("reduce.npz")
    names = sorted({k.rsplit("_", 1)[0] for k in g.files if k.endswith("_partials")})
    for n in names:
        part = torch.from_numpy(g[n + "_partials"]).cuda()
        out, lse = xq.lse_merge(part)
        out, lse = out.cpu().numpy(), lse.cpu().numpy()
        ro, rl = g[n + "_out"], g[n + "_lse"]
        assert np.array_equal(np.isnan(out), np.isnan(ro)), n
        assert np.array_equal(np.isnan(lse), np.isnan(rl)), n
        fin = ~np.isnan(ro)
        np.testing.assert_allclose(out[fin], ro[fin], rtol=1e-6, atol=1e-7, err_msg=n)
        fl = ~np.isnan(rl)
        np.testing.assert_allclose(lse[fl], rl[fl], rtol=1e-6, atol=1e-6, err_msg=n)


def test_partials_merge_equals_flash_attn_and_is_shard_invariant():
    """Fixed global splits: computing them in 1, 2, 4 or 8 shards and merging
    in split order gives bit-identical output."""
    xq = _xq()
    rng = np.random.default_rng(8)
    D, H, Hkv, n_kv, n_seq = 256, 24, 4, 8192, 2
    q = torch.from_numpy(rng.normal(0, 1, (n_seq, H, 1, D)).astype(np.float32)).cuda()
    kf = rng.normal(0, 1, (n_seq, n_kv, Hkv, D)).astype(np.float32)
    vf = rng.normal(0, 1, (n_seq, n_kv, Hkv, D)).astype(np.float32)
    k = torch.from_numpy(oracle.quantize(oracle.Q8_0, kf)).cuda()
    v = torch.from_numpy(oracle.quantize(oracle.Q8_0, vf)).cuda()
    rows, n_splits = 256, n_kv // 256
    ref = None
    for shards in (1, 2, 4, 8):
        per = n_splits // shards
        parts = [xq.fa_partials(q, k, v, oracle.Q8_0, rows, i * per, (i + 1) * per, scale=1 / 16)
                 for i in range(shards)]
        out, _ = xq.lse_merge(torch.cat(parts, 0).contiguous())
        out = out.cpu().numpy()
        if ref is None:
            ref = out
        assert np.array_equal(out.view(np.uint32), ref.view(np.uint32)), shards
    want = oracle.flash_attn_ext(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), oracle.Q8_0,
                                 oracle.Q8_0, scale=1 / 16)
    np.testing.assert_allclose(ref.reshape(want.shape), want, rtol=1e-2, atol=2e-3)


@pytest.mark.parametrize("ty,key", [(oracle.Q8_0, "q8"), (oracle.Q4_0, "q4")])
def test_codecs_bit_exact(ty, key):
    xq = _xq()
    g = golden("codecs.npz")
    raw = torch.from_numpy(g[key]).cuda()
    deq = xq.dequantize_rows(ty, raw.view(g["x"].shape[0], -1), g["x"].shape[1]).cpu().numpy()
    assert np.array_equal(deq.view(np.uint32), g[key + "_deq"].astype(np.float32).view(np.uint32))
    q = xq.quantize_rows(ty, torch.from_numpy(g["x"]).cuda()).cpu().numpy()
    assert np.array_equal(q.reshape(-1), g[key].reshape(-1))


def test_f16_codec_bit_exact():
    xq = _xq()
    g = golden("codecs.npz")
    x = g["f16_in"][: (g["f16_in"].size // 32) * 32].reshape(-1, 32)
    raw = xq.quantize_rows(oracle.F16, torch.from_numpy(x).cuda()).cpu().numpy()
    bits = raw.view(np.uint16).reshape(-1)
    assert np.array_equal(bits, g["f16_bits"][: bits.size])
    back = xq.dequantize_rows(oracle.F16, torch.from_numpy(raw).cuda(), 32).cpu().numpy()
    assert np.array_equal(back.reshape(-1), bits.view(np.float16).astype(np.float32))


@pytest.mark.parametrize("rows", [24, 64])  # cluster kernel / warp-per-row kernel
def test_lse_merge_records_two_level(rows):
    """Group records (O, lse, 1) of xq_lse_merge_records match the oracle's
    per-group merge; empty groups give (0, -FLT_MAX, 0), poisoned rows NaN;
    merging the records equals merging all splits at once."""
    xq = _xq()
    rng = np.random.default_rng(11)
    G, per, D = 4, 5, 256
    part = np.zeros((G * per, rows, D + 2), np.float32)
    part[:, :, :D] = rng.normal(0, 1, (G * per, rows, D))
    part[:, :, D] = rng.normal(0, 2, (G * per, rows))
    part[:, :, D + 1] = rng.uniform(0.5, 3, (G * per, rows))
    part[per:2 * per, 3, :D] = 0.0            # group 1, row 3: empty
    part[per:2 * per, 3, D] = -3.402823466e38
    part[per:2 * per, 3, D + 1] = 0.0
    part[2 * per + 1, 5, 7] = np.nan         # group 2, row 5: poisoned
    rec = xq.lse_merge_records(torch.from_numpy(part).cuda(), per).cpu().numpy()
    for g in range(G):
        o, lse = oracle.lse_merge(part[g * per:(g + 1) * per])
        for r in range(rows):
            if np.isnan(lse[r]):
                assert np.isnan(rec[g, r]).all(), (g, r)
            elif np.isneginf(lse[r]):
                assert (rec[g, r, :D] == 0).all() and rec[g, r, D + 1] == 0
                assert rec[g, r, D] == np.float32(-3.402823466e38)
            else:
                np.testing.assert_allclose(rec[g, r, :D], o[r], rtol=1e-5, atol=1e-6)
                np.testing.assert_allclose(rec[g, r, D], lse[r], rtol=1e-6, atol=1e-6)
                assert rec[g, r, D + 1] == 1.0
    out2, lse2 = xq.lse_merge(torch.from_numpy(rec).cuda())
    out1, lse1 = oracle.lse_merge(part)
    out2, lse2 = out2.cpu().numpy(), lse2.cpu().numpy()
    assert np.array_equal(np.isnan(out2), np.isnan(out1))
    fin = ~np.isnan(out1)
    np.testing.assert_allclose(out2[fin], out1[fin], rtol=1e-4, atol=1e-5)
    fl = ~np.isnan(lse1)
    np.testing.assert_allclose(lse2[fl], lse1[fl], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("rows", [12, 48])  # D = 256: one-wave (staged) / larger grid
@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("n_splits", [1, 37, 148, 2500])
def test_lse_merge_variants_bit_identical(D, n_splits, rows):
    """The cluster merge picks its lane width (and, at D = 128, numerators
    staged in shared memory) from the partials' alignment; every variant sums
    each dim over the same splits in the same order, so partials at an 8-byte
    aligned address and the same records 4 bytes off give the same bits --
    plain, empty, poisoned and record-mode rows alike -- and agree with the
    oracle."""
    xq = _xq()
    rng = np.random.default_rng(D * 7919 + n_splits + rows)
    part = np.zeros((n_splits, rows, D + 2), np.float32)
    part[:, :, :D] = rng.normal(0, 1, (n_splits, rows, D))
    part[:, :, D] = rng.normal(0, 3, (n_splits, rows))
    part[:, :, D + 1] = rng.uniform(0.5, 2.0, (n_splits, rows))
    empty = rng.random((n_splits, rows)) < 0.2
    part[:, :, D + 1][empty] = 0.0
    part[:, :, D][empty] = -3.402823466e38
    part[:, 2, D + 1] = 0.0                         # row 2: every split empty
    part[:, 2, D] = -3.402823466e38
    live = np.nonzero(part[:, 4, D + 1] != 0.0)[0]
    if live.size:
        part[live[-1], 4, 5] = np.inf               # row 4: poisoned
    n = part.size
    buf = torch.zeros(n + 2, dtype=torch.float32, device="cuda")
    aligned = buf[:n].view(part.shape)               # 8-byte aligned (allocator: 256)
    shifted = buf[1:n + 1]                           # 4 bytes off
    assert aligned.data_ptr() % 8 == 0 and shifted.data_ptr() % 8 == 4
    results = []
    for view in (aligned, shifted):
        view.copy_(torch.from_numpy(part).reshape(view.shape).cuda())
        o, lse = xq.lse_merge(view.view(part.shape))
        torch.cuda.synchronize()
        results.append((o.cpu().numpy().view(np.int32), lse.cpu().numpy().view(np.int32)))
    assert np.array_equal(results[0][0], results[1][0])
    assert np.array_equal(results[0][1], results[1][1])
    o_ref, lse_ref = oracle.lse_merge(part)
    o = results[0][0].view(np.float32)
    assert np.array_equal(np.isnan(o), np.isnan(o_ref))
    fin = ~np.isnan(o_ref)
    np.testing.assert_allclose(o[fin], o_ref[fin], rtol=1e-4, atol=1e-5)
    if n_splits % 2 == 0 and n_splits > 1:
        # record mode (two groups), both alignments
        recs = []
        for view in (aligned, shifted):
            view.copy_(torch.from_numpy(part).reshape(view.shape).cuda())
            r = xq.lse_merge_records(view.view(part.shape), n_splits // 2)
            torch.cuda.synchronize()
            recs.append(r.cpu().numpy().view(np.int32))
        assert np.array_equal(recs[0], recs[1])


@pytest.mark.parametrize("D", [128, 256])
@pytest.mark.parametrize("n_splits", [1, 33, 70])
def test_lse_merge_many_rows_four_warps_equal_one_warp(D, n_splits):
    """The warp-per-row merges (many rows, and every record merge) take four
    warps per row when the rows fit one wave (at most two per SM) and one warp
    per row beyond; both add every dim over the splits in split order, so the
    first 160 rows merged alone (four warps) equal the same rows of a 400-row
    merge (one warp) bit for bit -- outputs, lse and records, with empty,
    poisoned and partial-chunk rows -- and match the oracle.  At D = 256 the
    160 rows 4 bytes off (one warp per row: unaligned pairs) agree too."""
    xq = _xq()
    rows, sub = 400, 160
    rng = np.random.default_rng(D + n_splits)
    part = np.zeros((n_splits, rows, D + 2), np.float32)
    part[:, :, :D] = rng.normal(0, 1, (n_splits, rows, D))
    part[:, :, D] = rng.normal(0, 3, (n_splits, rows))
    part[:, :, D + 1] = rng.uniform(0.5, 2.0, (n_splits, rows))
    empty = rng.random((n_splits, rows)) < 0.2
    part[:, :, D + 1][empty] = 0.0
    part[:, :, D][empty] = -3.402823466e38
    part[:, 2, D + 1] = 0.0
    part[:, 2, D] = -3.402823466e38
    live = np.nonzero(part[:, 4, D + 1] != 0.0)[0]
    if live.size:
        part[live[-1], 4, D - 1] = np.nan

    def merged(t):
        o, lse = xq.lse_merge(t)
        r = xq.lse_merge_records(t, n_splits)
        torch.cuda.synchronize()
        return [x.cpu().numpy() for x in (o, lse, r)]

    whole = merged(torch.from_numpy(part).cuda())
    head = np.ascontiguousarray(part[:, :sub])
    alone = merged(torch.from_numpy(head).cuda())
    for a, w in zip(alone, (whole[0][:sub], whole[1][:sub], whole[2][:, :sub])):
        assert np.array_equal(a.view(np.int32), np.ascontiguousarray(w).view(np.int32))
    if D == 256:
        n = head.size
        buf = torch.zeros(n + 2, dtype=torch.float32, device="cuda")
        buf[1:n + 1].copy_(torch.from_numpy(head).reshape(-1).cuda())
        off = merged(buf[1:n + 1].view(head.shape))
        for a, b in zip(alone, off):
            assert np.array_equal(a.view(np.int32), b.view(np.int32))
    o_ref, lse_ref = oracle.lse_merge(head)
    assert np.array_equal(np.isnan(alone[0]), np.isnan(o_ref))
    fin = ~np.isnan(o_ref)
    np.testing.assert_allclose(alone[0][fin], o_ref[fin], rtol=1e-4, atol=1e-5)
    fl = ~np.isnan(lse_ref)
    np.testing.assert_allclose(alone[1][fl], lse_ref[fl], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("rows", [6, 48, 200])
def test_lse_merge_records_of_a_group_block_equal_the_whole(rows):
    """The records of any block of groups equal the same groups' records of
    the whole merge, bit for bit, at few rows as at many: a record comes out of
    one kernel however the groups are spread over GPUs."""
    import xq
    rng = np.random.default_rng(rows)
    n_groups, per, D = 8, 4, 256
    part = rng.normal(0, 1, (n_groups * per, rows, D + 2)).astype(np.float32)
    part[:, :, D] = rng.normal(0, 2, (n_groups * per, rows))
    part[:, :, D + 1] = rng.uniform(0.5, 4, (n_groups * per, rows))
    tp = torch.from_numpy(part).cuda()
    whole = xq.lse_merge_records(tp, per)
    for blocks in (1, 2, 4, 8):
        size = n_groups // blocks
        for b in range(blocks):
            sub = xq.lse_merge_records(tp[b * size * per:(b + 1) * size * per].contiguous(), per)
            torch.cuda.synchronize()
            assert torch.equal(sub, whole[b * size:(b + 1) * size]), (rows, blocks, b)
