"""B200: the KV-sharded decode through the C ABI (xq_fa_shard_push /
xq_fa_shard_finish: group records exchanged with NVLink peer stores), its
ranks emulated on one GPU.

All ranks' pushes run before any rank's finish, so no kernel ever waits for
a launch that comes after it on the same GPU; every finish finds its records
complete.  The output must be bit-identical for 1, 2, 4 and 8 ranks, equal
the split records merged in two levels by xq_lse_merge_records /
xq_lse_merge, and match the oracle.  A finish whose peers never push runs
its bounded wait out: the host then reads the error status and the output
is NaN -- the failure path, exercised without faulting anything.
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

H, HKV, D, N_SEQ = 24, 4, 256, 2
ROWS, SPLITS, GROUPS = 256, 32, 8   # 8192 KV rows per sequence
PER = SPLITS // GROUPS


def _case():
    import xq
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    q = torch.randn((N_SEQ, H, 1, D), generator=g, device="cuda")
    k = xq.quantize_rows(xq.Q8_0, torch.randn((N_SEQ, ROWS * SPLITS, HKV, D), generator=g,
                                              device="cuda"))
    v = xq.quantize_rows(xq.Q8_0, torch.randn((N_SEQ, ROWS * SPLITS, HKV, D), generator=g,
                                              device="cuda"))
    return q, k, v


def _run(world, q, k, v, steps=3):
    import xq
    from xq import shard
    n_rows = N_SEQ * H
    bufs = shard.ShardExchange.alloc_local(GROUPS, n_rows, D, world)
    ex = shard.ShardExchange(GROUPS, n_rows, D, buffers=bufs)
    outs = [torch.full((n_rows, D), float("nan"), device="cuda") for _ in range(world)]
    wss = [torch.empty(1 << 24, dtype=torch.uint8, device="cuda") for _ in range(world)]
    try:
        for t in range(steps):
            for r in range(world):  # every rank's push first ...
                g0, g1 = shard.split_block(GROUPS, world, r)
                lo, hi = g0 * PER * ROWS, g1 * PER * ROWS
                shard.shard_decode_step(q, k[:, lo:hi], v[:, lo:hi], xq.Q8_0, ex, r, world, ROWS,
                                        PER, t, scale=1 / 16, ws=wss[r], finish=False)
            for r in range(world):  # ... then every rank's wait + merge
                shard.shard_decode_step(q, None, None, xq.Q8_0, ex, r, world, ROWS, PER, t,
                                        scale=1 / 16, out=outs[r], push=False)
        torch.cuda.synchronize()
        for r in range(world):
            err = np.zeros(1, np.int32)
            import ctypes as C
            from xq import _lib
            e = C.c_int32()
            _lib.check(_lib.lib().xq_shard_exchange_error(bufs[r], GROUPS, n_rows, D, None,
                                                          C.byref(e)))
            assert e.value == 0
        return [o.clone() for o in outs]
    finally:
        torch.cuda.synchronize()
        from xq import _lib
        for b in bufs:
            _lib.lib().xq_shard_exchange_free(b)


def test_sharded_decode_is_bit_identical_for_1_2_4_8_ranks():
    import xq
    q, k, v = _case()
    one = _run(1, q, k, v)[0]
    # the same plan merged by the two-level record merge in one process
    part = xq.fa_partials(q, k, v, xq.Q8_0, ROWS, 0, SPLITS, scale=1 / 16)
    rec = xq.lse_merge_records(part, PER)
    two, _ = xq.lse_merge(rec, want_lse=False)
    torch.cuda.synchronize()
    assert torch.equal(one, two)
    for world in (2, 4, 8):
        for o in _run(world, q, k, v):
            assert torch.equal(o, one), world
    want = oracle.flash_attn_ext(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), oracle.Q8_0,
                                 oracle.Q8_0, scale=1 / 16, nth=8)
    np.testing.assert_allclose(one.view(N_SEQ, 1, H, D).cpu().numpy(), want, rtol=1e-2,
                               atol=2e-3)


def test_finish_without_peers_times_out_with_an_error_status():
    """Rank 0 of a two-rank plan finishes a step no peer pushed: its bounded
    wait (2 s) runs out, the host reads status 1, the output is NaN, and the
    call itself returns normally (the context stays usable)."""
    import ctypes as C

    import xq
    from xq import _lib, shard
    q, k, v = _case()
    n_rows = N_SEQ * H
    bufs = shard.ShardExchange.alloc_local(GROUPS, n_rows, D, 2)
    try:
        ex = shard.ShardExchange(GROUPS, n_rows, D, buffers=bufs)
        out = torch.zeros((n_rows, D), device="cuda")
        shard.shard_decode_step(q, None, None, xq.Q8_0, ex, 0, 2, ROWS, PER, 0, out=out,
                                push=False)
        e = C.c_int32()
        _lib.check(_lib.lib().xq_shard_exchange_error(bufs[0], GROUPS, n_rows, D, None,
                                                      C.byref(e)))
        assert e.value == 1
        assert bool(torch.isnan(out).all())
        # the device still runs work afterwards
        assert float(torch.ones(4, device="cuda").sum()) == 4.0
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            _lib.lib().xq_shard_exchange_free(b)
