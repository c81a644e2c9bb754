"""KV-sharded decode host logic on CPU: world_size 2 and 4 gloo ranks.

Each rank owns a contiguous block of the fixed split groups
(xq.shard.split_block), computes partial records for its rows only (here a
float64 numpy stand-in for xq.fa_partials, since there is no GPU), merges each
of its groups into one (O, lse, 1) record (the oracle's LSE merge standing in
for xq.lse_merge_records), the group records are all-gathered in group order
(xq.shard.gather_partials) and merged with the oracle's LSE merge.  The output
must be bit-identical to the same two-level merge in one process, and match
plain softmax attention over all rows; unequal blocks gather in order too.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

D, H, N_KV, ROWS = 64, 4, 780, 100  # 8 splits (the last one short)
N_GROUPS = 4
SCALE = 0.125


def _inputs():
    rng = np.random.default_rng(5)
    q = rng.normal(0, 1, (H, D)).astype(np.float32)
    k = rng.normal(0, 1, (N_KV, D)).astype(np.float32)
    v = rng.normal(0, 1, (N_KV, D)).astype(np.float32)
    return q, k, v


def _partials(q, k_rows, v_rows, n_local, rows):
    """(n_local, H, D + 2) records (acc, max, denom) of consecutive splits."""
    out = np.zeros((n_local, H, D + 2), np.float32)
    for s in range(n_local):
        kk = k_rows[s * rows:(s + 1) * rows].astype(np.float64)
        vv = v_rows[s * rows:(s + 1) * rows].astype(np.float64)
        if len(kk) == 0:
            out[s, :, D] = -3.402823466e38
            continue
        sc = SCALE * (q.astype(np.float64) @ kk.T)
        m = sc.max(axis=1)
        p = np.exp(sc - m[:, None])
        out[s, :, :D] = p @ vv
        out[s, :, D] = m
        out[s, :, D + 1] = p.sum(axis=1)
    return torch.from_numpy(out)


def _records(part, per_group):
    """Reference record merge: each group -> (O, lse, 1); empty -> (0, -FLT_MAX, 0)."""
    import oracle
    part = np.asarray(part)
    n, rows, d2 = part.shape
    out = np.zeros((n // per_group, rows, d2), np.float32)
    for g in range(n // per_group):
        o, lse = oracle.lse_merge(part[g * per_group:(g + 1) * per_group])
        out[g, :, :d2 - 2] = o
        empty = np.isneginf(lse)
        out[g, :, d2 - 2] = np.where(empty, np.float32(-3.402823466e38), lse)
        out[g, :, d2 - 1] = np.where(empty, 0.0, 1.0)
    return torch.from_numpy(out)


def _rank(rank, world, port, n_splits, result):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "xllama-qwen35-xbox_b200")]
    import torch.distributed as dist

    import oracle
    from xq import shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v = _inputs()
        per = n_splits // N_GROUPS
        gb, ge = shard.split_block(N_GROUPS, world, rank)
        k_local, v_local = k[gb * per * ROWS:ge * per * ROWS], v[gb * per * ROWS:ge * per * ROWS]

        def partials_fn(qq, kl, vl, ty, rows, n_local, sc):
            return _partials(qq, kl, vl, n_local, rows)

        out, lse = shard.sharded_flash_decode(
            q, k_local, v_local, 0, ROWS, n_splits, SCALE, n_groups=N_GROUPS,
            partials_fn=partials_fn, records_fn=_records,
            merge_fn=lambda p: oracle.lse_merge(p.numpy()))
        # unequal blocks (7 of 8 splits over the ranks) gather in split order
        n7 = 7
        b, e = shard.split_block(n7, world, rank)
        mine = torch.arange(b, e, dtype=torch.float32).reshape(-1, 1, 1).repeat(1, 2, 3)
        allp = shard.gather_partials(mine, n7)
        result[rank] = (out, lse, allp[:, 0, 0].numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, n_splits):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, world, port, n_splits, result))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        return [result[r] for r in range(world)]


def test_split_block_partitions_in_order():
    from xq import shard
    for n in (7, 8, 256):
        for world in (1, 2, 3, 4, 8):
            if n < world:
                continue
            blocks = [shard.split_block(n, world, r) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == n
            assert all(blocks[r][1] == blocks[r + 1][0] for r in range(world - 1))
            sizes = [e - b for b, e in blocks]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.split_block(2, 4, 0)


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_merge_is_rank_count_invariant(world):
    import oracle
    q, k, v = _inputs()
    n_splits = -(-N_KV // ROWS)
    part = _partials(q, k, v, n_splits, ROWS)
    full, full_lse = oracle.lse_merge(_records(part, n_splits // N_GROUPS).numpy())
    outs = _run(world, n_splits)
    for out, lse, order in outs:
        assert np.array_equal(out, full) and np.array_equal(lse, full_lse)
        assert np.array_equal(order, np.arange(7, dtype=np.float32))
    sc = SCALE * (q.astype(np.float64) @ k.T.astype(np.float64))
    p = np.exp(sc - sc.max(axis=1, keepdims=True))
    ref = (p @ v.astype(np.float64)) / p.sum(axis=1, keepdims=True)
    np.testing.assert_allclose(full, ref, rtol=1e-5, atol=1e-6)
