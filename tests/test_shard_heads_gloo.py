"""Head-sharded host logic on CPU: world_size 2 and 4 gloo ranks.

GATED_DELTA_NET sharded by value head: rank r takes value heads
xq.shard.head_block(H, world, r), runs them with the whole q/k and the head
offset that keeps the fork's key-head map (h mod H_k) -- here through the C
oracle's block mode, which takes the same (head_begin, n_head_total) pair as
xq_gated_delta_net_heads -- and the y blocks are all-gathered in head order
(xq.shard.gather_heads).  Every rank must then hold exactly the unsharded
op's y, and its snapshot block must equal the unsharded op's snapshot slots
for its heads, bit for bit.

Prefill FLASH_ATTN_EXT sharded by KV-head group: xq.shard.prefill_block
plans (query heads, KV heads, query rows) per rank; each rank runs the oracle
on its views; the blocks cover every (row, head) once and equal the unsharded
output bit for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

H, H_K, S, T, N_SEQ, SLOTS = 8, 4, 128, 5, 2, 2


def _gdn_inputs():
    rng = np.random.default_rng(11)

    def l2n(x):
        return (x / np.linalg.norm(x, axis=-1, keepdims=True)).astype(np.float32)
    q = l2n(rng.normal(0, 1, (N_SEQ, T, H_K, S)))
    k = l2n(rng.normal(0, 1, (N_SEQ, T, H_K, S)))
    v = rng.normal(0, 1, (N_SEQ, T, H, S)).astype(np.float32)
    g = (-np.log1p(np.exp(rng.normal(0, 1, (N_SEQ, T, H, 1))))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.normal(0, 1, (N_SEQ, T, H, 1))))).astype(np.float32)
    st = (0.1 * rng.normal(0, 1, (N_SEQ, H, S, S))).astype(np.float32)
    return q, k, v, g, beta, st


def _rank(rank, world, port, result):
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
        q, k, v, g, beta, st = _gdn_inputs()
        h0, h1 = shard.head_block(H, world, rank)
        _, y, snaps = oracle.gated_delta_net(
            q, k, np.ascontiguousarray(v[:, :, h0:h1]), np.ascontiguousarray(g[:, :, h0:h1]),
            np.ascontiguousarray(beta[:, :, h0:h1]), np.ascontiguousarray(st[:, h0:h1]),
            slots=SLOTS, head_begin=h0, n_head_total=H, n_workers=1)
        y_all = shard.gather_heads(torch.from_numpy(np.ascontiguousarray(y)), H)
        result[rank] = (h0, h1, y_all.numpy(), snaps.copy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, world, port, result)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        return [result[r] for r in range(world)]


@pytest.mark.parametrize("world", [2, 4])
def test_gdn_value_head_shards_gather_to_the_whole_op(world):
    import oracle
    q, k, v, g, beta, st = _gdn_inputs()
    _, y_full, snaps_full = oracle.gated_delta_net(q, k, v, g, beta, st, slots=SLOTS,
                                                   n_workers=1)
    outs = _run(world)
    assert [o[:2] for o in outs] == [(r * H // world, (r + 1) * H // world)
                                     for r in range(world)]
    for h0, h1, y_all, snaps in outs:
        assert np.array_equal(y_all, y_full)
        assert np.array_equal(snaps, snaps_full[:, :, h0:h1])


def test_gdn_block_mode_keeps_the_key_head_map():
    """A block that starts past H_k and wraps (value heads 6..9 of 12 with
    H_k = 4) reads key heads 2, 3, 0, 1 -- the unsharded op's h mod H_k."""
    import oracle
    rng = np.random.default_rng(2)
    Hv, Hk = 12, 4
    q = rng.normal(0, 0.1, (1, 3, Hk, S)).astype(np.float32)
    k = rng.normal(0, 0.1, (1, 3, Hk, S)).astype(np.float32)
    v = rng.normal(0, 1, (1, 3, Hv, S)).astype(np.float32)
    g = -np.abs(rng.normal(0, 1, (1, 3, Hv, 1))).astype(np.float32)
    beta = rng.uniform(0, 1, (1, 3, Hv, 1)).astype(np.float32)
    st = rng.normal(0, 0.1, (1, Hv, S, S)).astype(np.float32)
    _, y_full, _ = oracle.gated_delta_net(q, k, v, g, beta, st, n_workers=1)
    _, y, _ = oracle.gated_delta_net(q, k, np.ascontiguousarray(v[:, :, 6:10]),
                                     np.ascontiguousarray(g[:, :, 6:10]),
                                     np.ascontiguousarray(beta[:, :, 6:10]),
                                     np.ascontiguousarray(st[:, 6:10]), head_begin=6,
                                     n_head_total=Hv, n_workers=1)
    assert np.array_equal(y, y_full[:, :, 6:10])
    with pytest.raises(ValueError):  # a block past the op's last head
        oracle.gated_delta_net(q, k, v[:, :, :4].copy(), g[:, :, :4].copy(),
                               beta[:, :, :4].copy(), st[:, :4].copy(), head_begin=10,
                               n_head_total=Hv, n_workers=1)


def test_key_heads_of_a_block():
    from xq import shard
    assert shard.key_heads(0, 16, 16) == list(range(16))
    assert shard.key_heads(16, 24, 16) == list(range(8))
    assert shard.key_heads(14, 18, 16) == [0, 1, 14, 15]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_prefill_blocks_cover_the_op_once_and_match(world):
    import oracle
    from xq import shard
    Hq, Hkv, D, n_q, n_kv = 8, 4, 64, 300, 340
    rng = np.random.default_rng(world)
    q = rng.normal(0, 1, (1, Hq, n_q, D)).astype(np.float32)
    k = oracle.quantize(oracle.Q8_0, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))
    v = oracle.quantize(oracle.Q8_0, rng.normal(0, 1, (1, n_kv, Hkv, D)).astype(np.float32))
    m = np.zeros((1, 1, n_q, n_kv), np.float16)
    for i in range(n_q):
        m[0, 0, i, n_kv - n_q + i + 1:] = -np.inf
    full = oracle.flash_attn_ext(q, k, v, oracle.Q8_0, oracle.Q8_0, mask=m, scale=0.125)
    seen = np.zeros((n_q, Hq), np.int32)
    for r in range(world):
        (h0, h1), (c0, c1), (r0, r1) = shard.prefill_block(Hq, Hkv, n_q, n_kv, world, r,
                                                           tile=128)
        assert h1 - h0 == (c1 - c0) * (Hq // Hkv) and r0 % 128 == 0
        seen[r0:r1, h0:h1] += 1
        part = oracle.flash_attn_ext(np.ascontiguousarray(q[:, h0:h1, r0:r1]),
                                     np.ascontiguousarray(k[:, :, c0:c1]),
                                     np.ascontiguousarray(v[:, :, c0:c1]), oracle.Q8_0,
                                     oracle.Q8_0, mask=np.ascontiguousarray(m[:, :, r0:r1]),
                                     scale=0.125)
        assert np.array_equal(part, full[:, r0:r1, h0:h1])
    assert np.all(seen == 1)


def test_prefill_row_blocks_balance_causal_work():
    from xq import shard
    blocks = [shard.prefill_block(24, 4, 8192, 8192, 8, r) for r in range(8)]
    assert blocks[0] == ((0, 6), (0, 1), (0, 5760)) and blocks[1] == ((0, 6), (0, 1), (5760, 8192))
    work = [sum(min(8192, i + 1) for i in range(r0, r1)) for _, _, (r0, r1) in blocks[:2]]
    assert abs(work[0] - work[1]) / sum(work) < 0.02
    with pytest.raises(ValueError):
        shard.prefill_block(24, 4, 8192, 8192, 3, 0)
