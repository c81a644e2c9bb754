"""B200: the head-sharded partitions of the hot path, every rank's share run
on one GPU and compared bit for bit with the unsharded call.

* GATED_DELTA_NET by value head (xq_gated_delta_net_heads through
  xq.shard.gdn_heads): the per-token kernel (8 sequences x 1 token), the
  chunked tensor-core form (300 tokens), and the chunked form followed by the
  per-token tail that writes K > 1 snapshot slots.
* Prefill FLASH_ATTN_EXT by KV-head group (xq.shard.prefill_part): blocks of
  KV heads for up to 4 ranks, then causal-work-balanced query-row blocks for
  8 ranks, F16 and Q8_0 caches.
"""
import numpy as np
import pytest
import torch

import oracle
from test_gdn_gpu import c3_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n_seq,T,K", [(8, 1, 1), (1, 300, 1), (1, 200, 3)])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_gdn_value_head_blocks_are_bit_identical(world, n_seq, T, K):
    import xq
    from xq import shard
    ins = [torch.from_numpy(x).cuda() for x in c3_inputs(500 + T, n_seq, T)]
    _, y_full, s_full = xq.gated_delta_net(*ins, slots=K)
    y_full, s_full = y_full.clone(), s_full.clone()
    for r in range(world):
        h0, h1 = shard.head_block(32, world, r)
        _, y, snaps = shard.gdn_heads(*ins, slots=K, world=world, rank=r)
        torch.cuda.synchronize()
        assert torch.equal(y, y_full[:, :, h0:h1]), (world, r)
        assert torch.equal(snaps, s_full[:, :, h0:h1]), (world, r)


def test_gdn_head_block_against_the_oracle():
    """A block whose heads wrap the key heads (value heads 12..19 of 32, key
    heads 12..15 then 0..3) against the oracle's block mode."""
    import xq
    q, k, v, g, beta, st = c3_inputs(9, 2, 70)
    sl = slice(12, 20)
    blk = [np.ascontiguousarray(x[:, :, sl]) for x in (v, g, beta)] + \
        [np.ascontiguousarray(st[:, sl])]
    dev = [torch.from_numpy(x).cuda() for x in (q, k, *blk)]
    _, y, snaps = xq.gated_delta_net(*dev, slots=2, head_begin=12, n_head_total=32)
    _, yo, so = oracle.gated_delta_net(q, k, *blk, slots=2, head_begin=12, n_head_total=32)
    np.testing.assert_allclose(y.cpu().numpy(), yo, rtol=1e-2, atol=2e-3)
    np.testing.assert_allclose(snaps.cpu().numpy(), so, rtol=1e-2, atol=2e-3)


@pytest.mark.parametrize("ty", [oracle.F16, oracle.Q8_0])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_prefill_kv_head_blocks_are_bit_identical(world, ty):
    import xq
    from xq import shard
    H, Hkv, D, N = 24, 4, 256, 1024
    g = torch.Generator(device="cuda")
    g.manual_seed(world)
    q = torch.randn((1, H, N, D), generator=g, device="cuda")
    k = xq.quantize_rows(ty, torch.randn((1, N, Hkv, D), generator=g, device="cuda"))
    v = xq.quantize_rows(ty, torch.randn((1, N, Hkv, D), generator=g, device="cuda"))
    mask = torch.zeros((1, 1, N, N), dtype=torch.float16, device="cuda")
    mask.masked_fill_(torch.triu(torch.ones(N, N, dtype=torch.bool, device="cuda"), 1)[None, None],
                      float("-inf"))
    full = xq.flash_attn_ext(q, k, v, ty, mask=mask, scale=1 / 16)
    seen = torch.zeros((N, H), dtype=torch.int32)
    for r in range(world):
        out, ((h0, h1), _, (r0, r1)) = shard.prefill_part(q, k, v, ty, mask, world, r,
                                                          scale=1 / 16)
        torch.cuda.synchronize()
        assert torch.equal(out, full[:, r0:r1, h0:h1]), (world, r)
        seen[r0:r1, h0:h1] += 1
    assert bool((seen == 1).all())
