"""The hot path spread over several GPUs (one process per GPU).

Three partitions, one per op shape:
  * decode (FLASH_ATTN_EXT, one query): KV rows sharded (below);
  * GATED_DELTA_NET: value heads sharded (`head_block`, `gdn_heads`): rank r
    runs value heads head_block(H, world, r) through xq_gated_delta_net_heads
    with the whole q/k (each value head h reads key head h % H_k); outputs and
    state stay sharded -- there is no exchange step (`gather_heads` is the
    optional all-gather of y when a caller wants it whole);
  * prefill (FLASH_ATTN_EXT, many queries): KV-head groups (`prefill_block`):
    up to n_head_kv ranks take blocks of KV heads with their query heads;
    beyond that each KV head's query rows are cut into blocks of equal causal
    work (whole 128-row tiles); outputs are disjoint, no exchange step.

KV-sharded flash decode:

The KV rows of every sequence are cut into a fixed global list of splits of
`rows_per_split` rows, and the splits into a fixed list of `n_groups` groups
of consecutive splits.  Rank r holds and reads a contiguous block of groups
(`split_block` over groups) and:
  1. writes one partial record (acc[D], max, denom) per (split, sequence,
     head) with `xq.fa_partials`;
  2. merges each of its groups in split order into one record (O, lse, 1)
     with `xq.lse_merge_records`;
  3. all-gathers the group records in group order (`gather_partials`, NCCL on
     GPUs: n_groups x n_rows x (D + 2) floats in total);
  4. merges the group records with `xq.lse_merge`.
The grouping and both merge orders are fixed by (n_splits, n_groups) alone,
so the output is bit-identical for any rank count that divides n_groups.
There is no other exchange step.
"""
from __future__ import annotations


def split_block(n_splits: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of the global splits owned by `rank`: contiguous blocks,
    the first n_splits % world ranks one split longer."""
    if n_splits < world:
        raise ValueError(f"{n_splits} splits cannot feed {world} ranks")
    base, extra = divmod(n_splits, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def gather_partials(part_local, n_splits: int, group=None, out=None):
    """All-gather every rank's block of partial records (split-major) into one
    (n_splits, n_rows, D + 2) tensor in global split order (`out` if given)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    sizes = [split_block(n_splits, world, r) for r in range(world)]
    longest = max(e - b for b, e in sizes)
    rest = tuple(part_local.shape[1:])
    if all(e - b == longest for b, e in sizes):
        if out is None:
            out = torch.empty((n_splits,) + rest, dtype=part_local.dtype,
                              device=part_local.device)
        if dist.get_backend(group) == "nccl":
            dist.all_gather_into_tensor(out, part_local.contiguous(), group=group)
        else:
            dist.all_gather(list(out.chunk(world)), part_local.contiguous(), group=group)
        return out
    # unequal blocks: pad to the longest, gather, drop the padding
    pad = torch.zeros((longest,) + rest, dtype=part_local.dtype, device=part_local.device)
    pad[: part_local.shape[0]] = part_local
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    full = torch.cat([bufs[r][: e - b] for r, (b, e) in enumerate(sizes)])
    if out is not None:
        out.copy_(full)
        return out
    return full


def sharded_flash_decode(q, k_local, v_local, k_type: int, rows_per_split: int, n_splits: int,
                         scale: float = 1.0, group=None, out=None, n_groups: int = 8,
                         partials_fn=None, records_fn=None, merge_fn=None):
    """One decode step whose KV rows are spread over the ranks of `group`.

    k_local / v_local hold this rank's rows only: the splits of groups
    split_block(n_groups, world, rank), row 0 = first row of its first split.
    Returns the merged (out (n_seq * n_q * n_head, D), lse) on every rank.
    `partials_fn(q, k, v, k_type, rows_per_split, n_local_splits, scale)`,
    `records_fn(partials, splits_per_group)` and `merge_fn(records)` default to
    the B200 kernels (xq.fa_partials, xq.lse_merge_records, xq.lse_merge)."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    if n_splits % n_groups or n_groups % world:
        raise ValueError(f"{n_splits} splits / {n_groups} groups / {world} ranks do not divide")
    per_group = n_splits // n_groups
    gb, ge = split_block(n_groups, world, rank)
    from . import ops
    if partials_fn is None:
        def partials_fn(q, k, v, ty, rows, n_local, sc):
            return ops.fa_partials(q, k, v, ty, rows, 0, n_local, scale=sc)
    if records_fn is None:
        records_fn = ops.lse_merge_records
    if merge_fn is None:
        def merge_fn(r):
            return ops.lse_merge(r, out=out)
    local = partials_fn(q, k_local, v_local, k_type, rows_per_split, (ge - gb) * per_group,
                        scale)
    records = records_fn(local, per_group)
    return merge_fn(gather_partials(records, n_groups, group))


# ---------------------------------------------------------------------------
# GATED_DELTA_NET sharded by value head

def head_block(n_head: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of the value heads `rank` owns: contiguous blocks."""
    return split_block(n_head, world, rank)


def key_heads(h0: int, h1: int, n_head_kv: int) -> list[int]:
    """The key heads value heads [h0, h1) read (h % n_head_kv)."""
    return sorted({h % n_head_kv for h in range(h0, h1)})


def gdn_heads(q, k, v, g, beta, state, slots: int = 1, world: int = 1, rank: int = 0,
              out=None, stream=None):
    """This rank's share of one GATED_DELTA_NET op sharded by value head.
    q, k: the whole (n_seq, T, H_k, S) key tensors; v, g, beta, state: the
    whole op's tensors (this rank's head block is viewed out of them, no
    copy).  Returns (dst, y (n_seq, T, h1 - h0, S), snapshots) of heads
    [h0, h1) = head_block(H, world, rank), bit-identical to the same heads of
    the unsharded op."""
    from . import ops
    H = v.shape[2]
    h0, h1 = head_block(H, world, rank)
    return ops.gated_delta_net(q, k, v[:, :, h0:h1], g[:, :, h0:h1], beta[:, :, h0:h1],
                               state[:, h0:h1], slots=slots, out=out, stream=stream,
                               head_begin=h0, n_head_total=H)


def gather_heads(y_local, n_head: int, group=None):
    """All-gather every rank's y block (n_seq, T, h1 - h0, S) into the whole
    (n_seq, T, n_head, S) on every rank (the optional exchange after a
    head-sharded GATED_DELTA_NET)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    blocks = [head_block(n_head, world, r) for r in range(world)]
    longest = max(e - b for b, e in blocks)
    n_seq, T, _, S = y_local.shape
    pad = torch.zeros((n_seq, T, longest, S), dtype=y_local.dtype, device=y_local.device)
    pad[:, :, : y_local.shape[2]] = y_local
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad.contiguous(), group=group)
    return torch.cat([bufs[r][:, :, : e - b] for r, (b, e) in enumerate(blocks)], dim=2)


# ---------------------------------------------------------------------------
# FLASH_ATTN_EXT prefill sharded by KV-head group

def prefill_block(n_head: int, n_head_kv: int, n_q: int, n_kv: int, world: int, rank: int,
                  causal: bool = True, tile: int = 128):
    """(head range, kv-head range, query-row range) of `rank` for one
    prefill FLASH_ATTN_EXT sharded by KV-head group.

    world <= n_head_kv: contiguous blocks of KV heads (n_head_kv % world ==
    0), each with its G = n_head / n_head_kv query heads and every query row.
    world > n_head_kv (world % n_head_kv == 0): rank r serves KV head
    r // parts (parts = world / n_head_kv) and its query heads, over one of
    `parts` blocks of query rows with equal attention work -- under a causal
    mask over the tail of the cache, row i sees n_kv - n_q + i + 1 keys --
    cut at whole `tile`-row query tiles, so each block computes exactly the
    tiles the unsharded kernel computes for those rows (bit-identical)."""
    G = n_head // n_head_kv
    if world <= n_head_kv:
        if n_head_kv % world:
            raise ValueError(f"{n_head_kv} KV heads do not split over {world} ranks")
        b, e = split_block(n_head_kv, world, rank)
        return (b * G, e * G), (b, e), (0, n_q)
    if world % n_head_kv:
        raise ValueError(f"{world} ranks are not a multiple of {n_head_kv} KV heads")
    parts = world // n_head_kv
    kvh, part = divmod(rank, parts)
    n_tiles = (n_q + tile - 1) // tile

    def cost(t):  # attention work of query tile t (keys seen, summed over its rows)
        r0, r1 = t * tile, min(n_q, (t + 1) * tile)
        if not causal:
            return (r1 - r0) * n_kv
        off = n_kv - n_q
        return sum(min(n_kv, off + i + 1) for i in range(r0, r1))
    costs = [cost(t) for t in range(n_tiles)]
    total = float(sum(costs))
    cuts, acc, t = [0], 0.0, 0
    for p in range(1, parts):
        while t < n_tiles and acc + costs[t] / 2 < total * p / parts:
            acc += costs[t]
            t += 1
        cuts.append(t)
    cuts.append(n_tiles)
    r0, r1 = cuts[part] * tile, min(n_q, cuts[part + 1] * tile)
    return (kvh * G, (kvh + 1) * G), (kvh, kvh + 1), (r0, r1)


def prefill_part(q, k, v, k_type: int, mask=None, world: int = 1, rank: int = 0,
                 scale: float = 1.0, out=None, stream=None):
    """This rank's share of one prefill FLASH_ATTN_EXT sharded by KV-head
    group: views of the whole q (n_seq, n_head, n_q, D), caches (n_seq_kv,
    n_kv, n_head_kv, row_bytes) and mask (m3, 1, >= n_q, n_kv) -- the mask
    must broadcast over heads, as llama.cpp's KQ mask does -- through one
    xq_flash_attn_ext call.  Returns (out (n_seq, r1 - r0, h1 - h0, D),
    ((h0, h1), (c0, c1), (r0, r1)))."""
    from . import ops
    n_seq, n_head, n_q, D = q.shape
    n_kv, n_hkv = k.shape[1], k.shape[2]
    if mask is not None and mask.shape[1] != 1:
        raise ValueError("a head-sharded prefill needs a mask that broadcasts over heads")
    plan = prefill_block(n_head, n_hkv, n_q, n_kv, world, rank, causal=mask is not None)
    (h0, h1), (c0, c1), (r0, r1) = plan
    m = mask[:, :, r0:r1] if mask is not None else None
    o = ops.flash_attn_ext(q[:, h0:h1, r0:r1], k[:, :, c0:c1], v[:, :, c0:c1], k_type,
                           mask=m, scale=scale, out=out, stream=stream)
    return o, plan


# ---------------------------------------------------------------------------
# KV-sharded decode through the C ABI: group records exchanged with NVLink
# peer stores (xq_fa_shard_push / xq_fa_shard_finish) instead of NCCL.

class ShardExchange:
    """This rank's exchange buffer (library-allocated, zeroed) and every
    rank's buffer as this process maps it (CUDA IPC handles moved with an
    all-gather of the process group).  `buffers` may instead be given: a list
    of buffers all mapped in this process (one GPU emulating several ranks,
    for tests)."""

    def __init__(self, n_groups: int, n_rows: int, D: int, group=None, buffers=None):
        import ctypes as C

        from ._lib import IpcHandle, check, lib
        self.n_groups, self.n_rows, self.D = n_groups, n_rows, D
        self._L = lib()
        self.bytes = self._L.xq_shard_exchange_bytes(n_groups, n_rows, D)
        self._opened, self._owned = [], []
        if buffers is not None:
            self.ptrs = list(buffers)
            return
        import torch.distributed as dist
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        own = C.c_void_p()
        check(self._L.xq_shard_exchange_alloc(self.bytes, C.byref(own)))
        self._owned.append(own.value)
        h = IpcHandle()
        check(self._L.xq_ipc_export(own, C.byref(h)))
        handles = [None] * world
        dist.all_gather_object(handles, bytes(h.bytes), group=group)
        self.ptrs = []
        for r in range(world):
            if r == rank:
                self.ptrs.append(own.value)
                continue
            hr = IpcHandle()
            C.memmove(hr.bytes, handles[r], 64)
            p = C.c_void_p()
            check(self._L.xq_ipc_open(C.byref(hr), C.byref(p)))
            self._opened.append(p.value)
            self.ptrs.append(p.value)

    @staticmethod
    def alloc_local(n_groups: int, n_rows: int, D: int, count: int):
        """`count` zeroed exchange buffers on the current GPU (emulation)."""
        import ctypes as C

        from ._lib import check, lib
        L = lib()
        nb = L.xq_shard_exchange_bytes(n_groups, n_rows, D)
        out = []
        for _ in range(count):
            p = C.c_void_p()
            check(L.xq_shard_exchange_alloc(nb, C.byref(p)))
            out.append(p.value)
        return out

    def plan(self, rank: int, world: int, rows_per_split: int, splits_per_group: int,
             step: int):
        from ._lib import ShardPlan
        s = ShardPlan()
        s.rows_per_split, s.splits_per_group, s.n_groups = rows_per_split, splits_per_group, \
            self.n_groups
        s.rank, s.world, s.step = rank, world, step & 0xffffffff
        for r, p in enumerate(self.ptrs[:world]):
            s.exchange[r] = p
        return s

    def close(self):
        for p in self._opened:
            self._L.xq_ipc_close(p)
        for p in self._owned:
            self._L.xq_shard_exchange_free(p)
        self._opened, self._owned = [], []


def shard_decode_step(q, k_local, v_local, k_type: int, exchange: ShardExchange, rank: int,
                      world: int, rows_per_split: int, splits_per_group: int, step: int,
                      scale: float = 1.0, out=None, lse=None, ws=None, push=True, finish=True,
                      stream=None):
    """One KV-sharded decode step of this rank through the C ABI (push, then
    finish).  k_local / v_local: this rank's rows (groups head_block-style
    split_block(n_groups, world, rank)).  Returns out (n_rows, D)."""
    import ctypes as C

    import torch

    from ._lib import check, lib
    from .ops import _fa_params, _stream, _workspace
    n_seq, n_head, n_q, D = q.shape
    n_rows = n_seq * n_q * n_head
    o = out if out is not None else torch.empty((n_rows, D), dtype=torch.float32,
                                                device=q.device)
    L = lib()
    s = exchange.plan(rank, world, rows_per_split, splits_per_group, step)
    st = _stream(stream)
    if push:
        dummy = o
        p = _fa_params(q, k_local, v_local, k_type, k_type, None, None, dummy, scale, 0.0, 0.0, 0)
        nbytes = L.xq_fa_shard_workspace(C.byref(p), C.byref(s))
        w = ws if ws is not None else _workspace(nbytes, q.device)
        check(L.xq_fa_shard_push(C.byref(p), C.byref(s), w.data_ptr(), w.numel(), st))
    if finish:
        check(L.xq_fa_shard_finish(C.byref(s), n_rows, D, None, n_head, o.data_ptr(),
                                   lse.data_ptr() if lse is not None else None, st))
    return o
