"""KV-sharded flash decode over several GPUs (one process per GPU).

The KV rows of every sequence are cut into a fixed global list of splits of
`rows_per_split` rows.  Rank r holds and reads a contiguous block of those
splits (`split_block`), writes one partial record (acc[D], max, denom) per
(split, sequence, head) with `xq.fa_partials`, the blocks are all-gathered in
global split order (`gather_partials`, NCCL on GPUs), and every rank merges
them with `xq.lse_merge`.  Because the list of splits and the merge order do
not depend on the number of ranks, the output is bit-identical for any GPU
count.  There is no other exchange step.
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
                         scale: float = 1.0, group=None, out=None, partials_fn=None,
                         merge_fn=None):
    """One decode step whose KV rows are spread over the ranks of `group`.

    k_local / v_local hold this rank's rows only: split_block(n_splits, ...)
    of the global splits, row 0 = first row of its first split.  Returns the
    merged output (n_seq * n_q * n_head, D) and the lse on every rank.
    `partials_fn(q, k, v, k_type, rows_per_split, n_local, scale)` and
    `merge_fn(partials)` default to the B200 kernels (xq.fa_partials,
    xq.lse_merge)."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    b, e = split_block(n_splits, world, rank)
    if partials_fn is None:
        from . import ops

        def partials_fn(q, k, v, ty, rows, n_local, sc):
            return ops.fa_partials(q, k, v, ty, rows, 0, n_local, scale=sc)
    if merge_fn is None:
        from . import ops

        def merge_fn(p):
            return ops.lse_merge(p, out=out)
    local = partials_fn(q, k_local, v_local, k_type, rows_per_split, e - b, scale)
    full = gather_partials(local, n_splits, group)
    return merge_fn(full)
