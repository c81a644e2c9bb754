"""KV-sharded flash decode over several GPUs (one process per GPU).

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
