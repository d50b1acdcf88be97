"""Output-column split (N-split) of one linear across ranks, one GPU per rank.

Rank r owns W rows [n0, n1) (a multiple of 128 wide, so every rank's tiles are whole) and computes
Y[:, n0:n1]; the shards are then all-gathered.  Row-major Y column shards are not contiguous, so
the gather lands rank-major in a [world, M, per] buffer and one strided copy restores [M, N].
"""


def shard_bounds(n, world, rank, align=128):
    """(n0, n1, per): rank's column range and the padded per-rank width (equal on every rank)."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"rank {rank} outside world {world}")
    per = -(-n // world)
    per = -(-per // align) * align
    n0 = min(n, rank * per)
    n1 = min(n, n0 + per)
    return n0, n1, per


def segment_rows(segments, world, rank, align=128):
    """Rows of a weight made of row blocks `segments` (e.g. Q, K, V heads, gate, up of the FLUX
    single-stream linear1, quicknn_transformers.pas:1503) that rank holds when each block is
    N-split in the same proportion: block s contributes its rows shard_bounds(segments[s], ...).
    With align = head_dim, every rank holds whole heads of Q, K and V and matching gate/up rows,
    so attention per head and the SiLU gate per pair need only the rank's own columns.  Returns the
    row indices in the rank's local order (block by block)."""
    import numpy as np

    parts, off = [], 0
    for n in segments:
        n0, n1, _ = shard_bounds(n, world, rank, align)
        parts.append(np.arange(off + n0, off + n1, dtype=np.int64))
        off += n
    return np.concatenate(parts)


def gather_columns(y_shard, n, group=None, out=None, buf=None):
    """All-gather the per-rank [M, per] shards (zero-padded past n1 - n0) into out [M, n]."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    M, per = y_shard.shape
    if buf is None:
        buf = torch.empty(world, M, per, dtype=y_shard.dtype, device=y_shard.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(buf, y_shard.contiguous(), group=group)
    else:
        dist.all_gather(list(buf.unbind(0)), y_shard.contiguous(), group=group)
    if out is None:
        out = torch.empty(M, n, dtype=y_shard.dtype, device=y_shard.device)
    out.copy_(buf.permute(1, 0, 2).reshape(M, world * per)[:, :n])
    return out
