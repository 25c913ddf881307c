"""N-sharding of the int4 GEMM over the GPUs of one node.

Output columns are independent: Y[:, n] needs only W[:, n], scales[n, :] and
LoRA B[:, n].  In the reference layout a contiguous column range of W and of
the scales is one contiguous byte range (packed byte n*(K/2) + k/2, scale
n*(K/32) + k/32), so rank r uploads columns [begin, end) with no repacking
(spaceslug_q4_weights_create with col_begin/col_end) and computes its Y shard
locally.  The only exchange is an all-gather of the fp32 Y shards over
NVLink (NCCL through torch.distributed), followed by the re-layout from the
rank-major [P][M][N/P] gather buffer to row-major [M][N].
"""
from __future__ import annotations


def shard_columns(n: int, world: int, rank: int, align: int = 8) -> tuple[int, int]:
    """Column range [begin, end) of `rank`; equal shards of a multiple of `align`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    per = -(-n // world)
    per = -(-per // align) * align
    begin = min(n, rank * per)
    end = min(n, begin + per)
    if end <= begin:
        raise ValueError(f"{n} columns cannot be split over {world} ranks in units of {align}")
    return begin, end


def shard_width(n: int, world: int, align: int = 8) -> int:
    per = -(-n // world)
    return -(-per // align) * align


def allgather_columns(y_shard, n_total: int, pg, stream=None):
    """All-gather column shards [M][w] of every rank into Y [M][n_total].

    Every rank passes a shard of the same width w = shard_width(n_total, P)
    (the last rank's shard is zero-padded by the caller if n_total % P != 0).
    """
    import torch
    world = pg.get_world_size()
    m, w = y_shard.shape
    buf = torch.empty((world, m, w), dtype=y_shard.dtype, device=y_shard.device)
    if y_shard.is_cuda:
        pg.all_gather_into_tensor(buf, y_shard.contiguous())
    else:  # gloo (CPU): list form
        pg.all_gather(list(buf.unbind(0)), y_shard.contiguous())
    return buf.permute(1, 0, 2).reshape(m, world * w)[:, :n_total]
