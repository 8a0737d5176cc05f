"""Row sharding of quantized weight matrices across the GPUs of one node.

Rows of a GEMV/GEMM are independent, so each rank holds a contiguous, whole-block-row slice of
every large matrix, computes its slice of the output with the same kernels, and one all-gather
per matrix assembles the full output on every rank (the only exchange step; no other data moves).
This has no counterpart in cuda-for-intel, which is single-GPU.

Output layout follows ggml's mul_mat_vec_q/mul_mat_q dst: column-major, `ncols` columns of
`nrows` fp32 values.
"""
from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    nrows: int        # rows of the whole matrix
    row0: int         # first row of this rank
    rows: int         # rows held by this rank
    rows_padded: int  # rows of the largest shard (all-gather chunk size)


def row_split(nrows, world, rank):
    """Balanced contiguous split: the first nrows % world ranks hold one extra row."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank %d of %d" % (rank, world))
    base, extra = divmod(nrows, world)
    row0 = rank * base + min(rank, extra)
    rows = base + (1 if rank < extra else 0)
    return Shard(rank, world, nrows, row0, rows, base + (1 if extra else 0))


def weight_slice(weights_2d, shard):
    """The rank's rows of a row-major block matrix (any array/tensor indexable by rows)."""
    return weights_2d[shard.row0:shard.row0 + shard.rows]


def gather_columns(y_local, shard, ncols, all_gather_into_tensor, empty):
    """Assemble the full column-major output from every rank's (ncols, rows_padded) slice.

    `y_local` is a contiguous tensor of ncols * rows_padded fp32 values (rows beyond shard.rows
    are padding); `all_gather_into_tensor(out, inp)` is the collective (torch.distributed over
    NCCL on GPUs, gloo on CPU); `empty(n)` allocates a flat fp32 tensor like y_local.  Returns a
    (ncols, nrows) tensor."""
    rp = shard.rows_padded
    buf = empty(shard.world * ncols * rp)
    all_gather_into_tensor(buf, y_local.reshape(-1))
    parts = buf.reshape(shard.world, ncols, rp)
    cols = []
    for r in range(shard.world):
        s = row_split(shard.nrows, shard.world, r)
        cols.append(parts[r, :, :s.rows])
    import torch

    return torch.cat(cols, dim=1)
