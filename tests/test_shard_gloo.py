"""Row sharding + all-gather on CPU ranks (gloo, world size 2 and 3): each rank evaluates its
rows with the oracle's decode step and the gathered output must equal the unsharded result bit
for bit (rows are independent, so sharding cannot change any value)."""
import os
import socket
import tempfile

import numpy as np
import pytest

import cfi_b200 as cfi
import shard

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def test_row_split_covers_every_row_once():
    for nrows in (1, 7, 8192, 151936, 8960):
        for world in (1, 2, 3, 4, 8):
            s = [shard.row_split(nrows, world, r) for r in range(world)]
            assert s[0].row0 == 0 and sum(x.rows for x in s) == nrows
            for a, b in zip(s, s[1:]):
                assert b.row0 == a.row0 + a.rows
            assert max(x.rows for x in s) == s[0].rows_padded
    with pytest.raises(ValueError):
        shard.row_split(10, 2, 2)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rank_main(rank, world, port, outdir, ty, rows, k, ncols):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import oracle_py as O

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = cfi.synthetic_weights(ty, rows, k, seed=3).reshape(rows, -1)
        x = np.random.default_rng(4).normal(size=(ncols, k)).astype(np.float32)
        sh = shard.row_split(rows, world, rank)
        wl = np.ascontiguousarray(shard.weight_slice(w, sh))
        y, _, _ = O.cpu_decode_step(ty, wl, sh.rows, k, x, ncols, 1)
        yl = torch.zeros(ncols, sh.rows_padded)
        yl[:, :sh.rows] = torch.from_numpy(y.reshape(ncols, sh.rows))
        full = shard.gather_columns(yl, sh, ncols, dist.all_gather_into_tensor, lambda n: torch.empty(n))
        np.save(os.path.join(outdir, "rank%d.npy" % rank), full.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,ty,rows,k,ncols", [(2, cfi.Q4_K, 301, 512, 3), (3, cfi.Q8_0, 100, 896, 2)])
def test_sharded_decode_equals_unsharded(world, ty, rows, k, ncols):
    import oracle_py as O

    with tempfile.TemporaryDirectory() as td:
        ctx = mp.get_context("spawn")
        port = free_port()
        ps = [ctx.Process(target=rank_main, args=(r, world, port, td, ty, rows, k, ncols)) for r in range(world)]
        for p in ps:
            p.start()
        for p in ps:
            p.join(120)
            assert p.exitcode == 0
        w = cfi.synthetic_weights(ty, rows, k, seed=3)
        x = np.random.default_rng(4).normal(size=(ncols, k)).astype(np.float32)
        want, _, _ = O.cpu_decode_step(ty, w, rows, k, x, ncols, 1)
        want = want.reshape(ncols, rows)
        for r in range(world):
            got = np.load(os.path.join(td, "rank%d.npy" % r))
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
