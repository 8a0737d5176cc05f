"""The host side of the peer-memory all-gather on CPU ranks (gloo, world size 2 and 3).

cfi_b200.PeerGroup exchanges every rank's buffer handle with torch.distributed, maps the other
ranks' buffers and fills the CfiPeerSet that the kernels read: delta[r] (rank r's buffer as mapped
here minus this rank's), sig_remote[r] (this rank's signal slot inside rank r's buffer) and the
local slots.  Here the library's allocation and mapping calls are replaced by a stand-in that
hands out distinct fake addresses (no device memory is touched), and every rank checks its set
against the others' bases: the layout the kernels rely on, as the GPU test on two GPUs uses it."""
import ctypes as C
import os
import socket
import tempfile

import numpy as np
import pytest

import cfi_b200 as cfi

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

BASE = 0x7f0000000000
STRIDE = 1 << 32   # rank r's buffer at BASE + r * STRIDE in its own process
MAP = 1 << 36      # rank q's buffer as mapped by rank r: BASE + MAP * (r + 1) + q * STRIDE


class FakePeerLib:
    """cfi_peer_alloc / open / close / free over fake addresses; the handle names the rank."""

    def __init__(self, rank):
        self.rank = rank
        self.opened, self.closed, self.freed = [], [], []

    def cfi_peer_alloc(self, nbytes, ptr, handle):
        ptr._obj.value = BASE + self.rank * STRIDE
        C.memmove(handle, C.create_string_buffer(b"rank%02d" % self.rank, cfi.PEER_HANDLE_BYTES),
                  cfi.PEER_HANDLE_BYTES)
        self.nbytes = nbytes
        return 0

    def cfi_peer_open(self, handle, ptr):
        q = int(bytes(handle)[4:6])
        ptr._obj.value = BASE + MAP * (self.rank + 1) + q * STRIDE
        self.opened.append(q)
        return 0

    def cfi_peer_close(self, p):
        self.closed.append(p.value)
        return 0

    def cfi_peer_free(self, p):
        self.freed.append(p.value)
        return 0


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rank_main(rank, world, port, outdir, nbytes):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fake = FakePeerLib(rank)
        cfi._lib = fake  # the library calls PeerGroup makes go to the stand-in

        def exchange(obj):
            got = [None] * world
            dist.all_gather_object(got, obj)
            return got

        pg = cfi.PeerGroup(rank, world, nbytes, exchange)
        ps = pg.peers
        np.savez(os.path.join(outdir, "rank%d.npz" % rank), data=pg.data, data_bytes=pg.data_bytes,
                 delta=np.array(ps.delta[:world], dtype=np.int64),
                 sig_remote=np.array([v or 0 for v in ps.sig_remote[:world]], dtype=np.uint64),
                 sig_local=ps.sig_local, expect=ps.expect, alloc=fake.nbytes, opened=np.array(sorted(fake.opened)))
        pg.close()
        assert sorted(fake.closed) == sorted(BASE + MAP * (rank + 1) + q * STRIDE for q in range(world) if q != rank)
        assert fake.freed == [BASE + rank * STRIDE]
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,nbytes", [(2, 1000), (3, 491520)])
def test_peer_group_layout_over_gloo_ranks(world, nbytes):
    with tempfile.TemporaryDirectory() as td:
        ctx = mp.get_context("spawn")
        port = free_port()
        ps = [ctx.Process(target=rank_main, args=(r, world, port, td, nbytes)) for r in range(world)]
        for p in ps:
            p.start()
        for p in ps:
            p.join(120)
            assert p.exitcode == 0
        res = [np.load(os.path.join(td, "rank%d.npz" % r)) for r in range(world)]
    data_bytes = (nbytes + 255) // 256 * 256
    for r, d in enumerate(res):
        base = BASE + r * STRIDE
        assert int(d["data"]) == base and int(d["data_bytes"]) == data_bytes
        # own signal slots right after the data, the wait counts after them, all in the allocation
        assert int(d["sig_local"]) == base + data_bytes and int(d["expect"]) == base + data_bytes + 4 * world
        assert int(d["alloc"]) >= data_bytes + 8 * world
        assert list(d["opened"]) == [q for q in range(world) if q != r]
        for q in range(world):
            mapped = base if q == r else BASE + MAP * (r + 1) + q * STRIDE
            assert int(d["delta"][q]) == mapped - base
            # rank q adds rank r's signal into slot r of q's buffer: q's sig_local + 4 r, as mapped here
            assert int(d["sig_remote"][q]) == mapped + data_bytes + 4 * r
