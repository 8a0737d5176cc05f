"""The all-gather of row-sharded products over NVLink peer memory (cfi_peer.h).

Two GPUs, one process each (spawned; gloo carries the IPC handles).  Every rank holds a row
slice of each weight matrix (shard.row_split) and runs the skinny mul_mat_q on it with
cfi_mmq_skinny_group_peers: the launch stores its rows into its own and the other rank's copy of
ggml's column-major output, and ends once the other rank's rows have arrived.  Over several
iterations with new activations each time (so a missed wait would show the last iteration's
rows), both ranks' gathered outputs must equal, bit for bit, the ranks' own shards computed
without peers, and the unsharded products of the oracle within the skinny kernel's tolerance.
The bounded waits are tested on one GPU: a signal that nothing sends ends the wait with the
error word set and the context still usable.  Skipped with fewer GPUs than needed."""
import ctypes as C
import os
import socket
import tempfile

import numpy as np
import pytest

import cfi_b200 as cfi
import oracle_py as O
import shard

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SKINNY_REL = 1e-5
UNIT = 65536  # what one launch adds to its slot on each peer, over all its CTAs
# (type, K, rows of each product of one launch, columns): a q, k, v-like group with ragged
# shards, and one Q8_0 product with an odd column count
GROUPS = [(cfi.Q4_K, 1536, (1536, 256, 257), 64), (cfi.Q8_0, 1536, (5001,), 37)]
ITERS = 3
GATHER_BYTES = 200000  # one rank's slice of the cfi_peer_all_gather test (a multiple of 16)


def gather_slice(rank, it):
    return np.arange(GATHER_BYTES // 4, dtype=np.float32) + np.float32(1000.0 * rank + 0.5 * it)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def cases():
    """Per group: the (params, weights) of each product, and ITERS activation sets."""
    out = []
    for gi, (ty, k, rows, ncols) in enumerate(GROUPS):
        ws = [O.mmq_case(ty, k, r, ncols, 1, 1, 1, 700 + 10 * gi + i)[:2] for i, r in enumerate(rows)]
        ys = [O.mmq_case(ty, k, 16, ncols, 1, 1, 1, 900 + 10 * gi + it)[2] for it in range(ITERS)]
        out.append((ws, ys))
    return out


def layout():
    """Byte offset of each product's gathered output (ncols x nrows fp32) in the peer buffer."""
    off, o = [], 0
    for ty, k, rows, ncols in GROUPS:
        og = []
        for r in rows:
            og.append(o)
            o += (ncols * r * 4 + 255) // 256 * 256
        off.append(og)
    return off, o


class _DevArray:
    """A device range as a torch tensor (no copy; __cuda_array_interface__ without a stream)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "strides": None}


def device_floats(ptr, n):
    return torch.as_tensor(_DevArray(ptr, n), device="cuda")


def rank_main(rank, world, port, outdir):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    pg = None
    try:
        cs = cases()
        off, total = layout()

        def exchange(obj):
            got = [None] * world
            dist.all_gather_object(got, obj)
            return got

        pg = cfi.PeerGroup(rank, world, total, exchange)
        s = torch.cuda.current_stream().cuda_stream
        dev = []
        for (ty, k, rows, ncols), (ws, ys) in zip(GROUPS, cs):
            sh = [shard.row_split(r, world, rank) for r in rows]
            xs = [torch.from_numpy(np.ascontiguousarray(w[1].reshape(r, -1)[h.row0:h.row0 + h.rows]).ravel()).cuda()
                  for w, r, h in zip(ws, rows, sh)]
            dys = [torch.from_numpy(y).cuda() for y in ys]
            dev.append((sh, xs, dys))
        snaps, shards = {}, {}
        for it in range(ITERS):
            for gi, ((ty, k, rows, ncols), (sh, xs, dys)) in enumerate(zip(GROUPS, dev)):
                dsts = [pg.data + off[gi][i] + 4 * h.row0 for i, h in enumerate(sh)]
                cfi.mmq_skinny_group_peers(ty, [x.data_ptr() for x in xs], dys[it].data_ptr(), dsts,
                                           [h.rows for h in sh], k, ncols, pg, stride_col_dst=list(rows), stream=s)
                for i, r in enumerate(rows):  # the gathered outputs as this rank sees them after the launch
                    snaps[it, gi, i] = device_floats(pg.data + off[gi][i], ncols * r).clone()
                # this rank's shard alone, without peers
                loc = [torch.full((ncols * h.rows,), float("nan"), device="cuda") for h in sh]
                cfi.mmq_skinny_group(ty, [x.data_ptr() for x in xs], dys[it].data_ptr(), [t.data_ptr() for t in loc],
                                     [h.rows for h in sh], k, ncols, stream=s)
                for i in range(len(rows)):
                    shards[it, gi, i] = loc[i]
        # cfi_peer_all_gather: a new slice per iteration, the gathered range read after each
        pg2 = cfi.PeerGroup(rank, world, world * GATHER_BYTES, exchange)
        gat = {}
        for it in range(ITERS):
            src = torch.from_numpy(gather_slice(rank, it)).cuda()
            pg2.all_gather(src.data_ptr(), GATHER_BYTES, 0, stream=s)
            gat[it] = device_floats(pg2.data, world * GATHER_BYTES // 4).clone()
        torch.cuda.synchronize()
        err = cfi.lib().cfi_device_error()
        np.savez(os.path.join(outdir, "rank%d.npz" % rank), err=np.uint32(err),
                 **{"g_%d_%d_%d" % key: t.cpu().numpy() for key, t in snaps.items()},
                 **{"s_%d_%d_%d" % key: t.cpu().numpy() for key, t in shards.items()},
                 **{"a_%d" % it: t.cpu().numpy() for it, t in gat.items()})
        dist.barrier()  # every rank done with the others' buffers before any is unmapped
        pg2.close()
    finally:
        if pg is not None:
            pg.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_all_gather_matches_the_shards_and_the_oracle():
    world = 2
    with tempfile.TemporaryDirectory() as td:
        ctx = torch.multiprocessing.get_context("spawn")
        port = free_port()
        ps = [ctx.Process(target=rank_main, args=(r, world, port, td)) for r in range(world)]
        for p in ps:
            p.start()
        for p in ps:
            p.join(300)
        assert [p.exitcode for p in ps] == [0] * world
        res = [np.load(os.path.join(td, "rank%d.npz" % r)) for r in range(world)]
        assert [int(r["err"]) for r in res] == [0] * world
        cs = cases()
        for it in range(ITERS):
            for gi, ((ty, k, rows, ncols), (ws, ys)) in enumerate(zip(GROUPS, cs)):
                for i, r in enumerate(rows):
                    parts = []
                    for rk in range(world):
                        h = shard.row_split(r, world, rk)
                        parts.append(res[rk]["s_%d_%d_%d" % (it, gi, i)].reshape(ncols, h.rows))
                    want = np.concatenate(parts, axis=1)
                    for rk in range(world):
                        got = res[rk]["g_%d_%d_%d" % (it, gi, i)].reshape(ncols, r)
                        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (it, gi, i, rk)
                    p, x = ws[i]
                    ref = O.mmq_ref(ty, p, x, ys[it], ncols * r)
                    assert O.rel_l2(want.ravel(), ref) < SKINNY_REL, (it, gi, i)
        # cfi_peer_all_gather: every rank's slice in rank order on every rank, each iteration's own
        for it in range(ITERS):
            want = np.concatenate([gather_slice(rk, it) for rk in range(world)])
            for rk in range(world):
                assert np.array_equal(res[rk]["a_%d" % it], want), (it, rk)


def one_gpu_group(ctr, scratch):
    """Rank 0 of a group of two on one GPU whose peer never runs: its slot on the 'peer' is a
    scratch word here; sig_local = ctr[0:2], expect = ctr[4:6]."""
    ps = cfi.PeerSet()
    ps.rank, ps.world = 0, 2
    ps.sig_remote[1] = scratch.data_ptr()
    ps.sig_local, ps.expect = ctr.data_ptr(), ctr.data_ptr() + 16
    return ps


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_peer_barrier_gives_up_with_the_error_word(monkeypatch):
    """A rank whose peer never signals: the barrier's wait ends after CFI_PEER_WAIT_MS with
    0x9e0000 | peer in the error word, later waits give up at once until the word is read, and
    the next kernels run normally."""
    L = cfi.lib()
    torch.cuda.synchronize()
    assert L.cfi_device_error() == 0
    ctr = torch.zeros(16, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(4, dtype=torch.int32, device="cuda")
    ps = one_gpu_group(ctr, scratch)
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    monkeypatch.setenv("CFI_PEER_WAIT_MS", "200")
    assert L.cfi_peer_barrier(C.byref(ps), s) == 0
    assert L.cfi_peer_barrier(C.byref(ps), s) == 0  # gives up at once: the first one's code is still set
    torch.cuda.synchronize()
    assert L.cfi_device_error() == 0x9e0001
    assert int(scratch[0]) == 2 * UNIT  # it signalled its peer each time
    # a peer that has signalled three times satisfies the next wait
    ctr[1] = 3 * UNIT
    assert L.cfi_peer_barrier(C.byref(ps), s) == 0
    torch.cuda.synchronize()
    assert L.cfi_device_error() == 0
    assert ctr.cpu().tolist()[4:6] == [0, 3 * UNIT]
    y = torch.ones(1024, device="cuda") * 3
    assert float(y.sum()) == 3072.0


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_peer_product_whose_peer_never_signals_ends_with_the_error_word(monkeypatch):
    """The product launch's own wait is bounded the same way; its local rows are written."""
    L = cfi.lib()
    torch.cuda.synchronize()
    assert L.cfi_device_error() == 0
    ty, k, rows, ncols = cfi.Q4_K, 1536, 300, 16
    p, x, y, n = O.mmq_case(ty, k, rows, ncols, 1, 1, 1, 77)
    ctr = torch.zeros(16, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(4, dtype=torch.int32, device="cuda")
    remote = torch.zeros(n, dtype=torch.float32, device="cuda")  # the 'peer' copy of the output
    dst = torch.full((n,), float("nan"), device="cuda")
    ps = one_gpu_group(ctr, scratch)
    ps.delta[1] = remote.data_ptr() - dst.data_ptr()
    monkeypatch.setenv("CFI_PEER_WAIT_MS", "200")
    dx, dy = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    P, U = C.c_void_p * 1, C.c_uint32 * 1
    rc = L.cfi_mmq_skinny_group_peers(ty, 1, P(dx.data_ptr()), C.c_void_p(dy.data_ptr()), P(dst.data_ptr()), U(rows),
                                      U(k // 256), U(rows), k, ncols, ncols, C.byref(ps),
                                      C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert L.cfi_device_error() == 0x9e0001
    want = O.mmq_ref(ty, p, x, y, n)
    got = dst.cpu().numpy()
    assert O.rel_l2(got, want) < SKINNY_REL
    assert np.array_equal(remote.cpu().numpy().view(np.uint32), got.view(np.uint32))
    assert int(scratch[0]) == UNIT  # one launch's whole signal, over all its CTAs


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_peer_all_gather_of_a_group_of_one_copies():
    """world 1: the slice lands at dst (no signal, no wait)."""
    L = cfi.lib()
    ps = cfi.PeerSet()
    ps.rank, ps.world = 0, 1
    src = torch.arange(4096, dtype=torch.float32, device="cuda")
    dst = torch.full((4096 + 16,), float("nan"), device="cuda")
    assert L.cfi_peer_all_gather(C.c_void_p(src.data_ptr()), 16384, C.c_void_p(dst.data_ptr() + 64), C.byref(ps),
                                 C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    torch.cuda.synchronize()
    assert L.cfi_device_error() == 0
    assert torch.equal(dst[16:], src) and torch.isnan(dst[:16]).all()


def test_peer_calls_refuse_bad_arguments():
    L = cfi.lib()
    buf = C.c_void_p(1 << 20)
    ps = cfi.PeerSet()
    ps.rank, ps.world = 0, 9
    assert L.cfi_peer_barrier(C.byref(ps), None) != 0    # more ranks than a node's GPUs
    ps.rank, ps.world = 2, 2
    assert L.cfi_peer_barrier(C.byref(ps), None) != 0    # rank outside the group
    ps.rank, ps.world = 0, 2
    ps.sig_local, ps.expect = buf.value, buf.value
    assert L.cfi_peer_barrier(C.byref(ps), None) != 0    # no slot on the peer
    ps.sig_remote[1] = buf.value
    ps.expect = None
    assert L.cfi_peer_barrier(C.byref(ps), None) != 0    # no wait counts
    assert L.cfi_peer_barrier(None, None) != 0
    P, U = C.c_void_p * 1, C.c_uint32 * 1
    args = (P(buf), buf, P(buf), U(16), U(8), U(16), 256, 8, 8)
    assert L.cfi_mmq_skinny_group_peers(cfi.Q4_K, 1, *args, C.byref(ps), None) != 0
    assert L.cfi_mmq_skinny_group_peers(cfi.Q4_K, 1, *args, None, None) != 0
    one = cfi.PeerSet()
    one.rank, one.world = 0, 1
    assert L.cfi_peer_all_gather(buf, 24, buf, C.byref(one), None) != 0               # not 16-byte sized
    assert L.cfi_peer_all_gather(C.c_void_p(buf.value + 8), 32, buf, C.byref(one), None) != 0  # source alignment
    assert L.cfi_peer_all_gather(buf, 32, C.c_void_p(buf.value + 4), C.byref(one), None) != 0  # destination alignment
    assert L.cfi_peer_all_gather(buf, 32, buf, None, None) != 0
