"""GPU test of cfi_glue_gather_row_shards, the assembly of row-sharded outputs after an all-gather
(the multi-GPU split of the weight rows): the gathered rank slices, with padding rows and, for a
group of products gathered together, a rank stride wider than one product's slice, must give
ggml's column-major output -- the layout shard.gather_columns builds on the CPU ranks."""
import numpy as np
import pytest

import cfi_b200 as cfi
import shard

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nrows,ncols,world,extra_before,extra_after", [
    (8960, 64, 8, 0, 0), (301, 3, 2, 0, 0), (100, 2, 3, 0, 0), (151936, 5, 4, 0, 0),
    (1536, 64, 8, 512, 1000),  # one product inside a group: slices at an offset, rank stride wider
    (257, 7, 5, 33, 11)])
def test_gather_row_shards_matches_the_cpu_assembly(nrows, ncols, world, extra_before, extra_after):
    rng = np.random.default_rng(nrows + world)
    full = rng.normal(size=(ncols, nrows)).astype(np.float32)
    rp = shard.row_split(nrows, world, 0).rows_padded
    stride = extra_before + ncols * rp + extra_after
    gathered = np.full(world * stride, np.nan, dtype=np.float32)
    for r in range(world):
        sh = shard.row_split(nrows, world, r)
        sl = np.full((ncols, rp), np.nan, dtype=np.float32)  # padding rows stay NaN: never read
        sl[:, :sh.rows] = full[:, sh.row0:sh.row0 + sh.rows]
        gathered[r * stride + extra_before:r * stride + extra_before + ncols * rp] = sl.ravel()
    src = torch.from_numpy(gathered).cuda()
    dst = torch.full((ncols * nrows,), np.nan, dtype=torch.float32, device="cuda")
    rc = cfi.lib().cfi_glue_gather_row_shards(src.data_ptr() + 4 * extra_before, dst.data_ptr(), nrows, ncols, world,
                                              stride if (extra_before or extra_after) else 0,
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert np.array_equal(dst.cpu().numpy().reshape(ncols, nrows), full)


def test_gather_row_shards_refuses_bad_shapes():
    src = torch.zeros(16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    L = cfi.lib()
    assert L.cfi_glue_gather_row_shards(src.data_ptr(), src.data_ptr(), 4, 2, 5, 0, s) != 0   # more ranks than rows
    assert L.cfi_glue_gather_row_shards(src.data_ptr(), src.data_ptr(), 8, 2, 2, 3, s) != 0   # stride below a slice
    assert L.cfi_glue_gather_row_shards(src.data_ptr(), src.data_ptr(), 0, 2, 1, 0, s) != 0
