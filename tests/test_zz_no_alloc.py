"""GPU test of cfi_mmq_static_scratch, the prefill GEMM for callers that may not allocate device
memory (a launch hook inside the application's cuLaunchKernel, a serving process whose pool holds
all free HBM, code that cannot take cudaMalloc's implicit synchronisation): its fp16 activation
scratch is a fixed array inside the library instead of a cudaMalloc'd buffer.

Collected last on purpose.  Each call goes through the C ABI and is checked against the regular
entry point (cfi_subst_launch of mul_mat_q) on the same inputs, for two calls in a row that leave
different contents behind in the shared array; the device's free memory is the same before and
after a repeated call (the first call on a device may still load the library's kernels, which
takes memory once); a problem too large for the array is refused before anything runs."""
import ctypes as C

import numpy as np
import pytest

import cfi_b200 as cfi
import oracle_py as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REL_L2 = 1e-3
LIMIT = 8 * 1024 * 1024


def stream():
    return torch.cuda.current_stream().cuda_stream


def mmq_args(x, y, dst, words):
    vals = [("ptr", x), ("ptr", y), ("ptr", 0), ("ptr", 0), ("ptr", dst), ("ptr", 0)] + [("u32", w) for w in words]
    return cfi.KernelArgs(vals)


def words(p):
    return [p.ncols_x, p.nrows_x, p.ncols_dst, p.stride_row_x, p.ncols_y, p.stride_col_dst, p.channel_ratio,
            p.nchannels_y, p.stride_channel_x, p.stride_channel_y, p.stride_channel_dst, p.sample_ratio, p.nsamples_y,
            p.stride_sample_x, p.stride_sample_y, p.stride_sample_dst, p.ncols_dst]


def static_call(ty, args):
    why = C.create_string_buffer(256)
    rc = cfi.lib().cfi_mmq_static_scratch(ty, args.ptrs, C.c_void_p(stream()), why, 256)
    return rc, why.value.decode()


def test_static_scratch_gemm_matches_the_regular_entry_point_twice_in_a_row():
    assert torch.cuda.is_available()
    torch.cuda.set_device(0)
    ctx = cfi.Ctx(0)
    g = cfi.GgmlCaller(ctx, "all")
    cases = [(cfi.Q8_0, (896, 300, 631, 1, 1, 1), 41), (cfi.Q4_K, (2048, 129, 77, 2, 1, 1), 42)]
    for ty, (ncols_x, nrows, ncols, nch, ratio, ns), seed in cases:
        p, x, y, n = O.mmq_case(ty, ncols_x, nrows, ncols, nch, ratio, ns, seed)
        dx, dy = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
        d_static = torch.full((n,), float("nan"), dtype=torch.float32, device="cuda")
        d_regular = torch.zeros(n, dtype=torch.float32, device="cuda")
        rc, why = static_call(ty, mmq_args(dx.data_ptr(), dy.data_ptr(), d_static.data_ptr(), words(p)))
        assert rc == 0, why
        g.mmq_words(ty, dx.data_ptr(), dy.data_ptr(), d_regular.data_ptr(), words(p), stream=stream())
        torch.cuda.synchronize()
        assert cfi.lib().cfi_device_error() == 0
        got, want = d_static.cpu().numpy(), d_regular.cpu().numpy()
        assert np.all(np.isfinite(got))
        assert O.rel_l2(got, want) < REL_L2
        assert O.rel_l2(got, O.mmq_ref(ty, p, x, y, n)) < REL_L2
        # the same call again: no device memory taken (a cudaMalloc'd scratch or workspace would
        # lower the free bytes; nothing else allocates between the two readings)
        d_static.fill_(float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rc, why = static_call(ty, mmq_args(dx.data_ptr(), dy.data_ptr(), d_static.data_ptr(), words(p)))
        assert rc == 0, why
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free_before
        assert np.array_equal(d_static.cpu().numpy(), got)
    ctx.close()


def test_static_scratch_refuses_problems_larger_than_its_array():
    torch.cuda.set_device(0)
    k, ncols = 4096, 1100  # 1100 x 4096 x 2 bytes > 8 MiB
    assert ncols * k * 2 > LIMIT
    dst = torch.zeros(16, dtype=torch.float32, device="cuda")
    w = [k, 128, ncols, k // 32, ncols, 128, 1, 1, 0, 0, 0, 1, 1, 0, 0, 0, ncols]
    rc, why = static_call(cfi.Q8_0, mmq_args(dst.data_ptr(), dst.data_ptr(), dst.data_ptr(), w))
    assert rc != 0 and "static scratch holds 8388608" in why
    torch.cuda.synchronize()
