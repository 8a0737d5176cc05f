"""GPU tests of the cuBLAS-compatible GEMM (tcgen05 for ggml's f16/bf16 layout, SIMT otherwise),
against a plain PyTorch fp32 reference of the same op (fp16/bf16 inputs are exact in fp32) and the
oracle's literal cuBLAS-semantics reference (crates/cublas_shim/src/plan.rs:346-362) on a slice.
Shapes: ggml's prefill GEMMs (tests/gpu/hw_xmx_gemm.rs:688-727) and attention GEMMs with heads 14 /
GQA ratio 7 (hw_xmx_gemm.rs:456-470)."""
import ctypes as C

import numpy as np
import pytest

import cfi_b200 as cfi
import oracle_py as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REL_L2 = 1e-3
B = cfi.Blas


@pytest.fixture(scope="module")
def blas():
    assert torch.cuda.is_available()
    b = cfi.Blas(torch.cuda.current_stream().cuda_stream)
    yield b
    b.close()


def rel(a, b):
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).norm() / b.norm())


def sync():
    torch.cuda.synchronize()
    assert cfi.lib().cfi_device_error() == 0


@pytest.mark.parametrize("m,n,k", [(4864, 631, 896), (896, 631, 4864), (128, 1, 64), (300, 17, 200), (4096, 512, 4096)])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_gemm_ex_tn_on_tensor_cores(blas, m, n, k, dt):
    torch.manual_seed(m + n + k)
    at = B.R_16F if dt == torch.float16 else B.R_16BF
    A = torch.randn(m, k, device="cuda").to(dt)        # column-major k x m == row-major m x k
    Bm = torch.randn(n, k, device="cuda").to(dt)       # column-major k x n
    Cm = torch.zeros(n, m, device="cuda")              # column-major m x n, ldc = m
    st = blas.gemm_ex(B.OP_T, B.OP_N, m, n, k, 1.0, A.data_ptr(), at, k, Bm.data_ptr(), at, k, 0.0, Cm.data_ptr(),
                      B.R_32F, m)
    assert st == 0
    sync()
    assert blas.last_path() == (3 if n <= 8 else 1), "expected the skinny (n <= 8) or the tcgen05 path"
    want = (A.float() @ Bm.float().T).T
    assert rel(Cm, want) < REL_L2
    if m * n <= 5000000 and dt == torch.float16:
        cols = min(n, 3)
        a16 = A.cpu().numpy()
        b16 = np.ascontiguousarray(Bm[:cols].cpu().numpy())
        c = np.zeros((cols, m), dtype=np.float32)
        O.lib().cfo_reference_gemm(1, 0, m, cols, k, C.c_float(1.0), a16.ctypes.data, 2, k, b16.ctypes.data, k,
                                   C.c_float(0.0), c.ctypes.data, 0, m)
        assert O.rel_l2(Cm[:cols].cpu().numpy(), c) < REL_L2


def test_gemm_ex_alpha_beta_f16_out_and_device_scalars(blas):
    torch.manual_seed(1)
    m, n, k = 257, 129, 320
    A = torch.randn(m, k, device="cuda").half()
    Bm = torch.randn(n, k, device="cuda").half()
    C0 = torch.randn(n, m, device="cuda").half()
    Cm = C0.clone()
    st = blas.gemm_ex(B.OP_T, B.OP_N, m, n, k, 0.5, A.data_ptr(), B.R_16F, k, Bm.data_ptr(), B.R_16F, k, -2.0,
                      Cm.data_ptr(), B.R_16F, m, compute=B.COMPUTE_16F)
    assert st == 0
    sync()
    want = 0.5 * (A.float() @ Bm.float().T).T - 2.0 * C0.float()
    assert rel(Cm.float(), want) < 2e-3  # fp16 output rounding
    # device pointer mode: alpha/beta read on the GPU
    dal = torch.tensor([0.25], device="cuda")
    dbe = torch.tensor([0.0], device="cuda")
    Cf = torch.full((n, m), 7.0, device="cuda")
    assert blas.set_pointer_mode(1) == 0
    st = blas.gemm_ex(B.OP_T, B.OP_N, m, n, k, 0, A.data_ptr(), B.R_16F, k, Bm.data_ptr(), B.R_16F, k, 0,
                      Cf.data_ptr(), B.R_32F, m, dev_scalars=(C.c_void_p(dal.data_ptr()), C.c_void_p(dbe.data_ptr())))
    assert blas.set_pointer_mode(0) == 0
    assert st == 0
    sync()
    assert rel(Cf, 0.25 * (A.float() @ Bm.float().T).T) < REL_L2


def test_attention_gemms_strided_and_pointer_arrays(blas):
    """KQ: m = n_kv, n = n_tokens, k = 64 per head (f16 -> f32); KQV: m = 64, n = n_tokens,
    k = n_kv (f16 -> f16, COMPUTE_16F); 14 query heads over 2 KV heads (ratio 7)."""
    torch.manual_seed(2)
    heads, kv_heads, d, n_kv, n_tok = 14, 2, 64, 631, 7
    K = torch.randn(kv_heads, n_kv, d, device="cuda").half()
    Q = torch.randn(heads, n_tok, d, device="cuda").half()
    KQ = torch.zeros(heads, n_tok, n_kv, device="cuda")
    # strided over the first kv head only (one GEMM per head with its own K): use pointer arrays for GQA
    ks = [K[h // (heads // kv_heads)] for h in range(heads)]
    Aarr = torch.tensor([t.data_ptr() for t in ks], dtype=torch.int64, device="cuda")
    Barr = torch.tensor([Q[h].data_ptr() for h in range(heads)], dtype=torch.int64, device="cuda")
    Carr = torch.tensor([KQ[h].data_ptr() for h in range(heads)], dtype=torch.int64, device="cuda")
    st = blas.gemm_batched_ex(B.OP_T, B.OP_N, n_kv, n_tok, d, 0.125, Aarr.data_ptr(), B.R_16F, d, Barr.data_ptr(),
                              B.R_16F, d, 0.0, Carr.data_ptr(), B.R_32F, n_kv, heads)
    assert st == 0
    sync()
    want = torch.stack([0.125 * (ks[h].float() @ Q[h].float().T).T for h in range(heads)])
    assert rel(KQ, want) < REL_L2
    # strided batched on the tensor cores (one KV head per query head here)
    Kf = K.repeat_interleave(heads // kv_heads, dim=0).contiguous()
    KQ2 = torch.zeros_like(KQ)
    st = blas.gemm_strided_batched_ex(B.OP_T, B.OP_N, n_kv, n_tok, d, 0.125, Kf.data_ptr(), B.R_16F, d, n_kv * d,
                                      Q.data_ptr(), B.R_16F, d, n_tok * d, 0.0, KQ2.data_ptr(), B.R_32F, n_kv,
                                      n_tok * n_kv, heads)
    assert st == 0
    sync()
    assert blas.last_path() == 3  # 7 columns: the skinny kernel
    assert rel(KQ2, want) < REL_L2
    # KQV: V^T (d x n_kv per head, stored n_kv x d column-major... op(A) = A^T with A stored n_kv x d)
    V = torch.randn(heads, d, n_kv, device="cuda").half()      # column-major n_kv x d per head
    P = torch.softmax(want, dim=-1).half()                       # column-major n_kv x n_tok per head
    O16 = torch.zeros(heads, n_tok, d, device="cuda").half()
    st = blas.gemm_strided_batched_ex(B.OP_T, B.OP_N, d, n_tok, n_kv, 1.0, V.data_ptr(), B.R_16F, n_kv, d * n_kv,
                                      P.data_ptr(), B.R_16F, n_kv, n_tok * n_kv, 0.0, O16.data_ptr(), B.R_16F, d,
                                      n_tok * d, heads, compute=B.COMPUTE_16F)
    assert st == 0
    sync()
    wantv = torch.stack([(V[h].float() @ P[h].float().T).T for h in range(heads)])
    assert rel(O16.float(), wantv) < 2e-3


@pytest.mark.parametrize("n", [1, 3, 7, 8])
@pytest.mark.parametrize("k", [64, 63, 680, 1000])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_skinny_gemm_batched_beta_and_tails(blas, n, k, dt):
    """n <= 8 columns: the warp-per-row kernel, strided batches, k not a multiple of 8 (lda = ldb
    rounded up to 8 so the rows stay 16-byte aligned), 16-bit output with beta, f32 output."""
    torch.manual_seed(n * 1000 + k)
    at = B.R_16F if dt == torch.float16 else B.R_16BF
    m, batch = 300, 3
    ld = (k + 7) // 8 * 8
    A = torch.randn(batch, m, ld, device="cuda").to(dt)
    Bm = torch.randn(batch, n, ld, device="cuda").to(dt)
    C0 = torch.randn(batch, n, m, device="cuda").to(dt)  # output in the input type (cuBLAS rule)
    Cm = C0.clone()
    st = blas.gemm_strided_batched_ex(B.OP_T, B.OP_N, m, n, k, 0.5, A.data_ptr(), at, ld, m * ld, Bm.data_ptr(), at,
                                      ld, n * ld, 1.5, Cm.data_ptr(), at, m, n * m, batch)
    assert st == 0
    sync()
    assert blas.last_path() == 3
    want = torch.stack([0.5 * (A[z, :, :k].float() @ Bm[z, :, :k].float().T).T + 1.5 * C0[z].float()
                        for z in range(batch)])
    assert rel(Cm.float(), want) < (2e-3 if dt == torch.float16 else 1e-2)  # output rounding
    Cf = torch.zeros(batch, n, m, device="cuda")
    st = blas.gemm_strided_batched_ex(B.OP_T, B.OP_N, m, n, k, 1.0, A.data_ptr(), at, ld, m * ld, Bm.data_ptr(), at,
                                      ld, n * ld, 0.0, Cf.data_ptr(), B.R_32F, m, n * m, batch)
    assert st == 0
    sync()
    want = torch.stack([(A[z, :, :k].float() @ Bm[z, :, :k].float().T).T for z in range(batch)])
    assert rel(Cf, want) < 1e-5


def test_skinny_switch_routes_to_tensor_cores(blas, monkeypatch):
    """CFI_GEMM_SKINNY=0 sends n <= 8 to the tcgen05 kernel; both give the same result."""
    torch.manual_seed(9)
    m, n, k = 680, 7, 64
    A = torch.randn(m, k, device="cuda").half()
    Bm = torch.randn(n, k, device="cuda").half()
    out = []
    for env, path in (("1", 3), ("0", 1)):
        monkeypatch.setenv("CFI_GEMM_SKINNY", env)
        Cm = torch.zeros(n, m, device="cuda")
        assert blas.gemm_ex(B.OP_T, B.OP_N, m, n, k, 1.0, A.data_ptr(), B.R_16F, k, Bm.data_ptr(), B.R_16F, k, 0.0,
                            Cm.data_ptr(), B.R_32F, m) == 0
        sync()
        assert blas.last_path() == path
        out.append(Cm)
    want = (A.float() @ Bm.float().T).T
    assert rel(out[0], want) < 1e-5 and rel(out[1], want) < 1e-5


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 1), (0, 1), (1, 0)])
def test_other_transposes_and_sgemm(blas, ta, tb):
    torch.manual_seed(3 + ta * 2 + tb)
    m, n, k = 77, 45, 130
    # a column-major R x Cc matrix is the row-major torch tensor of shape (Cc, R)
    A = torch.randn(m, k, device="cuda") if ta else torch.randn(k, m, device="cuda")
    Bm = torch.randn(k, n, device="cuda") if tb else torch.randn(n, k, device="cuda")
    lda = A.shape[1]
    ldb = Bm.shape[1]
    opA = A if ta else A.T   # op(A) as an m x k matrix
    opB = Bm if tb else Bm.T
    Cm = torch.zeros(n, m, device="cuda")
    assert blas.sgemm(ta, tb, m, n, k, 1.5, A.data_ptr(), lda, Bm.data_ptr(), ldb, 0.0, Cm.data_ptr(), m) == 0
    sync()
    assert blas.last_path() == 2
    want = 1.5 * (opA @ opB).T
    assert rel(Cm, want) < 1e-5
    Ah, Bh = A.half(), Bm.half()
    Ch = torch.zeros(n, m, device="cuda")
    assert blas.gemm_ex(ta, tb, m, n, k, 1.0, Ah.data_ptr(), B.R_16F, lda, Bh.data_ptr(), B.R_16F, ldb, 0.0,
                        Ch.data_ptr(), B.R_32F, m) == 0
    sync()
    wanth = ((Ah.float() if ta else Ah.float().T) @ (Bh.float() if tb else Bh.float().T)).T
    assert rel(Ch, wanth) < REL_L2
