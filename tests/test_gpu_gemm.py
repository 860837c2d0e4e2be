"""Parity of the 3xTF32 tcgen05 GEMM.

Small shapes are checked against the oracle (reference summation order) and a
float64 product; tolerance: per-element |gpu - ref| <= 1e-4 * sum_k |a_ik b_kj|
(and in practice ~1e-6).  Full-size (4096^3, config 3) results are checked
against float64 torch norm-relative <= 1e-4 (the GEMM tolerance of the
target); measured ~3e-5, dominated by the tensor cores' fp32 accumulation
over 3 x 512 chained MMAs.
"""
import numpy as np
import pytest
import torch

from ferrograd_b200 import data, kernels
from ferrograd_b200._lib import EPI_BIAS, EPI_BIAS_RELU, EPI_NONE, EPI_RELU_MASK

pytestmark = pytest.mark.gpu


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def elemwise_bound(A, B):
    """sum_k |A[m,k]| |B[n,k]| in float64 (A: [M,K], B: [N,K])."""
    return np.abs(A.astype(np.float64)) @ np.abs(B.astype(np.float64)).T


def check_close(got, ref, bound, rtol=1e-4):
    err = np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64))
    worst = np.max(err / np.maximum(bound, 1e-30))
    assert worst <= rtol, worst


SHAPES = [(128, 128, 32), (256, 128, 784), (200, 136, 100), (1, 16, 4), (130, 260, 36),
          (384, 512, 1024)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_layouts_vs_oracle(oracle, M, N, K, a_mn, b_mn):
    if (a_mn and M % 4) or (b_mn and N % 4):
        pytest.skip("MN-major pitch must be a multiple of 4")
    A = data.uniform((M, K), 8, -1 / 64, 1 / 64)
    B = data.uniform((N, K), 9, -1 / 64, 1 / 64)
    ta = cuda(A.T) if a_mn else cuda(A)
    tb = cuda(B.T) if b_mn else cuda(B)
    got = kernels.gemm(ta, tb, a_mn_major=a_mn, b_mn_major=b_mn).cpu().numpy()
    ref = oracle.gemm_fwd(A, B)
    check_close(got, ref, elemwise_bound(A, B))
    exact = A.astype(np.float64) @ B.astype(np.float64).T
    check_close(got, exact, elemwise_bound(A, B), rtol=2e-6)


def test_gemm_backward_contractions_vs_oracle(oracle):
    """dA = G.B (ReduceAxis over N) and dBt = G^T.A (over M), routed as GEMMs."""
    M, N, K = 256, 192, 160
    A = data.uniform((M, K), 8, -1 / 64, 1 / 64)
    Bt = data.uniform((N, K), 9, -1 / 64, 1 / 64)
    G = data.normal((M, N), 10, std=1e-2)
    # dA[m,k] = sum_n G[m,n] Bt[n,k]: A-operand G (K-major over n), B-operand Bt [n,k] = [K,N]
    dA = kernels.gemm(cuda(G), cuda(Bt), b_mn_major=True).cpu().numpy()
    check_close(dA, oracle.gemm_dx(G, Bt), elemwise_bound(G, Bt.T))
    # dBt[n,k] = sum_m G[m,n] A[m,k]: both operands MN-major over the batch
    dBt = kernels.gemm(cuda(G), cuda(A), a_mn_major=True, b_mn_major=True).cpu().numpy()
    check_close(dBt, oracle.gemm_dw(A, G), elemwise_bound(G.T, A.T))


def test_gemm_epilogues(oracle):
    M, N, K = 256, 256, 128
    A = data.uniform((M, K), 1, -1, 1)
    B = data.uniform((N, K), 2, -1, 1)
    bias = data.normal(N, 3)
    base = A.astype(np.float64) @ B.astype(np.float64).T
    bound = elemwise_bound(A, B) + 1e-3
    z = kernels.gemm(cuda(A), cuda(B), epilogue=EPI_BIAS, bias=cuda(bias)).cpu().numpy()
    check_close(z, base + bias, bound)
    out_lo = torch.empty((M, N), device="cuda")
    r = kernels.gemm(cuda(A), cuda(B), epilogue=EPI_BIAS_RELU, bias=cuda(bias), out_lo=out_lo)
    rn = r.cpu().numpy()
    check_close(rn, np.maximum(base + bias, 0), bound)
    assert np.all(rn[(base + bias) < -1e-3] == 0)
    hi = (r.view(torch.int32) & -8192).view(torch.float32)
    assert torch.equal(hi + out_lo, r)
    mask = cuda(data.normal((M, N), 4))
    mz = kernels.gemm(cuda(A), cuda(B), epilogue=EPI_RELU_MASK, mask=mask).cpu().numpy()
    check_close(mz, np.where(mask.cpu().numpy() > 0, base, 0), bound)


def test_tensor_core_reads_fp32_as_truncated_tf32():
    """The 3xTF32 split assumes the MMA drops the low 13 mantissa bits; one
    pass on 1 + 3*2^-12 tells truncation (1.0) from rounding (1 + 2^-10)."""
    a = torch.zeros((1, 4), device="cuda")
    a[0, 0] = 1.0 + 3 * 2.0 ** -12
    b = torch.zeros((16, 4), device="cuda")
    b[:, 0] = 1.0
    got = kernels.gemm(a, b, one_pass=True)
    assert got[0, 0].item() == 1.0
    full = kernels.gemm(a, b)
    assert full[0, 0].item() == 1.0 + 3 * 2.0 ** -12


def test_gemm_full_size_precision():
    """Config 3: A,B U(+-1/64) [4096,4096] (matmul via Linear-style [N,K] rhs),
    plus the two backward contractions with G N(0, 1e-2)."""
    n = data.C3_N
    g = torch.Generator(device="cuda").manual_seed(8)
    A = (torch.rand((n, n), device="cuda", generator=g) * 2 - 1) / 64
    Bm = (torch.rand((n, n), device="cuda", generator=g) * 2 - 1) / 64   # B[k, n]
    G = torch.randn((n, n), device="cuda", generator=g) * 1e-2

    def nrel(got, ref):
        return (torch.max(torch.abs(got.double() - ref)) / torch.max(torch.abs(ref))).item()

    # C = A.B: A [M,K] K-major, B stored [K,N] -> MN-major
    C = kernels.gemm(A, Bm, b_mn_major=True)
    err_c = nrel(C, A.double() @ Bm.double())
    print(f"config-3 GEMM norm-relative error vs float64: {err_c:.3e}")
    assert err_c <= 1e-4
    # dA = G.B^T: A-operand G [M, N] K-major, B-operand B [K, N] K-major over N
    dA = kernels.gemm(G, Bm)
    assert nrel(dA, G.double() @ Bm.double().T) <= 1e-4
    # dB = A^T.G: A-operand A [M,K] -> MN-major over M, B-operand G [M,N] MN-major
    dB = kernels.gemm(A, G, a_mn_major=True, b_mn_major=True)
    assert nrel(dB, A.double().T @ G.double()) <= 1e-4
    one = kernels.gemm(A, Bm, b_mn_major=True, one_pass=True)
    assert nrel(one, A.double() @ Bm.double()) > 2 * err_c
    kernels.check_device_error()


@pytest.mark.parametrize("M,N,K", [(256, 512, 2048), (128, 128, 8192), (1000, 300, 1000)])
def test_gemm_stream_k_tail_with_epilogues(M, N, K):
    """Few output tiles and a long K: the persistent grid splits the tiles'
    k-blocks over many CTAs (stream-K), and the CTA holding each tile's
    first k-block adds the others' partials before the fused epilogue.  The
    result must match float64 per element, keep the epilogue semantics and
    be bitwise reproducible run to run (partials are added in CTA order)."""
    A = data.uniform((M, K), 11, -1, 1)
    B = data.uniform((N, K), 12, -1, 1)
    bias = data.normal(N, 13)
    base = A.astype(np.float64) @ B.astype(np.float64).T
    bound = elemwise_bound(A, B) + 1e-3
    ta, tb, tbias = cuda(A), cuda(B), cuda(bias)
    plain = kernels.gemm(ta, tb).cpu().numpy()
    check_close(plain, base, bound)
    out_lo = torch.empty((M, N), device="cuda")
    r = kernels.gemm(ta, tb, epilogue=EPI_BIAS_RELU, bias=tbias, out_lo=out_lo)
    rn = r.cpu().numpy()
    check_close(rn, np.maximum(base + bias, 0), bound)
    hi = (r.view(torch.int32) & -8192).view(torch.float32)
    assert torch.equal(hi + out_lo, r)
    mask = cuda(data.normal((M, N), 14))
    mz = kernels.gemm(ta, tb, epilogue=EPI_RELU_MASK, mask=mask).cpu().numpy()
    check_close(mz, np.where(mask.cpu().numpy() > 0, base, 0), bound)
    for _ in range(3):
        assert np.array_equal(kernels.gemm(ta, tb).cpu().numpy(), plain)
    kernels.check_device_error()
