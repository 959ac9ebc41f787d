"""The W8A8 path (MarlinGemmEngine::forward_cutlass_int8, marlin_gemm.cu:327-377, 603-617): hq_w8_gemm
against the oracle's restatement, the oracle against the reference's own kernel (built from source in
oracle/_ref), and the engine shim's method."""
import ctypes

import numpy as np
import pytest
import torch

from nebula_b200 import _lib, hq
from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL = 1e-5  # max |Y - Y_ref| / max |Y_ref|: exact int32 sums rounded once vs an fp32 running sum


def case(M, K, N, seed):
    rng = np.random.default_rng(seed)
    X = (rng.standard_normal((M, K)) * 0.6).astype(np.float32)  # some |x * 127| clamp at +-128 / 127
    W = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
    S = rng.uniform(0.005, 0.02, size=N).astype(np.float32)
    return X, W, S


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")


@pytest.mark.parametrize("M,K,N", [(1, 4096, 4096), (3, 512, 132), (8, 4096, 1024), (13, 1024, 256),
                                   (2, 102, 8), (1, 65536, 64)])
def test_w8_gemm_matches_oracle(M, K, N):
    X, W, S = case(M, K, N, seed=M * 1000 + N)
    Y = hq.w8_gemm(dev(X), dev(W), dev(S)).cpu().numpy()
    assert o.max_rel_err(Y, o.w8_gemm(X, W, S)) <= TOL


def test_w8_gemm_deterministic():
    X, W, S = case(4, 4096, 2048, seed=3)
    dX, dW, dS = dev(X), dev(W), dev(S)
    a = hq.w8_gemm(dX, dW, dS)
    b = hq.w8_gemm(dX, dW, dS)
    assert torch.equal(a, b)


@pytest.mark.parametrize("M", [1, 8])
def test_oracle_pinned_to_reference_int8_kernel(M):
    """The restatement reproduces kernel_cutlass_int8_gemm bit for bit; hq_w8_gemm and the engine shim's
    forward_cutlass_int8 meet the tolerance against it."""
    r = o.ref_lib()
    if r is None or not hasattr(r, "ref_forward_cutlass_int8"):
        pytest.skip("oracle/_ref/libref_marlin.so not present")
    r.ref_forward_cutlass_int8.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_uint32]
    K, N = 1024, 512
    X, W, S = case(M, K, N, seed=40 + M)
    h = r.ref_engine_create(8, K, N, 128)
    assert h, r.ref_last_error()
    try:
        dX, dW, dS = dev(X), dev(W), dev(S)
        Yr = torch.zeros((M, N), device="cuda:0")
        P = lambda t: ctypes.c_void_p(t.data_ptr())
        assert r.ref_forward_cutlass_int8(ctypes.c_void_p(h), P(dX), P(dW), P(dS), P(Yr), M) == 0
        torch.cuda.synchronize()
        ref = Yr.cpu().numpy()
        assert np.array_equal(ref, o.w8_gemm(X, W, S))
    finally:
        r.ref_engine_destroy(ctypes.c_void_p(h))
    L = _lib.lib()
    e = L.hq_marlin_engine_create(8, K, N, 128)
    assert e
    try:
        Ye = torch.zeros((M, N), device="cuda:0")
        assert L.hq_marlin_forward_cutlass_int8(e, P(dX), P(dW), P(dS), P(Ye), M) == _lib.HQ_OK
        torch.cuda.synchronize()
        assert o.max_rel_err(Ye.cpu().numpy(), ref) <= TOL
    finally:
        L.hq_marlin_engine_destroy(e)
