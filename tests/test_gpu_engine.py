"""GPU tests of the MarlinGemmEngine drop-in and of the oracle pin against the reference's
own kernels.

* The shim (include/hq_marlin_gemm.hpp, via the hq_marlin_* C wrappers) is driven with the
  reference's argument conventions: fp32 X, Marlin-quad weights, fp32 scales and biases.
* oracle/_ref/libref_marlin.so is the reference's unmodified marlin_gemm.cu compiled for
  sm_100a.  Its kernel_reference_gemm (marlin_gemm.cu:52-70) must equal the oracle's
  hqo_gemm_f32 bit for bit, and its Marlin kernel (:130-237) must meet its own 1e-3 bound
  against the oracle: this pins the oracle to the reference on the GPU.
"""
import ctypes

import numpy as np
import pytest
import torch

from nebula_b200 import hq
from oracle import oracle as o

pytestmark = pytest.mark.gpu


def ref_case(M, K, N, g, seed):
    rng = np.random.default_rng(seed)
    X = (rng.standard_normal((M, K)) * 0.25).astype(np.float32)
    S = (0.05 + rng.integers(0, 1000, size=(K // g, N)) * 1e-4).astype(np.float32)
    B = (-8.0 * S).astype(np.float32)
    q = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    lin = o.pack_linear_u4(q)
    return X, S, B, lin


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.float32:
        return torch.from_numpy(a).cuda()
    return torch.from_numpy(a.view(np.uint8).reshape(-1)).cuda()


def P(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("M", [1, 2, 4, 8, 13])
def test_engine_shim_matches_reference_semantics(M):
    K, N, g = 2048, 1024, 128
    X, S, B, lin = ref_case(M, K, N, g, seed=M)
    quad = o.repack_marlin_quad(lin, K, N)
    W = o.dequant_u4(lin, S, B, K, N, g)
    eng = hq.MarlinGemmEngine(max(M, 8), K, N, g)
    dX, dQ, dL, dS, dB, dW = dev(X), dev(quad), dev(lin), dev(S), dev(B), dev(W)
    Yr = torch.empty((M, N), device="cuda"); Ym = torch.empty_like(Yr); Yb = torch.empty_like(Yr)
    eng.forward_reference(dX, dW, Yr, M)
    eng.forward_marlin_int4(dX, dQ, dS, dB, Ym, M)
    eng.forward_baseline_int4(dX, dL, dS, dB, Yb, M)
    torch.cuda.synchronize()
    # forward_reference is bit-identical to kernel_reference_gemm's arithmetic (the oracle)
    assert np.array_equal(Yr.cpu().numpy(), o.gemm_f32(X, W))
    mx, mse = eng.verify_fidelity(Yr, Ym, M)
    assert mx < 1e-3  # the reference's numerical_match bound (marlin_gemm.cu:747)
    # the un-optimised baseline rounds the dequant as the reference's host code does and sums in
    # k order with fma: bit-identical to kernel_reference_gemm on the dequantised weights
    assert np.array_equal(Yb.cpu().numpy(), o.gemm_f32(X, W))
    eng.close()


def test_engine_repack_matches_oracle():
    K, N = 4096, 512
    rng = np.random.default_rng(0)
    lin = rng.integers(0, 2**32, size=(K // 8, N), dtype=np.uint64).astype(np.uint32)
    eng = hq.MarlinGemmEngine(8, K, N, 128)
    quad, ms = eng.repack_q4k_to_marlin(lin, K, N)
    assert np.array_equal(quad, o.repack_marlin_quad(lin, K, N))
    assert ms < 1000.0
    eng.close()


def _ref():
    r = o.ref_lib()
    if r is None:
        pytest.skip("oracle/_ref/libref_marlin.so not present")
    r.ref_forward_reference.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_uint32]
    r.ref_forward_marlin.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_uint32]
    return r


@pytest.mark.parametrize("M", [1, 2, 4, 8])
@pytest.mark.parametrize("g", [128, 32])
def test_oracle_pinned_to_reference_kernels(M, g):
    r = _ref()
    K, N = 512, 256  # the reference's split-K needs K % 512 == 0 and group % 32 == 0 (marlin_gemm.cu:156-159)
    X, S, B, lin = ref_case(M, K, N, g, seed=10 + M + g)
    quad = o.repack_marlin_quad(lin, K, N)
    W = o.dequant_u4(lin, S, B, K, N, g)
    h = r.ref_engine_create(8, K, N, g)
    assert h, r.ref_last_error()
    try:
        dX, dW, dQ, dS, dB = dev(X), dev(W), dev(quad), dev(S), dev(B)
        Yr = torch.zeros((M, N), device="cuda"); Ym = torch.zeros_like(Yr)
        assert r.ref_forward_reference(ctypes.c_void_p(h), P(dX), P(dW), P(Yr), M) == 0
        assert r.ref_forward_marlin(ctypes.c_void_p(h), P(dX), P(dQ), P(dS), P(dB), P(Ym), M) == 0
        torch.cuda.synchronize()
        # the oracle restates kernel_reference_gemm exactly
        assert np.array_equal(Yr.cpu().numpy(), o.gemm_f32(X, W))
        # the reference's own Marlin kernel meets its bound against the oracle
        assert np.max(np.abs(Ym.cpu().numpy() - o.w4_gemm(X, lin, S, B, group=g))) < 1e-3
    finally:
        r.ref_engine_destroy(ctypes.c_void_p(h))


@pytest.mark.parametrize("M", [1, 3, 8, 13])
def test_engine_group32_against_reference_kernel(M):
    """Group 32, which the reference's Marlin engine accepts (group % 32 == 0): the drop-in's
    forward_marlin_int4 and the reference's own kernel on identical inputs, both within the
    reference's 1e-3 bound of the oracle."""
    K, N, g = 1024, 256, 32
    X, S, B, lin = ref_case(M, K, N, g, seed=40 + M)
    quad = o.repack_marlin_quad(lin, K, N)
    ref = o.w4_gemm(X, lin, S, B, group=g)
    dX, dQ, dS, dB = dev(X), dev(quad), dev(S), dev(B)
    eng = hq.MarlinGemmEngine(max(M, 8), K, N, g)
    Ym = torch.zeros((M, N), device="cuda")
    eng.forward_marlin_int4(dX, dQ, dS, dB, Ym, M)
    torch.cuda.synchronize()
    ours = Ym.cpu().numpy()
    assert np.max(np.abs(ours - ref)) < 1e-3
    assert o.max_rel_err(ours, ref) <= 1e-5
    eng.close()
    # the reference's kernels hold at most 8 rows (acc[8], marlin_gemm.cu:260): no M > 8 there
    if o.ref_lib() is None or M > 8:
        return
    r = _ref()
    h = r.ref_engine_create(8, K, N, g)
    assert h, r.ref_last_error()
    try:
        Yr = torch.zeros((M, N), device="cuda")
        assert r.ref_forward_marlin(ctypes.c_void_p(h), P(dX), P(dQ), P(dS), P(dB), P(Yr), M) == 0
        torch.cuda.synchronize()
        theirs = Yr.cpu().numpy()
        assert np.max(np.abs(theirs - ref)) < 1e-3
        assert np.max(np.abs(ours - theirs)) < 1e-3
    finally:
        r.ref_engine_destroy(ctypes.c_void_p(h))
