"""GPU parity of the tcgen05 tensor-core kernel (M > 16) through the C ABI, against the CPU oracle.

Tolerance: max|y - y_ref| / max|y_ref| <= 1e-2 (fp16) / 2e-2 (bf16) against the fp32
oracle.  The dequantised weight q * s is rounded to the activation type before the
tensor-core product, the only rounding beyond the output cast.
"""
import numpy as np
import pytest
import torch

from nebula_b200 import _lib, hq
from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL = {"f16": 1e-2, "bf16": 2e-2}
TDT = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def cuda(x, dtype=None):
    x = np.ascontiguousarray(x)
    if dtype is None:
        return torch.from_numpy(x.view(np.uint8).reshape(-1)).to("cuda:0")
    return torch.from_numpy(x.astype(np.float32)).to("cuda:0").to(TDT[dtype])


def run(A, W, S, N, g, dtype, wfmt=_lib.HQ_WFMT_TILE_U4, out_dtype=None):
    y = hq.gemm(cuda(A, dtype), W, cuda(S, dtype), N=N, group=g, wfmt=wfmt, out_dtype=out_dtype)
    torch.cuda.synchronize()
    hq.check_device_error()
    return y.float().cpu().numpy()


@pytest.mark.parametrize("M,K,N,g", [(17, 64, 16, 64), (64, 256, 48, 128), (128, 512, 256, 128),
                                     (130, 384, 272, 128), (300, 1024, 1040, 128), (257, 640, 896, 128),
                                     (200, 512, 272, 64), (200, 1024, 400, 256), (40, 192, 32, 64)])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_prefill_int4_small(M, K, N, g, dtype):
    A, q, S = o.gen_int4_case(M, K, N, group=g, seed=M + K + N, a_dtype=dtype)
    ref = o.w4_gemm(A, o.pack_linear_u4(q), S, group=g)
    W = cuda(o.pack_tile(q, 4))
    y = run(A, W, S, N, g, dtype)
    assert o.max_rel_err(y, ref) <= TOL[dtype]
    y32 = run(A, W, S, N, g, dtype, out_dtype=torch.float32)
    assert o.max_rel_err(y32, ref) <= TOL[dtype]


@pytest.mark.parametrize("M,K,N", [(100, 256, 48), (300, 512, 272)])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_prefill_ternary(M, K, N, dtype):
    A, t, S = o.gen_ternary_case(M, K, N, group=128, seed=M + N, a_dtype=dtype)
    ref = o.t2_gemm(A, o.pack_linear_t2(t), S, group=128)
    y = run(A, cuda(o.pack_tile(t, 2)), S, N, 128, dtype, wfmt=_lib.HQ_WFMT_TILE_T2)
    assert o.max_rel_err(y, ref) <= TOL[dtype]


def test_prefill_is_deterministic():
    M, K, N = 384, 1024, 512
    A, q, S = o.gen_int4_case(M, K, N, seed=3, a_dtype="bf16")
    At, St, W = cuda(A, "bf16"), cuda(S, "bf16"), cuda(o.pack_tile(q, 4))
    ys = [hq.gemm(At, W, St, N=N).clone() for _ in range(3)]
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])


@pytest.mark.parametrize("name,K,N", [("qkv", 5120, 7168), ("o", 5120, 5120), ("gate_up", 5120, 34816),
                                      ("down", 17408, 5120)])
@pytest.mark.parametrize("M", [512, 2048, 8192])
def test_prefill_27b_shapes(name, K, N, M):
    """BASELINE config 2 at every shape and token count (bf16 activations and scales), checked on a
    sample of rows."""
    rng = np.random.default_rng(M + K + N)
    A, q, S = o.gen_int4_case(M, K, N, group=128, seed={"qkv": 1, "o": 2, "gate_up": 3, "down": 4}[name],
                              a_dtype="bf16")
    W = hq.repack(cuda(o.pack_linear_u4(q)), _lib.HQ_WFMT_LINEAR_U4, _lib.HQ_WFMT_TILE_U4, K, N)
    y = run(A, W, S, N, 128, "bf16")
    rows = np.sort(rng.choice(M, size=24, replace=False))
    ref = o.w4_gemm(np.ascontiguousarray(A[rows]), o.pack_linear_u4(q), S, group=128)
    assert o.max_rel_err(y[rows], ref) <= TOL["bf16"]


@pytest.mark.parametrize("name,K,N", [("qkv", 5120, 7168), ("o", 5120, 5120), ("gate_up", 5120, 34816),
                                      ("down", 17408, 5120)])
def test_prefill_ternary_27b_shapes(name, K, N):
    """BASELINE config 3 at M = 2048 on the 27B shapes (2-bit ternary codes, fp16 activations and
    scales ~U(0.01, 0.05)): the tensor-core path, checked on a sample of rows."""
    M = 2048
    rng = np.random.default_rng(K + N + 7)
    A, t, S = o.gen_ternary_case(M, K, N, group=128, seed={"qkv": 11, "o": 12, "gate_up": 13, "down": 14}[name],
                                 a_dtype="f16")
    W = hq.repack(cuda(o.pack_linear_t2(t)), _lib.HQ_WFMT_LINEAR_T2, _lib.HQ_WFMT_TILE_T2, K, N)
    y = run(A, W, S, N, 128, "f16", wfmt=_lib.HQ_WFMT_TILE_T2)
    rows = np.sort(rng.choice(M, size=24, replace=False))
    ref = o.t2_gemm(np.ascontiguousarray(A[rows]), o.pack_linear_t2(t), S, group=128)
    assert o.max_rel_err(y[rows], ref) <= TOL["f16"]
