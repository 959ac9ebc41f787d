"""GPU parity of GGUF Q4_K at model load and of the group-32 GEMM that runs it, through the
C ABI (libhq.so), against the CPU oracle (whose Q4_K restatement tests/test_q4k.py pins to
the gguf-py fixtures).

Tolerances: conversions bit for bit; fp32 outputs <= 1e-4 of max|y_ref| (fp32 accumulation
in another order); fp16 / bf16 outputs 1e-2 / 2e-2, as in tests/test_gpu_decode.py.
"""
import os

import numpy as np
import pytest
import torch

from nebula_b200 import hq
from oracle import oracle as o

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "q4_k.npz")
TDT = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}
TOL16 = {"f16": 1e-2, "bf16": 2e-2}


def dev_u8(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1)).to("cuda:0")


def check_conversion(blob, K, N):
    tile, s, b = hq.q4_k_to_tile(dev_u8(blob), K, N)
    torch.cuda.synchronize()
    with np.errstate(invalid="ignore"):
        t_ref, s_ref, b_ref = o.q4_k_to_tile(blob, K, N)
    assert np.array_equal(tile.cpu().numpy(), t_ref)
    for got, want in ((s.cpu().numpy(), s_ref), (b.cpu().numpy(), b_ref)):
        # bit for bit, except that a NaN's payload is the hardware's own (Inf * 0 gives
        # 0x7FFFFFFF on the GPU, 0xFFC00000 on x86): NaN positions must agree
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(got), nan)
        assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


@pytest.mark.parametrize("name", ["rand", "edge"])
def test_device_conversion_matches_oracle_on_fixtures(name):
    g = np.load(GOLDEN)
    check_conversion(g[f"{name}_blocks"], int(g[f"{name}_K"]), int(g[f"{name}_N"]))


@pytest.mark.parametrize("K,N", [(768, 272), (5120, 7168)])
def test_device_conversion_matches_oracle(K, N):
    check_conversion(o.gen_q4_k_blocks(K, N, seed=K + N), K, N)


def q4k_case(M, K, N, seed, a_dtype):
    blob = o.gen_q4_k_blocks(K, N, seed=seed)
    X = o.round_to((np.random.default_rng(seed).standard_normal((M, K)) * 0.5).astype(np.float32), a_dtype)
    return blob, X


@pytest.mark.parametrize("M", [1, 2, 5, 8, 9, 16])
@pytest.mark.parametrize("a_dtype", ["f16", "f32"])
def test_q4_k_gemm_parity(M, a_dtype):
    """Q4_K blocks -> device conversion -> hq_gemm(group 32, f32 scale and bias) on the decode
    kernel against the fused oracle.  N = 272 leaves a one-strip group."""
    K, N = 1024, 272
    blob, X = q4k_case(M, K, N, 100 + M, a_dtype)
    ref = o.q4_k_gemm(X, blob, K, N)
    tile, s, b = hq.q4_k_to_tile(dev_u8(blob), K, N)
    Xt = torch.from_numpy(X).to("cuda:0").to(TDT[a_dtype])
    y32 = hq.gemm(Xt, tile, s, N=N, group=32, bias=b, out_dtype=torch.float32)
    torch.cuda.synchronize()
    y = y32.cpu().numpy()
    assert o.max_rel_err(y, ref) <= 1e-4
    y2 = hq.gemm(Xt, tile, s, N=N, group=32, bias=b, out_dtype=torch.float32).cpu().numpy()
    assert np.array_equal(y, y2)  # deterministic
    if a_dtype == "f16":
        y16 = hq.gemm(Xt, tile, s, N=N, group=32, bias=b).float().cpu().numpy()
        assert o.max_rel_err(y16, ref) <= TOL16["f16"]
    # and against llama.cpp's dequantised weights (float64 product)
    W = o.dequant_q4_k(blob, K, N).astype(np.float64)
    y64 = X.astype(np.float64) @ W
    assert np.max(np.abs(y - y64)) <= 1e-4 * np.max(np.abs(y64))


def rounded_weight_ref(X, u, scale, bias, dtype):
    """float64 product with the weights u * s + b rounded to the tensor-core operand type, as the
    prefill kernel's dequantiser forms them (fp32 fma, one rounding)."""
    g = u.shape[0] // scale.shape[0]
    s = np.repeat(scale.astype(np.float64), g, axis=0)
    b = np.repeat(bias.astype(np.float64), g, axis=0)
    W = o.round_to((u.astype(np.float64) * s + b).astype(np.float32), dtype).astype(np.float64)
    return X.astype(np.float64) @ W


@pytest.mark.parametrize("M", [17, 40, 300])
def test_q4_k_prefill(M):
    """M > 16: the tcgen05 kernel's f32-scale form (two scale and bias rows per 64-k block)."""
    K, N = 1024, 272
    blob, X = q4k_case(M, K, N, 200 + M, "f16")
    tile, s, b = hq.q4_k_to_tile(dev_u8(blob), K, N)
    Xt = torch.from_numpy(X).to("cuda:0").half()
    y = hq.gemm(Xt, tile, s, N=N, group=32, bias=b, out_dtype=torch.float32).cpu().numpy()
    hq.check_device_error()
    u, scale, bias = o.unpack_q4_k(blob, K, N)
    assert o.max_rel_err(y, rounded_weight_ref(X, u, scale, bias, "f16")) <= 1e-5
    assert o.max_rel_err(y, o.q4_k_gemm(X, blob, K, N)) <= TOL16["f16"]
    y16 = hq.gemm(Xt, tile, s, N=N, group=32, bias=b).float().cpu().numpy()
    assert o.max_rel_err(y16, o.q4_k_gemm(X, blob, K, N)) <= TOL16["f16"]
    y2 = hq.gemm(Xt, tile, s, N=N, group=32, bias=b, out_dtype=torch.float32).cpu().numpy()
    assert np.array_equal(y, y2)


@pytest.mark.parametrize("M,K,N,g", [(64, 512, 144, 32), (200, 1024, 272, 128), (130, 768, 256, 64)])
@pytest.mark.parametrize("a_dtype,with_bias", [("f16", True), ("f16", False), ("bf16", False)])
def test_prefill_f32_scales(M, K, N, g, a_dtype, with_bias):
    """f32 scale rows (and the reference's bias form) at M > 16 with 16-bit activations: group 32
    and groups of 64 / 128 on the one-CTA tcgen05 kernel."""
    rng = np.random.default_rng(M + K + g)
    A, q, _ = o.gen_int4_case(M, K, N, group=g, seed=M + N, a_dtype=a_dtype)
    S = (0.005 + rng.random((K // g, N)) * 0.015).astype(np.float32)
    B = (-8.0 * S + 0.01 * rng.standard_normal(S.shape)).astype(np.float32) if with_bias else None
    W = dev_u8(o.pack_tile_k32(q) if g == 32 else o.pack_tile(q, 4))
    At = torch.from_numpy(A).to("cuda:0").to(TDT[a_dtype])
    Bt = torch.from_numpy(B).to("cuda:0") if with_bias else None
    y = hq.gemm(At, W, torch.from_numpy(S).to("cuda:0"), N=N, group=g, bias=Bt, out_dtype=torch.float32)
    y = y.cpu().numpy()
    hq.check_device_error()
    u = (q.astype(np.int16) + 8).astype(np.uint8)
    bias = B if with_bias else (-8.0 * S).astype(np.float32)
    assert o.max_rel_err(y, rounded_weight_ref(A, u, S, bias, a_dtype)) <= 1e-5
    ref = o.w4_gemm(A, o.pack_linear_u4(q), S, B, group=g)
    assert o.max_rel_err(y, ref) <= TOL16[a_dtype]


@pytest.mark.parametrize("M", [1, 16, 2048])
def test_q4_k_27b_qkv_shape(M):
    """The 27B QKV projection (K 5120, N 7168) held as Q4_K."""
    K, N = 5120, 7168
    blob, X = q4k_case(M, K, N, 7 + M, "f16")
    rows = np.arange(M) if M <= 16 else np.arange(0, M, 61)  # sampled rows at M = 2048
    ref = o.q4_k_gemm(X[rows], blob, K, N)
    tile, s, b = hq.q4_k_to_tile(dev_u8(blob), K, N)
    y = hq.gemm(torch.from_numpy(X).to("cuda:0").half(), tile, s, N=N, group=32, bias=b,
                out_dtype=torch.float32).cpu().numpy()
    assert o.max_rel_err(y[rows], ref) <= (1e-4 if M <= 16 else TOL16["f16"])


@pytest.mark.parametrize("M", [1, 8, 16, 33])
@pytest.mark.parametrize("a_dtype", ["f16", "bf16", "f32"])
def test_group32_symmetric(M, a_dtype):
    """Group 32 without a bias (w = (u - 8) * scale, f32 scales): every activation type."""
    K, N = 512, 144
    A, q, S = o.gen_int4_case(M, K, N, group=32, seed=M + 3, a_dtype=a_dtype, s_dtype="f32")
    ref = o.w4_gemm(A, o.pack_linear_u4(q), S, group=32)
    W = dev_u8(o.pack_tile_k32(q))
    At = torch.from_numpy(A).to("cuda:0").to(TDT[a_dtype])
    St = torch.from_numpy(S).to("cuda:0")
    y = hq.gemm(At, W, St, N=N, group=32, out_dtype=torch.float32).cpu().numpy()
    if M > 16 and a_dtype != "f32":  # tcgen05 kernel: weights rounded to the operand type
        u = (q.astype(np.int16) + 8).astype(np.uint8)
        assert o.max_rel_err(y, rounded_weight_ref(A, u, S, (-8.0 * S).astype(np.float32), a_dtype)) <= 1e-5
        assert o.max_rel_err(y, ref) <= TOL16[a_dtype]
    else:
        assert o.max_rel_err(y, ref) <= 1e-4
    if a_dtype != "f32":
        y16 = hq.gemm(At, W, St, N=N, group=32).float().cpu().numpy()
        assert o.max_rel_err(y16, ref) <= TOL16[a_dtype]


def test_group32_reference_layouts():
    """Group 32 through the drop-in's reference layouts (linear / Marlin quad, re-tiled in the
    workspace) with the reference's fp32 X, scale and bias."""
    M, K, N = 3, 1024, 256
    rng = np.random.default_rng(9)
    X = (rng.standard_normal((M, K)) * 0.25).astype(np.float32)
    S = (0.05 + rng.integers(0, 1000, size=(K // 32, N)) * 1e-4).astype(np.float32)
    B = (-8.0 * S).astype(np.float32)
    q = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    lin = o.pack_linear_u4(q)
    ref = o.w4_gemm(X, lin, S, B, group=32)
    quad = o.repack_marlin_quad(lin, K, N)
    Xt, St, Bt = (torch.from_numpy(a).to("cuda:0") for a in (X, S, B))
    for fmt, w in ((hq.HQ_WFMT_LINEAR_U4, lin), (hq.HQ_WFMT_MARLIN_QUAD, quad)):
        y = hq.gemm(Xt, dev_u8(w), St, N=N, group=32, wfmt=fmt, bias=Bt).cpu().numpy()
        assert np.max(np.abs(y - ref)) < 1e-3  # the reference's own acceptance bound


def test_group32_unsupported_combinations_fail_loudly():
    K, N = 512, 144
    A, q, S = o.gen_int4_case(4, K, N, group=32, seed=1, a_dtype="f16")
    W = dev_u8(o.pack_tile_k32(q))
    At = torch.from_numpy(A).to("cuda:0").half()
    with pytest.raises(hq.HQError):  # group 32 takes f32 scales only
        hq.gemm(At, W, torch.from_numpy(S).to("cuda:0").half(), N=N, group=32)
    S32 = torch.from_numpy(S).to("cuda:0")
    with pytest.raises(hq.HQError):  # group 32 takes the TILE_U4_K32 order, not TILE_U4
        hq.gemm(At, W, S32, N=N, group=32, wfmt=hq.HQ_WFMT_TILE_U4)
    with pytest.raises(hq.HQError):  # and TILE_U4_K32 is only for group 32
        hq.gemm(At, W, torch.ones((K // 64, N), device="cuda:0"), N=N, group=64, wfmt=hq.HQ_WFMT_TILE_U4_K32)
    S96 = torch.ones((K // 96 + 1, N), device="cuda:0")
    with pytest.raises(hq.HQError):  # 96 is neither 32 nor a multiple of 64
        hq.gemm(At, W, S96, N=N, group=96)


def test_q4_k_quant_linear_and_smallest_shape():
    """hq.QuantLinear.from_q4_k at the smallest Q4_K layer (one super-block, one strip: K 256,
    N 16), across the decode / prefill boundary, and M = 0."""
    K, N = 256, 16
    blob = o.gen_q4_k_blocks(K, N, seed=5)
    layer = hq.QuantLinear.from_q4_k(dev_u8(blob), K, N)
    for M in (1, 16, 17, 64):
        X = o.round_to((np.random.default_rng(M).standard_normal((M, K)) * 0.5).astype(np.float32), "f16")
        y = layer(torch.from_numpy(X).to("cuda:0").half(), out_dtype=torch.float32).cpu().numpy()
        ref = o.q4_k_gemm(X, blob, K, N)
        assert o.max_rel_err(y, ref) <= (1e-4 if M <= 16 else TOL16["f16"])
    y0 = layer(torch.empty((0, K), device="cuda:0", dtype=torch.float16))
    assert tuple(y0.shape) == (0, N)


@pytest.mark.parametrize("K,N", [(512, 272), (5120, 7168)])
def test_device_repack_k32(K, N):
    """hq_repack_device LINEAR_U4 / MARLIN_QUAD -> TILE_U4_K32 and back, bit for bit."""
    q = np.random.default_rng(K).integers(-8, 8, size=(K, N), dtype=np.int8)
    lin = o.pack_linear_u4(q)
    want = o.pack_tile_k32(q)
    for fmt, src in ((hq.HQ_WFMT_LINEAR_U4, lin), (hq.HQ_WFMT_MARLIN_QUAD, o.repack_marlin_quad(lin, K, N))):
        t = hq.repack(dev_u8(src), fmt, hq.HQ_WFMT_TILE_U4_K32, K, N)
        assert np.array_equal(t.cpu().numpy(), want)
    back = hq.repack(dev_u8(want), hq.HQ_WFMT_TILE_U4_K32, hq.HQ_WFMT_LINEAR_U4, K, N)
    assert np.array_equal(back.cpu().numpy().view(np.uint32).reshape(lin.shape), lin)


@pytest.mark.parametrize("M", [1, 5, 8])
@pytest.mark.parametrize("a_dtype,with_bias", [("f16", True), ("f32", True), ("bf16", False), ("f16", False)])
def test_group32_wide_layer(M, a_dtype, with_bias):
    """Group 32 on a layer of >= 56 strip groups at M <= 8 (N = 8192: the three-stage ring)."""
    K, N = 512, 8192
    rng = np.random.default_rng(M + N)
    A, q, _ = o.gen_int4_case(M, K, N, group=32, seed=M + 17, a_dtype=a_dtype)
    S = (0.005 + rng.random((K // 32, N)) * 0.015).astype(np.float32)
    B = (-8.0 * S + 0.01 * rng.standard_normal(S.shape)).astype(np.float32) if with_bias else None
    ref = o.w4_gemm(A, o.pack_linear_u4(q), S, B, group=32)
    y = hq.gemm(torch.from_numpy(A).to("cuda:0").to(TDT[a_dtype]), dev_u8(o.pack_tile_k32(q)),
                torch.from_numpy(S).to("cuda:0"), N=N, group=32,
                bias=torch.from_numpy(B).to("cuda:0") if with_bias else None, out_dtype=torch.float32)
    assert o.max_rel_err(y.cpu().numpy(), ref) <= 1e-4
