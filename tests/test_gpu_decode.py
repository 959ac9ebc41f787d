"""GPU parity of the decode (M <= 16) kernel, the repacks and the TQ1_0 path, all called
through the C ABI (libhq.so) and checked against the CPU oracle.

Tolerance (from the task statement): max|y - y_ref| / max|y_ref| <= 1e-2 for fp16
and <= 2e-2 for bf16 against the fp32 oracle; integer/byte work (repacks) is
compared bit for bit.
"""
import numpy as np
import pytest
import torch

from nebula_b200 import _lib, hq
from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL = {"f16": 1e-2, "bf16": 2e-2, "f32": 1e-4}
TDT = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def cuda(x, dtype="f32"):
    """Upload: float arrays converted to `dtype` (exact: values are representable); dtype None
    uploads the raw bytes as uint8."""
    x = np.ascontiguousarray(x)
    if dtype is None:
        return torch.from_numpy(x.view(np.uint8).reshape(-1)).to("cuda:0")
    return torch.from_numpy(x.astype(np.float32)).to("cuda:0").to(TDT[dtype])


def run_gemm(A, W_dev, S, N, group, dtype, wfmt=_lib.HQ_WFMT_TILE_U4, out_dtype=None, bias=None, s_dtype=None):
    At = cuda(A, dtype)
    St = cuda(S, s_dtype or dtype)
    Bt = cuda(bias, "f32") if bias is not None else None
    Y = hq.gemm(At, W_dev, St, N=N, group=group, wfmt=wfmt, bias=Bt, out_dtype=out_dtype)
    torch.cuda.synchronize()
    return Y.float().cpu().numpy()


SHAPES = [(256, 48, 128), (512, 144, 64), (384, 256, 128), (1024, 1040, 128), (5120, 5120, 128), (1024, 272, 256)]


@pytest.mark.parametrize("K,N,g", SHAPES)
@pytest.mark.parametrize("M", [1, 2, 3, 8, 9, 16])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_decode_int4_parity(K, N, g, M, dtype):
    A, q, S = o.gen_int4_case(M, K, N, group=g, seed=M * 131 + K + N, a_dtype=dtype)
    lin = o.pack_linear_u4(q)
    ref = o.w4_gemm(A, lin, S, group=g)
    W = cuda(o.pack_tile(q, 4), None)
    y16 = run_gemm(A, W, S, N, g, dtype)
    assert o.max_rel_err(y16, ref) <= TOL[dtype]
    y32 = run_gemm(A, W, S, N, g, dtype, out_dtype=torch.float32)
    # fp32 output: accumulation order plus the raw-code offset correction (the MMA
    # accumulates (magic + code) * x and subtracts magic * sum(x)), ~1e-5 relative.
    assert o.max_rel_err(y32, ref) <= 1e-4


@pytest.mark.parametrize("M", [1, 5, 16])
def test_reference_layouts_give_identical_results(M):
    K, N, g = 1024, 272, 128
    A, q, S = o.gen_int4_case(M, K, N, group=g, seed=99)
    lin = o.pack_linear_u4(q)
    quad = o.repack_marlin_quad(lin, K, N)
    y_tile = run_gemm(A, cuda(o.pack_tile(q, 4), None), S, N, g, "f16")
    y_lin = run_gemm(A, cuda(lin, None), S, N, g, "f16", wfmt=_lib.HQ_WFMT_LINEAR_U4)
    y_quad = run_gemm(A, cuda(quad, None), S, N, g, "f16", wfmt=_lib.HQ_WFMT_MARLIN_QUAD)
    assert np.array_equal(y_tile, y_lin) and np.array_equal(y_tile, y_quad)


@pytest.mark.parametrize("K,N", [(17408, 5120), (5120, 34816), (256, 48)])
def test_decode_is_deterministic(K, N):
    """Strip groups split between CTAs are summed in CTA order by whichever CTA arrives last:
    repeated calls (sharing one workspace, whose counters every call leaves at zero) are bitwise equal."""
    g, M = 128, 16
    A, q, S = o.gen_int4_case(M, K, N, group=g, seed=5)
    W = cuda(o.pack_tile(q, 4), None)
    At, St = cuda(A, "f16"), cuda(S, "f16")
    ws = hq.make_workspace(M, N, K, g, _lib.HQ_WFMT_TILE_U4, At.device)
    ys = [hq.gemm(At, W, St, N=N, group=g, workspace=ws).clone() for _ in range(3)]
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])
    ref = o.w4_gemm(A, o.pack_linear_u4(q), S, group=g)
    assert o.max_rel_err(ys[0].float().cpu().numpy(), ref) <= TOL["f16"]
    hq.check_device_error()


def test_launch_overlap_chain_matches_serial():
    """A chain of dependent GEMMs (each output is the next input) gives the same result with the
    launch overlap on and off: activations are read only after the previous kernel finished."""
    K = N = 1024
    rng = np.random.default_rng(3)
    layers = []
    for i in range(6):
        _, q, S = o.gen_int4_case(1, K, N, group=128, seed=50 + i)
        layers.append((cuda(o.pack_tile(q, 4), None), cuda(S * 0.25, "f16")))
    x0 = cuda(o.round_to(rng.standard_normal((4, K)).astype(np.float32), "f16"), "f16")

    def chain():
        x = x0
        for W, S in layers:
            x = hq.gemm(x, W, S, N=N, group=128)
        return x
    outs = []
    for flag in (1, 0, 1):
        _lib.lib().hq_set_launch_overlap(flag)
        outs.append(chain().clone())
    torch.cuda.synchronize()
    _lib.lib().hq_set_launch_overlap(1)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


@pytest.mark.parametrize("name,K,N", [("qkv", 5120, 7168), ("o", 5120, 5120), ("gate_up", 5120, 34816),
                                      ("down", 17408, 5120)])
@pytest.mark.parametrize("M", [1, 2, 4, 8, 16])
def test_decode_27b_shapes(name, K, N, M):
    """BASELINE config 1 at full size: every shape at every M of the decode sweep (the oracle runs
    these in well under a second each)."""
    A, q, S = o.gen_int4_case(M, K, N, group=128, seed={"qkv": 1, "o": 2, "gate_up": 3, "down": 4}[name] * 100 + M, a_dtype="f16")
    ref = o.w4_gemm(A, o.pack_linear_u4(q), S, group=128)
    W = hq.repack(cuda(o.pack_linear_u4(q), None), _lib.HQ_WFMT_LINEAR_U4, _lib.HQ_WFMT_TILE_U4, K, N)
    y = run_gemm(A, W, S, N, 128, "f16")
    assert o.max_rel_err(y, ref) <= TOL["f16"]


def test_config0_against_golden():
    """BASELINE config 0 (A fp16 [16,4096], int4 [4096,4096] g128, seed 0) vs the committed oracle output."""
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    A, q, S = o.gen_int4_case(16, 4096, 4096, group=128, seed=0, a_dtype="f16")
    y = run_gemm(A, cuda(o.pack_tile(q, 4), None), S, 4096, 128, "f16")
    assert o.max_rel_err(y, g["cfg0_Y"]) <= TOL["f16"]


@pytest.mark.parametrize("K,N", [(256, 32), (512, 144), (5120, 7168)])
@pytest.mark.parametrize("M", [1, 7, 16])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_decode_ternary_parity(K, N, M, dtype):
    A, t, S = o.gen_ternary_case(M, K, N, group=128, seed=K + M, a_dtype=dtype)
    ref = o.t2_gemm(A, o.pack_linear_t2(t), S, group=128)
    W = cuda(o.pack_tile(t, 2), None)
    y = run_gemm(A, W, S.astype(np.float32), N, 128, dtype, wfmt=_lib.HQ_WFMT_TILE_T2, s_dtype=dtype)
    assert o.max_rel_err(y, ref) <= TOL[dtype]


@pytest.mark.parametrize("K,N,g", [(512, 16384, 128), (1024, 16400, 64), (2048, 16640, 256), (5120, 34816, 128)])
@pytest.mark.parametrize("M", [1, 2, 3, 4])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_decode_ternary_integer_path(K, N, g, M, dtype):
    """Ternary weights on the integer-MMA stream kernel (layers of >= 128 strip groups, M <= 4):
    codes q + 1 as u8 MMA operands, the "- 1" restored from per-k-block sums of the fixed-point
    activations.  Ragged width (16400 = 1025 strips), groups 64 / 128 / 256, 16-bit and fp32 outputs."""
    A, t, S = o.gen_ternary_case(M, K, N, group=g, seed=K + N + M, a_dtype=dtype)
    ref = o.t2_gemm(A, o.pack_linear_t2(t), S, group=g)
    W = cuda(o.pack_tile(t, 2), None)
    y = run_gemm(A, W, S.astype(np.float32), N, g, dtype, wfmt=_lib.HQ_WFMT_TILE_T2, s_dtype=dtype)
    assert o.max_rel_err(y, ref) <= TOL[dtype]
    if dtype == "f16":  # scales exact in fp16 (the generator rounds them so): fp32 output to 1e-4
        y32 = run_gemm(A, W, S.astype(np.float32), N, g, dtype, wfmt=_lib.HQ_WFMT_TILE_T2, s_dtype=dtype,
                       out_dtype=torch.float32)
        assert o.max_rel_err(y32, ref) <= 1e-4


@pytest.mark.parametrize("M", [1, 4, 8])
def test_f32_activations_with_bias_match_reference_semantics(M):
    """The reference's own form: fp32 X, fp32 scale and bias, w = u*s + b (marlin_gemm.cu:208-209),
    with its synthetic distributions (:470-487) and its acceptance bound max_abs_error < 1e-3."""
    rng = np.random.default_rng(42)
    K, N, g = 4096, 4096, 128
    X = (rng.standard_normal((M, K)) * 0.25).astype(np.float32)
    S = (0.05 + rng.integers(0, 1000, size=(K // g, N)) * 1e-4).astype(np.float32)
    B = (-8.0 * S).astype(np.float32)
    q = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    lin = o.pack_linear_u4(q)
    ref = o.w4_gemm(X, lin, S, B, group=g)
    quad = o.repack_marlin_quad(lin, K, N)
    y = run_gemm(X, cuda(quad, None), S, N, g, "f32", wfmt=_lib.HQ_WFMT_MARLIN_QUAD, bias=B)
    assert np.max(np.abs(y - ref)) < 1e-3
    y2 = run_gemm(X, cuda(quad, None), S, N, g, "f32", wfmt=_lib.HQ_WFMT_MARLIN_QUAD)  # symmetric form
    ref2 = o.w4_gemm(X, lin, S, None, group=g)
    assert np.max(np.abs(y2 - ref2)) < 1e-3


@pytest.mark.parametrize("K,N,g", [(256, 48, 128), (4096, 4096, 128), (262144, 144, 64), (180224, 272, 256),
                                   (17408, 5120, 128), (5120, 34816, 128)])
@pytest.mark.parametrize("M", [1, 2, 3, 4])
@pytest.mark.parametrize("with_bias", [False, True])
def test_f32_activations_integer_path(K, N, g, M, with_bias):
    """fp32 X at M <= 4.  Layers of >= 8192 (strip group, k-block) units run the integer-MMA
    stream kernel with each activation held as two fixed-point parts (30 bits) and, with a bias,
    the (8 s + b) * sum(x) term per scale group: ragged widths (N % 128 != 0) with group 64 / 256,
    and the 27B down / gate_up shapes, whose scale groups straddle CTAs.  The two smaller
    shapes run the cluster split-K kernel (two fp16 terms)."""
    rng = np.random.default_rng(K + N + M + (7 if with_bias else 0))
    X = (rng.standard_normal((M, K)) * 0.25).astype(np.float32)
    X[0, :5] *= 40.0  # one large-magnitude group: the rest of the group keeps its bits in the second part
    S = (0.05 + rng.integers(0, 1000, size=(K // g, N)) * 1e-4).astype(np.float32)
    B = (-8.0 * S + 0.01 * rng.standard_normal(S.shape)).astype(np.float32) if with_bias else None
    q = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    lin = o.pack_linear_u4(q)
    ref = o.w4_gemm(X, lin, S, B, group=g)
    y = run_gemm(X, cuda(o.pack_tile(q, 4), None), S, N, g, "f32", bias=B)
    assert o.max_rel_err(y, ref) <= TOL["f32"]
    y2 = run_gemm(X, cuda(o.pack_tile(q, 4), None), S, N, g, "f32", bias=B)
    assert np.array_equal(y, y2)  # deterministic


@pytest.mark.parametrize("M", [1, 4])
@pytest.mark.parametrize("dtype", ["f16"])
def test_16bit_activations_with_fp32_scales_and_bias_wide_layer(M, dtype):
    """fp16 X with the reference's fp32 scale and bias on a layer wide enough (>= 128 strip groups)
    for the integer-MMA kernel; fp32 and fp16 outputs.  (A bias goes with f16 or f32 activations,
    as hq.h states.)"""
    K, N, g = 512, 16384, 128
    rng = np.random.default_rng(M)
    A, q, _ = o.gen_int4_case(M, K, N, group=g, seed=M + 5, a_dtype=dtype)
    S = (0.05 + rng.integers(0, 1000, size=(K // g, N)) * 1e-4).astype(np.float32)
    B = (-8.0 * S + 0.01 * rng.standard_normal(S.shape)).astype(np.float32)
    lin = o.pack_linear_u4(q)
    ref = o.w4_gemm(A, lin, S, B, group=g)
    W = cuda(o.pack_tile(q, 4), None)
    y32 = run_gemm(A, W, S, N, g, dtype, bias=B, s_dtype="f32", out_dtype=torch.float32)
    assert o.max_rel_err(y32, ref) <= 1e-4
    y16 = run_gemm(A, W, S, N, g, dtype, bias=B, s_dtype="f32")
    assert o.max_rel_err(y16, ref) <= TOL[dtype]


def test_f32_activations_nan_group_poisons_only_its_token():
    """A scale group of fp32 activations holding NaN makes that token's outputs NaN, others finite."""
    M, K, N, g = 3, 1024, 272, 128
    rng = np.random.default_rng(3)
    X = rng.standard_normal((M, K)).astype(np.float32)
    X[1, 300] = np.nan
    S = (0.05 + rng.integers(0, 1000, size=(K // g, N)) * 1e-4).astype(np.float32)
    q = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    y = run_gemm(X, cuda(o.pack_tile(q, 4), None), S, N, g, "f32")
    assert np.all(np.isnan(y[1])) and np.all(np.isfinite(y[[0, 2]]))
    ref = o.w4_gemm(X[[0, 2]], o.pack_linear_u4(q), S, None, group=g)
    assert o.max_rel_err(y[[0, 2]], ref) <= TOL["f32"]


@pytest.mark.parametrize("K,N", [(64, 16), (512, 144), (5120, 7168)])
def test_device_repacks_bit_exact(K, N):
    rng = np.random.default_rng(K + N)
    q = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    lin = o.pack_linear_u4(q)
    quad = o.repack_marlin_quad(lin, K, N)
    tile = o.pack_tile(q, 4)
    got = lambda src, sf, df: hq.repack(cuda(src, None), sf, df, K, N).cpu().numpy()  # noqa: E731
    assert np.array_equal(got(lin, _lib.HQ_WFMT_LINEAR_U4, _lib.HQ_WFMT_TILE_U4), tile)
    assert np.array_equal(got(quad, _lib.HQ_WFMT_MARLIN_QUAD, _lib.HQ_WFMT_TILE_U4), tile)
    assert np.array_equal(got(tile, _lib.HQ_WFMT_TILE_U4, _lib.HQ_WFMT_LINEAR_U4).view(np.uint32), lin.ravel())
    assert np.array_equal(got(lin, _lib.HQ_WFMT_LINEAR_U4, _lib.HQ_WFMT_MARLIN_QUAD).view(np.uint32), quad.ravel())
    assert np.array_equal(got(quad, _lib.HQ_WFMT_MARLIN_QUAD, _lib.HQ_WFMT_LINEAR_U4).view(np.uint32), lin.ravel())
    t = rng.integers(-1, 2, size=(K, N), dtype=np.int8)
    lin2, tile2 = o.pack_linear_t2(t), o.pack_tile(t, 2)
    assert np.array_equal(got(lin2, _lib.HQ_WFMT_LINEAR_T2, _lib.HQ_WFMT_TILE_T2), tile2)
    assert np.array_equal(got(tile2, _lib.HQ_WFMT_TILE_T2, _lib.HQ_WFMT_LINEAR_T2).view(np.uint32), lin2.ravel())


def test_tq1_0_gemv_golden_and_conversion():
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    K, N, _ = (int(v) for v in g["tq1_meta"])
    x, blob = cuda(g["tq1_x"], "f32"), cuda(g["tq1_blob"], None)
    y = hq.tq1_0_gemv(x, blob, N)
    torch.cuda.synchronize()
    assert o.max_rel_err(y.cpu().numpy(), g["tq1_y"]) <= 1e-5


@pytest.mark.parametrize("K,N", [(512, 48), (768, 144)])
def test_tq1_0_to_tile_t2_then_gemm(K, N):
    """Offline conversion of TQ1_0 into the 2-bit tile order (N % 16 == 0), then the decode kernel."""
    rng = np.random.default_rng(N)
    t = rng.integers(-1, 2, size=(N, K), dtype=np.int8)
    d = rng.uniform(0.01, 0.05, size=(N, K // 256)).astype(np.float16).view(np.uint16)
    d[1, 0] = 0x7C00  # non-finite block scale: contributes nothing, as in the reference
    blob = o.pack_tq1_0(t, d)
    tile, scales = hq.tq1_0_to_tile_t2(cuda(blob, None), K, N)
    torch.cuda.synchronize()
    assert np.array_equal(tile.cpu().numpy(), o.pack_tile(np.ascontiguousarray(t.T), 2))
    x16 = o.round_to(rng.standard_normal(K).astype(np.float32), "f16")
    y2 = hq.gemm(cuda(x16[None, :], "f16"), tile, scales, N=N, group=128, wfmt=_lib.HQ_WFMT_TILE_T2,
                 out_dtype=torch.float32)
    ref2 = o.gemv_tq1_0(x16, blob, K, N)
    assert o.max_rel_err(y2.cpu().numpy()[0], ref2) <= TOL["f16"]


@pytest.mark.parametrize("K,N", [(512, 48), (5120, 7168), (17408, 5120)])
@pytest.mark.parametrize("M", [1, 3, 16])
def test_tq1_0_layers_at_load_with_fp32_x(K, N, M):
    """TQ1_0 layers converted once at load (hq_tq1_0_to_tile_t2), then hq_gemm with the reference's
    fp32 x (two fp16 terms on the split-K kernel) and fp32 output: against the oracle's
    restatement of kernel_gemv_tq1_0, row by row, within 1e-5 of max|out|."""
    rng = np.random.default_rng(K + N + M)
    t = rng.integers(-1, 2, size=(N, K), dtype=np.int8)
    d = rng.uniform(0.01, 0.05, size=(N, K // 256)).astype(np.float16).view(np.uint16)
    d[1, 0] = 0x7E00  # NaN block scale: skipped, as in the reference
    blob = o.pack_tq1_0(t, d)
    tile, scales = hq.tq1_0_to_tile_t2(cuda(blob, None), K, N)
    X = (rng.standard_normal((M, K)) * 0.5).astype(np.float32)
    Y = hq.gemm(cuda(X, "f32"), tile, scales, N=N, group=128, wfmt=_lib.HQ_WFMT_TILE_T2,
                out_dtype=torch.float32).cpu().numpy()
    for m in range(M):
        assert o.max_rel_err(Y[m], o.gemv_tq1_0(X[m], blob, K, N)) <= 1e-5


@pytest.mark.parametrize("K,N", [(1024, 1), (1024, 45), (2048, 100), (768, 37), (4096, 4097)])
def test_tq1_0_gemv_edge_shapes(K, N):
    """Tensor-core path (K % 1024 == 0) with ragged row counts, and the row-per-warp path (K = 768);
    non-finite block scales and malformed bytes (>= 243) follow the reference's digit arithmetic."""
    rng = np.random.default_rng(K + N)
    t = rng.integers(-1, 2, size=(N, K), dtype=np.int8)
    d = rng.uniform(0.01, 0.05, size=(N, K // 256)).astype(np.float16).view(np.uint16)
    d[0, 0] = 0x7E00  # NaN
    d[N - 1, K // 256 - 1] = 0xFC00  # -Inf
    blob = o.pack_tq1_0(t, d).reshape(N, -1)
    blob[:, 2:54:9] = 250  # bytes outside 0..242
    blob = blob.ravel()
    x = rng.standard_normal(K).astype(np.float32)
    ref = o.gemv_tq1_0(x, blob, K, N)
    y = hq.tq1_0_gemv(cuda(x, "f32"), cuda(blob, None), N)
    torch.cuda.synchronize()
    assert o.max_rel_err(y.cpu().numpy(), ref) <= 1e-5


def test_tq1_0_gemv_x_offset_by_one_float():
    """x only 4-byte aligned (a view one float into a buffer) takes the scalar staging loop."""
    K, N = 1024, 64
    rng = np.random.default_rng(11)
    t = rng.integers(-1, 2, size=(N, K), dtype=np.int8)
    d = rng.uniform(0.01, 0.05, size=(N, K // 256)).astype(np.float16).view(np.uint16)
    blob = o.pack_tq1_0(t, d)
    x = rng.standard_normal(K + 1).astype(np.float32)
    y = hq.tq1_0_gemv(cuda(x, "f32")[1:], cuda(blob, None), N)
    assert o.max_rel_err(y.cpu().numpy(), o.gemv_tq1_0(x[1:], blob, K, N)) <= 1e-5


@pytest.mark.parametrize("kind", ["zero", "tiny", "huge", "nonfinite"])
def test_tq1_0_gemv_x_ranges(kind):
    """x = 0, x near the fp32 minimum, x near the fp32 maximum, and x holding Inf/NaN (the float path)."""
    K, N = 2048, 96
    rng = np.random.default_rng(7)
    t = rng.integers(-1, 2, size=(N, K), dtype=np.int8)
    d = rng.uniform(0.01, 0.05, size=(N, K // 256)).astype(np.float16).view(np.uint16)
    blob = o.pack_tq1_0(t, d)
    x = rng.standard_normal(K).astype(np.float32)
    if kind == "zero":
        x[:] = 0
    elif kind == "tiny":
        x *= np.float32(1e-37)
    elif kind == "huge":
        x *= np.float32(1e30)
    else:
        x[5] = np.inf
        x[700] = np.nan
    ref = o.gemv_tq1_0(x, blob, K, N)
    y = hq.tq1_0_gemv(cuda(x, "f32"), cuda(blob, None), N).cpu().numpy()
    if kind == "nonfinite":
        assert np.array_equal(np.isnan(y), np.isnan(ref)) and np.array_equal(np.isinf(y), np.isinf(ref))
        fin = np.isfinite(ref)
        assert np.allclose(y[fin], ref[fin], rtol=1e-5, atol=1e-5)
    elif kind == "zero":
        assert np.array_equal(y, np.zeros_like(y))
    else:
        assert o.max_rel_err(y, ref) <= 1e-5


@pytest.mark.parametrize("K,N", [(5120, 7168), (17408, 5120), (5120, 248320)])
def test_tq1_0_gemv_full_size(K, N):
    """The layer shapes and the output projection (vocab 248320 x hidden 5120)."""
    rng = np.random.default_rng(K)
    if N * K <= 100_000_000:
        t = rng.integers(-1, 2, size=(N, K), dtype=np.int8)
        d = rng.uniform(0.01, 0.05, size=(N, K // 256)).astype(np.float16).view(np.uint16)
        blob = o.pack_tq1_0(t, d)
    else:  # well-formed blocks drawn directly as bytes: packed values 0..242, d ~ U(0.01, 0.05), pad 0
        blk = rng.integers(0, 243, size=(N, K // 256, 56), dtype=np.uint8)
        d = rng.uniform(0.01, 0.05, size=(N, K // 256)).astype(np.float16).view(np.uint8).reshape(N, K // 256, 2)
        blk[:, :, 0:2] = d
        blk[:, :, 54:56] = 0
        blob = blk.ravel()
    x = rng.standard_normal(K).astype(np.float32)
    ref = o.gemv_tq1_0(x, blob, K, N)
    y = hq.tq1_0_gemv(cuda(x, "f32"), cuda(blob, None), N)
    torch.cuda.synchronize()
    assert o.max_rel_err(y.cpu().numpy(), ref) <= 1e-5
