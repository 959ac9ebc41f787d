"""GGUF Q4_K at model load, on the CPU: the oracle's restatement of the format against the
committed gguf-py fixtures, and the library's host conversion against the oracle.

The device conversion and the group-32 GEMM it feeds are in tests/test_gpu_q4k.py.
"""
import os

import numpy as np
import pytest

from nebula_b200 import hq
from oracle import oracle as o

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "q4_k.npz")


def _cases():
    g = np.load(GOLDEN)
    return [(name, int(g[f"{name}_K"]), int(g[f"{name}_N"]), g[f"{name}_blocks"], g[f"{name}_w_nk"])
            for name in ("rand", "edge")]


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c[0])
def test_oracle_dequant_matches_gguf_fixture(case):
    """unpack_q4_k / dequant_q4_k == gguf-py's dequantize bit for bit (NaN where it has NaN)."""
    _, K, N, blob, w_nk = case
    with np.errstate(invalid="ignore"):
        w = o.dequant_q4_k(blob, K, N)
    assert w.shape == (K, N)
    assert np.array_equal(w.T, w_nk, equal_nan=True)


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c[0])
@pytest.mark.parametrize("nthreads", [1, 0])
def test_host_conversion_matches_oracle(case, nthreads):
    """hq_q4_k_to_tile_host: tile codes, scales and biases identical to the oracle's."""
    _, K, N, blob, _ = case
    tile, scale, bias = hq.q4_k_to_tile_host(blob, K, N, nthreads)
    with np.errstate(invalid="ignore"):
        t_ref, s_ref, b_ref = o.q4_k_to_tile(blob, K, N)
    assert np.array_equal(tile, t_ref)
    assert np.array_equal(scale.view(np.uint32), s_ref.view(np.uint32))
    assert np.array_equal(bias.view(np.uint32), b_ref.view(np.uint32))


def test_host_conversion_ragged_strip_group():
    """N = 272: the last strip group holds one strip (ragged), K spans several super-blocks."""
    K, N = 768, 272
    blob = o.gen_q4_k_blocks(K, N, seed=11)
    tile, scale, bias = hq.q4_k_to_tile_host(blob, K, N)
    t_ref, s_ref, b_ref = o.q4_k_to_tile(blob, K, N)
    assert np.array_equal(tile, t_ref)
    assert np.array_equal(scale, s_ref) and np.array_equal(bias, b_ref)
    # the tile codes decode back to u - 8 of the block codes
    u, _, _ = o.unpack_q4_k(blob, K, N)
    assert np.array_equal(o.unpack_tile_k32(tile, K, N), u.astype(np.int8) - 8)


@pytest.mark.parametrize("src", ["linear", "quad"])
def test_host_repack_to_k32_layout(src):
    """hq_repack_host LINEAR_U4 / MARLIN_QUAD -> TILE_U4_K32 equals the oracle's K32 packer, and
    TILE_U4_K32 -> LINEAR_U4 inverts it bit for bit."""
    K, N = 512, 272
    q = np.random.default_rng(3).integers(-8, 8, size=(K, N), dtype=np.int8)
    lin = o.pack_linear_u4(q)
    s = lin if src == "linear" else o.repack_marlin_quad(lin, K, N)
    fmt = hq.HQ_WFMT_LINEAR_U4 if src == "linear" else hq.HQ_WFMT_MARLIN_QUAD
    t = hq.repack_host(s, fmt, hq.HQ_WFMT_TILE_U4_K32, K, N)
    assert np.array_equal(t.view(np.uint8).reshape(-1), o.pack_tile_k32(q))
    back = hq.repack_host(t, hq.HQ_WFMT_TILE_U4_K32, hq.HQ_WFMT_LINEAR_U4, K, N)
    assert np.array_equal(back.reshape(lin.shape), lin)
    assert not np.array_equal(o.pack_tile_k32(q), o.pack_tile(q, 4))  # the two orders differ


def test_scale_and_bias_exact_in_f32():
    """d * sc and dmin * m need at most 11 + 6 significant bits: the f32 rows hold them exactly."""
    g = np.load(GOLDEN)
    K, N, blob = int(g["rand_K"]), int(g["rand_N"]), g["rand_blocks"]
    _, scale, bias = o.unpack_q4_k(blob, K, N)
    blk = blob.reshape(N, K // 256, 144)
    d = blk[:, :, 0:2].copy().view(np.float16)[..., 0].astype(np.float64)
    s64 = scale.astype(np.float64).T.reshape(N, K // 256, 8) / d[:, :, None]
    assert np.array_equal(s64, np.round(s64)) and s64.max() <= 63 and s64.min() >= 0


def test_oracle_gemm_matches_dequantised_product():
    """q4_k_gemm (the fused int4 oracle, group 32, biased form) against a float64 product of
    the fixture's dequantised weights."""
    g = np.load(GOLDEN)
    K, N, blob, w_nk = int(g["rand_K"]), int(g["rand_N"]), g["rand_blocks"], g["rand_w_nk"]
    X = np.random.default_rng(5).standard_normal((3, K)).astype(np.float32)
    Y = o.q4_k_gemm(X, blob, K, N)
    Y64 = X.astype(np.float64) @ w_nk.T.astype(np.float64)
    assert np.max(np.abs(Y - Y64)) <= 1e-5 * np.max(np.abs(Y64))


@pytest.mark.parametrize("K,N", [(255, 16), (256, 8), (0, 16), (512, 24)])
def test_host_conversion_rejects_bad_shapes(K, N):
    blob = np.zeros(max(1, N * max(K, 256) // 256 * 144), np.uint8)
    with pytest.raises(hq.HQError):
        hq.q4_k_to_tile_host(blob, K, N)
