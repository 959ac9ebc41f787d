"""numpy front end of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loads ``oracle/liboracle.so`` (this project's C restatement of the reference path,
see ``hq_oracle.c``) and, when present, ``oracle/_ref/libref_marlin.so`` (the
reference's own ``marlin_gemm.cu`` compiled from source).  Also holds the seeded
input generators that the parity tests, smoke() and bench.py's CPU baseline share.

Nothing in the product package imports this module.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_lib = None
_ref = None

c_int, c_size_t, c_void_p, c_double = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_double


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            from oracle.build import build_oracle
            build_oracle()
        _lib = ctypes.CDLL(path)
        _lib.hqo_tile_bytes.restype = c_size_t
        _lib.hqo_tile_bytes.argtypes = [c_int, c_int, c_int]
        _lib.hqo_half_to_float.restype = ctypes.c_float
        _lib.hqo_half_to_float.argtypes = [ctypes.c_uint16]
    return _lib


def ref_lib():
    """The reference's own Marlin engine library, or None when it was not built."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libref_marlin.so")
        if not os.path.exists(path):
            return None
        _ref = ctypes.CDLL(path)
        _ref.ref_last_error.restype = ctypes.c_char_p
        _ref.ref_engine_create.restype = c_void_p
        _ref.ref_engine_create.argtypes = [ctypes.c_uint32] * 4
        _ref.ref_engine_destroy.argtypes = [c_void_p]
        for f in ("ref_forward_reference", "ref_forward_marlin", "ref_forward_baseline", "ref_forward_cutlass_int8"):
            getattr(_ref, f).restype = c_int
        _ref.ref_engine_repack_q4k_to_marlin.argtypes = [c_void_p, c_void_p, c_void_p, ctypes.c_uint32,
                                                         ctypes.c_uint32, ctypes.POINTER(c_double)]
    return _ref


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(c_void_p)


def _ck(rc: int, what: str):
    if rc != 0:
        raise ValueError(f"oracle {what} rejected its arguments (rc={rc})")


# ------------------------------------------------------------------ dtypes

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to fp16/bf16 and return them as float32."""
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    if dtype == "f32":
        return x.astype(np.float32)
    raise ValueError(dtype)


def to_bits(x32: np.ndarray, dtype: str) -> np.ndarray:
    """float32 (already representable) -> raw uint16 bits of fp16/bf16."""
    if dtype == "f16":
        return x32.astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        return f32_to_bf16_bits(x32)
    raise ValueError(dtype)


# --------------------------------------------------------------- generators

def gen_int4_case(M, K, N, group=128, seed=0, a_dtype="f16", s_dtype=None,
                  s_lo=0.005, s_hi=0.02):
    """BASELINE-style int4 case: A ~ N(0,1), codes U{-8..7}, scales ~ U(lo,hi).

    Returns float32 arrays holding values already rounded to the storage dtypes.
    """
    s_dtype = s_dtype or a_dtype
    rng = np.random.Generator(np.random.PCG64(seed))
    A = round_to(rng.standard_normal((M, K), dtype=np.float32), a_dtype)
    q = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    S = round_to(rng.uniform(s_lo, s_hi, size=(K // group, N)).astype(np.float32), s_dtype)
    return A, q, S


def gen_ternary_case(M, K, N, group=128, seed=0, a_dtype="f16", s_lo=0.01, s_hi=0.05):
    rng = np.random.Generator(np.random.PCG64(seed))
    A = round_to(rng.standard_normal((M, K), dtype=np.float32), a_dtype)
    t = rng.integers(-1, 2, size=(K, N), dtype=np.int8)
    S = round_to(rng.uniform(s_lo, s_hi, size=(K // group, N)).astype(np.float32), "f16")
    return A, t, S


# ------------------------------------------------------------------ formats

def pack_linear_u4(q: np.ndarray) -> np.ndarray:
    K, N = q.shape
    out = np.empty((K // 8, N), np.uint32)
    _ck(lib().hqo_pack_linear_u4(_p(np.ascontiguousarray(q, np.int8)), _p(out), K, N), "pack_linear_u4")
    return out


def unpack_linear_u4(w: np.ndarray, K: int, N: int) -> np.ndarray:
    q = np.empty((K, N), np.int8)
    _ck(lib().hqo_unpack_linear_u4(_p(np.ascontiguousarray(w, np.uint32)), _p(q), K, N), "unpack_linear_u4")
    return q


def repack_marlin_quad(linear: np.ndarray, K: int, N: int) -> np.ndarray:
    out = np.empty((K // 32, N, 4), np.uint32)
    _ck(lib().hqo_repack_marlin_quad(_p(np.ascontiguousarray(linear, np.uint32)), _p(out), K, N), "repack_marlin_quad")
    return out


def unrepack_marlin_quad(quad: np.ndarray, K: int, N: int) -> np.ndarray:
    out = np.empty((K // 8, N), np.uint32)
    _ck(lib().hqo_unrepack_marlin_quad(_p(np.ascontiguousarray(quad, np.uint32)), _p(out), K, N), "unrepack")
    return out


def pack_linear_t2(t: np.ndarray) -> np.ndarray:
    K, N = t.shape
    out = np.empty((K // 16, N), np.uint32)
    _ck(lib().hqo_pack_linear_t2(_p(np.ascontiguousarray(t, np.int8)), _p(out), K, N), "pack_linear_t2")
    return out


def unpack_linear_t2(w: np.ndarray, K: int, N: int) -> np.ndarray:
    t = np.empty((K, N), np.int8)
    _ck(lib().hqo_unpack_linear_t2(_p(np.ascontiguousarray(w, np.uint32)), _p(t), K, N), "unpack_linear_t2")
    return t


def tile_bytes(K: int, N: int, wbits: int) -> int:
    return int(lib().hqo_tile_bytes(K, N, wbits))


def pack_tile(q: np.ndarray, wbits: int) -> np.ndarray:
    K, N = q.shape
    out = np.empty(tile_bytes(K, N, wbits), np.uint8)
    _ck(lib().hqo_pack_tile(_p(np.ascontiguousarray(q, np.int8)), _p(out), K, N, wbits), "pack_tile")
    return out


def unpack_tile(tile: np.ndarray, K: int, N: int, wbits: int) -> np.ndarray:
    q = np.empty((K, N), np.int8)
    _ck(lib().hqo_unpack_tile(_p(np.ascontiguousarray(tile, np.uint8)), _p(q), K, N, wbits), "unpack_tile")
    return q


def _k32_perm(K: int) -> np.ndarray:
    """Row order that turns TILE_U4 into TILE_U4_K32: tile position 16t + 8j + e of a 64-k
    block holds k = 8t + 32j + e (hq.h HQ_WFMT_TILE_U4_K32)."""
    d = np.arange(64)
    t, j, e = d // 16, (d // 8) % 2, d % 8
    src = 8 * t + 32 * j + e
    return (np.arange(K) // 64) * 64 + src[np.arange(K) % 64]


def pack_tile_k32(q: np.ndarray) -> np.ndarray:
    """TILE_U4_K32 bytes of int4 codes q [K][N]: the tile packer on k-permuted rows."""
    return pack_tile(np.ascontiguousarray(q[_k32_perm(q.shape[0])]), 4)


def unpack_tile_k32(tile: np.ndarray, K: int, N: int) -> np.ndarray:
    q = np.empty((K, N), np.int8)
    q[_k32_perm(K)] = unpack_tile(tile, K, N, 4)
    return q


def pack_tq1_0(t_nk: np.ndarray, d_bits: np.ndarray) -> np.ndarray:
    N, K = t_nk.shape
    out = np.empty(N * (K // 256) * 56, np.uint8)
    _ck(lib().hqo_pack_tq1_0(_p(np.ascontiguousarray(t_nk, np.int8)),
                             _p(np.ascontiguousarray(d_bits, np.uint16)), _p(out), K, N), "pack_tq1_0")
    return out


def unpack_tq1_0(blob: np.ndarray, K: int, N: int):
    t = np.empty((N, K), np.int8)
    d = np.empty((N, K // 256), np.uint16)
    _ck(lib().hqo_unpack_tq1_0(_p(np.ascontiguousarray(blob, np.uint8)), _p(t), _p(d), K, N), "unpack_tq1_0")
    return t, d


# --------------------------------------------------------------------- math

def dequant_u4(linear, scales, bias, K, N, group):
    W = np.empty((K, N), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    _ck(lib().hqo_dequant_u4(_p(np.ascontiguousarray(linear, np.uint32)),
                             _p(np.ascontiguousarray(scales, np.float32)),
                             None if b is None else _p(b), _p(W), K, N, group), "dequant_u4")
    return W


def gemm_f32(X, W, nthreads=0):
    M, K = X.shape
    N = W.shape[1]
    Y = np.empty((M, N), np.float32)
    _ck(lib().hqo_gemm_f32(_p(np.ascontiguousarray(X, np.float32)), _p(np.ascontiguousarray(W, np.float32)),
                           _p(Y), M, K, N, nthreads), "gemm_f32")
    return Y


def w4_gemm(X, linear, scales, bias=None, group=128, nthreads=0):
    """Fused dequant-then-matmul (fp32, k ascending, FMA per step)."""
    M, K = X.shape
    N = linear.shape[1]
    Y = np.empty((M, N), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    _ck(lib().hqo_w4_gemm(_p(np.ascontiguousarray(X, np.float32)), _p(np.ascontiguousarray(linear, np.uint32)),
                          _p(np.ascontiguousarray(scales, np.float32)), None if b is None else _p(b),
                          _p(Y), M, K, N, group, nthreads), "w4_gemm")
    return Y


def t2_gemm(X, linear_t2, scales, group=128, nthreads=0):
    M, K = X.shape
    N = linear_t2.shape[1]
    Y = np.empty((M, N), np.float32)
    _ck(lib().hqo_t2_gemm(_p(np.ascontiguousarray(X, np.float32)), _p(np.ascontiguousarray(linear_t2, np.uint32)),
                          _p(np.ascontiguousarray(scales, np.float32)), _p(Y), M, K, N, group, nthreads), "t2_gemm")
    return Y


def gemv_tq1_0(x, blob, in_dim, out_dim, nthreads=0):
    out = np.empty(out_dim, np.float32)
    _ck(lib().hqo_gemv_tq1_0(_p(np.ascontiguousarray(x, np.float32)), _p(np.ascontiguousarray(blob, np.uint8)),
                             _p(out), in_dim, out_dim, nthreads), "gemv_tq1_0")
    return out


def w8_gemm(X, W, scales, nthreads=0):
    """kernel_cutlass_int8_gemm (marlin_gemm.cu:327-377) restated: X fp32 [M][K], W int8 [K][N], scales fp32 [N]."""
    X = np.ascontiguousarray(X, np.float32)
    W = np.ascontiguousarray(W, np.int8)
    M, K = X.shape
    N = W.shape[1]
    Y = np.empty((M, N), np.float32)
    _ck(lib().hqo_w8_gemm(_p(X), _p(W), _p(np.ascontiguousarray(scales, np.float32)), _p(Y), M, K, N, nthreads),
        "w8_gemm")
    return Y


GGML_F32, GGML_Q8_0, GGML_BF16, GGML_TQ1_0 = 0, 8, 30, 34  # gguf_parser.hpp:33-64


def output_projection(x, w, w_type, embedding_dim, vocab_size, nthreads=0):
    """kernel_output_projection (forward_baseline.cu:178-257) restated: logits = W x."""
    out = np.empty(vocab_size, np.float32)
    wa = np.ascontiguousarray(w)
    _ck(lib().hqo_output_projection(_p(np.ascontiguousarray(x, np.float32)), _p(wa), w_type, _p(out),
                                    embedding_dim, vocab_size, nthreads), "output_projection")
    return out


def embedding_lookup(table, w_type, token_id, embedding_dim):
    """kernel_embedding_lookup (forward_baseline.cu:55-109) restated: row token_id as fp32."""
    out = np.empty(embedding_dim, np.float32)
    _ck(lib().hqo_embedding_lookup(_p(np.ascontiguousarray(table)), w_type, token_id, _p(out), embedding_dim),
        "embedding_lookup")
    return out


def pack_q8_0(q, d_bits):
    """Q8_0 blocks (forward_baseline.cu:30-33): per 32 weights fp16 d (bits) + 32 int8, 34 bytes.
    q int8 [N][K], d_bits uint16 [N][K/32] -> uint8 [N * K/32 * 34]."""
    q = np.asarray(q, np.int8)
    N, K = q.shape
    blk = np.empty((N, K // 32, 34), np.uint8)
    blk[:, :, 0:2] = np.asarray(d_bits, np.uint16).reshape(N, K // 32, 1).view(np.uint8)
    blk[:, :, 2:] = q.reshape(N, K // 32, 32).view(np.uint8)
    return blk.ravel()


def max_rel_err(y, y_ref) -> float:
    """max|y - y_ref| / max|y_ref| over the whole output tensor."""
    y = np.asarray(y, np.float64)
    y_ref = np.asarray(y_ref, np.float64)
    den = np.max(np.abs(y_ref))
    return float(np.max(np.abs(y - y_ref)) / (den if den > 0 else 1.0))


# --------------------------------------------------------------- GGUF Q4_K
#
# The reference names Q4_K only as a GGUF block type (hydrogen/include/
# gguf_parser.hpp:44 type 12, :130 256 weights in 144 bytes); its field layout
# and dequantisation are llama.cpp's (ggml/src/ggml-common.h block_q4_K,
# ggml/src/ggml-quants.c dequantize_row_q4_K / get_scale_min_k4), a pinned but
# un-vendored dependency of the reference.  Restated here from that published
# format; pinned against gguf-py 0.19.0 (gguf.quants.dequantize, llama.cpp's own
# Python copy of the format) by tests/golden/make_q4k_golden.py.

Q4K_BLOCK_BYTES = 144


def unpack_q4_k(blob: np.ndarray, K: int, N: int):
    """Q4_K blocks [N][K/256] -> (codes u uint8 [K][N], scale f32 [K/32][N], bias f32 [K/32][N])
    with weight = u * scale + bias, scale = d * sc_i, bias = -(dmin * m_i)."""
    nb = K // 256
    blk = np.ascontiguousarray(blob, np.uint8).reshape(N, nb, Q4K_BLOCK_BYTES)
    d = blk[:, :, 0:2].copy().view(np.float16)[..., 0].astype(np.float32)        # [N, nb]
    dmin = blk[:, :, 2:4].copy().view(np.float16)[..., 0].astype(np.float32)
    p = blk[:, :, 4:16].astype(np.int32)                                         # [N, nb, 12]
    sc = np.empty((N, nb, 8), np.int32)
    mn = np.empty((N, nb, 8), np.int32)
    sc[..., 0:4] = p[..., 0:4] & 63
    mn[..., 0:4] = p[..., 4:8] & 63
    sc[..., 4:8] = (p[..., 8:12] & 0xF) | ((p[..., 0:4] >> 6) << 4)
    mn[..., 4:8] = (p[..., 8:12] >> 4) | ((p[..., 4:8] >> 6) << 4)
    qs = blk[:, :, 16:].reshape(N, nb, 4, 32)
    codes = np.stack([qs & 0xF, qs >> 4], axis=3).reshape(N, K)                  # k = 64j + 32h + l
    scale = (d[:, :, None] * sc.astype(np.float32)).reshape(N, K // 32)
    bias = -(dmin[:, :, None] * mn.astype(np.float32)).reshape(N, K // 32)
    return (np.ascontiguousarray(codes.T), np.ascontiguousarray(scale.T.astype(np.float32)),
            np.ascontiguousarray(bias.T.astype(np.float32)))


def dequant_q4_k(blob: np.ndarray, K: int, N: int) -> np.ndarray:
    """llama.cpp's dequantize_row_q4_K per row, as float32 [K][N]: y = (d sc) u - dmin m."""
    u, scale, bias = unpack_q4_k(blob, K, N)
    s = np.repeat(scale, 32, axis=0)
    m = -np.repeat(bias, 32, axis=0)
    return (s * u.astype(np.float32)).astype(np.float32) - m


def q4_k_to_tile(blob: np.ndarray, K: int, N: int):
    """The oracle's Q4_K -> (TILE_U4_K32 bytes, scale, bias): the packer on q = u - 8."""
    u, scale, bias = unpack_q4_k(blob, K, N)
    return pack_tile_k32(u.astype(np.int8) - 8), scale, bias


def q4_k_gemm(X, blob, K, N, nthreads=0):
    """X [M][K] fp32 times the Q4_K weights, through the fused int4 oracle (group 32, biased form)."""
    u, scale, bias = unpack_q4_k(blob, K, N)
    linear = pack_linear_u4(u.astype(np.int8) - 8)
    return w4_gemm(X, linear, scale, bias, group=32, nthreads=nthreads)


def gen_q4_k_blocks(K: int, N: int, seed: int = 0, d_range=(1e-3, 4e-3), dmin_range=(1e-3, 4e-3)) -> np.ndarray:
    """Seeded Q4_K tensor [N][K/256] of 144-byte blocks: random scale/min/code bytes and
    fp16 d / dmin drawn uniformly from the given ranges (weights of order 0.1)."""
    rng = np.random.default_rng(seed)
    nb = K // 256
    blk = rng.integers(0, 256, size=(N, nb, Q4K_BLOCK_BYTES), dtype=np.uint8)
    d = rng.uniform(*d_range, size=(N, nb)).astype(np.float16)
    dmin = rng.uniform(*dmin_range, size=(N, nb)).astype(np.float16)
    blk[:, :, 0:2] = d.view(np.uint8).reshape(N, nb, 2)
    blk[:, :, 2:4] = dmin.view(np.uint8).reshape(N, nb, 2)
    return blk.reshape(-1)


# ----------------------------------------------------- reference (compiled)

def ref_repack_q4k_to_marlin(linear: np.ndarray, K: int, N: int):
    """Run the reference's own repack (marlin_gemm.cu:432-467) through a constructed
    MarlinGemmEngine.  The engine's constructor allocates device memory, so this needs a
    GPU; returns None when the reference library is absent or no engine can be built."""
    r = ref_lib()
    if r is None:
        return None
    eng = r.ref_engine_create(1, K, N, 32)
    if not eng:
        return None
    try:
        out = np.zeros((K // 32, N, 4), np.uint32)
        ms = c_double(0.0)
        rc = r.ref_engine_repack_q4k_to_marlin(c_void_p(eng), _p(np.ascontiguousarray(linear, np.uint32)), _p(out),
                                               K, N, ctypes.byref(ms))
        if rc != 0:
            raise RuntimeError(r.ref_last_error().decode())
        return out
    finally:
        r.ref_engine_destroy(c_void_p(eng))
