"""CPU tests of the oracle: pinned against the reference's own code and the golden fixtures.

The oracle (oracle/hq_oracle.c) is test infrastructure; these tests establish
that it restates the reference before any GPU result is compared with it.
"""
import os

import numpy as np
import pytest

from oracle import oracle as o

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


# ----------------------------------------------------------- reference pins

@pytest.mark.gpu
def test_repack_matches_reference_binary_random():
    """Oracle repack == MarlinGemmEngine::repack_q4k_to_marlin (marlin_gemm.cu:432-467) on random words
    and on benchmark_repacking's constant fill (:648), through a constructed reference engine (its
    constructor allocates device memory, hence the GPU)."""
    if o.ref_lib() is None:
        pytest.skip("reference library not built (no reference tree at build time)")
    rng = np.random.default_rng(5)
    for K, N in [(32, 1), (64, 3), (512, 40), (4096, 64)]:
        lin = rng.integers(0, 2**32, size=(K // 8, N), dtype=np.uint64).astype(np.uint32)
        ref = o.ref_repack_q4k_to_marlin(lin, K, N)
        assert ref is not None, o.ref_lib().ref_last_error().decode()
        assert np.array_equal(o.repack_marlin_quad(lin, K, N), ref)
    K, N = 4096, 64
    lin = np.full((K // 8, N), 0x12345678, np.uint32)
    assert np.array_equal(o.repack_marlin_quad(lin, K, N), o.ref_repack_q4k_to_marlin(lin, K, N))


def test_repack_kat_constant_fill():
    """benchmark_repacking's constant fill (marlin_gemm.cu:648): every output word is the input word."""
    K, N = 4096, 64
    lin = np.full((K // 8, N), 0x12345678, np.uint32)
    assert np.all(o.repack_marlin_quad(lin, K, N) == 0x12345678)


def test_golden_reference_repack_vectors(golden):
    """The committed reference-repack outputs equal the oracle restatement."""
    for p in ("i4a", "i4b", "i4c"):
        M, K, N, g, seed, _ = golden[f"{p}_meta"]
        assert np.array_equal(o.repack_marlin_quad(golden[f"{p}_linear"], int(K), int(N)), golden[f"{p}_ref_quad"])


# ------------------------------------------------------------ golden fixtures

@pytest.mark.parametrize("p", ["i4a", "i4b", "i4c"])
def test_golden_int4(golden, p):
    M, K, N, g, seed, isbf = (int(v) for v in golden[f"{p}_meta"])
    A, q, S = o.gen_int4_case(M, K, N, group=g, seed=seed, a_dtype="bf16" if isbf else "f16")
    assert np.array_equal(A, golden[f"{p}_A"]) and np.array_equal(q, golden[f"{p}_q"])
    lin = o.pack_linear_u4(q)
    assert np.array_equal(lin, golden[f"{p}_linear"])
    assert np.array_equal(o.pack_tile(q, 4), golden[f"{p}_tile"])
    assert np.array_equal(o.w4_gemm(A, lin, S, None, group=g), golden[f"{p}_Y"])
    assert np.array_equal(o.w4_gemm(A, lin, S, -8.0 * S, group=g), golden[f"{p}_Ybias"])


@pytest.mark.parametrize("p", ["t2a", "t2b"])
def test_golden_ternary(golden, p):
    M, K, N, g, seed, isbf = (int(v) for v in golden[f"{p}_meta"])
    A, t, S = o.gen_ternary_case(M, K, N, group=g, seed=seed, a_dtype="bf16" if isbf else "f16")
    lin = o.pack_linear_t2(t)
    assert np.array_equal(lin, golden[f"{p}_linear"])
    assert np.array_equal(o.pack_tile(t, 2), golden[f"{p}_tile"])
    assert np.array_equal(o.t2_gemm(A, lin, S, group=g), golden[f"{p}_Y"])


def test_golden_tq1(golden):
    K, N, seed = (int(v) for v in golden["tq1_meta"])
    blob = o.pack_tq1_0(golden["tq1_t"], golden["tq1_d"])
    assert np.array_equal(blob, golden["tq1_blob"])
    assert np.array_equal(o.gemv_tq1_0(golden["tq1_x"], blob, K, N), golden["tq1_y"])


@pytest.mark.parametrize("prefix", ["pf32", "pbf16", "pq8", "ptq1"])
def test_golden_projection(golden, prefix):
    w_type, K, N, _ = (int(v) for v in golden[f"{prefix}_meta"])
    w = golden[f"{prefix}_w"]
    y = o.output_projection(golden[f"{prefix}_x"], w, w_type, K, N)
    assert np.array_equal(y, golden[f"{prefix}_y"], equal_nan=True)
    for tk, row in zip(golden[f"{prefix}_tokens"], golden[f"{prefix}_emb"]):
        assert np.array_equal(o.embedding_lookup(w, w_type, int(tk), K), row)


def test_projection_restatement_against_float64():
    """The restated projection against an independent float64 dot product of the decoded weights."""
    rng = np.random.default_rng(3)
    K, N = 320, 9
    x = rng.standard_normal(K).astype(np.float32)
    W = rng.standard_normal((N, K)).astype(np.float32)
    assert o.max_rel_err(o.output_projection(x, W, o.GGML_F32, K, N), W.astype(np.float64) @ x) < 1e-6
    bf = (W.view(np.uint32) >> 16).astype(np.uint16)
    Wb = (bf.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    assert o.max_rel_err(o.output_projection(x, bf, o.GGML_BF16, K, N), Wb @ x) < 1e-6
    q = rng.integers(-128, 128, (N, K), dtype=np.int8)
    d = rng.uniform(0.01, 0.02, (N, K // 32)).astype(np.float16)
    blob = o.pack_q8_0(q, d.view(np.uint16))
    Wq = (q.reshape(N, K // 32, 32) * d.astype(np.float64)[:, :, None]).reshape(N, K)
    assert o.max_rel_err(o.output_projection(x, blob, o.GGML_Q8_0, K, N), Wq @ x) < 1e-6
    for tk in (0, N - 1):
        assert np.array_equal(o.embedding_lookup(blob, o.GGML_Q8_0, tk, K), Wq[tk].astype(np.float32))
    # TQ1_0: the projection's restatement and the decoder GEMV's agree where every d is finite
    t = rng.integers(-1, 2, (N, 512), dtype=np.int8)
    dt = rng.uniform(0.01, 0.05, (N, 2)).astype(np.float16).view(np.uint16)
    tb = o.pack_tq1_0(t, dt)
    x2 = rng.standard_normal(512).astype(np.float32)
    assert o.max_rel_err(o.output_projection(x2, tb, o.GGML_TQ1_0, 512, N), o.gemv_tq1_0(x2, tb, 512, N)) < 1e-6
    emb = o.embedding_lookup(tb, o.GGML_TQ1_0, 4, 512)
    dd = dt[4].view(np.float16).astype(np.float32)
    assert np.array_equal(emb, (t[4].reshape(2, 256) * dd[:, None]).ravel().astype(np.float32))


def test_w8_restatement_against_int64():
    """kernel_cutlass_int8_gemm restated: against an int64 product of the same q8 activations (K % 4 tail ignored)."""
    rng = np.random.default_rng(8)
    M, K, N = 3, 102, 12
    X = (rng.standard_normal((M, K)) * 0.6).astype(np.float32)
    W = rng.integers(-128, 128, (K, N), dtype=np.int8)
    S = rng.uniform(0.01, 0.02, N).astype(np.float32)
    q = np.clip(X * np.float32(127), -128, 127).astype(np.int64)  # float -> int truncates toward zero
    kk = (K // 4) * 4
    ref = (q[:, :kk] @ W[:kk].astype(np.int64)).astype(np.float64) / 127 * S
    assert o.max_rel_err(o.w8_gemm(X, W, S), ref) < 1e-6


def test_golden_config0_checksums(golden):
    import hashlib
    A, q, S = o.gen_int4_case(16, 4096, 4096, group=128, seed=0, a_dtype="f16")
    lin = o.pack_linear_u4(q)
    sh = [hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest() for x in (A, lin, S)]
    assert list(golden["cfg0_sha"]) == sh
    assert np.array_equal(o.w4_gemm(A, lin, S, None, group=128), golden["cfg0_Y"])


# ------------------------------------------------------------ restatement

@pytest.mark.parametrize("K,N", [(64, 16), (128, 48), (256, 144), (512, 272), (192, 1040)])
def test_tile_roundtrip(K, N):
    rng = np.random.default_rng(K + N)
    q = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    assert np.array_equal(o.unpack_tile(o.pack_tile(q, 4), K, N, 4), q)
    t = rng.integers(-1, 2, size=(K, N), dtype=np.int8)
    assert np.array_equal(o.unpack_tile(o.pack_tile(t, 2), K, N, 2), t)


def test_tile_is_a_permutation_of_linear_words():
    """Each tile word carries exactly the 8 codes of one linear word (k-aligned), reordered."""
    rng = np.random.default_rng(3)
    K, N = 128, 144
    q = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    lin = o.pack_linear_u4(q)
    tile = o.pack_tile(q, 4).view(np.uint32)
    nib = lambda w: sorted(((int(w) >> (4 * i)) & 15) for i in range(8))  # noqa: E731
    assert sorted(map(tuple, (nib(w) for w in lin.ravel()))) == sorted(map(tuple, (nib(w) for w in tile)))


def test_linear_roundtrips():
    rng = np.random.default_rng(1)
    q = rng.integers(-8, 8, size=(256, 40), dtype=np.int8)
    lin = o.pack_linear_u4(q)
    assert np.array_equal(o.unpack_linear_u4(lin, 256, 40), q)
    assert np.array_equal(o.unrepack_marlin_quad(o.repack_marlin_quad(lin, 256, 40), 256, 40), lin)
    t = rng.integers(-1, 2, size=(256, 40), dtype=np.int8)
    assert np.array_equal(o.unpack_linear_t2(o.pack_linear_t2(t), 256, 40), t)


def test_pack_rejects_out_of_range():
    with pytest.raises(ValueError):
        o.pack_linear_u4(np.full((8, 4), 8, np.int8))
    with pytest.raises(ValueError):
        o.pack_tile(np.full((64, 16), 2, np.int8), 2)
    with pytest.raises(ValueError):
        o.pack_tile(np.zeros((60, 16), np.int8), 4)


def test_w4_gemm_matches_float64():
    A, q, S = o.gen_int4_case(4, 512, 96, seed=2)
    lin = o.pack_linear_u4(q)
    Y = o.w4_gemm(A, lin, S)
    W = q.astype(np.float64) * np.repeat(S.astype(np.float64), 128, axis=0)
    assert o.max_rel_err(Y, A.astype(np.float64) @ W) < 1e-6
    # fused path == separate dequant + reference GEMM, bit for bit (both forms)
    assert np.array_equal(Y, o.gemm_f32(A, o.dequant_u4(lin, S, None, 512, 96, 128)))
    B = -8.0 * S
    assert np.array_equal(o.w4_gemm(A, lin, S, B), o.gemm_f32(A, o.dequant_u4(lin, S, B, 512, 96, 128)))


def test_w4_gemm_thread_count_invariant():
    A, q, S = o.gen_int4_case(16, 1024, 512, seed=4)
    lin = o.pack_linear_u4(q)
    assert np.array_equal(o.w4_gemm(A, lin, S, nthreads=1), o.w4_gemm(A, lin, S, nthreads=8))


def test_tq1_decode_matches_digit_arithmetic():
    """TQ1_0 element decode (native_decoder.cu:81-101): digit j%5 of byte j/5, LS digit first."""
    rng = np.random.default_rng(9)
    t = rng.integers(-1, 2, size=(3, 512), dtype=np.int8)
    d = np.full((3, 2), 0x3C00, np.uint16)  # 1.0
    blob = o.pack_tq1_0(t, d).reshape(3, 2, 56)
    for n in range(3):
        for b in range(2):
            packed = blob[n, b, 2:54].astype(np.int64)
            for j in range(256):
                byte, dig = (j // 5, j % 5) if j < 250 else (50 + (j - 250) // 3, (j - 250) % 3)
                assert (packed[byte] // 3 ** dig) % 3 - 1 == t[n, b * 256 + j]


def test_tq1_gemv_skips_nonfinite_blocks():
    rng = np.random.default_rng(4)
    K, N = 512, 4
    t = rng.integers(-1, 2, size=(N, K), dtype=np.int8)
    d = np.full((N, 2), np.float16(0.5).view(np.uint16), np.uint16)
    d[2, 1] = 0x7C00
    blob = o.pack_tq1_0(t, d)
    x = rng.standard_normal(K).astype(np.float32)
    y = o.gemv_tq1_0(x, blob, K, N)
    ref = (t.astype(np.float64) * 0.5) @ x
    ref[2] = 0.5 * (t[2, :256].astype(np.float64) @ x[:256])
    assert np.allclose(y, ref, rtol=1e-5, atol=1e-5)
