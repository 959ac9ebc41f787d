"""Generate the committed golden fixtures (tests/golden/*.npz).

Needs oracle/liboracle.so and, for the reference columns, oracle/_ref/libref_marlin.so
compiled from the reference source (both built by __graft_entry__.build()), on a machine
with a GPU: the reference repack runs on a constructed MarlinGemmEngine, whose
constructor allocates device memory.

    python tests/golden/make_golden.py           # (re)write golden.npz
    python tests/golden/make_golden.py --check   # regenerate in memory, compare with golden.npz

Contents
  * int4 / ternary / TQ1_0 cases at small and ragged shapes: the seeded inputs,
    every packed layout, and the oracle's fp32 outputs;
  * ``*_ref_quad``: the Marlin-quad repack produced by the reference's own
    MarlinGemmEngine::repack_q4k_to_marlin (hydrogen/src/model/marlin_gemm.cu
    :432-467) run through oracle/_ref -- the vector that pins the oracle's
    restatement of that repack;
  * ``cfg0_*``: BASELINE config 0 (A fp16 [16,4096] ~N(0,1), int4 [4096,4096]
    g128, fp16 scales ~U(0.005,0.02), seed 0): input checksums and the oracle
    output, so the GPU box can check the full-size CPU-reference case without
    re-running the oracle.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as o  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def int4_case(prefix, M, K, N, group, seed, dtype, out):
    A, q, S = o.gen_int4_case(M, K, N, group=group, seed=seed, a_dtype=dtype)
    lin = o.pack_linear_u4(q)
    quad = o.repack_marlin_quad(lin, K, N)
    ref_quad = o.ref_repack_q4k_to_marlin(lin, K, N)
    if ref_quad is None:
        raise SystemExit("no reference engine: oracle/_ref/libref_marlin.so is missing or no GPU is visible")
    assert np.array_equal(quad, ref_quad), "oracle repack differs from the reference repack"
    tile = o.pack_tile(q, 4)
    Y = o.w4_gemm(A, lin, S, None, group=group, nthreads=1)
    Yb = o.w4_gemm(A, lin, S, -8.0 * S, group=group, nthreads=1)
    out.update({f"{prefix}_A": A, f"{prefix}_q": q, f"{prefix}_S": S, f"{prefix}_linear": lin,
                f"{prefix}_quad": quad, f"{prefix}_ref_quad": ref_quad, f"{prefix}_tile": tile,
                f"{prefix}_Y": Y, f"{prefix}_Ybias": Yb,
                f"{prefix}_meta": np.array([M, K, N, group, seed, 0 if dtype == "f16" else 1], np.int64)})


def t2_case(prefix, M, K, N, group, seed, dtype, out):
    A, t, S = o.gen_ternary_case(M, K, N, group=group, seed=seed, a_dtype=dtype)
    lin = o.pack_linear_t2(t)
    tile = o.pack_tile(t, 2)
    Y = o.t2_gemm(A, lin, S, group=group, nthreads=1)
    out.update({f"{prefix}_A": A, f"{prefix}_t": t, f"{prefix}_S": S, f"{prefix}_linear": lin,
                f"{prefix}_tile": tile, f"{prefix}_Y": Y,
                f"{prefix}_meta": np.array([M, K, N, group, seed, 0 if dtype == "f16" else 1], np.int64)})


def tq1_case(prefix, K, N, seed, out):
    rng = np.random.Generator(np.random.PCG64(seed))
    t = rng.integers(-1, 2, size=(N, K), dtype=np.int8)
    d = rng.uniform(0.01, 0.05, size=(N, K // 256)).astype(np.float16).view(np.uint16)
    d[0, 0] = 0x7C00  # +Inf block: skipped by the reference (native_decoder.cu:174)
    d[1, -1] = 0x7E00  # NaN block: skipped
    blob = o.pack_tq1_0(t, d)
    x = rng.standard_normal(K, dtype=np.float32)
    y = o.gemv_tq1_0(x, blob, K, N, nthreads=1)
    out.update({f"{prefix}_t": t, f"{prefix}_d": d, f"{prefix}_blob": blob, f"{prefix}_x": x, f"{prefix}_y": y,
                f"{prefix}_meta": np.array([K, N, seed], np.int64)})


def proj_case(prefix, w_type, K, N, seed, out):
    """Output projection and embedding rows (forward_baseline.cu:55-109, 178-257) over a GGML type."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal(K, dtype=np.float32)
    if w_type == o.GGML_F32:
        w = rng.standard_normal((N, K), dtype=np.float32).view(np.uint8).ravel()
    elif w_type == o.GGML_BF16:
        w = (rng.standard_normal((N, K), dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).ravel()
    elif w_type == o.GGML_Q8_0:
        q = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
        d = rng.uniform(0.005, 0.02, size=(N, K // 32)).astype(np.float16).view(np.uint16)
        d[2, 1] = 0x7E00  # NaN d: applied unchecked, the row's logit is NaN as in the reference
        w = o.pack_q8_0(q, d)
    else:
        t = rng.integers(-1, 2, size=(N, K), dtype=np.int8)
        d = rng.uniform(0.01, 0.05, size=(N, K // 256)).astype(np.float16).view(np.uint16)
        d[1, 0] = 0x7C00  # Inf d: read as 0 (forward_baseline.cu:223)
        w = o.pack_tq1_0(t, d)
    y = o.output_projection(x, w, w_type, K, N, nthreads=1)
    tokens = np.array([0, N // 2, N - 1], np.int64)
    emb = np.stack([o.embedding_lookup(w, w_type, int(tk), K) for tk in tokens])
    out.update({f"{prefix}_x": x, f"{prefix}_w": w, f"{prefix}_y": y, f"{prefix}_tokens": tokens,
                f"{prefix}_emb": emb, f"{prefix}_meta": np.array([w_type, K, N, seed], np.int64)})


def main():
    out: dict[str, np.ndarray] = {}
    int4_case("i4a", 3, 256, 48, 128, 7, "f16", out)       # N=48: one ragged strip group
    int4_case("i4b", 5, 512, 144, 64, 11, "bf16", out)     # 9 strips: 8 + 1; group 64
    int4_case("i4c", 16, 384, 256, 128, 13, "f16", out)    # K = 3 groups
    t2_case("t2a", 2, 256, 32, 128, 17, "f16", out)
    t2_case("t2b", 9, 512, 144, 128, 19, "bf16", out)
    tq1_case("tq1", 768, 40, 23, out)
    proj_case("pf32", o.GGML_F32, 200, 37, 29, out)     # K % 8 != 0
    proj_case("pbf16", o.GGML_BF16, 264, 37, 31, out)
    proj_case("pq8", o.GGML_Q8_0, 320, 37, 37, out)      # one NaN block scale
    proj_case("ptq1", 143, 512, 21, 41, out)             # TQ1_0 under its alternate type id; one Inf d
    # BASELINE config 0, full size: store checksums of the inputs and the output.
    A, q, S = o.gen_int4_case(16, 4096, 4096, group=128, seed=0, a_dtype="f16")
    lin = o.pack_linear_u4(q)
    Y = o.w4_gemm(A, lin, S, None, group=128)
    out["cfg0_Y"] = Y
    out["cfg0_sha"] = np.array([sha(A), sha(lin), sha(S)])
    path = os.path.join(HERE, "golden.npz")
    if "--check" in sys.argv[1:]:
        old = np.load(path)
        def same(a, b):  # byte equality, so NaN outputs compare equal to themselves
            return a.dtype == b.dtype and a.shape == b.shape and a.tobytes() == b.tobytes()
        bad = sorted(k for k in set(old.files) | set(out) if k not in old.files or k not in out
                     or not same(old[k], np.asarray(out[k])))
        print("golden.npz reproduced: " + ("yes" if not bad else "NO, differs in " + ", ".join(bad)))
        raise SystemExit(1 if bad else 0)
    np.savez_compressed(path, **out)
    print("wrote", path, sum(v.nbytes for v in out.values()), "bytes raw")


if __name__ == "__main__":
    main()
