"""CPU tests of the C ABI: libhq.so loads, exports what include/hq.h declares, host-side
repacks are bit-exact against the oracle, and argument errors come back as status codes
(no device work is issued by any call here)."""
import ctypes
import os
import re

import numpy as np
import pytest

from nebula_b200 import _lib
from oracle import oracle as o

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "hq.h")).read()
    return re.findall(r"HQ_API\s+[\w\s\*]+?\b(hq_\w+)\s*\(", src)


def test_library_loads_and_reports_version():
    L = _lib.lib()
    assert L.hq_version().decode().startswith("hq ")


def test_every_declared_symbol_is_exported_and_bound():
    L = _lib.lib()
    syms = header_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(L, s), f"{s} declared in include/hq.h but not exported"
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(syms)


def test_only_abi_symbols_are_exported():
    """Internal C++ symbols stay hidden (-fvisibility=hidden); the dynamic table holds hq_* only."""
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    ours = {s for s in exported if s.startswith("hq_")}
    assert ours == set(header_symbols())


def test_weight_bytes():
    L = _lib.lib()
    assert L.hq_weight_bytes(_lib.HQ_WFMT_TILE_U4, 5120, 7168) == 5120 * 7168 // 2
    assert L.hq_weight_bytes(_lib.HQ_WFMT_TILE_T2, 5120, 7168) == 5120 * 7168 // 4
    assert L.hq_weight_bytes(_lib.HQ_WFMT_TQ1_0, 5120, 7168) == 7168 * 20 * 56
    assert L.hq_weight_bytes(_lib.HQ_WFMT_TILE_U4, 5120, 7160) == 0


def _host_repack(src, sf, df, K, N, nthreads=0):
    from nebula_b200 import hq
    return hq.repack_host(src, sf, df, K, N, nthreads)


@pytest.mark.parametrize("K,N", [(64, 16), (256, 48), (512, 144), (1024, 272)])
def test_host_repack_matches_oracle(K, N):
    rng = np.random.default_rng(K * 7 + N)
    q = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    lin = o.pack_linear_u4(q)
    quad = o.repack_marlin_quad(lin, K, N)
    tile = o.pack_tile(q, 4).view(np.uint32)
    assert np.array_equal(_host_repack(lin, _lib.HQ_WFMT_LINEAR_U4, _lib.HQ_WFMT_MARLIN_QUAD, K, N), quad.ravel())
    assert np.array_equal(_host_repack(quad, _lib.HQ_WFMT_MARLIN_QUAD, _lib.HQ_WFMT_LINEAR_U4, K, N), lin.ravel())
    assert np.array_equal(_host_repack(lin, _lib.HQ_WFMT_LINEAR_U4, _lib.HQ_WFMT_TILE_U4, K, N), tile)
    assert np.array_equal(_host_repack(quad, _lib.HQ_WFMT_MARLIN_QUAD, _lib.HQ_WFMT_TILE_U4, K, N, 3), tile)
    assert np.array_equal(_host_repack(tile, _lib.HQ_WFMT_TILE_U4, _lib.HQ_WFMT_LINEAR_U4, K, N), lin.ravel())
    t = rng.integers(-1, 2, size=(K, N), dtype=np.int8)
    lin2 = o.pack_linear_t2(t)
    tile2 = o.pack_tile(t, 2).view(np.uint32)
    assert np.array_equal(_host_repack(lin2, _lib.HQ_WFMT_LINEAR_T2, _lib.HQ_WFMT_TILE_T2, K, N), tile2)
    assert np.array_equal(_host_repack(tile2, _lib.HQ_WFMT_TILE_T2, _lib.HQ_WFMT_LINEAR_T2, K, N), lin2.ravel())


def test_host_repack_reference_kat():
    """benchmark_repacking's constant input (marlin_gemm.cu:648) repacks to itself."""
    K, N = 4096, 4096
    src = np.full((K // 8) * N, 0x12345678, np.uint32)
    out = _host_repack(src, _lib.HQ_WFMT_LINEAR_U4, _lib.HQ_WFMT_MARLIN_QUAD, K, N)
    assert np.all(out == 0x12345678)


@pytest.mark.gpu
def test_host_repack_matches_reference_binary():
    """hq_repack_host to Marlin quads == the reference's repack on a constructed engine (needs a GPU)."""
    if o.ref_lib() is None:
        pytest.skip("reference library not built (no reference tree at build time)")
    rng = np.random.default_rng(11)
    K, N = 2048, 96
    lin = rng.integers(0, 2**32, size=(K // 8, N), dtype=np.uint64).astype(np.uint32)
    ours = _host_repack(lin, _lib.HQ_WFMT_LINEAR_U4, _lib.HQ_WFMT_MARLIN_QUAD, K, N)
    assert np.array_equal(ours, o.ref_repack_q4k_to_marlin(lin, K, N).ravel())


def test_repack_errors():
    L = _lib.lib()
    buf = np.zeros(1024, np.uint32)
    p = buf.ctypes.data_as(ctypes.c_void_p)
    assert L.hq_repack_host(None, 0, p, 1, 64, 16, 0) == _lib.HQ_ERR_INVALID_ARG
    assert L.hq_repack_host(p, 0, p, 1, 48, 16, 0) == _lib.HQ_ERR_UNSUPPORTED_SHAPE
    assert L.hq_repack_host(p, 0, p, 2, 64, 8, 0) == _lib.HQ_ERR_UNSUPPORTED_SHAPE
    assert L.hq_repack_host(p, 4, p, 2, 64, 16, 0) == _lib.HQ_ERR_INVALID_ARG
    assert b"unsupported" in L.hq_last_error_string()


def test_gemm_argument_errors_need_no_device():
    """Shape, enum, null and alignment checks run before any device call."""
    L = _lib.lib()
    buf = np.zeros(4096, np.uint8)
    base = buf.ctypes.data
    al = base + (-base) % 16
    P = lambda a: ctypes.c_void_p(a)  # noqa: E731
    args = lambda **kw: dict(A=P(al), at=_lib.HQ_F16, W=P(al), wf=_lib.HQ_WFMT_TILE_U4, S=P(al),  # noqa: E731
                             st=_lib.HQ_F16, bias=None, C=P(al), ct=_lib.HQ_F16, M=1, N=16, K=64, g=64,
                             ws=P(al), wsb=1 << 20, stream=None) | kw
    call = lambda a: L.hq_gemm(a["A"], a["at"], a["W"], a["wf"], a["S"], a["st"], a["bias"], a["C"],  # noqa: E731
                               a["ct"], a["M"], a["N"], a["K"], a["g"], a["ws"], a["wsb"], a["stream"])
    assert call(args(N=24)) == _lib.HQ_ERR_UNSUPPORTED_SHAPE
    assert call(args(K=96)) == _lib.HQ_ERR_UNSUPPORTED_SHAPE
    assert call(args(g=16)) == _lib.HQ_ERR_UNSUPPORTED_SHAPE  # groups: 32 or multiples of 64
    assert call(args(g=96, K=192)) == _lib.HQ_ERR_UNSUPPORTED_SHAPE
    assert call(args(g=32, K=96)) == _lib.HQ_ERR_UNSUPPORTED_SHAPE
    assert call(args(M=-1)) == _lib.HQ_ERR_INVALID_ARG
    assert call(args(at=7)) == _lib.HQ_ERR_INVALID_ARG
    assert call(args(wf=_lib.HQ_WFMT_TQ1_0)) == _lib.HQ_ERR_INVALID_ARG
    assert call(args(A=None)) == _lib.HQ_ERR_INVALID_ARG
    assert call(args(C=P(al + 4))) == _lib.HQ_ERR_MISALIGNED
    assert call(args(M=0)) == _lib.HQ_OK  # empty problem: nothing to do
    assert call(args(wf=_lib.HQ_WFMT_TILE_T2, bias=P(al))) == _lib.HQ_ERR_INVALID_ARG


def test_tq1_gemv_argument_errors():
    L = _lib.lib()
    buf = np.zeros(4096, np.uint8)
    p = ctypes.c_void_p(buf.ctypes.data + (-buf.ctypes.data) % 16)
    assert L.hq_tq1_0_gemv(None, p, p, 256, 4, None) == _lib.HQ_ERR_INVALID_ARG
    assert L.hq_tq1_0_gemv(p, p, p, 200, 4, None) == _lib.HQ_ERR_UNSUPPORTED_SHAPE


def test_projection_argument_errors():
    L = _lib.lib()
    buf = np.zeros(4096, np.uint8)
    p = ctypes.c_void_p(buf.ctypes.data + (-buf.ctypes.data) % 16)
    odd = ctypes.c_void_p(p.value + 1)
    assert L.hq_output_projection(None, p, _lib.HQ_GGML_BF16, p, 256, 4, None) == _lib.HQ_ERR_INVALID_ARG
    assert L.hq_output_projection(p, p, 12, p, 256, 4, None) == _lib.HQ_ERR_INVALID_ARG  # Q4_K: not a projection type
    assert L.hq_output_projection(p, p, _lib.HQ_GGML_Q8_0, p, 48, 4, None) == _lib.HQ_ERR_UNSUPPORTED_SHAPE
    assert L.hq_output_projection(p, p, _lib.HQ_GGML_TQ1_0_ALT, p, 200, 4, None) == _lib.HQ_ERR_UNSUPPORTED_SHAPE
    assert L.hq_output_projection(p, odd, _lib.HQ_GGML_BF16, p, 256, 4, None) == _lib.HQ_ERR_MISALIGNED
    assert L.hq_embedding_lookup(p, _lib.HQ_GGML_F32, 4, p, 256, 4, None) == _lib.HQ_ERR_INVALID_ARG  # token >= vocab
    assert L.hq_embedding_lookup(p, _lib.HQ_GGML_F32, -1, p, 256, 4, None) == _lib.HQ_ERR_INVALID_ARG
    assert L.hq_embedding_lookup(p, _lib.HQ_GGML_Q8_0, 0, p, 40, 4, None) == _lib.HQ_ERR_UNSUPPORTED_SHAPE
    assert L.hq_embedding_lookup(p, 2, 0, p, 256, 4, None) == _lib.HQ_ERR_INVALID_ARG


def test_w8_gemm_argument_errors():
    L = _lib.lib()
    buf = np.zeros(4096, np.uint8)
    p = ctypes.c_void_p(buf.ctypes.data + (-buf.ctypes.data) % 16)
    odd = ctypes.c_void_p(p.value + 2)
    assert L.hq_w8_gemm(None, p, p, p, 1, 64, 64, None) == _lib.HQ_ERR_INVALID_ARG
    assert L.hq_w8_gemm(p, p, p, p, 1, 64, 66, None) == _lib.HQ_ERR_UNSUPPORTED_SHAPE
    assert L.hq_w8_gemm(p, p, p, p, 1, 65540, 64, None) == _lib.HQ_ERR_UNSUPPORTED_SHAPE
    assert L.hq_w8_gemm(p, odd, p, p, 1, 64, 64, None) == _lib.HQ_ERR_MISALIGNED
    assert L.hq_marlin_forward_cutlass_int8(None, p, p, p, p, 1) == _lib.HQ_ERR_INVALID_ARG
