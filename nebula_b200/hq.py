"""Python host side of the quantized linear layer (torch tensors in, libhq.so underneath).

Mirrors the reference's operator interface for this path:
  * ``MarlinGemmEngine`` -- the methods of hydrogen::MarlinGemmEngine
    (hydrogen/include/marlin_gemm.hpp:59-172) with the same argument meaning
    (device tensors for X / weights / scales / biases / Y, M rows), raising
    ``HQError`` where the reference throws std::runtime_error;
  * ``tq1_0_gemv`` -- kernel_gemv_tq1_0 (hydrogen/src/model/native_decoder.cu:155-206);
  * ``QuantLinear`` / ``gemm`` -- the production entry (hq_gemm) on tile-order
    weights produced once by ``repack``.
All device work runs on the caller's current torch stream.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import (HQ_BF16, HQ_F16, HQ_F32, HQ_WFMT_LINEAR_T2, HQ_WFMT_LINEAR_U4, HQ_WFMT_MARLIN_QUAD,
                   HQ_WFMT_TILE_T2, HQ_WFMT_TILE_U4, HQ_WFMT_TILE_U4_K32, HQ_WFMT_TQ1_0, HQError, check, lib)

__all__ = ["HQError", "weight_bytes", "repack_host", "repack", "make_workspace", "gemm", "QuantLinear",
           "tq1_0_gemv", "tq1_0_to_tile_t2", "q4_k_to_tile", "q4_k_to_tile_host", "output_projection", "embedding_lookup", "w8_gemm", "check_device_error",
           "MarlinGemmEngine",
           "HQ_WFMT_LINEAR_U4", "HQ_WFMT_MARLIN_QUAD", "HQ_WFMT_TILE_U4", "HQ_WFMT_LINEAR_T2",
           "HQ_WFMT_TILE_T2", "HQ_WFMT_TQ1_0", "HQ_WFMT_TILE_U4_K32"]

_DT = {torch.float32: HQ_F32, torch.float16: HQ_F16, torch.bfloat16: HQ_BF16}


def _dt(t: torch.dtype) -> int:
    try:
        return _DT[t]
    except KeyError:
        raise HQError(_lib.HQ_ERR_INVALID_ARG, f"unsupported dtype {t}") from None


def _stream(stream=None) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _ptr(t) -> ctypes.c_void_p | None:
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def weight_bytes(fmt: int, K: int, N: int) -> int:
    return int(lib().hq_weight_bytes(fmt, K, N))


def repack_host(src: np.ndarray, src_fmt: int, dst_fmt: int, K: int, N: int, nthreads: int = 0) -> np.ndarray:
    """Bit-exact host repack (hq_repack_host); returns a uint32 array in dst_fmt."""
    src = np.ascontiguousarray(src)
    nb = weight_bytes(dst_fmt, K, N)
    if nb == 0:
        raise HQError(_lib.HQ_ERR_UNSUPPORTED_SHAPE, f"no {dst_fmt} layout for K={K} N={N}")
    dst = np.empty(nb // 4, np.uint32)
    check(lib().hq_repack_host(src.ctypes.data_as(ctypes.c_void_p), src_fmt, dst.ctypes.data_as(ctypes.c_void_p),
                               dst_fmt, K, N, nthreads))
    return dst


def repack(src: torch.Tensor, src_fmt: int, dst_fmt: int, K: int, N: int, stream=None) -> torch.Tensor:
    """Bit-exact device repack (hq_repack_device) into a new uint8 tensor."""
    nb = weight_bytes(dst_fmt, K, N)
    if nb == 0:
        raise HQError(_lib.HQ_ERR_UNSUPPORTED_SHAPE, f"no {dst_fmt} layout for K={K} N={N}")
    dst = torch.empty(nb, dtype=torch.uint8, device=src.device)
    check(lib().hq_repack_device(_ptr(src), src_fmt, _ptr(dst), dst_fmt, K, N, _stream(stream)))
    return dst


def make_workspace(M: int, N: int, K: int, group: int, wfmt: int, device) -> torch.Tensor:
    """Zero-filled workspace for hq_gemm (split-K partials + self-resetting counters)."""
    if K <= 0 or N <= 0 or N % 16 or K % 64 or group <= 0 or K % group:
        raise HQError(_lib.HQ_ERR_UNSUPPORTED_SHAPE, f"bad shape M={M} N={N} K={K} group={group}")
    with torch.cuda.device(device):
        nb = int(lib().hq_gemm_workspace_size(M, N, K, group, wfmt))
    return torch.zeros(max(nb, 16), dtype=torch.uint8, device=device)


def gemm(A: torch.Tensor, W: torch.Tensor, scales: torch.Tensor, *, N: int, group: int = 128,
         wfmt: int | None = None, bias: torch.Tensor | None = None, out: torch.Tensor | None = None,
         out_dtype: torch.dtype | None = None, workspace: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """C = A @ dequant(W) through hq_gemm.  A: [M, K] device tensor.  wfmt defaults to the tile
    order of the group: TILE_U4_K32 for group 32, TILE_U4 otherwise."""
    M, K = A.shape
    if wfmt is None:
        wfmt = HQ_WFMT_TILE_U4_K32 if group == 32 else HQ_WFMT_TILE_U4
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype or A.dtype, device=A.device)
    if workspace is None:
        workspace = make_workspace(M, N, K, group, wfmt, A.device)
    check(lib().hq_gemm(_ptr(A), _dt(A.dtype), _ptr(W), wfmt, _ptr(scales), _dt(scales.dtype), _ptr(bias),
                        _ptr(out), _dt(out.dtype), M, N, K, group, _ptr(workspace), workspace.numel(),
                        _stream(stream)))
    return out


class QuantLinear:
    """A packed quantized linear layer: tile-order weights + group scales + workspace."""

    def __init__(self, W_tile: torch.Tensor, scales: torch.Tensor, K: int, N: int, group: int = 128,
                 wbits: int = 4, max_m: int = 16, bias: torch.Tensor | None = None):
        self.W, self.scales, self.K, self.N, self.group, self.bias = W_tile, scales, K, N, group, bias
        self.wfmt = (HQ_WFMT_TILE_U4_K32 if group == 32 else HQ_WFMT_TILE_U4) if wbits == 4 else HQ_WFMT_TILE_T2
        self.max_m = max_m
        self.workspace = make_workspace(max_m, N, K, group, self.wfmt, W_tile.device)

    @classmethod
    def from_q4_k(cls, w_q4k: torch.Tensor, K: int, N: int, max_m: int = 16, stream=None) -> "QuantLinear":
        """A layer from GGUF Q4_K blocks [N][K/256] on the device (converted once, exactly)."""
        tile, scales, bias = q4_k_to_tile(w_q4k, K, N, stream=stream)
        return cls(tile, scales, K, N, group=32, max_m=max_m, bias=bias)

    def __call__(self, A: torch.Tensor, out: torch.Tensor | None = None, out_dtype=None, stream=None):
        if A.shape[0] > self.max_m:
            self.max_m = A.shape[0]
            self.workspace = make_workspace(self.max_m, self.N, self.K, self.group, self.wfmt, A.device)
        return gemm(A, self.W, self.scales, N=self.N, group=self.group, wfmt=self.wfmt, bias=self.bias, out=out,
                    out_dtype=out_dtype, workspace=self.workspace, stream=stream)


def tq1_0_gemv(x: torch.Tensor, w: torch.Tensor, out_dim: int, out: torch.Tensor | None = None,
               stream=None) -> torch.Tensor:
    in_dim = x.numel()
    if out is None:
        out = torch.empty(out_dim, dtype=torch.float32, device=x.device)
    check(lib().hq_tq1_0_gemv(_ptr(x), _ptr(w), _ptr(out), in_dim, out_dim, _stream(stream)))
    return out


def w8_gemm(X: torch.Tensor, W: torch.Tensor, scales: torch.Tensor, out: torch.Tensor | None = None,
            stream=None) -> torch.Tensor:
    """forward_cutlass_int8 (marlin_gemm.cu:327-377): Y = scale * q8(X) W / 127; X fp32 [M][K], W int8 [K][N],
    scales fp32 [N]."""
    M, K = X.shape
    N = W.shape[1]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=X.device)
    check(lib().hq_w8_gemm(_ptr(X), _ptr(W), _ptr(scales), _ptr(out), M, K, N, _stream(stream)))
    return out


def output_projection(x: torch.Tensor, w: torch.Tensor, w_type: int, vocab_size: int,
                      out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """kernel_output_projection (forward_baseline.cu:178-257): logits = W x over GGML F32 / BF16 / Q8_0 /
    TQ1_0 rows (w_type: _lib.HQ_GGML_*), fp32 x and logits."""
    embedding_dim = x.numel()
    if out is None:
        out = torch.empty(vocab_size, dtype=torch.float32, device=x.device)
    check(lib().hq_output_projection(_ptr(x), _ptr(w), w_type, _ptr(out), embedding_dim, vocab_size,
                                     _stream(stream)))
    return out


def embedding_lookup(table: torch.Tensor, w_type: int, token_id: int, embedding_dim: int, vocab_size: int,
                     out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """kernel_embedding_lookup (forward_baseline.cu:55-109): row token_id of a GGML table as fp32."""
    if out is None:
        out = torch.empty(embedding_dim, dtype=torch.float32, device=table.device)
    check(lib().hq_embedding_lookup(_ptr(table), w_type, token_id, _ptr(out), embedding_dim, vocab_size,
                                    _stream(stream)))
    return out


def tq1_0_to_tile_t2(w: torch.Tensor, K: int, N: int, stream=None):
    tile = torch.empty(weight_bytes(HQ_WFMT_TILE_T2, K, N), dtype=torch.uint8, device=w.device)
    scales = torch.empty((K // 128, N), dtype=torch.float16, device=w.device)
    check(lib().hq_tq1_0_to_tile_t2(_ptr(w), _ptr(tile), _ptr(scales), K, N, _stream(stream)))
    return tile, scales


def q4_k_to_tile(w: torch.Tensor, K: int, N: int, stream=None):
    """GGUF Q4_K blocks [N][K/256] (uint8, device) -> (TILE_U4_K32 codes, f32 scales [K/32, N],
    f32 bias [K/32, N]) for gemm(..., bias=bias, group=32)."""
    tile = torch.empty(weight_bytes(HQ_WFMT_TILE_U4_K32, K, N), dtype=torch.uint8, device=w.device)
    scales = torch.empty((K // 32, N), dtype=torch.float32, device=w.device)
    bias = torch.empty((K // 32, N), dtype=torch.float32, device=w.device)
    check(lib().hq_q4_k_to_tile(_ptr(w), _ptr(tile), _ptr(scales), _ptr(bias), K, N, _stream(stream)))
    return tile, scales, bias


def q4_k_to_tile_host(w: np.ndarray, K: int, N: int, nthreads: int = 0):
    """Host-thread form of q4_k_to_tile on numpy arrays."""
    src = np.ascontiguousarray(w, dtype=np.uint8)
    tile = np.empty(weight_bytes(HQ_WFMT_TILE_U4_K32, K, N), np.uint8)
    scales = np.empty((K // 32, N), np.float32)
    bias = np.empty((K // 32, N), np.float32)
    vp = ctypes.c_void_p
    check(lib().hq_q4_k_to_tile_host(src.ctypes.data_as(vp), tile.ctypes.data_as(vp), scales.ctypes.data_as(vp),
                                        bias.ctypes.data_as(vp), K, N, nthreads))
    return tile, scales, bias


def check_device_error() -> None:
    check(lib().hq_check_device_error())


class MarlinGemmEngine:
    """hydrogen::MarlinGemmEngine (marlin_gemm.hpp:59-172) through the C wrappers."""

    def __init__(self, M: int, K: int, N: int, group_size: int = 128):
        self._h = lib().hq_marlin_engine_create(M, K, N, group_size)
        if not self._h:
            raise HQError(_lib.HQ_ERR_CUDA, lib().hq_last_error_string().decode(errors="replace"))
        self.M, self.K, self.N, self.group_size = M, K, N, group_size

    def close(self):
        if self._h:
            lib().hq_marlin_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def repack_q4k_to_marlin(self, h_src: np.ndarray, K: int, N: int):
        src = np.ascontiguousarray(h_src, dtype=np.uint32)
        dst = np.zeros((K // 32, N, 4), np.uint32)
        ms = ctypes.c_double(0)
        check(lib().hq_marlin_repack_q4k_to_marlin(self._h, src.ctypes.data_as(ctypes.c_void_p),
                                                   dst.ctypes.data_as(ctypes.c_void_p), K, N, ctypes.byref(ms)))
        return dst, ms.value

    def forward_marlin_int4(self, X, W_marlin, scales, biases, Y, M):
        check(lib().hq_marlin_forward_marlin_int4(self._h, _ptr(X), _ptr(W_marlin), _ptr(scales), _ptr(biases),
                                                  _ptr(Y), M))

    def forward_baseline_int4(self, X, W_linear, scales, biases, Y, M):
        check(lib().hq_marlin_forward_baseline_int4(self._h, _ptr(X), _ptr(W_linear), _ptr(scales),
                                                    _ptr(biases), _ptr(Y), M))

    def forward_reference(self, X, W_dequant, Y_ref, M):
        check(lib().hq_marlin_forward_reference(self._h, _ptr(X), _ptr(W_dequant), _ptr(Y_ref), M))

    def verify_fidelity(self, Y_ref, Y, M):
        mx, mse = ctypes.c_double(0), ctypes.c_double(0)
        check(lib().hq_marlin_verify_fidelity(self._h, _ptr(Y_ref), _ptr(Y), M, ctypes.byref(mx), ctypes.byref(mse)))
        return mx.value, mse.value
