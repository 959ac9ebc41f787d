"""Split-fuse continuous batching over libhq.so (hq_batcher_*): the scheduling of hydrogen::SplitFuseBatcher
(batcher.hpp:98-199, split_fuse.cpp:70-193) with a step executor that runs real hq_gemm layers at the fused M.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from ._lib import check, lib

QUEUED, RUNNING_PREFILL, RUNNING_DECODE, COMPLETED = range(4)


class _Config(ctypes.Structure):
    _fields_ = [("max_prefill_chunk_tokens", ctypes.c_uint32), ("max_decode_streams", ctypes.c_uint32),
                ("max_batch_tokens", ctypes.c_uint32)]


class _Chunk(ctypes.Structure):
    _fields_ = [("request_id", ctypes.c_uint32), ("start_token", ctypes.c_uint32),
                ("num_tokens", ctypes.c_uint32), ("is_prefill", ctypes.c_int)]


class _Info(ctypes.Structure):
    _fields_ = [("num_decode_requests", ctypes.c_uint32), ("num_prefill_tokens", ctypes.c_uint32),
                ("total_batch_tokens", ctypes.c_uint32), ("assembly_overhead_us", ctypes.c_double)]


class _State(ctypes.Structure):
    _fields_ = [("prompt_tokens", ctypes.c_uint32), ("prefill_completed_tokens", ctypes.c_uint32),
                ("decode_tokens_generated", ctypes.c_uint32), ("max_decode_tokens", ctypes.c_uint32),
                ("status", ctypes.c_int)]


class LinearLayer(ctypes.Structure):
    """hq_linear_layer: one quantized linear layer (device pointers)."""
    _fields_ = [("W", ctypes.c_void_p), ("wfmt", ctypes.c_int), ("scales", ctypes.c_void_p),
                ("s_dtype", ctypes.c_int), ("bias", ctypes.c_void_p), ("K", ctypes.c_int), ("N", ctypes.c_int),
                ("group", ctypes.c_int)]


@dataclass
class BatchChunk:
    request_id: int
    start_token: int
    num_tokens: int
    is_prefill: bool


@dataclass
class FusedBatch:
    chunks: list
    num_decode_requests: int
    num_prefill_tokens: int
    total_batch_tokens: int
    assembly_overhead_us: float


class SplitFuseBatcher:
    """SplitFuseBatcher's scheduling surface: submit_request, assemble_step_batch, update_step_completion,
    has_active_work, num_active_requests, reset; plus execute_step over real quantized layers."""

    def __init__(self, max_prefill_chunk_tokens=64, max_decode_streams=16, max_batch_tokens=512):
        cfg = _Config(max_prefill_chunk_tokens, max_decode_streams, max_batch_tokens)
        self._h = lib().hq_batcher_create(ctypes.byref(cfg))
        if not self._h:
            raise MemoryError("hq_batcher_create")

    def close(self):
        if self._h:
            lib().hq_batcher_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        lib().hq_batcher_reset(self._h)

    def submit_request(self, prompt_tokens: int, max_decode_tokens: int) -> int:
        return int(lib().hq_batcher_submit(self._h, prompt_tokens, max_decode_tokens))

    def assemble_step_batch(self) -> FusedBatch:
        cap = int(lib().hq_batcher_active_requests(self._h)) + 2
        buf = (_Chunk * cap)()
        info = _Info()
        n = lib().hq_batcher_assemble(self._h, buf, cap, ctypes.byref(info))
        if n < 0:
            raise RuntimeError("hq_batcher_assemble: chunk buffer too small")
        chunks = [BatchChunk(c.request_id, c.start_token, c.num_tokens, bool(c.is_prefill)) for c in buf[:n]]
        return FusedBatch(chunks, info.num_decode_requests, info.num_prefill_tokens, info.total_batch_tokens,
                          info.assembly_overhead_us)

    def update_step_completion(self, batch: FusedBatch):
        arr = (_Chunk * max(1, len(batch.chunks)))(
            *[_Chunk(c.request_id, c.start_token, c.num_tokens, int(c.is_prefill)) for c in batch.chunks])
        check(lib().hq_batcher_complete(self._h, arr, len(batch.chunks)))

    def has_active_work(self) -> bool:
        return bool(lib().hq_batcher_has_work(self._h))

    def num_active_requests(self) -> int:
        return int(lib().hq_batcher_active_requests(self._h))

    def request_state(self, request_id: int) -> dict:
        st = _State()
        check(lib().hq_batcher_request_state(self._h, request_id, ctypes.byref(st)))
        return {f: getattr(st, f) for f, _ in _State._fields_}

    def execute_step(self, rows: int, layers, act0, act1, a_dtype: int, workspace=None, stream=None):
        """Run `rows` rows of act0 through `layers` (LinearLayer list) with hq_gemm; returns the output buffer."""
        import torch
        arr = (LinearLayer * max(1, len(layers)))(*layers)
        s = stream if stream is not None else torch.cuda.current_stream()
        ws = ctypes.c_void_p(workspace.data_ptr()) if workspace is not None else None
        ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
        check(lib().hq_batcher_execute(self._h, rows, arr, len(layers), ctypes.c_void_p(act0.data_ptr()),
                                       ctypes.c_void_p(act1.data_ptr()), a_dtype, ws, ws_bytes,
                                       ctypes.c_void_p(s.cuda_stream)))
        return act1 if len(layers) % 2 else act0
