"""ctypes binding of libhq.so (the C ABI declared in include/hq.h).

The product path is this shared library and nothing else: if it is missing or
cannot be loaded, every call raises -- there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libhq.so")

# enums (include/hq.h)
HQ_OK, HQ_ERR_INVALID_ARG, HQ_ERR_UNSUPPORTED_SHAPE, HQ_ERR_WORKSPACE_TOO_SMALL, HQ_ERR_CUDA, \
    HQ_ERR_TIMEOUT, HQ_ERR_MISALIGNED, HQ_ERR_UNSUPPORTED_DEVICE = range(8)
HQ_F32, HQ_F16, HQ_BF16 = 0, 1, 2
(HQ_WFMT_LINEAR_U4, HQ_WFMT_MARLIN_QUAD, HQ_WFMT_TILE_U4, HQ_WFMT_LINEAR_T2, HQ_WFMT_TILE_T2, HQ_WFMT_TQ1_0,
 HQ_WFMT_TILE_U4_K32) = range(7)
HQ_NOALLOC_SCRATCH_BYTES = 64 << 20  # scratch array of hq_gemm_noalloc
HQ_GGML_F32, HQ_GGML_Q8_0, HQ_GGML_BF16, HQ_GGML_TQ1_0, HQ_GGML_TQ1_0_ALT = 0, 8, 30, 34, 143

STATUS_NAMES = {0: "HQ_OK", 1: "HQ_ERR_INVALID_ARG", 2: "HQ_ERR_UNSUPPORTED_SHAPE", 3: "HQ_ERR_WORKSPACE_TOO_SMALL",
                4: "HQ_ERR_CUDA", 5: "HQ_ERR_TIMEOUT", 6: "HQ_ERR_MISALIGNED", 7: "HQ_ERR_UNSUPPORTED_DEVICE"}

# Every symbol include/hq.h declares, with (restype, argtypes).
_vp, _i, _u32, _sz, _d = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_size_t, ctypes.c_double
SIGNATURES = {
    "hq_version": (ctypes.c_char_p, []),
    "hq_last_error_string": (ctypes.c_char_p, []),
    "hq_weight_bytes": (_sz, [_i, _i, _i]),
    "hq_gemm_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "hq_workspace_init": (_i, [_vp, _sz, _vp]),
    "hq_gemm": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    "hq_gemm_noalloc": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "hq_repack_host": (_i, [_vp, _i, _vp, _i, _i, _i, _i]),
    "hq_repack_device": (_i, [_vp, _i, _vp, _i, _i, _i, _vp]),
    "hq_tq1_0_gemv": (_i, [_vp, _vp, _vp, _i, _i, _vp]),
    "hq_tq1_0_to_tile_t2": (_i, [_vp, _vp, _vp, _i, _i, _vp]),
    "hq_q4_k_to_tile": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp]),
    "hq_q4_k_to_tile_host": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i]),
    "hq_w8_gemm": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "hq_output_projection": (_i, [_vp, _vp, _i, _vp, _i, _i, _vp]),
    "hq_embedding_lookup": (_i, [_vp, _i, _i, _vp, _i, _i, _vp]),
    "hq_check_device_error": (_i, []),
    "hq_set_launch_overlap": (None, [_i]),
    "hq_allreduce_sum": (_i, [_vp, _vp, _vp, _i, _i, _i, _sz, _u32, _i, _vp]),
    "hq_batcher_create": (_vp, [_vp]),
    "hq_batcher_destroy": (None, [_vp]),
    "hq_batcher_reset": (None, [_vp]),
    "hq_batcher_submit": (_u32, [_vp, _u32, _u32]),
    "hq_batcher_assemble": (_i, [_vp, _vp, _i, _vp]),
    "hq_batcher_complete": (_i, [_vp, _vp, _i]),
    "hq_batcher_has_work": (_i, [_vp]),
    "hq_batcher_active_requests": (_sz, [_vp]),
    "hq_batcher_request_state": (_i, [_vp, _u32, _vp]),
    "hq_batcher_execute": (_i, [_vp, _u32, _vp, _i, _vp, _vp, _i, _vp, _sz, _vp]),
    "hq_marlin_engine_create": (_vp, [_u32, _u32, _u32, _u32]),
    "hq_marlin_engine_destroy": (None, [_vp]),
    "hq_marlin_repack_q4k_to_marlin": (_i, [_vp, _vp, _vp, _u32, _u32, ctypes.POINTER(_d)]),
    "hq_marlin_forward_marlin_int4": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _u32]),
    "hq_marlin_forward_baseline_int4": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _u32]),
    "hq_marlin_forward_reference": (_i, [_vp, _vp, _vp, _vp, _u32]),
    "hq_marlin_forward_cutlass_int8": (_i, [_vp, _vp, _vp, _vp, _vp, _u32]),
    "hq_marlin_verify_fidelity": (_i, [_vp, _vp, _vp, _u32, ctypes.POINTER(_d), ctypes.POINTER(_d)]),
}

_lib = None


class HQError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load libhq.so (building it first when the sources are present and it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        from .build import build
        build()
    L = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def check(status: int) -> None:
    if status != HQ_OK:
        raise HQError(status, lib().hq_last_error_string().decode(errors="replace"))
