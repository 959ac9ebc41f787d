"""hq_gemm_noalloc: the GEMM for callers that cannot allocate device memory.

A host that embeds this library as a plugin in a serving process whose device
memory is pre-budgeted by that process cannot hand hq_gemm a workspace; this
entry point uses a fixed array compiled into the library instead.  These tests
call it through the C ABI with reference-layout weights (the case that needs
scratch: the weights are re-tiled into it) and compare its output with
hq_gemm's, which gets an ordinary caller workspace, on two calls in a row: the
second call finds the first call's data in the shared array and must not
depend on it.  Tolerance as for every parity test here: max relative error
1e-2 (fp16) / 2e-2 (bf16).

The file name sorts last so that a run stopping at the first failure has run
every other test already; it also passes run alone in a fresh process (the
first call then does the per-device set-up).
"""
import ctypes

import numpy as np
import pytest
import torch

from nebula_b200 import _lib, hq
from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL = {"f16": 1e-2, "bf16": 2e-2}
TDT = {"f16": torch.float16, "bf16": torch.bfloat16}
_DT = {"f16": _lib.HQ_F16, "bf16": _lib.HQ_BF16}


def _dev(x, dtype=None):
    x = np.ascontiguousarray(x)
    if dtype is None:
        return torch.from_numpy(x.view(np.uint8).reshape(-1)).to("cuda:0")
    return torch.from_numpy(x.astype(np.float32)).to("cuda:0").to(TDT[dtype])


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def _noalloc(A, W, wfmt, S, C, dt, M, N, K, g):
    L = _lib.lib()
    st = L.hq_gemm_noalloc(_vp(A), _DT[dt], _vp(W), wfmt, _vp(S), _DT[dt], None, _vp(C), _DT[dt], M, N, K, g,
                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(st)


CASES = [
    # (M, K, N, group, dtype, weight format)
    (4, 1024, 512, 128, "f16", _lib.HQ_WFMT_LINEAR_U4),
    (16, 2048, 272, 128, "bf16", _lib.HQ_WFMT_MARLIN_QUAD),
]


def test_noalloc_matches_hq_gemm_on_two_calls_in_a_row():
    torch.cuda.set_device(0)
    for i, (M, K, N, g, dt, wfmt) in enumerate(CASES):
        A, q, S = o.gen_int4_case(M, K, N, group=g, seed=500 + i, a_dtype=dt)
        lin = o.pack_linear_u4(q)
        packed = lin if wfmt == _lib.HQ_WFMT_LINEAR_U4 else o.repack_marlin_quad(lin, K, N)
        At, St, Wt = _dev(A, dt), _dev(S, dt), _dev(packed)
        y_ref = hq.gemm(At, Wt, St, N=N, group=g, wfmt=wfmt)  # existing entry point, caller workspace
        y = torch.full((M, N), float("nan"), dtype=TDT[dt], device="cuda:0")
        _noalloc(At, Wt, wfmt, St, y, dt, M, N, K, g)
        torch.cuda.synchronize()
        hq.check_device_error()
        a, b = y.float().cpu().numpy(), y_ref.float().cpu().numpy()
        assert np.isfinite(a).all()
        assert o.max_rel_err(a, b) <= TOL[dt], f"call {i}: differs from hq_gemm"
        # and both against the fp32 oracle
        assert o.max_rel_err(a, o.w4_gemm(A, lin, S, group=g)) <= TOL[dt]


def test_noalloc_rejects_problems_beyond_its_scratch():
    """Re-tiling LINEAR_U4 weights of K=16384, N=16384 needs 128 MiB > the 64 MiB array."""
    torch.cuda.set_device(0)
    L = _lib.lib()
    K = N = 16384
    assert L.hq_gemm_workspace_size(1, N, K, 128, _lib.HQ_WFMT_LINEAR_U4) > _lib.HQ_NOALLOC_SCRATCH_BYTES
    buf = torch.zeros(64, dtype=torch.uint8, device="cuda:0")  # never read: the size check comes first
    st = L.hq_gemm_noalloc(_vp(buf), _lib.HQ_F16, _vp(buf), _lib.HQ_WFMT_LINEAR_U4, _vp(buf), _lib.HQ_F16, None,
                           _vp(buf), _lib.HQ_F16, 1, N, K, 128,
                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.HQ_ERR_WORKSPACE_TOO_SMALL
    msg = L.hq_last_error_string().decode()
    assert "scratch" in msg and str(_lib.HQ_NOALLOC_SCRATCH_BYTES) in msg


_FIRST_CALL_ON_SIDE_STREAM = r"""
import ctypes, sys
import numpy as np, torch
sys.path.insert(0, sys.argv[1])
from nebula_b200 import _lib, hq
from oracle import oracle as o
M, K, N, g = 8, 1024, 512, 128
A, q, S = o.gen_int4_case(M, K, N, group=g, seed=77, a_dtype="f16")
lin = o.pack_linear_u4(q)
dev = lambda x: torch.from_numpy(np.ascontiguousarray(x).view(np.uint8).reshape(-1)).to("cuda:0")
At = torch.from_numpy(A).to("cuda:0").half(); St = torch.from_numpy(S).to("cuda:0").half(); Wt = dev(lin)
side = torch.cuda.Stream()  # non-blocking: not ordered with the legacy default stream
y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda:0")
with torch.cuda.stream(side):
    vp = lambda t: ctypes.c_void_p(t.data_ptr())
    _lib.check(_lib.lib().hq_gemm_noalloc(vp(At), _lib.HQ_F16, vp(Wt), _lib.HQ_WFMT_LINEAR_U4, vp(St), _lib.HQ_F16,
                                          None, vp(y), _lib.HQ_F16, M, N, K, g, ctypes.c_void_p(side.cuda_stream)))
side.synchronize()
err = o.max_rel_err(y.float().cpu().numpy(), o.w4_gemm(A, lin, S, group=g))
print("max_rel_err", err)
sys.exit(0 if np.isfinite(err) and err <= 1e-2 else 1)
"""


def test_noalloc_first_call_on_a_side_stream_in_a_fresh_process():
    """The first call of a process does the set-up (address lookup and zero fill).  Made on a
    non-blocking stream, the GEMM it launches must still see the array fully zero-filled and
    the re-tiled weights intact."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _FIRST_CALL_ON_SIDE_STREAM, root], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
