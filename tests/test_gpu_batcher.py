"""The split-fuse batcher's step executor: each assembled step's rows (mixed decode + prefill M) run through a
two-layer int4 stack with real hq_gemm kernels; every step against direct hq_gemm calls (bit-identical) and the
first against the oracle."""
import ctypes

import numpy as np
import pytest
import torch

from nebula_b200 import _lib, hq
from nebula_b200.batcher import LinearLayer, SplitFuseBatcher
from oracle import oracle as o

pytestmark = pytest.mark.gpu


def test_batcher_drives_real_gemm_steps():
    K0, N0, N1, g = 512, 1024, 512, 128
    _, q0, S0 = o.gen_int4_case(1, K0, N0, g, seed=1)
    _, q1, S1 = o.gen_int4_case(1, N0, N1, g, seed=2)
    W0 = torch.from_numpy(o.pack_tile(q0, 4)).cuda()
    W1 = torch.from_numpy(o.pack_tile(q1, 4)).cuda()
    S0d = torch.from_numpy(S0).cuda().half()
    S1d = torch.from_numpy(S1).cuda().half()
    P = lambda t: t.data_ptr()
    layers = [LinearLayer(P(W0), _lib.HQ_WFMT_TILE_U4, P(S0d), _lib.HQ_F16, None, K0, N0, g),
              LinearLayer(P(W1), _lib.HQ_WFMT_TILE_U4, P(S1d), _lib.HQ_F16, None, N0, N1, g)]
    max_rows = 512
    width = max(K0, N0, N1)
    act0 = torch.zeros(max_rows * width, dtype=torch.float16, device="cuda")
    act1 = torch.zeros_like(act0)
    L = _lib.lib()
    ws_bytes = max(int(L.hq_gemm_workspace_size(max_rows, N0, K0, g, _lib.HQ_WFMT_TILE_U4)),
                   int(L.hq_gemm_workspace_size(max_rows, N1, N0, g, _lib.HQ_WFMT_TILE_U4)), 16)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")

    b = SplitFuseBatcher(64, 16, max_rows)
    for prompt, dec in ((100, 4), (300, 6), (5, 9), (0, 2), (70, 3)):
        b.submit_request(prompt, dec)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    steps, rows_seen = 0, set()
    while b.has_active_work():
        fb = b.assemble_step_batch()
        rows = fb.total_batch_tokens
        rows_seen.add(rows)
        if rows:
            X = torch.randn((rows, K0), device="cuda", generator=gen).half()
            act0[: rows * K0] = X.reshape(-1)
            out = b.execute_step(rows, layers, act0, act1, _lib.HQ_F16, workspace=ws)
            Y = out[: rows * N1].view(rows, N1)
            direct = hq.gemm(hq.gemm(X, W0, S0d, N=N0, group=g), W1, S1d, N=N1, group=g)
            torch.cuda.synchronize()
            assert torch.equal(Y, direct), steps
            if steps == 0:
                h = o.round_to(o.w4_gemm(X.float().cpu().numpy(), o.pack_linear_u4(q0), S0, group=g), "f16")
                ref = o.w4_gemm(h, o.pack_linear_u4(q1), S1, group=g)
                assert o.max_rel_err(Y.float().cpu().numpy(), ref) <= 2e-2
        b.update_step_completion(fb)
        steps += 1
        assert steps < 200
    assert len(rows_seen) > 3  # the steps ran at several different M
    b.close()
