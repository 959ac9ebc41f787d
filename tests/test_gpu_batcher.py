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


def _pin_to_reference(cfg, arrivals, max_steps=20000):
    """Drive the native scheduler and the reference's compiled SplitFuseBatcher with the same submissions;
    every assembled batch and every request's final state must be equal."""
    from nebula_b200.batcher import SplitFuseBatcher
    from oracle.batcher import CompiledRefSplitFuse
    nat, ref = SplitFuseBatcher(*cfg), CompiledRefSplitFuse(*cfg)
    n_sub = 0
    try:
        for step in range(max_steps):
            for prompt, dec in arrivals.get(step, []):
                assert nat.submit_request(prompt, dec) == ref.submit_request(prompt, dec)
                n_sub += 1
            if not nat.has_active_work() and step > max(arrivals, default=0):
                assert not ref.has_active_work()
                break
            assert nat.has_active_work() == ref.has_active_work()
            b = nat.assemble_step_batch()
            rc, n_dec, n_pre, total = ref.assemble_step_batch()
            got = [(c.request_id, c.start_token, c.num_tokens, c.is_prefill) for c in b.chunks]
            assert got == rc, step
            assert (b.num_decode_requests, b.num_prefill_tokens, b.total_batch_tokens) == (n_dec, n_pre, total)
            nat.update_step_completion(b)
            ref.update_step_completion()
        for rid in range(1, n_sub + 1):
            st, r = nat.request_state(rid), ref.request_state(rid)
            keys = ("prompt_tokens", "prefill_completed_tokens", "decode_tokens_generated", "max_decode_tokens",
                    "status")
            assert r is not None and tuple(st[k] for k in keys) == tuple(r[k] for k in keys), rid
    finally:
        nat.close()
        ref.close()


@pytest.mark.parametrize("seed", range(8))
def test_scheduler_pinned_to_reference_split_fuse(seed):
    """split_fuse.cpp:84-193 compiled from the reference tree (oracle/_ref/libref_batcher.so): random
    arrival traces over several configurations, including clamps below the default 64-token chunk."""
    import os
    if not os.path.exists(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle",
                                       "_ref", "libref_batcher.so")):
        pytest.skip("reference scheduler not built (oracle/build.py needs the reference tree)")
    rng = np.random.default_rng(100 + seed)
    cfg = [(64, 16, 512), (64, 16, 80), (32, 8, 40), (1, 4, 3), (64, 4, 70), (128, 16, 512), (16, 2, 17),
           (64, 16, 16)][seed]
    arrivals = {}
    for _ in range(int(rng.integers(5, 40))):
        step = int(rng.integers(0, 200))
        arrivals.setdefault(step, []).append((int(rng.integers(0, 1500)), int(rng.integers(0, 40))))
    _pin_to_reference(cfg, arrivals)


def test_scheduler_pinned_to_reference_1500_token_observation():
    """The reference's own H10 scenario: 8 decode streams, then a 1500-token observation."""
    import os
    if not os.path.exists(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle",
                                       "_ref", "libref_batcher.so")):
        pytest.skip("reference scheduler not built (oracle/build.py needs the reference tree)")
    arrivals = {0: [(1, 10_000)] * 8, 3: [(1500, 5)]}
    _pin_to_reference((64, 16, 512), arrivals, max_steps=200)
