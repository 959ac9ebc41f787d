"""Split-fuse batching: the native scheduler (hq_batcher_*) against the restatement of split_fuse.cpp, step by
step, and the reference's own invariants (batcher.hpp:76-94)."""
import math

import numpy as np
import pytest

from nebula_b200.batcher import SplitFuseBatcher, RUNNING_DECODE, COMPLETED
from oracle.batcher import RefSplitFuse


def run_both(cfg, arrivals, max_steps=20000):
    """arrivals: {step: [(prompt, max_decode), ...]}; returns the list of per-step native batches."""
    nat, ref = SplitFuseBatcher(*cfg), RefSplitFuse(*cfg)
    steps = []
    for step in range(max_steps):
        for prompt, dec in arrivals.get(step, []):
            assert nat.submit_request(prompt, dec) == ref.submit_request(prompt, dec)
        if not nat.has_active_work() and step > max(arrivals, default=0):
            assert not ref.has_active_work()
            break
        b = nat.assemble_step_batch()
        rc, n_dec, n_pre, total = ref.assemble_step_batch()
        got = [(c.request_id, c.start_token, c.num_tokens, c.is_prefill) for c in b.chunks]
        assert got == rc, step
        assert (b.num_decode_requests, b.num_prefill_tokens, b.total_batch_tokens) == (n_dec, n_pre, total)
        nat.update_step_completion(b)
        ref.update_step_completion(rc)
        steps.append(b)
    for rid in range(1, len(ref.requests) + 1):
        st, r = nat.request_state(rid), ref.requests[rid - 1]
        assert (st["prefill_completed_tokens"], st["decode_tokens_generated"], st["status"]) == \
            (r["prefilled"], r["generated"], r["status"])
    nat.close()
    return steps


@pytest.mark.parametrize("seed", range(6))
def test_native_scheduler_matches_restatement(seed):
    rng = np.random.default_rng(seed)
    cfg = [(64, 16, 512), (64, 16, 80), (32, 8, 40), (1, 4, 3)][seed % 4]
    arrivals = {}
    for _ in range(int(rng.integers(5, 40))):
        step = int(rng.integers(0, 200))
        arrivals.setdefault(step, []).append((int(rng.integers(0, 1500)), int(rng.integers(0, 40))))
    run_both(cfg, arrivals)


def test_reference_invariants_1500_token_observation():
    """One 1500-token prefill fused with 8 running decode streams: chunks clamped to 64 tokens, 24 prefill
    iterations (SplitFuseBenchmarkResult, batcher.hpp:88-90), one decode row per stream every step."""
    b = SplitFuseBatcher(64, 16, 512)
    for _ in range(8):
        b.submit_request(1, 10_000)
    while any(b.request_state(i)["status"] != RUNNING_DECODE for i in range(1, 9)):
        b.update_step_completion(b.assemble_step_batch())
    b.submit_request(1500, 5)
    prefill_iters, max_chunk = 0, 0
    while b.request_state(9)["status"] != RUNNING_DECODE:
        fb = b.assemble_step_batch()
        assert fb.num_decode_requests == 8
        assert fb.total_batch_tokens <= 512
        if fb.num_prefill_tokens:
            prefill_iters += 1
            max_chunk = max(max_chunk, fb.num_prefill_tokens)
        b.update_step_completion(fb)
    assert prefill_iters == math.ceil(1500 / 64) and max_chunk == 64
    for _ in range(5):
        b.update_step_completion(b.assemble_step_batch())
    assert b.request_state(9)["status"] == COMPLETED
    b.close()


def test_batch_budget_limits_prefill():
    b = SplitFuseBatcher(64, 16, 20)
    for _ in range(18):
        b.submit_request(1, 100)
    while b.num_active_requests() and any(b.request_state(i)["status"] != RUNNING_DECODE for i in range(1, 19)):
        b.update_step_completion(b.assemble_step_batch())
    b.submit_request(100, 1)
    fb = b.assemble_step_batch()
    assert fb.num_decode_requests == 18 and fb.num_prefill_tokens == 2 and fb.total_batch_tokens == 20
    b.close()


def test_failed_calls_change_nothing():
    """A too-small chunk buffer (assemble) or an unknown request id (complete) fails without changing state."""
    import ctypes
    from nebula_b200 import _lib
    from nebula_b200.batcher import _Chunk, _Info, QUEUED
    L = _lib.lib()
    b = SplitFuseBatcher(64, 16, 512)
    b.submit_request(100, 2)
    buf = (_Chunk * 1)()
    assert L.hq_batcher_assemble(b._h, buf, 0, ctypes.byref(_Info())) == -1
    assert b.request_state(1)["status"] == QUEUED
    fb = b.assemble_step_batch()
    bad = (_Chunk * 2)(_Chunk(fb.chunks[0].request_id, 0, fb.chunks[0].num_tokens, 1), _Chunk(99, 0, 1, 0))
    assert L.hq_batcher_complete(b._h, bad, 2) == _lib.HQ_ERR_INVALID_ARG
    assert b.request_state(1)["prefill_completed_tokens"] == 0
    b.update_step_completion(fb)
    assert b.request_state(1)["prefill_completed_tokens"] == 64
    b.close()
