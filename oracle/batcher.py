"""Restatement of hydrogen::SplitFuseBatcher's scheduling (batcher.hpp:98-199, split_fuse.cpp:70-193).

TEST INFRASTRUCTURE ONLY: tests drive nebula_b200's native batcher and this restatement with the same
submissions and compare every step.  Nothing in the product library imports it.
"""
from __future__ import annotations

QUEUED, RUNNING_PREFILL, RUNNING_DECODE, COMPLETED = range(4)  # RequestStatus, batcher.hpp:17-22


class RefSplitFuse:
    def __init__(self, max_prefill_chunk_tokens=64, max_decode_streams=16, max_batch_tokens=512):
        self.max_prefill = max_prefill_chunk_tokens
        self.max_batch = max_batch_tokens
        self.requests = []        # dicts, id r at index r - 1
        self.prefill_queue = []   # split_fuse.cpp:78 (deque)
        self.decode = []          # active_decode_streams_

    def submit_request(self, prompt_tokens, max_decode_tokens):  # split_fuse.cpp:76-90
        rid = len(self.requests) + 1
        self.requests.append({"prompt": prompt_tokens, "prefilled": 0, "generated": 0,
                              "max_decode": max_decode_tokens, "status": QUEUED})
        self.prefill_queue.append(rid)
        return rid

    def assemble_step_batch(self):  # split_fuse.cpp:92-152
        chunks, total, n_decode, n_prefill = [], 0, 0, 0
        for rid in self.decode:
            r = self.requests[rid - 1]
            if r["status"] == RUNNING_DECODE:
                chunks.append((rid, r["prompt"] + r["generated"], 1, False))
                n_decode += 1
                total += 1
        if self.prefill_queue:
            left = self.max_batch - total if self.max_batch > total else 0
            budget = min(self.max_prefill, left)
            if budget > 0:
                rid = self.prefill_queue[0]
                r = self.requests[rid - 1]
                r["status"] = RUNNING_PREFILL
                take = min(r["prompt"] - r["prefilled"], budget)
                take = min(take, self.max_prefill)
                chunks.append((rid, r["prefilled"], take, True))
                n_prefill = take
                total += take
        return chunks, n_decode, n_prefill, total

    def update_step_completion(self, chunks):  # split_fuse.cpp:154-193
        for rid, _start, n, is_prefill in chunks:
            r = self.requests[rid - 1]
            if is_prefill:
                r["prefilled"] += n
                if r["prefilled"] >= r["prompt"]:
                    r["status"] = RUNNING_DECODE
                    if self.prefill_queue and self.prefill_queue[0] == rid:
                        self.prefill_queue.pop(0)
                    self.decode.append(rid)
            else:
                r["generated"] += n
                if r["generated"] >= r["max_decode"]:
                    r["status"] = COMPLETED
        self.decode = [rid for rid in self.decode if self.requests[rid - 1]["status"] != COMPLETED]

    def has_active_work(self):
        return bool(self.prefill_queue or self.decode)
