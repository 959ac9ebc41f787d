"""Restatement of hydrogen::SplitFuseBatcher's scheduling (batcher.hpp:98-199, split_fuse.cpp:70-193).

TEST INFRASTRUCTURE ONLY: tests drive nebula_b200's native batcher and this restatement with the same
submissions and compare every step (on CPU), and, where a GPU is visible, the native batcher against the
reference's own compiled scheduler (``CompiledRefSplitFuse``).  Nothing in the product library imports it.
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


class CompiledRefSplitFuse:
    """The reference's own hydrogen::SplitFuseBatcher (split_fuse.cpp, compiled where it lies into
    oracle/_ref/libref_batcher.so by oracle/build.py).  Its constructor allocates device memory, so it
    exists only where a GPU is visible.  Same surface as RefSplitFuse."""

    def __init__(self, max_prefill_chunk_tokens=64, max_decode_streams=16, max_batch_tokens=512):
        import ctypes
        import os
        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libref_batcher.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = ctypes.CDLL(path)
        u32, vp = ctypes.c_uint32, ctypes.c_void_p
        L.refb_create.restype, L.refb_create.argtypes = vp, [u32, u32, u32]
        L.refb_destroy.argtypes = [vp]
        L.refb_submit.restype, L.refb_submit.argtypes = u32, [vp, u32, u32]
        L.refb_assemble.restype = ctypes.c_int
        L.refb_assemble.argtypes = [vp, ctypes.POINTER(u32), ctypes.c_int, ctypes.POINTER(u32)]
        L.refb_complete_last.restype, L.refb_complete_last.argtypes = ctypes.c_int, [vp]
        L.refb_has_work.restype, L.refb_has_work.argtypes = ctypes.c_int, [vp]
        L.refb_active.restype, L.refb_active.argtypes = ctypes.c_uint64, [vp]
        L.refb_state.restype, L.refb_state.argtypes = ctypes.c_int, [vp, u32, ctypes.POINTER(u32)]
        L.refb_last_error.restype = ctypes.c_char_p
        self._L, self._ct = L, ctypes
        self._h = L.refb_create(max_prefill_chunk_tokens, max_decode_streams, max_batch_tokens)
        if not self._h:
            raise RuntimeError(L.refb_last_error().decode())

    def close(self):
        if self._h:
            self._L.refb_destroy(self._h)
            self._h = None

    def submit_request(self, prompt, max_decode):
        return int(self._L.refb_submit(self._h, prompt, max_decode))

    def assemble_step_batch(self):
        """(chunks [(rid, start, n, is_prefill)], n_decode, n_prefill_tokens, total_tokens)"""
        ct = self._ct
        cap = int(self._L.refb_active(self._h)) + 2
        buf = (ct.c_uint32 * (4 * cap))()
        info = (ct.c_uint32 * 3)()
        n = self._L.refb_assemble(self._h, buf, cap, info)
        if n < 0:
            raise RuntimeError("refb_assemble failed")
        chunks = [(buf[4 * i], buf[4 * i + 1], buf[4 * i + 2], bool(buf[4 * i + 3])) for i in range(n)]
        return chunks, info[0], info[1], info[2]

    def update_step_completion(self):
        """Advance past the batch assembled last (the reference keeps it)."""
        if self._L.refb_complete_last(self._h) != 0:
            raise RuntimeError(self._L.refb_last_error().decode())

    def has_active_work(self):
        return bool(self._L.refb_has_work(self._h))

    def request_state(self, rid):
        out = (self._ct.c_uint32 * 5)()
        if self._L.refb_state(self._h, rid, out) != 0:
            return None
        return {"prompt_tokens": out[0], "prefill_completed_tokens": out[1], "decode_tokens_generated": out[2],
                "max_decode_tokens": out[3], "status": out[4]}
