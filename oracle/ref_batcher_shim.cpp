// ref_batcher_shim.cpp -- C entry points into the reference's own SplitFuseBatcher.
//
// TEST INFRASTRUCTURE ONLY.  Linked with the reference's unmodified
// hydrogen/src/batcher/split_fuse.cpp (compiled where it lies) into
// oracle/_ref/libref_batcher.so, so that a test can drive the reference
// scheduler and this library's hq_batcher_* with the same requests and compare
// every assembled batch and every request state.  The reference constructor
// allocates its workspace with cudaMalloc (split_fuse.cpp:41-54), so the
// scheduler can only be constructed where a GPU is visible.  Exceptions
// become return code -1 / a null handle.
#include "batcher.hpp"

#include <cstdint>
#include <cstring>
#include <exception>

namespace {

struct Handle {
    hydrogen::SplitFuseBatcher* b = nullptr;
    hydrogen::FusedBatch last;  // the batch that refb_complete_last hands back
};

char g_err[512];
void set_err(const char* s) {
    std::strncpy(g_err, s, sizeof g_err - 1);
    g_err[sizeof g_err - 1] = 0;
}

}  // namespace

extern "C" {

const char* refb_last_error() { return g_err; }

void* refb_create(uint32_t max_prefill_chunk_tokens, uint32_t max_decode_streams, uint32_t max_batch_tokens) {
    try {
        hydrogen::SplitFuseConfig c;
        c.max_prefill_chunk_tokens = max_prefill_chunk_tokens;
        c.max_decode_streams = max_decode_streams;
        c.max_batch_tokens = max_batch_tokens;
        auto* h = new Handle;
        h->b = new hydrogen::SplitFuseBatcher(c);
        return h;
    } catch (const std::exception& e) {
        set_err(e.what());
        return nullptr;
    }
}

void refb_destroy(void* p) {
    auto* h = static_cast<Handle*>(p);
    if (!h) return;
    delete h->b;
    delete h;
}

uint32_t refb_submit(void* p, uint32_t prompt_tokens, uint32_t max_decode_tokens) {
    return static_cast<Handle*>(p)->b->submit_request(prompt_tokens, max_decode_tokens);
}

// Assemble the next step: chunks as (request_id, start_token, num_tokens, is_prefill) quadruples in
// `out` (room for `cap`), counts in info[0..2] = (num_decode_requests, num_prefill_tokens,
// total_batch_tokens).  Returns the number of chunks, or -1 when `cap` is too small.
int refb_assemble(void* p, uint32_t* out, int cap, uint32_t* info) {
    auto* h = static_cast<Handle*>(p);
    try {
        h->last = h->b->assemble_step_batch();
    } catch (const std::exception& e) {
        set_err(e.what());
        return -1;
    }
    const int n = (int)h->last.chunks.size();
    if (n > cap) return -1;
    for (int i = 0; i < n; ++i) {
        const auto& c = h->last.chunks[i];
        out[4 * i + 0] = c.request_id;
        out[4 * i + 1] = c.start_token;
        out[4 * i + 2] = c.num_tokens;
        out[4 * i + 3] = c.is_prefill ? 1u : 0u;
    }
    info[0] = h->last.num_decode_requests;
    info[1] = h->last.num_prefill_tokens;
    info[2] = h->last.total_batch_tokens;
    return n;
}

int refb_complete_last(void* p) {
    auto* h = static_cast<Handle*>(p);
    try {
        h->b->update_step_completion(h->last);
        return 0;
    } catch (const std::exception& e) {
        set_err(e.what());
        return -1;
    }
}

int refb_has_work(void* p) { return static_cast<Handle*>(p)->b->has_active_work() ? 1 : 0; }

uint64_t refb_active(void* p) { return static_cast<Handle*>(p)->b->num_active_requests(); }

// Request state: out[0..4] = (prompt_tokens, prefill_completed_tokens, decode_tokens_generated,
// max_decode_tokens, status).  Returns -1 for an unknown id.
int refb_state(void* p, uint32_t request_id, uint32_t* out) {
    const hydrogen::SequenceRequest* r = static_cast<Handle*>(p)->b->get_request(request_id);
    if (!r) return -1;
    out[0] = r->prompt_tokens;
    out[1] = r->prefill_completed_tokens;
    out[2] = r->decode_tokens_generated;
    out[3] = r->max_decode_tokens;
    out[4] = (uint32_t)r->status;
    return 0;
}

void refb_reset(void* p) { static_cast<Handle*>(p)->b->reset(); }

}  // extern "C"
