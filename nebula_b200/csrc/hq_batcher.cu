// hq_batcher.cu -- split-fuse continuous batching that drives the quantized
// linear stack with the mixed M it decides.
//
// Scheduling restates hydrogen::SplitFuseBatcher (batcher.hpp:98-199,
// split_fuse.cpp:70-193): requests queue for prefill; every step takes one row
// per active decode stream (in the order the streams became active), then up
// to min(max_prefill_chunk_tokens, max_batch_tokens - decode rows) prompt
// tokens of the request at the head of the prefill queue; a request whose
// prompt is complete joins the decode streams, and one that generated
// max_decode_tokens leaves them.  As in the reference, max_decode_streams is a
// sizing hint and not enforced.
//
// The reference's execute_step (split_fuse.cpp:196-238) simulates the forward
// step with a formula and a device copy; hq_batcher_execute runs the step's
// rows through a chain of real hq_gemm layers (M = rows of the fused batch)
// on the caller's stream.
#include "hq.h"
#include "hq_internal.h"

#include <algorithm>
#include <chrono>
#include <deque>
#include <new>
#include <vector>

namespace {

struct Request {
    uint32_t id = 0, prompt = 0, prefilled = 0, generated = 0, max_decode = 0;
    int status = HQ_REQ_QUEUED;
};

}  // namespace

struct hq_batcher {
    hq_batcher_config cfg{};
    std::vector<Request> requests;       // request id r at index r - 1
    std::deque<uint32_t> prefill_queue;  // ids waiting for or in prefill
    std::vector<uint32_t> decode;        // ids of active decode streams
    std::vector<double> assembly_us;
};

extern "C" {

HQ_API hq_batcher* hq_batcher_create(const hq_batcher_config* cfg) {
    hq_batcher* b = new (std::nothrow) hq_batcher();
    if (!b) return nullptr;
    if (cfg) b->cfg = *cfg;
    else b->cfg = hq_batcher_config{64, 16, 512};
    b->decode.reserve(b->cfg.max_decode_streams + 2);
    return b;
}

HQ_API void hq_batcher_destroy(hq_batcher* b) { delete b; }

HQ_API void hq_batcher_reset(hq_batcher* b) {
    if (!b) return;
    b->requests.clear();
    b->prefill_queue.clear();
    b->decode.clear();
    b->assembly_us.clear();
}

HQ_API uint32_t hq_batcher_submit(hq_batcher* b, uint32_t prompt_tokens, uint32_t max_decode_tokens) {
    if (!b) return 0;
    Request r;
    r.id = (uint32_t)b->requests.size() + 1;
    r.prompt = prompt_tokens;
    r.max_decode = max_decode_tokens;
    b->requests.push_back(r);
    b->prefill_queue.push_back(r.id);
    return r.id;
}

HQ_API int hq_batcher_assemble(hq_batcher* b, hq_batch_chunk* chunks, int max_chunks, hq_batch_info* info) {
    if (!b || !chunks || max_chunks < 0) return -1;
    const auto t0 = std::chrono::steady_clock::now();
    int n = 0;
    uint32_t total = 0, n_decode = 0, n_prefill = 0;
    for (uint32_t id : b->decode) {  // one row per active decode stream
        const Request& r = b->requests[id - 1];
        if (r.status != HQ_REQ_RUNNING_DECODE) continue;
        if (n == max_chunks) return -1;
        chunks[n++] = hq_batch_chunk{id, r.prompt + r.generated, 1u, 0};
        ++n_decode;
        ++total;
    }
    if (!b->prefill_queue.empty()) {
        const uint32_t budget_left = b->cfg.max_batch_tokens > total ? b->cfg.max_batch_tokens - total : 0;
        const uint32_t budget = std::min(b->cfg.max_prefill_chunk_tokens, budget_left);
        if (budget > 0) {
            if (n == max_chunks) return -1;  // before any state changes: a failed call leaves none
            Request& r = b->requests[b->prefill_queue.front() - 1];
            r.status = HQ_REQ_RUNNING_PREFILL;
            uint32_t take = std::min(r.prompt - r.prefilled, budget);
            take = std::min(take, b->cfg.max_prefill_chunk_tokens);
            chunks[n++] = hq_batch_chunk{r.id, r.prefilled, take, 1};
            n_prefill = take;
            total += take;
        }
    }
    const double us = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
    b->assembly_us.push_back(us);
    if (info) *info = hq_batch_info{n_decode, n_prefill, total, us};
    return n;
}

HQ_API hq_status hq_batcher_complete(hq_batcher* b, const hq_batch_chunk* chunks, int n) {
    if (!b || (n > 0 && !chunks) || n < 0) return HQ_ERR_INVALID_ARG;
    for (int i = 0; i < n; ++i)  // validate the whole step first: an invalid one changes nothing
        if (chunks[i].request_id == 0 || chunks[i].request_id > b->requests.size()) return HQ_ERR_INVALID_ARG;
    for (int i = 0; i < n; ++i) {
        const hq_batch_chunk& c = chunks[i];
        Request& r = b->requests[c.request_id - 1];
        if (c.is_prefill) {
            r.prefilled += c.num_tokens;
            if (r.prefilled >= r.prompt) {
                r.status = HQ_REQ_RUNNING_DECODE;
                if (!b->prefill_queue.empty() && b->prefill_queue.front() == c.request_id) b->prefill_queue.pop_front();
                b->decode.push_back(c.request_id);
            }
        } else {
            r.generated += c.num_tokens;
            if (r.generated >= r.max_decode) r.status = HQ_REQ_COMPLETED;
        }
    }
    b->decode.erase(std::remove_if(b->decode.begin(), b->decode.end(),
                                   [b](uint32_t id) { return b->requests[id - 1].status == HQ_REQ_COMPLETED; }),
                    b->decode.end());
    return HQ_OK;
}

HQ_API int hq_batcher_has_work(const hq_batcher* b) {
    return b && (!b->prefill_queue.empty() || !b->decode.empty()) ? 1 : 0;
}

HQ_API size_t hq_batcher_active_requests(const hq_batcher* b) {
    return b ? b->prefill_queue.size() + b->decode.size() : 0;
}

HQ_API hq_status hq_batcher_request_state(const hq_batcher* b, uint32_t request_id, hq_request_state* out) {
    if (!b || !out || request_id == 0 || request_id > b->requests.size()) return HQ_ERR_INVALID_ARG;
    const Request& r = b->requests[request_id - 1];
    *out = hq_request_state{r.prompt, r.prefilled, r.generated, r.max_decode, r.status};
    return HQ_OK;
}

HQ_API hq_status hq_batcher_execute(hq_batcher* b, uint32_t rows, const hq_linear_layer* layers, int n_layers,
                                    void* act0, void* act1, hq_dtype a_dtype, void* workspace, size_t ws_bytes,
                                    hq_stream_t stream) {
    if (!b || (n_layers > 0 && (!layers || !act0 || !act1)) || n_layers < 0) return HQ_ERR_INVALID_ARG;
    for (int i = 0; i + 1 < n_layers; ++i)
        if (layers[i + 1].K != layers[i].N) return HQ_ERR_UNSUPPORTED_SHAPE;  // the layers must chain
    if (rows == 0) return HQ_OK;
    for (int i = 0; i < n_layers; ++i) {
        const hq_linear_layer& L = layers[i];
        void* in = (i & 1) ? act1 : act0;
        void* out = (i & 1) ? act0 : act1;
        const hq_status st = hq_gemm(in, a_dtype, L.W, L.wfmt, L.scales, L.s_dtype, L.bias, out, a_dtype, (int)rows,
                                     L.N, L.K, L.group, workspace, ws_bytes, stream);
        if (st != HQ_OK) return st;
    }
    return HQ_OK;
}

}  // extern "C"
