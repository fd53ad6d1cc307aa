// Continuous-batching scheduler on a decoder context: SchedCore's policy bound to the
// C ABI of the decoder (sequences, fa_forward_rows), exported as fa_sched_*.
#include "nvtx_range.hpp"
#include "funasr_dec.h"
#include "sched_core.hpp"

#include <algorithm>
#include <new>
#include <string>
#include <vector>

namespace fa {
int report_op_error(int code, const char* msg);                      // fa_api.cu
int report_ctx_error(const fa_ctx* ctx, int code, const char* msg);  // fa_api.cu
}  // namespace fa

namespace {

struct DeviceBackend {
    fa_ctx* ctx;
    fa_model_desc d{};
    long pages = 0;

    int open(int max_tokens, int* seq) { return fa_seq_open(ctx, max_tokens, seq); }
    int close(int seq) { return fa_seq_close(ctx, seq); }
    int forward(int n, const int* seqs, const int* toks, const float* embeds, int n_out, const int* out_rows,
                int* next) {
        return fa_forward_rows(ctx, n, seqs, toks, embeds, n_out, out_rows, next, nullptr);
    }
    long total_pages() const { return pages; }
    int max_rows() const { return d.max_rows; }
    int max_seqs() const { return d.max_seqs; }
    int hidden() const { return d.hidden; }
};

}  // namespace

struct fa_sched {
    DeviceBackend be;
    fa::SchedCore<DeviceBackend>* core = nullptr;
    std::vector<fa::SchedEvent> events;
    ~fa_sched() { delete core; }
};

extern "C" fa_sched* fa_sched_create(fa_ctx* ctx, const fa_sched_config* cfg) {
    if (!ctx || !cfg) {
        fa::report_op_error(FA_ERR_INVALID_ARG, "fa_sched_create: NULL argument");
        return nullptr;
    }
    fa_sched* s = new (std::nothrow) fa_sched;
    if (!s) {
        fa::report_op_error(FA_ERR_OOM, "fa_sched_create: out of host memory");
        return nullptr;
    }
    s->be.ctx = ctx;
    int n_pages = 0, n_free = 0;
    size_t pb = 0;
    if (fa_pool_info(ctx, &n_pages, &n_free, &pb) != FA_OK || fa_ctx_desc(ctx, &s->be.d) != FA_OK) {
        delete s;
        return nullptr;
    }
    // the pages already held by open sequences stay theirs
    s->be.pages = n_free;
    fa::SchedConfig c;
    c.max_batch_rows = cfg->max_batch_rows;
    c.prefill_chunk = cfg->prefill_chunk;
    c.max_running = cfg->max_running;
    c.eos_id = cfg->eos_id;
    s->core = new (std::nothrow) fa::SchedCore<DeviceBackend>(s->be, c);
    if (!s->core) {
        delete s;
        fa::report_op_error(FA_ERR_OOM, "fa_sched_create: out of host memory");
        return nullptr;
    }
    return s;
}

extern "C" void fa_sched_destroy(fa_sched* s) { delete s; }

extern "C" int fa_sched_submit(fa_sched* s, int64_t tag, const int* prompt_ids, const float* prompt_embeds,
                               int n_prompt, int max_new) {
    if (!s) return fa::report_op_error(FA_ERR_INVALID_ARG, "fa_sched_submit: NULL scheduler");
    if (s->core->submit(tag, prompt_ids, prompt_embeds, n_prompt, max_new) != 0)
        return fa::report_ctx_error(s->be.ctx, FA_ERR_CAPACITY,
                                    "fa_sched_submit: give n_prompt > 0, max_new > 0, ids or embeddings, and a "
                                    "stream that fits the page pool");
    return FA_OK;
}

extern "C" int fa_sched_step(fa_sched* s, fa_sched_event* events, int max_events, int* n_events) {
    fa::NvtxRange nv("fa_sched_step");
    if (!s || (max_events > 0 && !events) || !n_events)
        return fa::report_op_error(FA_ERR_INVALID_ARG, "fa_sched_step: bad argument");
    // events not yet handed out come first; a step runs only when none are left
    int rc = FA_OK;
    if (s->events.empty()) rc = s->core->step(s->events);
    if (rc != FA_OK && s->events.empty()) return rc;
    const int n = std::min<int>(max_events, (int)s->events.size());
    for (int i = 0; i < n; ++i) {
        events[i].tag = s->events[(size_t)i].tag;
        events[i].token = s->events[(size_t)i].token;
        events[i].finished = s->events[(size_t)i].finished;
    }
    s->events.erase(s->events.begin(), s->events.begin() + n);
    *n_events = n;
    return FA_OK;
}

extern "C" int fa_sched_idle(const fa_sched* s) { return s && s->core->idle() && s->events.empty() ? 1 : 0; }

extern "C" int fa_sched_get_stats(const fa_sched* s, fa_sched_stats* out) {
    if (!s || !out) return fa::report_op_error(FA_ERR_INVALID_ARG, "fa_sched_get_stats: bad argument");
    const fa::SchedStats st = s->core->stats();
    out->steps = st.steps;
    out->rows = st.rows;
    out->prompt_rows = st.prompt_rows;
    out->tokens = st.tokens;
    out->finished = st.finished;
    out->waiting = st.waiting;
    out->running = st.running;
    out->reserved_pages = st.reserved_pages;
    out->total_pages = st.total_pages;
    return FA_OK;
}
