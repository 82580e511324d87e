// ref_amp_sched_shim.cpp -- TEST INFRASTRUCTURE ONLY (a driver of AMP's own host code).
//
// AMP's continuous-batching Scheduler (src/scheduler.cpp) and PagePoolFast
// (src/pool_fast.cpp), compiled in place from the reference tree for AMP's CPU
// backend (AMP_MALLOC = malloc: the page buffers are host memory and are never
// touched; only the page ids matter), behind a C ABI so that the tests can run
// real schedule() batches through amp_b200's paged kernels.
//
// refsched_step runs one schedule(), exports every entry with the pages its
// sequence holds after scheduling, then calls step_complete() with one dummy
// token per decode entry.  Exported per entry: seq id, is_prefill, n_tokens,
// prefill_start, ctx (tokens whose K/V exist once this step has run:
// prefill_start + n_tokens for a prefill chunk, total_tokens() + 1 for a decode).
#include <cstdint>
#include <vector>

#include "scheduler.hpp"

#define REF_EXPORT extern "C" __attribute__((visibility("default")))

REF_EXPORT void* refsched_create(int page_tokens, int max_pages_total, int max_batch_tokens,
                                 int max_seqs_running, int max_prefill_tokens_per_step) {
    AMP::SchedulerConfig cfg;
    cfg.kv_page_size_tokens = page_tokens;
    cfg.max_pages_total = max_pages_total;
    cfg.page_bytes = 64;   // host buffers only; the kernels use their own pools
    cfg.max_batch_tokens = max_batch_tokens;
    cfg.max_seqs_running = max_seqs_running;
    cfg.max_prefill_tokens_per_step = max_prefill_tokens_per_step;
    return new AMP::Scheduler(cfg);
}

REF_EXPORT void refsched_destroy(void* s) { delete static_cast<AMP::Scheduler*>(s); }

REF_EXPORT int refsched_add(void* s, int prompt_len, int max_new_tokens) {
    std::vector<int> prompt(prompt_len, 7);
    return static_cast<AMP::Scheduler*>(s)->add_request(std::move(prompt), max_new_tokens);
}

// entries: [cap][5]; pages: flat page ids, page_start: [cap + 1] offsets into it.
REF_EXPORT int refsched_step(void* sp, int32_t* entries, int32_t* pages, int32_t* page_start,
                             int cap, int pages_cap) {
    auto* s = static_cast<AMP::Scheduler*>(sp);
    AMP::ScheduledBatch batch = s->schedule();
    const int n = (int)batch.entries.size();
    if (n > cap) return -1;
    int np = 0;
    page_start[0] = 0;
    std::vector<int> new_tokens;
    for (int i = 0; i < n; ++i) {
        const AMP::BatchEntry& e = batch.entries[i];
        const AMP::Sequence* q = e.seq;
        int32_t* row = entries + 5 * i;
        row[0] = q->id;
        row[1] = e.is_prefill ? 1 : 0;
        row[2] = e.n_tokens;
        row[3] = e.prefill_start;
        row[4] = e.is_prefill ? e.prefill_start + e.n_tokens : q->total_tokens() + 1;
        if (np + (int)q->kv_page_ids.size() > pages_cap) return -2;
        for (int p : q->kv_page_ids) pages[np++] = p;
        page_start[i + 1] = np;
        if (!e.is_prefill) new_tokens.push_back(1);
    }
    s->step_complete(batch, new_tokens);
    return n;
}
