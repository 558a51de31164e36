// Continuous batching over the executor's paged KV slots: the engine-side counterpart of the
// reference's ContinuousBatchScheduler (runtime/include/ggmlc/batch_scheduler.h:35-77,
// runtime/src/batch_scheduler.cpp:130-403), with the same request / step / result interface.
//
// Differences by design: every sequence decodes at its own position in its own slot (one
// batched step over all active sequences, rows padded to a bucket of 1/2/4/8/16 with a scratch
// slot), where the reference runs one shared position over all slots; the graph needs no batch
// dimension (rows of the sequence axis are the batch).  Prefix caching (on by default, as in the
// reference) indexes whole prompt pages in a PrefixTree whose page ids are pages of the
// executor's paged KV pool, each held by a reference of the tree: a hit maps the cached pages
// into the new slot's page table (no copy) and prefills only the rest of the prompt; a prefill
// hands its new whole pages to the tree.  A prompt cached whole re-evaluates its last token,
// so its last page is copied first (copy-on-write).
//
// Admission follows the pool: a request is admitted when the pages it can still claim
// (prompt + max_new_tokens, less the pages it shares) fit next to what the running sequences
// may still claim, after evicting least-recently-used prefix pages; otherwise it waits.  Pages
// are assigned as sequences grow (the prompt at admission, one page per tokens_per_page decode
// steps after), so the pool's mapped bytes follow the tokens in use.
#pragma once

#include <cstdint>
#include <deque>
#include <map>
#include <memory>
#include <random>
#include <string>
#include <utility>
#include <vector>

#include "executor.h"
#include "radix.h"

namespace gb {

struct GenRequest {
    uint64_t id = 0;
    std::vector<int32_t> prompt;
    std::vector<int32_t> generated;
    int slot = -1;
    int64_t pos = 0;       // position of the next token to decode
    int max_new = 32;
    float temperature = 0.0f;
    int eos = -1;
    bool finished = false;
    std::string finish_reason;  // "stop" (end token) or "length" (max_new reached)
    int64_t prefix_matched = 0;  // prompt tokens whose KV rows came from the prefix cache
};

struct StepOut {
    std::vector<std::pair<uint64_t, int32_t>> new_tokens;  // (request id, token)
    std::vector<uint64_t> completed;
};

class Scheduler {
public:
    // Initialises the executor's paged KV cache for max_batch sequences of up to max_ctx
    // positions (the reference uses 2048) and switches logits to the last row.
    Scheduler(Executor& ex, int max_batch, int eos, int64_t max_ctx = 2048);
    ~Scheduler();

    uint64_t add_request(const std::vector<int32_t>& prompt, int max_new, float temperature,
                         int eos);
    // One iteration: admit every pending request that finds a free slot (prefill, first token)
    // and return, or run one batched decode step over every active sequence.
    StepOut step();
    bool has_work() const;
    size_t active_count() const;
    size_t pending_count() const { return pending_.size(); }
    int max_batch() const { return max_batch_; }
    std::shared_ptr<GenRequest> get(uint64_t id) const;
    void enable_prefix_caching(bool on) { prefix_caching_ = on; }
    bool prefix_caching() const { return prefix_caching_; }
    int64_t prefix_cache_hits() const { return prefix_hits_; }
    int64_t prefix_tokens_saved() const { return prefix_saved_; }

private:
    int32_t sample(const float* logits, int64_t vocab, float temperature);
    void ensure_tree();
    int64_t pages_for(int64_t tokens) const;
    int64_t outstanding_pages() const;  // pages running sequences may still claim
    bool make_room(int64_t need);       // evict prefix pages until `need` pages are claimable
    void finish(const std::shared_ptr<GenRequest>& r, int32_t tok, StepOut& out);

    Executor& ex_;
    int max_batch_;
    int eos_;
    bool prefix_caching_ = true;
    uint64_t next_id_ = 1;
    uint32_t in_id_ = 0, out_id_ = 0;
    std::deque<std::shared_ptr<GenRequest>> pending_;
    std::vector<std::shared_ptr<GenRequest>> slots_;
    std::map<uint64_t, std::shared_ptr<GenRequest>> all_;
    std::mt19937 rng_{1337};
    std::unique_ptr<PrefixTree> tree_;
    int64_t tree_gen_ = -1;  // pool layout the tree's page ids belong to
    int64_t gen_ = -1;       // pool layout made by the constructor
    int64_t prefix_hits_ = 0, prefix_saved_ = 0;
};

}  // namespace gb
