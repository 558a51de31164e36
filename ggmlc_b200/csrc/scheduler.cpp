#include "scheduler.h"

#include <algorithm>
#include <cmath>

#include "common.h"
#include "kernels.h"

namespace gb {

Scheduler::Scheduler(Executor& ex, int max_batch, int eos, int64_t max_ctx)
    : ex_(ex), max_batch_(max_batch), eos_(eos) {
    GB_CHECK(max_batch >= 1 && max_batch <= kMaxRows, "scheduler: max_batch_size must be 1..16");
    const Graph& g = ex.graph();
    bool have_in = false;
    for (uint32_t id : g.inputs)
        if (g.t(id).type == T_I32) {
            in_id_ = id;
            have_in = true;
            break;
        }
    GB_CHECK(have_in, "scheduler: the graph has no int32 token-id input");
    GB_CHECK(!g.outputs.empty(), "scheduler: the graph has no output");
    out_id_ = g.outputs[0];
    ex.init_paged_kv_cache(max_batch, max_ctx);
    gen_ = ex.kv_pool_generation();
    ex.set_logits_last_only(true);
    slots_.assign((size_t)max_batch, nullptr);
}

Scheduler::~Scheduler() {
    // after another init_paged_kv_cache the slots and pages belong to the new pool's users
    const bool same_pool = gen_ == ex_.kv_pool_generation();
    for (size_t i = 0; i < slots_.size(); ++i)
        if (slots_[i] && same_pool) {
            try {
                ex_.paged_kv_free_slot((int64_t)i);
            } catch (...) {
            }
        }
    try {  // the prefix cache's page references
        if (tree_ && tree_gen_ == ex_.kv_pool_generation())
            for (int64_t pg; (pg = tree_->evict_lru()) >= 0;) ex_.kv_page_release(pg);
    } catch (...) {
    }
}

uint64_t Scheduler::add_request(const std::vector<int32_t>& prompt, int max_new, float temperature,
                                int eos) {
    GB_CHECK(!prompt.empty(), "scheduler: empty prompt");
    GB_CHECK(max_new >= 1, "scheduler: max_new_tokens must be at least 1");
    GB_CHECK((int64_t)prompt.size() + max_new <= ex_.kv_max_ctx(),
             "scheduler: prompt + max_new_tokens exceed the KV cache length");
    GB_CHECK(pages_for((int64_t)prompt.size() + max_new) <= ex_.kv_pool_pages(),
             "scheduler: prompt + max_new_tokens need more pages than the KV pool holds");
    auto r = std::make_shared<GenRequest>();
    r->id = next_id_++;
    r->prompt = prompt;
    r->max_new = max_new;
    r->temperature = temperature;
    r->eos = eos >= 0 ? eos : eos_;
    pending_.push_back(r);
    all_[r->id] = r;
    return r->id;
}

bool Scheduler::has_work() const { return !pending_.empty() || active_count() > 0; }

size_t Scheduler::active_count() const {
    size_t n = 0;
    for (auto& s : slots_) n += s ? 1 : 0;
    return n;
}

std::shared_ptr<GenRequest> Scheduler::get(uint64_t id) const {
    auto it = all_.find(id);
    return it == all_.end() ? nullptr : it->second;
}

// greedy: the first maximum; otherwise a draw from softmax(logits / temperature)
// (batch_scheduler.cpp:94-128)
int32_t Scheduler::sample(const float* logits, int64_t vocab, float temperature) {
    int64_t best = 0;
    for (int64_t i = 1; i < vocab; ++i)
        if (logits[i] > logits[best]) best = i;
    if (temperature <= 0.0f) return (int32_t)best;
    std::vector<float> p((size_t)vocab);
    float total = 0.0f;
    for (int64_t i = 0; i < vocab; ++i) {
        p[(size_t)i] = std::exp((logits[i] - logits[best]) / temperature);
        total += p[(size_t)i];
    }
    std::uniform_real_distribution<float> u(0.0f, total);
    float r = u(rng_), run = 0.0f;
    for (int64_t i = 0; i < vocab; ++i) {
        run += p[(size_t)i];
        if (run >= r) return (int32_t)i;
    }
    return (int32_t)(vocab - 1);
}

void Scheduler::finish(const std::shared_ptr<GenRequest>& r, int32_t tok, StepOut& out) {
    const bool stop = r->eos >= 0 && tok == r->eos;
    const bool length = (int)r->generated.size() >= r->max_new || r->pos >= ex_.kv_max_ctx();
    if (!stop && !length) return;
    r->finished = true;
    r->finish_reason = stop ? "stop" : "length";
    out.completed.push_back(r->id);
    ex_.paged_kv_free_slot(r->slot);
    slots_[(size_t)r->slot] = nullptr;
}

int64_t Scheduler::pages_for(int64_t tokens) const {
    const int64_t T = ex_.tokens_per_page();
    return (tokens + T - 1) / T;
}

int64_t Scheduler::outstanding_pages() const {
    int64_t n = 0;
    for (auto& r : slots_)
        if (r)
            n += std::max<int64_t>(0, pages_for((int64_t)r->prompt.size() + r->max_new) -
                                          ex_.paged_kv_slot_pages(r->slot));
    return n;
}

bool Scheduler::make_room(int64_t need) {
    const int64_t owed = outstanding_pages();
    while (ex_.kv_free_pages() - owed < need) {
        const int64_t pg = tree_ ? tree_->evict_lru() : -1;  // least recently used prefix page
        if (pg < 0) return false;
        ex_.kv_page_release(pg);
    }
    return true;
}

void Scheduler::ensure_tree() {
    const int64_t T = ex_.tokens_per_page();
    if (tree_ && tree_->tokens_per_page() == T && tree_gen_ == ex_.kv_pool_generation()) return;
    // a new pool layout: the old tree's page ids (and their references) went with the old pool
    tree_ = std::make_unique<PrefixTree>(T);
    tree_gen_ = ex_.kv_pool_generation();
}

StepOut Scheduler::step() {
    StepOut out;
    // admission (batch_scheduler.cpp:136-277): every pending request that finds a free slot is
    // prefilled alone into it, reusing the KV rows of the longest cached run of whole prompt
    // pages; a step that admits returns without decoding
    bool admitted = false;
    if (gen_ != ex_.kv_pool_generation()) {  // the pool was laid out again
        GB_CHECK(active_count() == 0, "scheduler: the KV pool was re-initialised under running "
                                      "requests");
        gen_ = ex_.kv_pool_generation();
    }
    if (tree_ && tree_gen_ != gen_) tree_.reset();
    while (!pending_.empty()) {
        int slot = -1;
        for (size_t i = 0; i < slots_.size(); ++i)
            if (!slots_[i]) {
                slot = (int)i;
                break;
            }
        if (slot < 0) break;
        auto r = pending_.front();
        const int64_t n = (int64_t)r->prompt.size();
        PrefixMatch m;
        if (prefix_caching_) {
            ensure_tree();
            m = tree_->match(r->prompt);
        }
        // the cached pages become the head of the slot's page table (a reference each)
        ex_.paged_kv_alloc_slot(slot);
        for (int64_t p = 0; p < m.matched_pages; ++p) ex_.kv_map_page(slot, m.pages[(size_t)p]);
        // a prompt cached whole re-evaluates its last token, which writes into its last page:
        // that page is copied first
        const bool whole = m.matched_pages > 0 && m.matched_tokens == n;
        const int64_t need = pages_for(n + r->max_new) - m.matched_pages + (whole ? 1 : 0);
        if (!make_room(need)) {
            ex_.paged_kv_free_slot(slot);
            GB_CHECK(active_count() > 0, "scheduler: the KV pool cannot hold request " +
                                             std::to_string(r->id) + " (" + std::to_string(need) +
                                             " pages) even with nothing else running");
            break;  // it waits for running sequences to return their pages
        }
        pending_.pop_front();
        r->slot = slot;
        slots_[(size_t)slot] = r;
        if (whole) ex_.kv_make_private(slot, m.matched_pages - 1);
        ex_.paged_kv_ensure_tokens(slot, n);
        const int64_t matched = m.matched_tokens;
        if (matched > 0) {
            ++prefix_hits_;
            prefix_saved_ += matched;
        }
        r->prefix_matched = matched;
        // the uncached tail; a prompt cached whole re-evaluates its last token
        const int64_t pos = matched < n ? matched : n - 1;
        const int64_t s = n - pos;
        SymEnv env;
        env["s"] = s;
        for (auto& sym : ex_.graph().symbol_table) env[sym] = s;
        env["pos"] = pos;
        env["slot"] = slot;
        ex_.prepare(env, true);
        ex_.set_input(in_id_, r->prompt.data() + pos, (size_t)s * 4);
        ex_.run();
        if (prefix_caching_) {  // the prompt's new whole pages join the tree (a reference each)
            const int64_t T = tree_->tokens_per_page();
            const int64_t first = m.matched_pages, full = n / T;
            if (full > first)
                tree_->insert(r->prompt, first, full - first, [&](int64_t i) {
                    const int64_t page = ex_.kv_slot_page(slot, first + i);
                    ex_.kv_page_retain(page);
                    return page;
                });
        }
        int32_t tok = 0;
        if (r->temperature <= 0.0f) {
            ex_.output_argmax(out_id_, 1, &tok);  // last row only
        } else {
            size_t bytes = 0;
            const float* logits = (const float*)ex_.get_output(out_id_, &bytes);
            tok = sample(logits, (int64_t)(bytes / 4), r->temperature);
        }
        r->generated.push_back(tok);
        r->pos = n;
        out.new_tokens.push_back({r->id, tok});
        finish(r, tok, out);
        admitted = true;
    }
    if (admitted) return out;
    // one batched decode step over every active sequence, rows padded to a bucket
    std::vector<std::shared_ptr<GenRequest>> act;
    for (auto& s : slots_)
        if (s) act.push_back(s);
    if (act.empty()) return out;
    int rows = 1;
    while (rows < (int)act.size()) rows *= 2;
    std::vector<int32_t> pos((size_t)rows, 0), slot((size_t)rows, max_batch_), tok((size_t)rows, 0);
    for (size_t i = 0; i < act.size(); ++i) {
        pos[i] = (int32_t)act[i]->pos;
        slot[i] = act[i]->slot;
        tok[i] = act[i]->generated.back();
    }
    GB_CHECK(make_room(0), "scheduler: the KV pool is overcommitted");
    for (auto& r : act) ex_.paged_kv_ensure_tokens(r->slot, r->pos + 1);  // the new position's page
    ex_.prepare_batch(rows, pos.data(), slot.data());
    ex_.set_input(in_id_, tok.data(), tok.size() * 4);
    ex_.run();
    // greedy rows take the device argmax; logits cross to the host only for sampled rows
    bool any_sampled = false;
    for (auto& r : act) any_sampled |= r->temperature > 0.0f;
    std::vector<int32_t> greedy((size_t)rows);
    ex_.output_argmax(out_id_, rows, greedy.data());
    const float* logits = nullptr;
    int64_t vocab = 0;
    if (any_sampled) {
        size_t bytes = 0;
        logits = (const float*)ex_.get_output(out_id_, &bytes);
        vocab = (int64_t)(bytes / 4 / (size_t)rows);
    }
    for (size_t i = 0; i < act.size(); ++i) {
        auto& r = act[i];
        const int32_t t = r->temperature > 0.0f
                              ? sample(logits + (int64_t)i * vocab, vocab, r->temperature)
                              : greedy[i];
        r->generated.push_back(t);
        r->pos += 1;
        out.new_tokens.push_back({r->id, t});
        finish(r, t, out);
    }
    return out;
}

}  // namespace gb
