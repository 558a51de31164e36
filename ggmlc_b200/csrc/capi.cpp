// extern "C" boundary of libggmlc_b200.so (declarations in include/ggmlc_b200.h).  Every entry
// point catches C++ exceptions and turns them into -1 + gb_last_error(), the C counterpart of
// the std::runtime_error -> Python exception path of the reference bindings.
#include "../../include/ggmlc_b200.h"

#include <cmath>
#include <cstring>
#include <memory>
#include <string>

#include "executor.h"
#include "tp.h"
#include "graph.h"
#include "radix.h"
#include "scheduler.h"
#include "kernels.h"
#include "kutil.cuh"

struct gb_graph {
    std::shared_ptr<gb::Graph> g;
    std::vector<uint32_t> tensor_ids;
};

struct gb_executor {
    std::unique_ptr<gb::Executor> e;
    std::string summary, mm_summary, ktimes;
};

struct gb_radix {
    std::unique_ptr<gb::PrefixTree> t;
    int64_t next_page = 0;  // page ids handed out by gb_radix_insert_prefix
};
struct gb_scheduler {
    std::unique_ptr<gb::Scheduler> s;
};

namespace {
thread_local std::string g_err;

template <class F>
int guard(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& ex) {
        g_err = ex.what();
    } catch (...) {
        g_err = "unknown error";
    }
    return -1;
}

gb_graph* wrap(std::shared_ptr<gb::Graph> g) {
    auto* h = new gb_graph();
    h->g = std::move(g);
    for (auto& [id, t] : h->g->tensors) h->tensor_ids.push_back(id);
    return h;
}

const std::vector<uint32_t>& ids_of(const gb_graph* g, int which) {
    switch (which) {
        case 0: return g->g->inputs;
        case 1: return g->g->outputs;
        default: return g->g->parameters;
    }
}
}  // namespace

extern "C" {

const char* gb_last_error(void) { return g_err.c_str(); }
int gb_version(void) { return 100; }

int gb_get_available_devices(char* buf, size_t cap) {
    std::string s;
    int rc = guard([&] {
        for (auto& d : gb::Executor::available_devices()) s += (s.empty() ? "" : "\n") + d;
    });
    if (rc) return -1;
    if (buf && cap) {
        std::strncpy(buf, s.c_str(), cap - 1);
        buf[cap - 1] = 0;
    }
    return (int)s.size() + 1;
}

int gb_loader_load_from_file(const char* path, gb_graph** out) {
    return guard([&] { *out = wrap(gb::load_gguf_file(path)); });
}
int gb_loader_load_from_bytes(const void* data, size_t size, gb_graph** out) {
    return guard([&] { *out = wrap(gb::load_gguf_bytes((const uint8_t*)data, size)); });
}
void gb_graph_free(gb_graph* g) { delete g; }

const char* gb_graph_name(const gb_graph* g) { return g->g->name.c_str(); }
int gb_graph_num_symbols(const gb_graph* g) { return (int)g->g->symbol_table.size(); }
const char* gb_graph_symbol(const gb_graph* g, int i) {
    if (i < 0 || i >= (int)g->g->symbol_table.size()) return nullptr;
    return g->g->symbol_table[(size_t)i].c_str();
}
int gb_graph_num_ids(const gb_graph* g, int which) { return (int)ids_of(g, which).size(); }
int gb_graph_id(const gb_graph* g, int which, int i, uint32_t* id) {
    const auto& v = ids_of(g, which);
    if (i < 0 || i >= (int)v.size()) {
        g_err = "index out of range";
        return -1;
    }
    *id = v[(size_t)i];
    return 0;
}
int gb_graph_num_tensors(const gb_graph* g) { return (int)g->tensor_ids.size(); }
int gb_graph_tensor_id(const gb_graph* g, int i, uint32_t* id) {
    if (i < 0 || i >= (int)g->tensor_ids.size()) {
        g_err = "index out of range";
        return -1;
    }
    *id = g->tensor_ids[(size_t)i];
    return 0;
}
int gb_graph_tensor_info(const gb_graph* g, uint32_t id, const char** name, int* type,
                         int* storage, uint64_t* data_size) {
    return guard([&] {
        const gb::GTensor& t = g->g->t(id);
        if (name) *name = t.name.c_str();
        if (type) *type = t.type;
        if (storage) *storage = t.storage;
        if (data_size) *data_size = t.data_size;
    });
}
int gb_graph_tensor_symbol_index(const gb_graph* g, uint32_t id, int axis) {
    auto it = g->g->tensors.find(id);
    if (it == g->g->tensors.end() || axis < 0 || axis > 3 || !it->second.ne[axis]) return -1;
    return it->second.ne[axis]->symbol_index(g->g->symbol_table);
}
int gb_graph_num_ops(const gb_graph* g) { return (int)g->g->ops.size(); }
int gb_graph_op_info(const gb_graph* g, int i, uint32_t* id, int* opcode, const char** name) {
    if (i < 0 || i >= (int)g->g->ops.size()) {
        g_err = "index out of range";
        return -1;
    }
    const auto& op = g->g->ops[(size_t)i];
    if (id) *id = op.id;
    if (opcode) *opcode = op.opcode;
    if (name) *name = op.name.c_str();
    return 0;
}
const char* gb_graph_metadata_str(const gb_graph* g, const char* key) {
    auto it = g->g->meta_str.find(key);
    return it == g->g->meta_str.end() ? nullptr : it->second.c_str();
}

int gb_executor_create(const gb_graph* g, const char* device, gb_executor** out) {
    return guard([&] {
        auto* h = new gb_executor();
        try {
            h->e.reset(new gb::Executor(g->g, device ? device : "cuda"));
        } catch (...) {
            delete h;
            throw;
        }
        *out = h;
    });
}
int gb_nccl_unique_id(void* out128) {
    return guard([&] { gb::Executor::nccl_unique_id(out128); });
}
int gb_executor_create_tp(const gb_graph* g, const char* device, int tp_rank, int tp_size,
                          const void* nccl_id, gb_executor** out) {
    return guard([&] {
        auto* h = new gb_executor();
        try {
            h->e.reset(new gb::Executor(g->g, device ? device : "cuda", tp_rank, tp_size, nccl_id));
        } catch (...) {
            delete h;
            throw;
        }
        *out = h;
    });
}
const char* gb_tp_plan(const gb_graph* g, int tp_rank, int tp_size) {
    static thread_local std::string buf;
    buf.clear();
    const int rc = guard([&] {
        gb::Graph copy = *g->g;
        const gb::TpPlan p = gb::plan_tensor_parallel(copy, tp_rank, tp_size);
        buf = gb::tp_plan_json(p, copy);
    });
    return rc == 0 ? buf.c_str() : nullptr;
}
int gb_executor_tp_size(const gb_executor* e) { return e->e->tp_size(); }
int gb_executor_tp_error(gb_executor* e) {
    int v = 0;
    const int rc = guard([&] { v = e->e->tp_allreduce_error(); });
    return rc == 0 ? v : -1;
}
int gb_executor_tp_rank(const gb_executor* e) { return e->e->tp_rank(); }
void gb_executor_free(gb_executor* e) { delete e; }
const char* gb_executor_device(const gb_executor* e) { return e->e->device().c_str(); }

int gb_executor_prepare(gb_executor* e, const char* const* names, const int64_t* values, int n,
                        int enable_arena_reuse) {
    return guard([&] {
        gb::SymEnv env;
        for (int i = 0; i < n; ++i) env[names[i]] = values[i];
        e->e->prepare(env, enable_arena_reuse != 0);
    });
}
int gb_executor_set_input(gb_executor* e, uint32_t tid, const void* data, size_t bytes) {
    return guard([&] { e->e->set_input(tid, data, bytes); });
}
int gb_executor_set_input_by_name(gb_executor* e, const char* name, const void* data,
                                  size_t bytes) {
    return guard([&] { e->e->set_input_by_name(name, data, bytes); });
}
int gb_executor_run(gb_executor* e, int) {
    return guard([&] { e->e->run(); });
}
int gb_executor_synchronize(gb_executor* e) {
    return guard([&] { e->e->synchronize(); });
}
int gb_executor_get_output(gb_executor* e, uint32_t tid, const void** data, size_t* bytes) {
    return guard([&] { *data = e->e->get_output(tid, bytes); });
}
int gb_executor_output_argmax(gb_executor* e, uint32_t tid, int rows, int32_t* out) {
    return guard([&] { e->e->output_argmax(tid, rows, out); });
}
int gb_executor_get_tensor_shape(gb_executor* e, uint32_t tid, int64_t ne[4]) {
    return guard([&] {
        auto s = e->e->tensor_shape(tid);
        for (int d = 0; d < 4; ++d) ne[d] = s[(size_t)d];
    });
}
int gb_executor_get_tensor_size_bytes(gb_executor* e, uint32_t tid, size_t* bytes) {
    return guard([&] { *bytes = e->e->tensor_size_bytes(tid); });
}
int gb_executor_set_state(gb_executor* e, uint32_t tid, const void* data, size_t bytes) {
    return guard([&] { e->e->set_state(tid, data, bytes); });
}
int gb_executor_get_state(gb_executor* e, uint32_t tid, const void** data, size_t* bytes) {
    return guard([&] { *data = e->e->get_state(tid, bytes); });
}
int gb_executor_reset_state(gb_executor* e) {
    return guard([&] { e->e->reset_state(); });
}
int gb_executor_init_kv_cache(gb_executor* e, int64_t max_ctx) {
    return guard([&] { e->e->init_kv_cache(max_ctx); });
}
int gb_executor_reset_kv_cache(gb_executor* e) {
    return guard([&] { e->e->reset_kv_cache(); });
}
int gb_executor_has_kv_cache(const gb_executor* e) { return e->e->has_kv_cache() ? 1 : 0; }
int gb_executor_init_paged_kv_cache(gb_executor* e, int64_t max_batch, int64_t max_ctx) {
    return guard([&] { e->e->init_paged_kv_cache(max_batch, max_ctx); });
}
int gb_executor_is_paged_kv_cache_enabled(const gb_executor* e) {
    return e->e->paged_kv_enabled() ? 1 : 0;
}
int gb_executor_paged_kv_alloc_slot(gb_executor* e, int64_t slot) {
    return guard([&] { e->e->paged_kv_alloc_slot(slot); });
}
int gb_executor_paged_kv_free_slot(gb_executor* e, int64_t slot) {
    return guard([&] { e->e->paged_kv_free_slot(slot); });
}
int gb_executor_paged_kv_ensure_tokens(gb_executor* e, int64_t slot, int64_t total_tokens) {
    return guard([&] { e->e->paged_kv_ensure_tokens(slot, total_tokens); });
}
int64_t gb_executor_paged_active_vram_bytes(const gb_executor* e) {
    return e->e->paged_active_vram_bytes();
}
int64_t gb_executor_tokens_per_page(const gb_executor* e) { return e->e->tokens_per_page(); }
int gb_executor_set_tokens_per_page(gb_executor* e, int64_t n) {
    return guard([&] { e->e->set_tokens_per_page(n); });
}
int gb_executor_prepare_batch(gb_executor* e, int rows, const int32_t* pos, const int32_t* slot) {
    return guard([&] { e->e->prepare_batch(rows, pos, slot); });
}

int gb_scheduler_create(gb_executor* e, int max_batch_size, int eos_token_id, gb_scheduler** out) {
    return guard([&] {
        auto* h = new gb_scheduler();
        try {
            h->s.reset(new gb::Scheduler(*e->e, max_batch_size, eos_token_id));
        } catch (...) {
            delete h;
            throw;
        }
        *out = h;
    });
}
void gb_scheduler_free(gb_scheduler* s) { delete s; }
int gb_scheduler_add_request(gb_scheduler* s, const int32_t* prompt, int64_t n, int max_new_tokens,
                             float temperature, int eos_token_id, uint64_t* request_id) {
    return guard([&] {
        GB_CHECK(n > 0 && prompt, "add_request: empty prompt");
        *request_id = s->s->add_request(std::vector<int32_t>(prompt, prompt + n), max_new_tokens,
                                        temperature, eos_token_id);
    });
}
int gb_scheduler_step(gb_scheduler* s, uint64_t* ids, int32_t* tokens, int cap, int* n_new,
                      uint64_t* done, int cap_done, int* n_done) {
    return guard([&] {
        const gb::StepOut r = s->s->step();
        GB_CHECK((int)r.new_tokens.size() <= cap && (int)r.completed.size() <= cap_done,
                 "scheduler step: result buffers too small");
        for (size_t i = 0; i < r.new_tokens.size(); ++i) {
            ids[i] = r.new_tokens[i].first;
            tokens[i] = r.new_tokens[i].second;
        }
        for (size_t i = 0; i < r.completed.size(); ++i) done[i] = r.completed[i];
        *n_new = (int)r.new_tokens.size();
        *n_done = (int)r.completed.size();
    });
}
int gb_scheduler_has_work(const gb_scheduler* s) { return s->s->has_work() ? 1 : 0; }
int64_t gb_scheduler_active_count(const gb_scheduler* s) { return (int64_t)s->s->active_count(); }
int64_t gb_scheduler_pending_count(const gb_scheduler* s) { return (int64_t)s->s->pending_count(); }
int gb_scheduler_max_batch_size(const gb_scheduler* s) { return s->s->max_batch(); }
int gb_scheduler_enable_prefix_caching(gb_scheduler* s, int enable) {
    s->s->enable_prefix_caching(enable != 0);
    return 0;
}
int gb_scheduler_is_prefix_caching_enabled(const gb_scheduler* s) {
    return s->s->prefix_caching() ? 1 : 0;
}
int gb_scheduler_prefix_stats(const gb_scheduler* s, int64_t* hits, int64_t* tokens_saved) {
    return guard([&] {
        if (hits) *hits = s->s->prefix_cache_hits();
        if (tokens_saved) *tokens_saved = s->s->prefix_tokens_saved();
    });
}
int gb_executor_configure_prefix_pool(gb_executor* e, int64_t pages) {
    return guard([&] { e->e->configure_prefix_pool(pages); });
}
int gb_executor_configure_kv_pool_pages(gb_executor* e, int64_t pages) {
    return guard([&] { e->e->configure_kv_pool_pages(pages); });
}
int64_t gb_executor_kv_pool_pages(const gb_executor* e) { return e->e->kv_pool_pages(); }
int64_t gb_executor_kv_free_pages(const gb_executor* e) { return e->e->kv_free_pages(); }

int gb_radix_create(int64_t tokens_per_page, gb_radix** out) {
    return guard([&] {
        auto* h = new gb_radix();
        try {
            h->t.reset(new gb::PrefixTree(tokens_per_page));
        } catch (...) {
            delete h;
            throw;
        }
        *out = h;
    });
}
void gb_radix_free(gb_radix* r) { delete r; }
int64_t gb_radix_tokens_per_page(const gb_radix* r) { return r->t->tokens_per_page(); }
int64_t gb_radix_total_cached_pages(const gb_radix* r) { return r->t->total_pages(); }
int64_t gb_radix_total_nodes(const gb_radix* r) { return r->t->total_nodes(); }
void gb_radix_reset(gb_radix* r) {
    r->t->reset();
    r->next_page = 0;
}
int gb_radix_match_prefix(gb_radix* r, const int32_t* tokens, int64_t n, int64_t* matched_pages,
                          int64_t* matched_tokens) {
    return guard([&] {
        GB_CHECK(n >= 0 && (n == 0 || tokens), "radix: bad token array");
        const gb::PrefixMatch m = r->t->match(std::vector<int32_t>(tokens, tokens + n));
        *matched_pages = m.matched_pages;
        *matched_tokens = m.matched_tokens;
    });
}
int gb_radix_insert_prefix(gb_radix* r, const int32_t* tokens, int64_t n, int64_t* added) {
    return guard([&] {
        GB_CHECK(n >= 0 && (n == 0 || tokens), "radix: bad token array");
        const std::vector<int32_t> v(tokens, tokens + n);
        const int64_t T = r->t->tokens_per_page();
        const gb::PrefixMatch m = r->t->match(v);
        *added = r->t->insert(v, m.matched_pages, n / T - m.matched_pages,
                              [&](int64_t) { return r->next_page++; });
    });
}
int64_t gb_radix_evict_lru(gb_radix* r) { return r->t->evict_lru(); }
int gb_scheduler_get_request(gb_scheduler* s, uint64_t request_id, gb_request_info* info) {
    return guard([&] {
        auto r = s->s->get(request_id);
        GB_CHECK(r != nullptr, "unknown request id " + std::to_string(request_id));
        info->request_id = r->id;
        info->slot_id = r->slot;
        info->current_pos = r->pos;
        info->max_new_tokens = r->max_new;
        info->temperature = r->temperature;
        info->eos_token_id = r->eos;
        info->finished = r->finished ? 1 : 0;
        info->finish_reason = r->finish_reason.c_str();
        info->n_prompt_tokens = (int64_t)r->prompt.size();
        info->n_generated_tokens = (int64_t)r->generated.size();
        info->prefix_tokens_matched = r->prefix_matched;
    });
}
int gb_scheduler_request_tokens(gb_scheduler* s, uint64_t request_id, int which, int32_t* buf,
                                int64_t cap, int64_t* n) {
    return guard([&] {
        auto r = s->s->get(request_id);
        GB_CHECK(r != nullptr, "unknown request id " + std::to_string(request_id));
        const std::vector<int32_t>& v = which == 0 ? r->prompt : r->generated;
        *n = (int64_t)v.size();
        const int64_t k = std::min<int64_t>(cap, (int64_t)v.size());
        if (k > 0 && buf) std::memcpy(buf, v.data(), (size_t)k * 4);
    });
}
int gb_executor_set_output_rows(gb_executor* e, const int32_t* rows, int n) {
    return guard([&] {
        GB_CHECK(n >= 0 && (n == 0 || rows), "set_output_rows: bad row array");
        e->e->set_output_rows(std::vector<int32_t>(rows, rows + n));
    });
}
int gb_executor_set_logits_last_only(gb_executor* e, int enable) {
    return guard([&] { e->e->set_logits_last_only(enable != 0); });
}
int gb_executor_logits_last_only(const gb_executor* e) { return e->e->logits_last_only() ? 1 : 0; }
int gb_executor_set_enable_cuda_graph(gb_executor* e, int enable) {
    return guard([&] { e->e->set_enable_cuda_graph(enable != 0); });
}
int gb_executor_is_cuda_graph_enabled(const gb_executor* e) {
    return e->e->cuda_graph_enabled() ? 1 : 0;
}
int gb_executor_set_decode_chain(gb_executor* e, int enable) {
    return guard([&] { e->e->set_decode_chain(enable != 0); });
}
int gb_executor_decode_chain(const gb_executor* e) { return e->e->decode_chain() ? 1 : 0; }
int gb_executor_is_cuda_graph_captured(const gb_executor* e) {
    return e->e->cuda_graph_captured() ? 1 : 0;
}
int gb_executor_set_enable_profile(gb_executor* e, int enable) {
    return guard([&] { e->e->set_enable_profile(enable != 0); });
}
int gb_executor_reset_profile(gb_executor* e) {
    return guard([&] { e->e->reset_profile(); });
}
int gb_executor_get_profile(gb_executor* e, double* prepare_ms, double* run_ms, int* n_prepare,
                            int* n_run) {
    return guard([&] {
        auto p = e->e->profile();
        if (prepare_ms) *prepare_ms = p.prepare_ms;
        if (run_ms) *run_ms = p.run_ms;
        if (n_prepare) *n_prepare = p.n_prepare;
        if (n_run) *n_run = p.n_run;
    });
}
const char* gb_executor_graph_summary(gb_executor* e) {
    e->summary = e->e->graph_summary();
    return e->summary.c_str();
}
const char* gb_executor_mul_mat_shape_summary(gb_executor* e) {
    e->mm_summary = e->e->mul_mat_shape_summary();
    return e->mm_summary.c_str();
}
int64_t gb_executor_launches_per_run(const gb_executor* e) { return e->e->launches_per_run(); }
int gb_executor_set_kernel_timing(gb_executor* e, int enable) {
    return guard([&] { e->e->set_kernel_timing(enable != 0); });
}
int gb_executor_reset_kernel_times(gb_executor* e) {
    return guard([&] { e->e->reset_kernel_times(); });
}
const char* gb_executor_kernel_times(gb_executor* e) {
    e->ktimes = e->e->kernel_times_json();
    return e->ktimes.c_str();
}
void* gb_executor_stream(const gb_executor* e) { return (void*)e->e->stream(); }

// ---- op level ----------------------------------------------------------------------------------

int64_t gb_weight_row_bytes(int type, int64_t K) {
    if ((type != gb::T_Q8_0 && type != gb::T_Q4_0) || K < 0 || K % 32) {
        g_err = "gb_weight_row_bytes: Q8_0 or Q4_0 with K a multiple of 32 required";
        return -1;
    }
    return gb::qrow_bytes(type, K);
}
int64_t gb_kv_row_offset(const int32_t* pages, int page_shift, int64_t H, int64_t ctx, int64_t h,
                         int64_t t, int64_t hd) {
    if (page_shift < 0 || page_shift > 16 || H < 0 || ctx < 0 || h < 0 || t < 0 || hd < 0) {
        g_err = "gb_kv_row_offset: negative argument or page_shift outside 0..16";
        return -1;
    }
    return gb::kv_row_off(pages, page_shift, H, ctx, h, t, hd);
}
int gb_repack_blocks(const void* gguf, int type, int64_t N, int64_t K, void* wq, void* stream) {
    return guard([&] {
        gb::launch_repack_blocks((const uint8_t*)gguf, type, N, K, wq, (cudaStream_t)stream);
    });
}
int gb_quantize_q8_0(const float* x, int64_t x_stride, int64_t M, int64_t K, int8_t* xq,
                     float* xd, void* stream) {
    return guard([&] { gb::launch_quantize_q8_0(x, x_stride, M, K, xq, xd, (cudaStream_t)stream); });
}
int gb_mul_mat_q(int type, const void* wq, int64_t N, int64_t K,
                 const int8_t* xq, const float* xd, int64_t M, float* y, const float* bias,
                 const float* residual, void* stream) {
    return guard([&] {
        GB_CHECK(type == gb::T_Q8_0 || type == gb::T_Q4_0, "gb_mul_mat_q: type must be Q8_0 or Q4_0");
        gb::QWeight w;
        w.type = type;
        w.N = N;
        w.K = K;
        w.qs = wq;
        gb::MatmulEpilogue ep;
        ep.bias = bias;
        ep.residual = residual;
        ep.res_stride = N;
        gb::launch_matmul_q(w, xq, xd, M, y, N, ep, (cudaStream_t)stream);
    });
}
int gb_gemm_tc(int type, const void* wq, int64_t N, int64_t K, const int8_t* xq, const float* xd,
               int64_t M, float* y, const float* bias, const float* residual, void* stream) {
    return guard([&] {
        GB_CHECK(type == gb::T_Q8_0 || type == gb::T_Q4_0, "gb_gemm_tc: type must be Q8_0 or Q4_0");
        gb::QWeight w;
        w.type = type;
        w.N = N;
        w.K = K;
        w.qs = wq;
        gb::MatmulEpilogue ep;
        ep.bias = bias;
        ep.residual = residual;
        ep.res_stride = N;
        gb::launch_gemm_tc(w, xq, xd, M, y, N, ep, (cudaStream_t)stream);
    });
}
int gb_gemm_tc_error(void) {
    int v = 0;
    const int rc = guard([&] { v = gb::gemm_tc_error(); });
    return rc == 0 ? v : -1;
}
int gb_gemv_error(void) {
    int v = 0;
    const int rc = guard([&] { v = gb::dgemv_error(); });
    return rc == 0 ? v : -1;
}
int gb_gemv(int type, const void* wq, int64_t N, int64_t K, int64_t M,
            const int8_t* xq, const float* xd, const float* xf, float eps, const float* gamma,
            int swiglu, float* y, int8_t* yq, float* yd, const float* bias,
            const float* residual, void* stream) {
    return guard([&] {
        GB_CHECK(type == gb::T_Q8_0 || type == gb::T_Q4_0, "gb_gemv: type must be Q8_0 or Q4_0");
        gb::GemvArgs a;
        a.w.type = type;
        a.w.N = N;
        a.w.K = K;
        a.w.qs = wq;
        a.M = (int)M;
        a.xq = xq;
        a.xd = xd;
        a.xf = xf;
        a.xf_stride = K;
        a.eps = eps;
        a.gamma = gamma;
        a.swiglu = swiglu != 0;
        a.F = N / 2;
        a.y = y;
        a.y_stride = swiglu ? N / 2 : N;
        a.yq = yq;
        a.yd = yd;
        a.bias = bias;
        a.residual = residual;
        a.res_stride = N;
        gb::launch_gemv_fused(a, (cudaStream_t)stream);
    });
}
size_t gb_attn_decode_workspace_bytes(int64_t Hq, int64_t Hkv, int64_t hd, int64_t ctx) {
    if (Hq <= 0 || Hkv <= 0 || hd <= 0 || ctx <= 0) return 0;
    return gb::attn_decode_workspace(Hq, hd, gb::attn_decode_splits(Hkv, ctx));
}
int gb_attn_decode(const float* qkv, int64_t Hq, int64_t Hkv, int64_t hd, void* k, void* v,
                   int64_t ctx, int64_t kv_pos, int n_dims, float freq_base, const void* table,
                   int64_t n_pos, float scale, float* o, int8_t* oq, float* od, void* work,
                   void* stream) {
    return guard([&] {
        GB_CHECK(Hq > 0 && Hkv > 0 && hd > 0, "gb_attn_decode: Hq, Hkv and hd must be positive");
        GB_CHECK(kv_pos >= 0 && kv_pos < ctx, "gb_attn_decode: kv_pos outside the cache");
        gb::AttnDecArgs a;
        a.qkv = qkv;
        a.q_off = 0;
        a.k_off = Hq * hd;
        a.v_off = (Hq + Hkv) * hd;
        a.Hq = (int)Hq;
        a.Hkv = (int)Hkv;
        a.hd = (int)hd;
        a.tab.cs = (const float2*)table;
        a.tab.n_pos = table ? n_pos : 0;
        a.tab.n_dims = n_dims;
        a.tab.theta_scale = n_dims ? powf(freq_base, -2.0f / (float)n_dims) : 1.0f;
        a.step = nullptr;
        a.pos_off = kv_pos;
        a.kc = (__half*)k;
        a.vc = (__half*)v;
        a.ctx = ctx;
        a.scale = scale;
        a.max_kv = ctx;
        a.splits = gb::attn_decode_splits(Hkv, ctx);
        a.part = (float*)work;
        a.o = o;
        a.oq = oq;
        a.od = od;
        gb::launch_attn_decode(a, (cudaStream_t)stream);
    });
}
size_t gb_attn_decode_noalloc_max_bytes(void) { return gb::kAttnDecStaticWorkBytes; }
int gb_attn_decode_noalloc(const float* qkv, int64_t Hq, int64_t Hkv, int64_t hd, void* k,
                           void* v, int64_t ctx, int64_t kv_pos, int n_dims, float freq_base,
                           const void* table, int64_t n_pos, float scale, float* o, int8_t* oq,
                           float* od, void* stream) {
    return guard([&] {
        GB_CHECK(Hq > 0 && Hkv > 0 && hd > 0, "gb_attn_decode_noalloc: head counts must be positive");
        GB_CHECK(kv_pos >= 0 && kv_pos < ctx, "gb_attn_decode_noalloc: kv_pos outside the cache");
        const int splits = gb::attn_decode_splits(Hkv, ctx);
        float* work = gb::attn_decode_static_work(gb::attn_decode_workspace(Hq, hd, splits));
        gb::AttnDecArgs a;
        a.qkv = qkv;
        a.q_off = 0;
        a.k_off = Hq * hd;
        a.v_off = (Hq + Hkv) * hd;
        a.Hq = (int)Hq;
        a.Hkv = (int)Hkv;
        a.hd = (int)hd;
        a.tab.cs = (const float2*)table;
        a.tab.n_pos = table ? n_pos : 0;
        a.tab.n_dims = n_dims;
        a.tab.theta_scale = n_dims ? powf(freq_base, -2.0f / (float)n_dims) : 1.0f;
        a.step = nullptr;
        a.pos_off = kv_pos;
        a.kc = (__half*)k;
        a.vc = (__half*)v;
        a.ctx = ctx;
        a.scale = scale;
        a.max_kv = ctx;
        a.splits = splits;
        a.part = work;
        a.o = o;
        a.oq = oq;
        a.od = od;
        gb::launch_attn_decode(a, (cudaStream_t)stream);
    });
}
int gb_get_rows(int type, const void* wq, int64_t N, int64_t K,
                const int32_t* ids, int64_t n, float* out, void* stream) {
    return guard([&] {
        gb::QWeight w;
        w.type = type;
        w.N = N;
        w.K = K;
        w.qs = wq;
        gb::launch_get_rows(w, ids, n, out, K, (cudaStream_t)stream);
    });
}
int gb_rms_norm(const float* x, int64_t M, int64_t D, float eps, const float* gamma, float* y,
                int8_t* yq, float* yd, void* stream) {
    return guard([&] {
        gb::launch_rms_norm(x, D, M, D, eps, gamma, y, D, yq, yd, (cudaStream_t)stream);
    });
}
int gb_layer_norm(const float* x, int64_t M, int64_t D, float eps, const float* gamma,
                  const float* beta, float* y, int8_t* yq, float* yd, void* stream) {
    return guard([&] {
        gb::launch_layer_norm(x, D, M, D, eps, gamma, beta, y, D, yq, yd, (cudaStream_t)stream);
    });
}
int gb_bias_gelu(const float* x, const float* bias, int64_t M, int64_t F, float* y, int8_t* yq,
                 float* yd, void* stream) {
    return guard([&] {
        gb::launch_bias_gelu(x, F, bias, M, F, y, F, yq, yd, (cudaStream_t)stream);
    });
}
int gb_swiglu(const float* x, int64_t M, int64_t F, float* y, int8_t* yq, float* yd,
              void* stream) {
    return guard([&] {
        gb::launch_swiglu(x, 2 * F, M, F, false, y, F, yq, yd, (cudaStream_t)stream);
    });
}
float gb_rope_table_fill(float* host_out, int64_t n_pos, int n_dims, float freq_base) {
    const float ts = powf(freq_base, -2.0f / (float)n_dims);
    const int half = n_dims / 2;
    for (int64_t p = 0; p < n_pos; ++p) {
        float theta = (float)p;
        for (int i = 0; i < half; ++i) {
            host_out[2 * (p * half + i)] = cosf(theta);
            host_out[2 * (p * half + i) + 1] = sinf(theta);
            theta *= ts;
        }
    }
    return ts;
}
int gb_rope_neox(const float* x, int64_t hd, int64_t H, int64_t s, const int32_t* pos,
                 int n_dims, float freq_base, const void* table, int64_t n_pos, float* y,
                 void* stream) {
    return guard([&] {
        gb::TView xv, yv;
        xv.data = (char*)x;
        yv.data = (char*)y;
        xv.type = yv.type = gb::T_F32;
        xv.ne[0] = yv.ne[0] = hd;
        xv.ne[1] = yv.ne[1] = H;
        xv.ne[2] = yv.ne[2] = s;
        xv.nb[0] = yv.nb[0] = 4;
        xv.nb[1] = yv.nb[1] = 4 * hd;
        xv.nb[2] = yv.nb[2] = 4 * hd * H;
        xv.nb[3] = yv.nb[3] = 4 * hd * H * s;
        gb::RopeTable rt;
        rt.cs = (const float2*)table;
        rt.n_pos = table ? n_pos : 0;
        rt.n_dims = n_dims;
        rt.theta_scale = powf(freq_base, -2.0f / (float)n_dims);
        gb::launch_rope_neox(xv, pos, false, nullptr, rt, &yv, nullptr, (cudaStream_t)stream);
    });
}
size_t gb_attention_workspace_bytes(int64_t s, int64_t Hq, int64_t hd, int64_t ctx) {
    return gb::attn_workspace_bytes(s, Hq, hd, ctx);
}
int gb_attention(const float* q, const void* k, const void* v, int64_t hd, int64_t s,
                 int64_t Hq, int64_t Hkv, int64_t ctx, int64_t kv_pos, float scale, float* o,
                 void* work, void* stream) {
    return guard([&] {
        GB_CHECK(kv_pos >= 0 && kv_pos + s <= ctx, "gb_attention: kv_pos + s exceeds ctx");
        gb::TView qv;
        qv.data = (char*)q;
        qv.type = gb::T_F32;
        qv.ne[0] = hd;  // view [hd, s, Hq] over q[s][Hq][hd]
        qv.ne[1] = s;
        qv.ne[2] = Hq;
        qv.nb[0] = 4;
        qv.nb[1] = 4 * hd * Hq;
        qv.nb[2] = 4 * hd;
        qv.nb[3] = 4 * hd * Hq * s;
        gb::launch_attention(qv, (const __half*)k, (const __half*)v, ctx, Hkv, nullptr, false,
                             kv_pos, scale, o, work, ctx, (cudaStream_t)stream);
    });
}

}  // extern "C"
