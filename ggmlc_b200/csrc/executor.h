// ModelExecutor for the B200 engine: the CUDA replacement of runtime/src/executor.cpp behind
// the same interface (runtime/include/ggmlc/executor.h:25-287).
//
// prepare(env) lowers the graph for one shape into a Program: a list of kernel launches over
// an activation arena, with the fusions this engine applies (norm/SwiGLU/GELU emit the Q8_0
// rows their matmul consumes; matmul epilogues add bias and the residual ADD).  Programs are
// cached per shape; the KV position is not part of the key — kernels read it from a device
// StepParams, so a decode Program (and its CUDA graph) is replayed for every token.
#pragma once

#include <cuda_runtime.h>

#include <array>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.h"
#include "graph.h"
#include "kernels.h"
#include "tp.h"

namespace gb {

struct BufRef {
    int buf = -1;           // arena buffer id (or -1)
    char* fixed = nullptr;  // persistent device memory (weights, KV cache, inputs)
    int64_t off = 0;
};

struct Val {
    BufRef ref;
    int type = T_F32;
    int64_t ne[4] = {1, 1, 1, 1};
    int64_t nb[4] = {0, 0, 0, 0};
    bool has_f = true;       // f32/f16/i32 data present at ref
    BufRef q, qd;            // Q8_0 rows (int8 quants, fp32 scales) when materialized
    bool has_q = false;
    const QWeight* w = nullptr;  // quantized weight
    // RMSNorm output left unmaterialized: the consuming decode GEMV normalizes rms_x itself
    bool virt_rms = false;
    BufRef rms_x;
    int64_t rms_stride = 0;
    float rms_eps = 0.0f;
    const float* rms_gamma = nullptr;
    // f32 rows whose Q8_0 form is left unmaterialized: every consumer is a decode GEMV that
    // quantizes them in its prologue (the SwiGLU output of a 1-2-row decode step)
    bool q_in_prologue = false;
    // RoPE output left unmaterialized: the attention lowering rotates q/k inside its kernels.
    // rsrc_* describe the un-rotated [hd, H, s] source view; rope_perm tracks a (0,2,1,3)
    // permute applied after the rotation.
    bool virt_rope = false;
    bool rope_perm = false;
    BufRef rsrc;
    int64_t rsrc_ne[4] = {1, 1, 1, 1};
    int64_t rsrc_nb[4] = {0, 0, 0, 0};
    RopeTable rtab;
    bool r_use_step = false;
    bool contiguous() const;
    int64_t nrows() const { return ne[1] * ne[2] * ne[3]; }
    bool rows_uniform() const { return nb[2] == nb[1] * ne[1] && nb[3] == nb[2] * ne[2]; }
};

struct Program;
using Launch = std::function<void(Program&, cudaStream_t)>;
// How a launch runs as one op of a decode chain (k_chain.cu): fills the op from the program's
// current buffers and returns whether the chain implements it.  Empty: the launch cannot join.
using ChainDesc = std::function<bool(const Program&, ChainOp&)>;
// A run of consecutive launches replaced by one chain launch.  The device table is rewritten
// before a run whenever the buffers it points at moved (arena growth, another KV slot); captured
// graphs keep the table's address.
struct ChainRun {
    std::vector<ChainDesc> descs;
    ChainOp* d_ops = nullptr;
    std::vector<ChainOp> h_ops;
    ChainSync* sync = nullptr;
    float* part = nullptr;
    char* key_arena = nullptr;
    int64_t key_slot = -1;
};

struct Program {
    std::string key;
    SymEnv env;
    bool kv = false;
    bool decode = false;
    bool batch = false;  // batched decode: row r is the next token of the sequence in a slot
    int64_t out_rows_of = 0;  // rows the output projections select from (out_rows), 0: none
    std::vector<int64_t> buf_size, buf_first, buf_last, buf_off;
    char* const* arena = nullptr;  // the executor's shared activation arena (grows on demand)
    size_t arena_bytes = 0;
    int64_t kv_slot = 0;           // KV slot of a single-sequence program (set by prepare)
    int64_t graph_slot = -1;       // kv_slot the captured graph was recorded with
    std::vector<Launch> launches;
    std::vector<std::string> launch_names;
    std::vector<double> launch_bytes;  // algorithmic HBM bytes of each launch (0 if untracked)
    std::vector<ChainDesc> chain_descs;  // per launch while lowering (empty: not chainable)
    std::vector<PfNext> launch_w;   // per launch: the quantized weights it streams (GEMVs)
    std::vector<PfNext> launch_pf;  // per launch: what it prefetches into L2 (the next launch_w)
    std::vector<std::shared_ptr<ChainRun>> chains;
    std::map<uint32_t, Val> vals;
    std::map<uint32_t, char*> input_bufs;  // graph inputs (device, persistent per program)
    std::vector<void*> owned;              // device allocations to free
    cudaGraphExec_t graph_exec = nullptr;
    int64_t s = 0;

    char* ptr(const BufRef& r) const {
        if (r.fixed) return r.fixed + r.off;
        if (r.buf < 0) return nullptr;
        return *arena + buf_off[r.buf] + r.off;
    }
    int new_buf(int64_t bytes, int first) {
        buf_size.push_back((bytes + 255) / 256 * 256);
        buf_first.push_back(first);
        buf_last.push_back(first);
        return (int)buf_size.size() - 1;
    }
    void use(const BufRef& r, int op) {
        if (!r.fixed && r.buf >= 0 && op > buf_last[r.buf]) buf_last[r.buf] = op;
    }
    TView view(const Val& v) const;
};

struct KVCache {
    __half* k = nullptr;
    __half* v = nullptr;
    int64_t hd = 0, Hkv = 0, batch = 1, ctx = 0;
    int64_t slots = 1;  // contiguous cache: sequence windows [slot][Hkv][ctx][hd], slot_elems apart
    int64_t elems = 0;  // halves allocated for k (and for v): windows, or pages [page][Hkv][T][hd]
    int64_t slot_elems() const { return Hkv * ctx * hd; }
};

class Executor {
public:
    // tp_size > 1: this executor is rank tp_rank of a tensor-parallel group (tp.h); nccl_id is
    // the group's 128-byte ncclUniqueId (made by rank 0 with nccl_unique_id and shared by the
    // caller).  Construction is collective: every rank of the group must construct its executor.
    Executor(std::shared_ptr<Graph> g, const std::string& device, int tp_rank = 0,
             int tp_size = 1, const void* nccl_id = nullptr);
    ~Executor();
    static void nccl_unique_id(void* out128);
    int tp_rank() const { return tp_.rank; }
    int tp_size() const { return tp_.size; }
    const TpPlan& tp_plan() const { return tp_; }

    static std::vector<std::string> available_devices();
    const std::string& device() const { return device_; }

    void prepare(const SymEnv& env, bool arena_reuse);
    void set_input(uint32_t tid, const void* data, size_t bytes);
    void set_input_by_name(const std::string& name, const void* data, size_t bytes);
    void run();
    void synchronize();
    const void* get_output(uint32_t tid, size_t* bytes);
    // greedy token of each of `rows` rows of an f32 output [rows][n] (first maximum), computed on
    // the device; only the indices cross to the host
    void output_argmax(uint32_t tid, int rows, int32_t* out);
    std::array<int64_t, 4> tensor_shape(uint32_t tid) const;
    size_t tensor_size_bytes(uint32_t tid) const;

    // persistent STATE tensors (executor.cpp:3063-3136); kept on the device
    void set_state(uint32_t tid, const void* data, size_t bytes);
    const void* get_state(uint32_t tid, size_t* bytes);
    void reset_state();

    void init_kv_cache(int64_t max_ctx);
    void reset_kv_cache();
    bool has_kv_cache() const { return kv_enabled_; }

    // Paged KV cache (executor.h:147-161 of the reference): max_batch sequence slots of up to
    // max_ctx positions.  Every attention layer keeps its K and its V in a page pool
    // [page][Hkv][T][hd] fp16 (T = tokens_per_page, a power of two); one page id names the same T
    // positions in every layer.  A device page table (max_batch + 1 rows of ceil(max_ctx / T)
    // entries) maps each slot's runs of T positions to pool pages, and the attention kernels
    // address the cache through it.  Pages are reference-counted: a slot holds the pages
    // assigned as it grows (paged_kv_ensure_tokens) until paged_kv_free_slot, and the prefix
    // cache holds references to the pages it indexes, so a prefix hit maps cached pages into a
    // new slot's table (kv_map_page) instead of copying rows.  Page 0 is the scratch page:
    // unassigned table entries and the scratch slot of padding rows (slot max_batch) point at it.
    // The pool holds max_batch full sequences plus the prefix pages of configure_prefix_pool,
    // or exactly configure_kv_pool_pages pages; both take effect at the next init.
    void init_paged_kv_cache(int64_t max_batch, int64_t max_ctx);
    bool paged_kv_enabled() const { return paged_; }
    void paged_kv_alloc_slot(int64_t slot);
    void paged_kv_free_slot(int64_t slot);
    void paged_kv_ensure_tokens(int64_t slot, int64_t total);  // assigns pages up to `total`
    int64_t paged_active_vram_bytes() const;  // bytes of the pages mapped into slots
    int64_t tokens_per_page() const { return tokens_per_page_; }
    void set_tokens_per_page(int64_t n);  // a power of two; re-lays an idle pool
    int64_t paged_max_batch() const { return paged_ ? paged_max_batch_ : 0; }
    int64_t kv_page_bytes() const;   // one page: T positions of K and V in every layer
    void configure_prefix_pool(int64_t pages);  // prefix-cache pages beyond max_batch sequences
    void configure_kv_pool_pages(int64_t pages);  // explicit pool size (0: the default rule)
    int64_t kv_pool_pages() const;   // pages sequences and the prefix cache can use
    int64_t kv_free_pages() const;   // pages nobody references
    int64_t paged_kv_slot_pages(int64_t slot) const;  // pages in the slot's table
    int64_t kv_pool_generation() const { return pool_gen_; }  // bumps on every re-layout
    // page sharing for the prefix cache
    int64_t kv_slot_page(int64_t slot, int64_t index) const;  // page of the slot's index-th run
    void kv_page_retain(int64_t page);
    void kv_page_release(int64_t page);
    // append `page` to the slot's table (a reference for the slot); the slot's next run
    void kv_map_page(int64_t slot, int64_t page);
    // give the slot its own copy of its index-th page (before writing into a shared page)
    void kv_make_private(int64_t slot, int64_t index);
    // Batched decode step over `rows` sequences: row r decodes the token at position pos[r] of
    // the sequence in slot slot[r] (rows padded up to a bucket use the scratch slot).
    void prepare_batch(int rows, const int32_t* pos, const int32_t* slot);
    int64_t kv_max_ctx() const { return kv_max_ctx_; }

    // Output rows (llama's out_ids; the reference's set_logits_last_only generalised): when set,
    // a prefill's output projections compute only these rows of the call's tokens, in this
    // order (at most kMaxOutRows, each below the call's token count); empty turns it off.  Takes
    // precedence over logits_last_only.
    void set_output_rows(const std::vector<int32_t>& rows);
    const std::vector<int32_t>& output_rows() const { return out_rows_; }
    void set_logits_last_only(bool on) { logits_last_only_ = on; }
    bool logits_last_only() const { return logits_last_only_; }
    void set_enable_cuda_graph(bool on) { cuda_graph_ = on; }
    // Decode chains (k_chain.cu): single-sequence decode steps run as one persistent launch.  Off
    // by default (measured slower than the per-op launches at the Llama-3-8B decode shape: every
    // op waits at a grid barrier and re-reads its operands through L2); toggling drops the
    // prepared programs (the next prepare rebuilds them).
    void set_decode_chain(bool on);
    bool decode_chain() const { return chain_enabled_; }
    bool cuda_graph_enabled() const { return cuda_graph_; }
    bool cuda_graph_captured() const;

    struct Profile {
        double prepare_ms = 0, run_ms = 0;
        int n_prepare = 0, n_run = 0;
    };
    void set_enable_profile(bool on) { profile_on_ = on; }
    void reset_profile() { profile_ = Profile(); }
    Profile profile() const { return profile_; }
    std::string graph_summary() const;
    std::string mul_mat_shape_summary() const;
    // Per-launch device timing: while on, run() skips graph replay, brackets every launch with
    // CUDA events and accumulates {name: [ms, launches, algorithmic bytes]}.
    void set_kernel_timing(bool on) { ktiming_ = on; }
    void reset_kernel_times() { ktimes_.clear(); }
    std::string kernel_times_json() const;

    cudaStream_t stream() const { return stream_; }
    const Graph& graph() const { return *g_; }
    // number of the engine's kernel launches of the active program per run (collectives excluded)
    int64_t launches_per_run() const;
    size_t weight_bytes() const { return weight_bytes_; }

private:
    void upload_weights();
    std::shared_ptr<Program> build(const SymEnv& env, bool kv);
    void fuse_chains(Program& pg);
    void refresh_chain(Program& p, ChainRun& c);
    const float2* rope_table(int n_dims, float freq_base, float freq_scale, int64_t* n_pos,
                             float* theta_scale);
    void free_program(Program& p);

    std::shared_ptr<Graph> g_;
    TpPlan tp_;
    void* nccl_ = nullptr;  // ncclComm_t of the tensor-parallel group
    QWeight tp_vocab_view_;  // this rank's rows of the vocabulary-split projection
    // peer-memory all-reduce of small partial sums (decode): this rank's buffer, the peers'
    // buffers mapped with CUDA IPC, per-CTA epochs and the error word
    void setup_peer_allreduce();
    char* ar_base_ = nullptr;
    std::vector<char*> ar_peer_;  // IPC mappings to close (index = rank; own rank null)
    TpPeers ar_peers_{};
    uint32_t* ar_epochs_ = nullptr;
    int* ar_err_ = nullptr;       // device address of ar_err_host_
    int* ar_err_host_ = nullptr;  // mapped pinned error word of the peer all-reduce
    int64_t ar_cap_ = 0;

public:
    // non-zero once a peer all-reduce gave up waiting for a peer (the sum of that call is not
    // valid)
    int tp_allreduce_error();
    void check_tp_error();

private:
    std::string device_;
    int dev_ = 0;
    cudaStream_t stream_ = nullptr;
    std::map<uint32_t, QWeight> qweights_;
    std::map<uint32_t, char*> consts_;  // f32/i32/f16 params and constants on device
    std::vector<void*> weight_allocs_;
    size_t weight_bytes_ = 0;
    std::map<uint32_t, KVCache> kv_;    // per FLASH_ATTN_EXT op id
    bool kv_enabled_ = false;
    int64_t kv_max_ctx_ = 0;
    bool paged_ = false;
    int64_t paged_max_batch_ = 0;
    int64_t tokens_per_page_ = 256;
    int64_t prefix_pool_want_ = 0;     // prefix pages; 0: about 2 GiB, at most max_batch seqs
    int64_t kv_pool_want_ = 0;         // explicit pool pages (0: the default rule)
    int64_t paged_max_ctx_ = 0;
    int64_t pool_gen_ = 0;
    int32_t ptab_stride_ = 0;          // page-table entries per slot
    int page_shift_ = 0;               // log2(tokens_per_page)
    std::vector<int32_t> h_ptab_;      // [(max_batch + 1) * ptab_stride_]
    int32_t* d_ptab_ = nullptr;
    bool ptab_dirty_ = false;
    static constexpr int kPtabRing = 4;  // pinned staging copies of the table
    static constexpr size_t kMaxPtabBytes = size_t(64) << 10;
    int32_t* ptab_ring_ = nullptr;
    cudaEvent_t ptab_ev_[kPtabRing] = {};
    int ptab_next_ = 0;
    std::vector<int32_t> page_ref_;    // references per pool page (slots + prefix cache)
    std::vector<int32_t> free_pages_;  // unreferenced pages (page 0 is never among them)
    std::vector<std::vector<int32_t>> slot_pages_;  // per slot: its table's pages in order
    std::vector<char> slot_live_;      // per slot: allocated
    void sync_page_table();            // stream-ordered upload of a changed table
    int32_t take_free_page();
    char* arena_ = nullptr;             // activation arena shared by every program
    size_t arena_cap_ = 0;
    void ensure_arena(size_t bytes);
    // contiguous windows for `slots` sequences, or (paged > 0) page pools sized for `paged`
    // sequences plus the prefix pages (init_paged_kv_cache)
    void alloc_kv(int64_t slots, int64_t max_ctx, int64_t paged = 0);
    void free_kv();
    bool logits_last_only_ = false;
    std::vector<int32_t> out_rows_;
    bool chain_enabled_ = false;  // decode chains (GGMLC_B200_CHAIN=1 turns them on by default)
    // most ops per chain launch (GGMLC_B200_CHAIN_OPS; 0: a whole run of chainable launches).  A
    // bound also chains runs shorter than three ops, so GGMLC_B200_CHAIN_OPS=1 times every op of
    // the chain kernel as its own launch.
    size_t chain_max_ops_ = 0;
    // tensor parallelism: decode-row all-reduces folded into the GEMV epilogue
    // (GGMLC_B200_GEMV_AR=0: the separate all-reduce launch instead)
    bool gemv_ar_ = true;
    int* chain_err_host_ = nullptr;  // mapped pinned word the chain kernel sets on failure
    int* chain_err_dev_ = nullptr;
    bool cuda_graph_ = false;
    bool profile_on_ = false;
    Profile profile_;
    StepParams* h_step_ = nullptr;  // working copy, rewritten by every prepare
    StepParams* d_step_ = nullptr;
    // Pinned staging ring of step parameters.  An async host-to-device copy reads its pinned
    // source when the stream reaches it, which can be many steps after run() returned; each run
    // copies from its own ring entry, and an entry is rewritten only after the event recorded
    // behind its previous copy has completed.
    static constexpr int kStepRing = 64;
    StepParams* step_ring_ = nullptr;
    cudaEvent_t step_ev_[kStepRing] = {};
    int step_next_ = 0;
    std::map<std::string, std::shared_ptr<Program>> programs_;
    std::shared_ptr<Program> active_;
    std::map<uint32_t, std::vector<uint8_t>> out_host_;
    std::map<uint32_t, char*> state_dev_;
    std::map<std::string, std::pair<float2*, std::pair<int64_t, float>>> rope_tabs_;
    void* pinned_out_ = nullptr;
    int32_t* d_argmax_ = nullptr;   // kMaxRows device indices
    int32_t* h_argmax_ = nullptr;   // pinned copy
    size_t pinned_out_bytes_ = 0;
    bool ktiming_ = false;
    struct KTime {
        double ms = 0, bytes = 0;
        int64_t n = 0;
    };
    std::map<std::string, KTime> ktimes_;
    std::vector<cudaEvent_t> kevents_;
};

}  // namespace gb
