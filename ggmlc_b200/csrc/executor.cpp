// Graph lowering and execution (see executor.h).  Op semantics follow the reference executor
// (runtime/src/executor.cpp: GET_ROWS :2034, ROPE :2053, FLASH_ATTN_EXT :2091-2354, MUL_MAT
// :2362-2447, RESHAPE/PERMUTE/VIEW :2448-2560, custom ops 200-203 :2703-2757).
#include "executor.h"

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <mutex>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <set>
#include <sstream>

#include "common.h"
#include "kutil.cuh"

namespace gb {

namespace {

void set_contig(Val& v) {
    const int64_t eb = v.type == T_F16 ? 2 : (v.type == T_I64 ? 8 : 4);
    v.nb[0] = eb;
    for (int d = 1; d < 4; ++d) v.nb[d] = v.nb[d - 1] * v.ne[d - 1];
}

int64_t nelem(const int64_t* ne) { return ne[0] * ne[1] * ne[2] * ne[3]; }

double now_ms() {
    return std::chrono::duration<double, std::milli>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

}  // namespace

bool Val::contiguous() const {
    int64_t e = type == T_F16 ? 2 : (type == T_I64 ? 8 : 4);
    if (nb[0] != e) return false;
    int64_t s = e * ne[0];
    for (int d = 1; d < 4; ++d) {
        if (ne[d] > 1 && nb[d] != s) return false;
        s *= ne[d];
    }
    return true;
}

TView Program::view(const Val& v) const {
    TView t;
    t.data = ptr(v.ref);
    t.type = v.type;
    for (int d = 0; d < 4; ++d) {
        t.ne[d] = v.ne[d];
        t.nb[d] = v.nb[d];
    }
    return t;
}

// ------------------------------------------------------------------------------ construction

std::vector<std::string> Executor::available_devices() {
    std::vector<std::string> out = {"cpu"};
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    for (int i = 0; i < n; ++i) out.push_back("cuda:" + std::to_string(i));
    if (n > 0) out.push_back("cuda");
    return out;
}

// NCCL is opened on first use (tensor parallelism only), preferring the libnccl.so.2 that the
// process has already loaded (PyTorch's), so the library carries no link-time NCCL dependency
// and never loads a second NCCL next to PyTorch's.
namespace {
struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                               ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};
const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
        api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
        api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
        api.all_reduce = (decltype(api.all_reduce))dlsym(h, "ncclAllReduce");
        api.all_gather = (decltype(api.all_gather))dlsym(h, "ncclAllGather");
        api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
    });
    GB_CHECK(api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce &&
                 api.all_gather && api.error_string,
             "tensor parallelism needs NCCL (libnccl.so.2), which could not be loaded");
    return api;
}
}  // namespace

#define GB_NCCL(call)                                                                     \
    do {                                                                                  \
        const ncclResult_t r_ = nccl().call;                                              \
        GB_CHECK(r_ == ncclSuccess,                                                       \
                 std::string("NCCL: ") + nccl().error_string(r_) + " (" #call ")");       \
    } while (0)

void Executor::nccl_unique_id(void* out128) {
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    ncclUniqueId id;
    GB_NCCL(get_unique_id(&id));
    std::memcpy(out128, &id, sizeof(id));
}

Executor::Executor(std::shared_ptr<Graph> g, const std::string& device, int tp_rank, int tp_size,
                   const void* nccl_id)
    : g_(std::move(g)) {
    std::string d = device;
    for (auto& c : d) c = (char)std::tolower((unsigned char)c);
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    if (d == "auto") d = "cuda:0";
    GB_CHECK(d.rfind("cuda", 0) == 0,
             "device '" + device + "' is not served by the B200 engine (CUDA only; the CPU path "
             "is the reference runtime)");
    GB_CHECK(n > 0, "no CUDA device is visible");
    dev_ = 0;
    if (d.size() > 5 && d[4] == ':') dev_ = std::stoi(d.substr(5));
    GB_CHECK(dev_ >= 0 && dev_ < n, "CUDA device index out of range: " + device);
    device_ = "cuda:" + std::to_string(dev_);
    GB_CUDA(cudaSetDevice(dev_));
    GB_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    GB_CUDA(cudaMallocHost(&h_step_, sizeof(StepParams)));
    GB_CUDA(cudaMallocHost(&step_ring_, kStepRing * sizeof(StepParams)));
    for (cudaEvent_t& ev : step_ev_) GB_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    GB_CUDA(cudaMalloc(&d_step_, sizeof(StepParams)));
    h_step_->pos = 0;
    GB_CUDA(cudaMemcpy(d_step_, h_step_, sizeof(StepParams), cudaMemcpyHostToDevice));
    if (const char* e = std::getenv("GGMLC_B200_CHAIN")) chain_enabled_ = std::string(e) == "1";
    if (const char* e = std::getenv("GGMLC_B200_CHAIN_OPS")) chain_max_ops_ = (size_t)std::max(0, std::atoi(e));
    if (const char* e = std::getenv("GGMLC_B200_GEMV_AR")) gemv_ar_ = std::string(e) != "0";
    int coop = 0;
    GB_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev_));
    if (!coop) chain_enabled_ = false;
    if (tp_size > 1) {
        GB_CHECK(nccl_id != nullptr, "tensor parallelism needs the group's NCCL unique id");
        g_ = std::make_shared<Graph>(*g_);  // this rank's shapes are rewritten in a copy
        tp_ = plan_tensor_parallel(*g_, tp_rank, tp_size);
        ncclUniqueId id;
        std::memcpy(&id, nccl_id, sizeof(id));
        ncclComm_t comm = nullptr;
        GB_NCCL(comm_init_rank(&comm, tp_size, id, tp_rank));
        nccl_ = comm;
        setup_peer_allreduce();
    }
    upload_weights();
}

// Buffers of the one-shot all-reduce (k_allreduce.cu): room for 16 rows of the widest K-split
// output, two parities, one slot per rank; handles exchanged with one NCCL all-gather.
void Executor::setup_peer_allreduce() {
    const int T = tp_.size, r = tp_.rank;
    GB_CHECK(T <= kMaxTp, "tensor parallelism: at most 8 ranks");
    SymEnv env;
    env["s"] = 1;
    for (auto& s : g_->symbol_table) env[s] = 1;
    int64_t width = 0;
    for (uint32_t id : tp_.partial) {
        const GTensor& t = g_->t(id);
        width = std::max<int64_t>(width, t.ne[0] ? t.ne[0]->eval(env) : 1);
    }
    ar_cap_ = (std::max<int64_t>(width, 1) * kMaxRows + 3) / 4 * 4;
    const size_t recv_bytes = (size_t)(2 * T * ar_cap_) * 4;
    const size_t flag_bytes = (size_t)(2 * T * kArCtas) * 4;
    // the decode GEMV's epilogue all-reduce has slots, flags and epochs of its own
    const size_t gflag_bytes = (size_t)(2 * T * kGemvArCtas) * 4;
    const size_t total = 2 * recv_bytes + flag_bytes + gflag_bytes;
    GB_CUDA(cudaMalloc(&ar_base_, total));
    GB_CUDA(cudaMemset(ar_base_, 0, total));
    GB_CUDA(cudaMalloc(&ar_epochs_, (kArCtas + kGemvArCtas) * sizeof(uint32_t)));
    GB_CUDA(cudaMemset(ar_epochs_, 0, (kArCtas + kGemvArCtas) * sizeof(uint32_t)));
    // the error word lives in mapped pinned host memory: every host synchronisation reads it
    // without a copy (check_tp_error)
    GB_CUDA(cudaHostAlloc((void**)&ar_err_host_, sizeof(int), cudaHostAllocMapped));
    *ar_err_host_ = 0;
    GB_CUDA(cudaHostGetDevicePointer((void**)&ar_err_, ar_err_host_, 0));
    cudaIpcMemHandle_t h;
    GB_CUDA(cudaIpcGetMemHandle(&h, ar_base_));
    char* dh = nullptr;
    GB_CUDA(cudaMalloc(&dh, (size_t)T * sizeof(h)));
    GB_CUDA(cudaMemcpy(dh + (size_t)r * sizeof(h), &h, sizeof(h), cudaMemcpyHostToDevice));
    GB_NCCL(all_gather(dh + (size_t)r * sizeof(h), dh, sizeof(h), ncclUint8, (ncclComm_t)nccl_,
                       stream_));
    GB_CUDA(cudaStreamSynchronize(stream_));
    std::vector<cudaIpcMemHandle_t> all((size_t)T);
    GB_CUDA(cudaMemcpy(all.data(), dh, (size_t)T * sizeof(h), cudaMemcpyDeviceToHost));
    GB_CUDA(cudaFree(dh));
    ar_peer_.assign((size_t)T, nullptr);
    for (int p = 0; p < T; ++p) {
        char* base = ar_base_;
        if (p != r) {
            void* m = nullptr;
            GB_CUDA(cudaIpcOpenMemHandle(&m, all[(size_t)p], cudaIpcMemLazyEnablePeerAccess));
            base = (char*)m;
            ar_peer_[(size_t)p] = base;
        }
        ar_peers_.recv[p] = (float*)base;
        ar_peers_.flags[p] = (uint32_t*)(base + recv_bytes);
        ar_peers_.grecv[p] = (float*)(base + recv_bytes + flag_bytes);
        ar_peers_.gflags[p] = (uint32_t*)(base + 2 * recv_bytes + flag_bytes);
    }
}

int Executor::tp_allreduce_error() {
    if (!ar_err_host_) return 0;
    GB_CUDA(cudaStreamSynchronize(stream_));
    return *(volatile int*)ar_err_host_;
}

// A peer all-reduce whose wait ran out wrote a sum that is not valid: every output read of this
// executor syncs through here and raises (once; the word is cleared) instead of handing it out.
void Executor::check_tp_error() {
    if (chain_err_host_ && *(volatile int*)chain_err_host_) {
        *(volatile int*)chain_err_host_ = 0;
        throw std::runtime_error(
            "decode chain: a wait ran out (about 2 s); the outputs of this run are not valid and "
            "later chain launches in this process do nothing");
    }
    if (ar_err_host_ && *(volatile int*)ar_err_host_) {
        *(volatile int*)ar_err_host_ = 0;
        throw std::runtime_error(
            "tensor-parallel all-reduce: a peer did not arrive within the wait limit (about 1 s); "
            "the outputs of this run are not valid");
    }
}

Executor::~Executor() {
    cudaSetDevice(dev_);
    if (stream_) cudaStreamSynchronize(stream_);
    if (chain_err_host_) cudaFreeHost(chain_err_host_);
    for (auto& [k, p] : programs_) free_program(*p);
    for (void* p : weight_allocs_) cudaFree(p);
    for (auto& [id, c] : kv_) {
        cudaFree(c.k);
        cudaFree(c.v);
    }
    for (auto& [id, p] : state_dev_) cudaFree(p);
    for (auto& [k, t] : rope_tabs_) cudaFree(t.first);
    for (cudaEvent_t ev : kevents_) cudaEventDestroy(ev);
    if (h_step_) cudaFreeHost(h_step_);
    if (step_ring_) cudaFreeHost(step_ring_);
    for (cudaEvent_t ev : step_ev_)
        if (ev) cudaEventDestroy(ev);
    if (d_step_) cudaFree(d_step_);
    if (d_ptab_) cudaFree(d_ptab_);
    if (ptab_ring_) cudaFreeHost(ptab_ring_);
    for (cudaEvent_t ev : ptab_ev_)
        if (ev) cudaEventDestroy(ev);
    if (pinned_out_) cudaFreeHost(pinned_out_);
    if (d_argmax_) cudaFree(d_argmax_);
    if (h_argmax_) cudaFreeHost(h_argmax_);
    if (arena_) cudaFree(arena_);
    for (char* m : ar_peer_)
        if (m) cudaIpcCloseMemHandle(m);
    if (ar_base_) cudaFree(ar_base_);
    if (ar_epochs_) cudaFree(ar_epochs_);
    if (ar_err_host_) cudaFreeHost(ar_err_host_);
    if (nccl_) nccl().comm_destroy((ncclComm_t)nccl_);  // after the graphs that captured its calls
    if (stream_) cudaStreamDestroy(stream_);
}

void Executor::free_program(Program& p) {
    if (p.graph_exec) cudaGraphExecDestroy(p.graph_exec);
    p.graph_exec = nullptr;
    for (void* q : p.owned) cudaFree(q);
    p.owned.clear();
}

// One activation arena for all programs (they run one at a time on the executor's stream).  It
// grows to the largest program's need; growing moves it, so captured graphs are dropped.
void Executor::ensure_arena(size_t bytes) {
    if (bytes <= arena_cap_) return;
    GB_CUDA(cudaStreamSynchronize(stream_));
    for (auto& [k, p] : programs_)
        if (p->graph_exec) {
            cudaGraphExecDestroy(p->graph_exec);
            p->graph_exec = nullptr;
        }
    if (arena_) GB_CUDA(cudaFree(arena_));
    arena_ = nullptr;
    const size_t cap = bytes + bytes / 4;
    GB_CUDA(cudaMalloc(&arena_, cap));
    arena_cap_ = cap;
}

namespace {

// This rank's part of a GGUF tensor [N0 rows][K0 elements]: concatenated row ranges, or one
// column range of every row (whole 32-element blocks for quantized types).
std::vector<uint8_t> slice_payload(const GTensor& t, const TpSlice& s, int64_t* N, int64_t* K) {
    const int64_t K0 = t.file_ne[0], N0 = t.file_ne[1] * t.file_ne[2] * t.file_ne[3];
    const int64_t rb = row_bytes(t.type, K0);
    GB_CHECK((uint64_t)(rb * N0) <= t.data_size, "tensor '" + t.name + "': payload too short");
    std::vector<uint8_t> out;
    if (!s.cols) {
        // a 1-D tensor (bias) is sliced by elements
        const bool vec = N0 == 1;
        const int64_t eb = vec ? row_bytes(t.type, 1) : rb;
        int64_t n = 0;
        for (auto& [a, b] : s.rows) {
            GB_CHECK(a >= 0 && b <= (vec ? K0 : N0) && a <= b, "tensor '" + t.name + "': bad slice");
            out.insert(out.end(), t.data + a * eb, t.data + b * eb);
            n += b - a;
        }
        *N = vec ? 1 : n;
        *K = vec ? n : K0;
        return out;
    }
    GB_CHECK(s.c0 >= 0 && s.c1 <= K0 && s.c0 < s.c1, "tensor '" + t.name + "': bad column slice");
    const int64_t b0 = row_bytes(t.type, s.c0), b1 = row_bytes(t.type, s.c1);
    out.resize((size_t)((b1 - b0) * N0));
    for (int64_t r = 0; r < N0; ++r)
        std::memcpy(out.data() + r * (b1 - b0), t.data + r * rb + b0, (size_t)(b1 - b0));
    *N = N0;
    *K = s.c1 - s.c0;
    return out;
}

}  // namespace

// Upload every tensor with a GGUF payload: quantized matrices are repacked into the SoA layout
// (aligned quants + fp16 scale rows), everything else is copied as is.  Under tensor
// parallelism each rank uploads only its slices.
void Executor::upload_weights() {
    size_t staging_bytes = 0;
    for (auto& [id, t] : g_->tensors)
        if (t.data && is_quant(t.type)) staging_bytes = std::max<size_t>(staging_bytes, t.data_size);
    uint8_t* staging = nullptr;
    if (staging_bytes) GB_CUDA(cudaMalloc(&staging, staging_bytes));
    for (auto& [id, t0] : g_->tensors) {
        if (!t0.data || t0.data_size == 0) continue;
        GTensor t = t0;
        std::vector<uint8_t> part;
        auto sl = tp_.slices.find(id);
        if (sl != tp_.slices.end()) {
            int64_t n = 0, k = 0;
            part = slice_payload(t0, sl->second, &n, &k);
            t.data = part.data();
            t.data_size = part.size();
            t.file_ne[0] = k;
            t.file_ne[1] = n;
            t.file_ne[2] = t.file_ne[3] = 1;
        }
        if (is_quant(t.type)) {
            const int64_t K = t.file_ne[0];
            const int64_t N = t.file_ne[1] * t.file_ne[2] * t.file_ne[3];
            QWeight w;
            w.type = t.type;
            w.N = N;
            w.K = K;
            GB_CHECK(K % QK == 0, "tensor '" + t.name + "': row length is not a multiple of 32");
            const size_t qbytes = (size_t)(N * qrow_bytes(t.type, K));
            void* qs = nullptr;
            GB_CUDA(cudaMalloc(&qs, qbytes));
            weight_allocs_.push_back(qs);
            GB_CUDA(cudaMemcpyAsync(staging, t.data, t.data_size, cudaMemcpyHostToDevice, stream_));
            launch_repack_blocks(staging, t.type, N, K, qs, stream_);
            GB_CUDA(cudaStreamSynchronize(stream_));
            w.qs = qs;
            qweights_[id] = w;
            weight_bytes_ += qbytes;
        } else {
            void* p = nullptr;
            GB_CUDA(cudaMalloc(&p, t.data_size));
            weight_allocs_.push_back(p);
            GB_CUDA(cudaMemcpy(p, t.data, t.data_size, cudaMemcpyHostToDevice));
            consts_[id] = (char*)p;
            weight_bytes_ += t.data_size;
            if (t.type == T_F32 || t.type == T_F16) {
                QWeight w;
                w.type = t.type;
                w.K = t.file_ne[0];
                w.N = t.file_ne[1] * t.file_ne[2] * t.file_ne[3];
                w.qs = p;
                qweights_[id] = w;
            }
        }
    }
    if (staging) cudaFree(staging);
    if (tp_.vocab_w != UINT32_MAX) {
        const QWeight& w = qweights_.at(tp_.vocab_w);
        tp_vocab_view_ = w;
        tp_vocab_view_.N = tp_.vocab_rows;
        tp_vocab_view_.qs = (const char*)w.qs + tp_.rank * tp_.vocab_rows * qrow_bytes(w.type, w.K);
    }
}

// ------------------------------------------------------------------------------ KV cache

void Executor::init_kv_cache(int64_t max_ctx) {
    if (kv_enabled_) return;
    alloc_kv(1, max_ctx);
}

void Executor::alloc_kv(int64_t slots, int64_t max_ctx, int64_t paged) {
    // enable rule of the reference (executor.cpp:505-539)
    bool has_rope = false, has_pos_sym = false, has_pos_in = false, has_arange = false;
    for (auto& op : g_->ops) has_rope |= op.opcode == OP_ROPE;
    for (auto& s : g_->symbol_table) has_pos_sym |= s == "pos";
    for (uint32_t id : g_->inputs) {
        auto it = g_->tensors.find(id);
        if (it != g_->tensors.end() &&
            (it->second.name == "position_ids" || it->second.name.find("pos") != std::string::npos))
            has_pos_in = true;
    }
    for (auto& [id, t] : g_->tensors)
        if (t.name.find("arange") != std::string::npos && t.data) has_arange = true;
    if (!has_rope && !has_pos_sym && !has_arange && !has_pos_in) return;
    SymEnv env;
    env["s"] = 1;
    for (auto& s : g_->symbol_table) env[s] = 1;
    std::map<uint32_t, KVCache> caches;
    for (auto& op : g_->ops) {
        if (op.opcode != OP_FLASH_ATTN_EXT) continue;
        const GTensor& k = g_->t(op.inputs.at(1));
        KVCache c;
        c.hd = k.ne[0]->eval(env);
        c.Hkv = k.ne[2]->eval(env);
        c.batch = k.ne[3]->eval(env);
        c.ctx = max_ctx;
        c.slots = slots;
        GB_CHECK(c.batch == 1, "KV caches with a graph batch dimension are not supported");
        caches[op.id] = c;
    }
    if (caches.empty()) return;
    int64_t pages = 0;
    if (paged) {
        // page bytes: T positions of K and V in every layer
        const int64_t T = tokens_per_page_;
        int64_t pb = 0;
        for (auto& [id, c] : caches) pb += 2 * c.Hkv * T * c.hd * 2;
        const int64_t per_seq = (max_ctx + T - 1) / T;
        if (kv_pool_want_ > 0) {
            pages = kv_pool_want_;
        } else {
            const int64_t warm = prefix_pool_want_ > 0
                                     ? prefix_pool_want_
                                     : std::min(std::max<int64_t>(1, (2LL << 30) / pb), paged * per_seq);
            pages = paged * per_seq + warm;
        }
        GB_CHECK(pages >= 1, "paged KV: the pool needs at least one page");
        GB_CHECK((size_t)((paged + 1) * per_seq) * 4 <= kMaxPtabBytes,
                 "paged KV: page table larger than " + std::to_string(kMaxPtabBytes) +
                     " bytes; raise tokens_per_page");
        pages += 1;  // + the scratch page 0
    }
    for (auto& [id, c] : caches) {
        c.elems = paged ? pages * c.Hkv * tokens_per_page_ * c.hd : c.hd * c.Hkv * slots * max_ctx;
        const size_t bytes = (size_t)c.elems * 2;
        GB_CUDA(cudaMalloc(&c.k, bytes));
        GB_CUDA(cudaMalloc(&c.v, bytes));
        GB_CUDA(cudaMemset(c.k, 0, bytes));
        GB_CUDA(cudaMemset(c.v, 0, bytes));
        kv_[id] = c;
    }
    if (paged) {
        int shift = 0;
        while ((int64_t(1) << shift) < tokens_per_page_) ++shift;
        page_shift_ = shift;
        ptab_stride_ = (int32_t)((max_ctx + tokens_per_page_ - 1) / tokens_per_page_);
        h_ptab_.assign((size_t)((paged + 1) * ptab_stride_), 0);
        GB_CUDA(cudaMalloc(&d_ptab_, h_ptab_.size() * 4));
        GB_CUDA(cudaMemset(d_ptab_, 0, h_ptab_.size() * 4));
        if (!ptab_ring_) {
            GB_CUDA(cudaMallocHost(&ptab_ring_, (size_t)kPtabRing * kMaxPtabBytes));
            for (cudaEvent_t& ev : ptab_ev_)
                GB_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        }
        page_ref_.assign((size_t)pages, 0);
        page_ref_[0] = 1;  // the scratch page is never handed out
        free_pages_.clear();
        for (int64_t p = pages - 1; p >= 1; --p) free_pages_.push_back((int32_t)p);
        slot_pages_.assign((size_t)paged, {});
        slot_live_.assign((size_t)paged, 0);
        ptab_dirty_ = false;
        ++pool_gen_;
    }
    kv_max_ctx_ = max_ctx;
    kv_enabled_ = true;
}

void Executor::set_decode_chain(bool on) {
    int coop = 0;
    GB_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev_));
    GB_CHECK(!on || coop, "decode chains need cooperative launch, which this device lacks");
    if (on == chain_enabled_) return;
    GB_CUDA(cudaStreamSynchronize(stream_));
    for (auto& [k, p] : programs_) free_program(*p);
    programs_.clear();
    active_.reset();
    chain_enabled_ = on;
}

void Executor::free_kv() {
    GB_CUDA(cudaStreamSynchronize(stream_));
    for (auto& [k, p] : programs_) free_program(*p);
    programs_.clear();
    active_.reset();
    for (auto& [id, c] : kv_) {
        cudaFree(c.k);
        cudaFree(c.v);
    }
    kv_.clear();
    kv_enabled_ = false;
    paged_ = false;
    if (d_ptab_) cudaFree(d_ptab_);
    d_ptab_ = nullptr;
    h_ptab_.clear();
    page_ref_.clear();
    free_pages_.clear();
    slot_pages_.clear();
    slot_live_.clear();
    ptab_dirty_ = false;
    ++pool_gen_;
}

void Executor::init_paged_kv_cache(int64_t max_batch, int64_t max_ctx) {
    GB_CHECK(max_batch >= 1 && max_batch <= kMaxRows, "paged KV: max_batch must be 1..16");
    GB_CHECK(max_ctx >= 1, "paged KV: max_ctx must be positive");
    if (kv_enabled_) free_kv();
    alloc_kv(max_batch + 1, max_ctx, max_batch);  // + the scratch slot of padding rows
    GB_CHECK(kv_enabled_, "paged KV: the graph has no attention over a KV cache");
    paged_ = true;
    paged_max_batch_ = max_batch;
    paged_max_ctx_ = max_ctx;
}

void Executor::paged_kv_alloc_slot(int64_t slot) {
    GB_CHECK(paged_, "paged KV cache not initialised");
    GB_CHECK(slot >= 0 && slot < paged_max_batch_, "paged KV: slot out of range");
    GB_CHECK(!slot_live_[(size_t)slot], "paged KV: slot already allocated");
    slot_live_[(size_t)slot] = 1;
}

void Executor::paged_kv_free_slot(int64_t slot) {
    GB_CHECK(paged_, "paged KV cache not initialised");
    GB_CHECK(slot >= 0 && slot < paged_max_batch_, "paged KV: slot out of range");
    auto& pages = slot_pages_[(size_t)slot];
    for (int32_t pg : pages) kv_page_release(pg);
    pages.clear();
    std::fill(h_ptab_.begin() + slot * ptab_stride_, h_ptab_.begin() + (slot + 1) * ptab_stride_, 0);
    ptab_dirty_ = true;
    slot_live_[(size_t)slot] = 0;
}

int32_t Executor::take_free_page() {
    GB_CHECK(!free_pages_.empty(), "paged KV: the page pool is exhausted (" +
                                       std::to_string(page_ref_.size() - 1) + " pages)");
    const int32_t pg = free_pages_.back();
    free_pages_.pop_back();
    return pg;
}

void Executor::paged_kv_ensure_tokens(int64_t slot, int64_t total) {
    GB_CHECK(paged_, "paged KV cache not initialised");
    GB_CHECK(slot >= 0 && slot < paged_max_batch_ && slot_live_[(size_t)slot],
             "paged KV: slot not allocated");
    GB_CHECK(total >= 0 && total <= kv_max_ctx_,
             "paged KV: " + std::to_string(total) + " tokens exceed max_ctx " +
                 std::to_string(kv_max_ctx_));
    const int64_t need = (total + tokens_per_page_ - 1) / tokens_per_page_;
    auto& pages = slot_pages_[(size_t)slot];
    while ((int64_t)pages.size() < need) {
        const int32_t pg = take_free_page();
        page_ref_[(size_t)pg] = 1;
        h_ptab_[(size_t)(slot * ptab_stride_) + pages.size()] = pg;
        pages.push_back(pg);
        ptab_dirty_ = true;
    }
}

int64_t Executor::paged_active_vram_bytes() const {
    if (!paged_) return 0;
    std::vector<char> mapped(page_ref_.size(), 0);
    int64_t n = 0;
    for (auto& pages : slot_pages_)
        for (int32_t pg : pages)
            if (!mapped[(size_t)pg]) {
                mapped[(size_t)pg] = 1;
                ++n;
            }
    return n * kv_page_bytes();
}

int64_t Executor::kv_page_bytes() const {
    int64_t b = 0;
    for (auto& [id, c] : kv_) b += 2 * c.Hkv * tokens_per_page_ * c.hd * 2;
    return b;
}

void Executor::configure_prefix_pool(int64_t pages) {
    GB_CHECK(pages >= 0, "prefix pool: page count must not be negative");
    prefix_pool_want_ = pages;
}

void Executor::configure_kv_pool_pages(int64_t pages) {
    GB_CHECK(pages >= 0, "paged KV: page count must not be negative");
    kv_pool_want_ = pages;
}

int64_t Executor::kv_pool_pages() const { return paged_ ? (int64_t)page_ref_.size() - 1 : 0; }
int64_t Executor::kv_free_pages() const { return paged_ ? (int64_t)free_pages_.size() : 0; }

int64_t Executor::paged_kv_slot_pages(int64_t slot) const {
    GB_CHECK(paged_ && slot >= 0 && slot < paged_max_batch_, "paged KV: slot out of range");
    return (int64_t)slot_pages_[(size_t)slot].size();
}

int64_t Executor::kv_slot_page(int64_t slot, int64_t index) const {
    GB_CHECK(paged_ && slot >= 0 && slot < paged_max_batch_, "paged KV: slot out of range");
    const auto& pages = slot_pages_[(size_t)slot];
    GB_CHECK(index >= 0 && index < (int64_t)pages.size(), "paged KV: page index out of range");
    return pages[(size_t)index];
}

void Executor::kv_page_retain(int64_t page) {
    GB_CHECK(paged_ && page >= 1 && page < (int64_t)page_ref_.size() && page_ref_[(size_t)page] > 0,
             "paged KV: retain of a page nobody holds");
    ++page_ref_[(size_t)page];
}

void Executor::kv_page_release(int64_t page) {
    GB_CHECK(paged_ && page >= 1 && page < (int64_t)page_ref_.size() && page_ref_[(size_t)page] > 0,
             "paged KV: release of a page nobody holds");
    if (--page_ref_[(size_t)page] == 0) free_pages_.push_back((int32_t)page);
}

void Executor::kv_map_page(int64_t slot, int64_t page) {
    GB_CHECK(paged_ && slot >= 0 && slot < paged_max_batch_ && slot_live_[(size_t)slot],
             "paged KV: slot not allocated");
    auto& pages = slot_pages_[(size_t)slot];
    GB_CHECK((int64_t)pages.size() < ptab_stride_, "paged KV: the slot's table is full");
    kv_page_retain(page);
    h_ptab_[(size_t)(slot * ptab_stride_) + pages.size()] = (int32_t)page;
    pages.push_back((int32_t)page);
    ptab_dirty_ = true;
}

// copy-on-write: page `index` of the slot is replaced by a fresh page holding the same rows of
// every layer (one device copy per layer and K / V: pages are contiguous in each pool)
void Executor::kv_make_private(int64_t slot, int64_t index) {
    const int64_t old = kv_slot_page(slot, index);
    if (page_ref_[(size_t)old] == 1) return;  // the slot is its only holder
    const int32_t pg = take_free_page();
    page_ref_[(size_t)pg] = 1;
    for (auto& [id, c] : kv_) {
        const int64_t pe = c.Hkv * tokens_per_page_ * c.hd;
        for (__half* pool : {c.k, c.v})
            GB_CUDA(cudaMemcpyAsync(pool + pg * pe, pool + old * pe, (size_t)pe * 2,
                                    cudaMemcpyDeviceToDevice, stream_));
    }
    kv_page_release(old);
    slot_pages_[(size_t)slot][(size_t)index] = pg;
    h_ptab_[(size_t)(slot * ptab_stride_ + index)] = pg;
    ptab_dirty_ = true;
}

// the host table into the device table, ordered on the stream before the next launch; each
// upload goes through its own pinned copy that no queued transfer still reads
void Executor::sync_page_table() {
    if (!ptab_dirty_) return;
    const size_t bytes = h_ptab_.size() * 4;
    int32_t* stage = ptab_ring_ + (size_t)ptab_next_ * (kMaxPtabBytes / 4);
    GB_CUDA(cudaEventSynchronize(ptab_ev_[ptab_next_]));
    std::memcpy(stage, h_ptab_.data(), bytes);
    GB_CUDA(cudaMemcpyAsync(d_ptab_, stage, bytes, cudaMemcpyHostToDevice, stream_));
    GB_CUDA(cudaEventRecord(ptab_ev_[ptab_next_], stream_));
    ptab_next_ = (ptab_next_ + 1) % kPtabRing;
    ptab_dirty_ = false;
}

void Executor::set_output_rows(const std::vector<int32_t>& rows) {
    GB_CHECK((int)rows.size() <= kMaxOutRows, "output rows: at most 64");
    out_rows_ = rows;
}

void Executor::set_tokens_per_page(int64_t n) {
    GB_CHECK(n >= 1 && n <= 65536 && (n & (n - 1)) == 0,
             "tokens_per_page must be a power of two (1 .. 65536)");
    if (n == tokens_per_page_) return;
    if (!paged_) {
        tokens_per_page_ = n;
        return;
    }
    for (char live : slot_live_) GB_CHECK(!live, "tokens_per_page: a slot is in use");
    const int64_t mb = paged_max_batch_, mc = paged_max_ctx_;
    tokens_per_page_ = n;
    init_paged_kv_cache(mb, mc);  // the pool is laid out again (the prefix cache starts empty)
}

void Executor::prepare_batch(int rows, const int32_t* pos, const int32_t* slot) {
    GB_CHECK(paged_, "batched decode needs init_paged_kv_cache");
    GB_CHECK(rows >= 1 && rows <= kMaxRows, "batched decode: 1..16 rows");
    for (int r = 0; r < rows; ++r) {
        GB_CHECK(slot[r] >= 0 && slot[r] <= paged_max_batch_, "batched decode: bad slot");
        GB_CHECK(pos[r] >= 0 && pos[r] < kv_max_ctx_, "batched decode: position outside the cache");
        if (slot[r] < paged_max_batch_)  // the scratch slot's table points at the scratch page
            GB_CHECK(slot_live_[(size_t)slot[r]] &&
                         pos[r] < (int64_t)slot_pages_[(size_t)slot[r]].size() * tokens_per_page_,
                     "batched decode: position " + std::to_string(pos[r]) + " of slot " +
                         std::to_string(slot[r]) + " has no page (paged_kv_ensure_tokens)");
    }
    SymEnv env;
    env["s"] = rows;
    env["__rows"] = rows;
    env["pos"] = 0;
    for (auto& s : g_->symbol_table)
        if (!env.count(s)) env[s] = rows;  // the sequence symbol(s) of the graph
    prepare(env, true);
    for (int r = 0; r < rows; ++r) {
        h_step_->row_pos[r] = pos[r];
        h_step_->row_slot[r] = slot[r];
    }
}

void Executor::reset_kv_cache() {
    for (auto& [id, c] : kv_) {
        const size_t bytes = (size_t)c.elems * 2;
        GB_CUDA(cudaMemsetAsync(c.k, 0, bytes, stream_));
        GB_CUDA(cudaMemsetAsync(c.v, 0, bytes, stream_));
    }
}

// Host table of (cos, sin) for positions 0..n_pos-1, computed exactly as ggml_rope_cache_init
// does on the CPU (ops.cpp:5910-5923): theta starts at the position, is multiplied by
// theta_scale = powf(base, -2/n_dims) once per pair in fp32, and cosf/sinf come from libm.
const float2* Executor::rope_table(int n_dims, float freq_base, float freq_scale, int64_t* n_pos,
                                   float* theta_scale) {
    const float ts = powf(freq_base, -2.0f / (float)n_dims);
    *theta_scale = ts;
    const int64_t np = std::max<int64_t>(4096, kv_max_ctx_);
    char key[96];
    snprintf(key, sizeof(key), "%d/%a/%a/%lld", n_dims, freq_base, freq_scale, (long long)np);
    auto it = rope_tabs_.find(key);
    if (it != rope_tabs_.end()) {
        *n_pos = it->second.second.first;
        return it->second.first;
    }
    const int half = n_dims / 2;
    std::vector<float2> h((size_t)(np * half));
    for (int64_t p = 0; p < np; ++p) {
        float theta = (float)p;
        for (int i = 0; i < half; ++i) {
            const float th = freq_scale * theta;
            h[(size_t)(p * half + i)] = make_float2(cosf(th), sinf(th));
            theta *= ts;
        }
    }
    float2* d = nullptr;
    GB_CUDA(cudaMalloc(&d, h.size() * sizeof(float2)));
    GB_CUDA(cudaMemcpy(d, h.data(), h.size() * sizeof(float2), cudaMemcpyHostToDevice));
    rope_tabs_[key] = {d, {np, ts}};
    *n_pos = np;
    return d;
}

// ------------------------------------------------------------------------------ lowering

std::shared_ptr<Program> Executor::build(const SymEnv& env, bool kv) {
    auto P = std::make_shared<Program>();
    Program& pg = *P;
    pg.env = env;
    pg.kv = kv;
    pg.batch = env.count("__rows") != 0;
    const Graph& G = *g_;
    const int nops = (int)G.ops.size();

    // concrete shapes
    std::map<uint32_t, std::array<int64_t, 4>> shape;
    for (auto& [id, t] : G.tensors) {
        std::array<int64_t, 4> ne{1, 1, 1, 1};
        for (int d = 0; d < 4; ++d) ne[d] = t.ne[d] ? t.ne[d]->eval(env) : 1;
        shape[id] = ne;
    }
    // consumers (op indices) per tensor
    std::map<uint32_t, std::vector<int>> consumers;
    for (int i = 0; i < nops; ++i)
        for (uint32_t in : G.ops[i].inputs) consumers[in].push_back(i);
    std::set<uint32_t> outputs(G.outputs.begin(), G.outputs.end());
    auto& vals = pg.vals;

    // graph inputs: persistent device buffers sized for this program
    for (uint32_t id : G.inputs) {
        const GTensor& t = G.t(id);
        Val v;
        v.type = t.type;
        for (int d = 0; d < 4; ++d) v.ne[d] = shape[id][d];
        set_contig(v);
        const size_t bytes = (size_t)(nelem(v.ne) * v.nb[0]);
        char* p = nullptr;
        GB_CUDA(cudaMalloc(&p, std::max<size_t>(bytes, 16)));
        pg.owned.push_back(p);
        pg.input_bufs[id] = p;
        v.ref.fixed = p;
        vals[id] = v;
    }
    // weights / constants
    auto weight_val = [&](uint32_t id) -> Val {
        const GTensor& t = G.t(id);
        Val v;
        v.type = t.type;
        for (int d = 0; d < 4; ++d) v.ne[d] = shape[id][d];
        auto qw = qweights_.find(id);
        if (qw != qweights_.end() && is_quant(t.type)) {
            v.w = &qw->second;
            v.has_f = false;
            return v;
        }
        auto c = consts_.find(id);
        GB_CHECK(c != consts_.end(), "tensor '" + t.name + "' has no data");
        if (qw != qweights_.end()) v.w = &qw->second;
        set_contig(v);
        v.ref.fixed = c->second;
        // the arange constant is offset by pos when the KV cache is in use (executor.cpp:2854)
        return v;
    };
    auto get = [&](uint32_t id) -> Val& {
        auto it = vals.find(id);
        if (it != vals.end()) return it->second;
        const GTensor& t = G.t(id);
        GB_CHECK(t.data != nullptr, "tensor '" + t.name + "' (id " + std::to_string(id) +
                                        ") is used before it is produced");
        vals[id] = weight_val(id);
        return vals[id];
    };

    auto add = [&](const std::string& name, Launch fn, double bytes = 0.0) {
        pg.launches.push_back(std::move(fn));
        pg.launch_names.push_back(name);
        pg.launch_bytes.push_back(bytes);
        pg.chain_descs.emplace_back();
        pg.launch_w.emplace_back();
    };
    // the last added launch streams the quantized weight qw (F: SwiGLU half width, 0: plain)
    auto streams = [&](const QWeight* qw, int64_t F) {
        pg.launch_w.back() = PfNext{qw->qs, qw->type, qw->N, qw->K, F};
    };
    // the last added launch can also run as an op of a decode chain
    auto chainable = [&](ChainDesc d) { pg.chain_descs.back() = std::move(d); };
    // algorithmic bytes of a quantized matmul: weight quants + scales once, Q8_0 activations,
    // f32 outputs (and residual reads)
    auto mm_bytes = [](const QWeight* w, int64_t M, bool residual) {
        const double wb = w->type == T_Q8_0 ? (double)w->N * w->K * (34.0 / 32.0)
                                            : (double)w->N * w->K * (18.0 / 32.0);
        return wb + (double)M * w->K * (34.0 / 32.0) + (double)M * w->N * 4.0 * (residual ? 2 : 1);
    };
    auto alloc = [&](Val& v, int op) {
        set_contig(v);
        v.ref = BufRef{};
        v.ref.buf = pg.new_buf(nelem(v.ne) * v.nb[0], op);
    };
    // Q8_0 rows for a value (rows of ne0); emits a quantize launch unless already present
    auto ensure_q = [&](Val& x, int op) {
        if (x.has_q) {
            pg.use(x.q, op);
            pg.use(x.qd, op);
            return;
        }
        GB_CHECK(x.has_f && x.type == T_F32, "matmul input is not f32");
        GB_CHECK(x.nb[0] == 4 && x.rows_uniform(), "matmul input rows are not uniform");
        const int64_t M = x.nrows(), K = x.ne[0];
        x.q.buf = pg.new_buf(M * K, op);
        x.qd.buf = pg.new_buf(M * (K / QK) * 4, op);
        x.has_q = true;
        pg.use(x.ref, op);
        const BufRef src = x.ref, qb = x.q, qdb = x.qd;
        const int64_t stride = x.nb[1] / 4;
        add("quantize_q8_0", [=](Program& p, cudaStream_t st) {
            launch_quantize_q8_0((const float*)p.ptr(src), stride, M, K, (int8_t*)p.ptr(qb),
                                 (float*)p.ptr(qdb), st);
        });
        if (chain_row_ok(M, K))
            chainable([=](const Program& p, ChainOp& c) {
                c.kind = CH_ROW;
                c.xf = (const float*)p.ptr(src);
                c.D = K;
                c.yq = (int8_t*)p.ptr(qb);
                c.yd = (float*)p.ptr(qdb);
                return true;
            });
    };
    auto cont = [&](Val x, int op) -> Val {
        Val y;
        y.type = x.type == T_F16 ? T_F16 : (x.type == T_I32 ? T_I32 : T_F32);
        for (int d = 0; d < 4; ++d) y.ne[d] = x.ne[d];
        alloc(y, op);
        pg.use(x.ref, op);
        const Val xs = x, ys = y;
        add("cont", [=](Program& p, cudaStream_t st) { launch_copy(p.view(xs), p.view(ys), st); });
        return y;
    };
    // which consumers need f32 / Q8_0 of tensor id
    auto needs = [&](uint32_t id, bool& need_f, bool& need_q) {
        need_f = outputs.count(id) != 0;
        need_q = false;
        for (int ci : consumers[id]) {
            const GOp& c = G.ops[ci];
            const bool qmm = c.opcode == OP_MUL_MAT && c.inputs.size() >= 2 && c.inputs[1] == id &&
                             is_quant(G.t(c.inputs[0]).type) && c.inputs[0] != id;
            if (qmm && !((logits_last_only_ || !out_rows_.empty()) && outputs.count(c.outputs[0])))
                need_q = true;
            else need_f = true;
        }
        if (!need_f && !need_q) need_f = true;
    };

    // tensor-parallel exchanges (NCCL on the executor's stream; captured with the program)
    ncclComm_t comm = (ncclComm_t)nccl_;
    // partial sums that fit the peer buffers (decode) take the one-shot peer all-reduce, larger
    // ones (prefill) NCCL's
    const TpPeers peers = ar_peers_;
    const int tp_rank = tp_.rank;
    uint32_t* const ar_epochs = ar_epochs_;
    int* const ar_err = ar_err_;
    const int64_t ar_cap = ar_cap_;
    auto tp_allreduce = [&](const Val& y) {
        const BufRef r = y.ref;
        const size_t n = (size_t)nelem(y.ne);
        const int T = tp_.size;
        if ((int64_t)n <= ar_cap) {
            add("allreduce_peer", [=](Program& p, cudaStream_t st) {
                launch_tp_allreduce((float*)p.ptr(r), (int64_t)n, peers, tp_rank, T, ar_epochs,
                                    ar_cap, ar_err, st);
            }, 8.0 * (double)n);
            return;
        }
        add("allreduce", [=](Program& p, cudaStream_t st) {
            float* d = (float*)p.ptr(r);
            GB_NCCL(all_reduce(d, d, n, ncclFloat32, ncclSum, comm, st));
        }, 8.0 * (double)n);
    };
    const int tp_n = tp_.size;
    auto tp_gather = [&](const Val& yl, int op) -> Val {
        Val yf = yl;
        yf.ne[0] = yl.ne[0] * tp_n;
        alloc(yf, op);
        const int64_t Vr = yl.ne[0], M = yl.nrows();
        const BufRef lr = yl.ref, fr = yf.ref;
        BufRef gr;
        if (M > 1) gr.buf = pg.new_buf(Vr * M * tp_n * 4, op);
        add("allgather", [=](Program& p, cudaStream_t st) {
            if (M == 1) {
                GB_NCCL(all_gather(p.ptr(lr), p.ptr(fr), (size_t)Vr, ncclFloat32, comm, st));
                return;
            }
            // rank-major [rank][M][Vr] -> row-major [M][rank * Vr + j]
            GB_NCCL(all_gather(p.ptr(lr), p.ptr(gr), (size_t)(Vr * M), ncclFloat32, comm, st));
            TView src, dst;
            src.data = p.ptr(gr);
            dst.data = p.ptr(fr);
            src.type = dst.type = T_F32;
            const int64_t ne[4] = {Vr, M, tp_n, 1};
            const int64_t sb[4] = {4, Vr * 4, Vr * M * 4, Vr * M * tp_n * 4};
            const int64_t db[4] = {4, Vr * tp_n * 4, Vr * 4, Vr * M * tp_n * 4};
            for (int d = 0; d < 4; ++d) {
                src.ne[d] = dst.ne[d] = ne[d];
                src.nb[d] = sb[d];
                dst.nb[d] = db[d];
            }
            launch_copy(src, dst, st);
        }, 8.0 * (double)(Vr * M * tp_n));
        return yf;
    };

    std::set<int> skip;  // ops folded into an earlier launch
    for (int oi = 0; oi < nops; ++oi) {
        if (skip.count(oi)) continue;
        const GOp& op = G.ops[oi];
        GB_CHECK(!op.outputs.empty(), "op without outputs");
        const uint32_t out = op.outputs[0];
        const auto& one = shape[out];
        auto in = [&](size_t k) -> Val& { return get(op.inputs.at(k)); };
        for (uint32_t iid : op.inputs) {
            Val& iv = get(iid);
            pg.use(iv.ref, oi);
            if (iv.has_q) {
                pg.use(iv.q, oi);
                pg.use(iv.qd, oi);
            }
            if (iv.virt_rms) pg.use(iv.rms_x, oi);
            if (iv.virt_rope) pg.use(iv.rsrc, oi);
        }
        Val o;
        o.type = T_F32;
        for (int d = 0; d < 4; ++d) o.ne[d] = one[d];

        switch (op.opcode) {
            case OP_GET_ROWS: {
                Val& w = in(0);
                Val ids = in(1);
                GB_CHECK(w.w, "GET_ROWS table must be a weight tensor");
                GB_CHECK(ids.type == T_I32, "GET_ROWS indices must be int32");
                if (!ids.contiguous()) ids = cont(ids, oi);
                const int64_t n = nelem(ids.ne);
                alloc(o, oi);
                const QWeight* qw = w.w;
                const BufRef ir = ids.ref, orf = o.ref;
                const int64_t K = qw->K;
                add("get_rows", [=](Program& p, cudaStream_t st) {
                    launch_get_rows(*qw, (const int32_t*)p.ptr(ir), n, (float*)p.ptr(orf), K, st);
                });
                break;
            }
            case OP_RMS_NORM_C:
            case OP_RMS_NORM:
            case OP_LAYER_NORM:
            case OP_NORM: {
                Val x = in(0);
                if (!(x.nb[0] == 4 && x.rows_uniform())) x = cont(x, oi);
                const float eps = (float)op.f("eps", 1e-5);
                const float* gamma = nullptr;
                const float* beta = nullptr;
                if (op.inputs.size() > 1) gamma = (const float*)get(op.inputs[1]).ref.fixed;
                if (op.inputs.size() > 2) beta = (const float*)get(op.inputs[2]).ref.fixed;
                bool nf, nq;
                needs(out, nf, nq);
                const int64_t D = x.ne[0], M = x.nrows();
                const bool rms_op = op.opcode == OP_RMS_NORM_C || op.opcode == OP_RMS_NORM;
                const bool fits = M >= 1 && gemv_fits(T_Q8_0, D, (int)M, true, gamma) &&
                                  gemv_fits(T_Q4_0, D, (int)M, true, gamma);
                if (rms_op && !nf && nq && M <= kGemvRouteRows && fits) {
                    // decode: every consumer is a quantized GEMV that normalizes in its prologue
                    o.has_f = false;
                    o.virt_rms = true;
                    o.rms_x = x.ref;
                    o.rms_stride = x.nb[1] / 4;
                    o.rms_eps = eps;
                    o.rms_gamma = gamma;
                    o.ne[0] = D;
                    break;
                }
                if (nf) alloc(o, oi);
                else o.has_f = false;
                if (nq) {
                    o.q.buf = pg.new_buf(M * D, oi);
                    o.qd.buf = pg.new_buf(M * (D / QK) * 4, oi);
                    o.has_q = true;
                }
                const BufRef xr = x.ref, orf = o.ref, qr = o.q, qdr = o.qd;
                const int64_t xs = x.nb[1] / 4;
                const bool rms = op.opcode == OP_RMS_NORM_C || op.opcode == OP_RMS_NORM;
                const bool hf = o.has_f, hq = o.has_q;
                add(rms ? "rms_norm" : "layer_norm", [=](Program& p, cudaStream_t st) {
                    float* y = hf ? (float*)p.ptr(orf) : nullptr;
                    int8_t* yq = hq ? (int8_t*)p.ptr(qr) : nullptr;
                    float* yd = hq ? (float*)p.ptr(qdr) : nullptr;
                    if (rms)
                        launch_rms_norm((const float*)p.ptr(xr), xs, M, D, eps, gamma, y, D, yq, yd, st);
                    else
                        launch_layer_norm((const float*)p.ptr(xr), xs, M, D, eps, gamma, beta, y, D,
                                          yq, yd, st);
                });
                if (rms && chain_row_ok(M, D))
                    chainable([=](const Program& p, ChainOp& c) {
                        c.kind = CH_ROW;
                        c.xf = (const float*)p.ptr(xr);
                        c.D = D;
                        c.rms = 1;
                        c.eps = eps;
                        c.gamma = gamma;
                        c.y = hf ? (float*)p.ptr(orf) : nullptr;
                        c.yq = hq ? (int8_t*)p.ptr(qr) : nullptr;
                        c.yd = hq ? (float*)p.ptr(qdr) : nullptr;
                        return true;
                    });
                break;
            }
            case OP_MUL_MAT: {
                Val& wv = in(0);
                GB_CHECK(wv.w, "MUL_MAT: first operand must be a weight matrix");
                // tensor parallelism: a K-split matmul yields a partial sum (all-reduced below;
                // only rank 0 adds bias and residual); the vocabulary-split projection computes
                // this rank's rows and all-gathers the logits
                const bool tp_partial = tp_.size > 1 && tp_.partial.count(out) != 0;
                const bool tp_vocab = tp_.size > 1 && out == tp_.vocab_out;
                const bool tp_skip_add = tp_partial && tp_.rank != 0;
                const QWeight* qw = tp_vocab ? &tp_vocab_view_ : wv.w;
                Val& xin = in(1);
                const int64_t K = qw->K, N = qw->N;
                if (tp_vocab) o.ne[0] = N;
                GB_CHECK(xin.ne[0] == K, "MUL_MAT: inner dimensions differ (" +
                                             std::to_string(xin.ne[0]) + " vs " +
                                             std::to_string(K) + ")");
                int64_t M = xin.nrows();
                int64_t row0 = 0;
                // output rows: the listed rows, or the last one
                const bool sel_rows = !out_rows_.empty() && outputs.count(out) && !pg.batch;
                const bool last_only =
                    !sel_rows && logits_last_only_ && outputs.count(out) && M > 1 && !pg.batch;
                const int64_t n_sel = sel_rows ? (int64_t)out_rows_.size() : 0;
                if (last_only || sel_rows) {
                    row0 = M - 1;
                    o.ne[1] = last_only ? 1 : n_sel;
                    o.ne[2] = 1;
                    o.ne[3] = 1;
                }
                const int64_t Mrun = last_only ? 1 : (sel_rows ? n_sel : M);
                // fused residual ADD: the only consumer is ADD(other, this) of equal shape
                int add_op = -1;
                const float* bias = nullptr;
                if (op.inputs.size() > 2 && !tp_skip_add)
                    bias = (const float*)get(op.inputs[2]).ref.fixed;
                Val res;
                if (!outputs.count(out) && consumers[out].size() == 1 && !last_only && !sel_rows) {
                    const int ci = consumers[out][0];
                    const GOp& c = G.ops[ci];
                    if (c.opcode == OP_ADD && c.inputs.size() == 2 && c.inputs[0] != c.inputs[1]) {
                        const uint32_t other = c.inputs[0] == out ? c.inputs[1] : c.inputs[0];
                        auto ov = vals.find(other);
                        if (ov != vals.end() && ov->second.has_f && ov->second.type == T_F32 &&
                            ov->second.contiguous() && nelem(ov->second.ne) == N * M &&
                            ov->second.ne[0] == N) {
                            add_op = ci;
                            res = ov->second;
                        }
                    }
                }
                // decode (M <= 16): SwiGLU / residual epilogue fused into the matmul launch; an
                // unmaterialized RMSNorm input (M <= 4) is normalized in the GEMV prologue
                bool dec = is_quant(qw->type) && !last_only && !sel_rows &&
                           (xin.virt_rms ? Mrun <= kGemvRouteRows && gemv_fused_fits(K, (int)Mrun)
                                         : Mrun <= kMmvMaxRows);
                GB_CHECK(!xin.virt_rms || dec, "internal: unfused RMSNorm without a decode GEMV");
                // SwiGLU consumer folded into the matmul epilogue: decode, and prefill whose gate
                // and up halves split into the block GEMM's 64-unit tiles
                const bool pre = is_quant(qw->type) && !last_only && !sel_rows && !xin.virt_rms &&
                                 Mrun > kMmvMaxRows && N % 128 == 0;
                int swi_op = -1;
                if ((dec || pre) && !bias && add_op < 0 && !outputs.count(out) &&
                    consumers[out].size() == 1) {
                    const int ci = consumers[out][0];
                    const GOp& c = G.ops[ci];
                    if ((c.opcode == OP_SWIGLU || c.opcode == OP_GLU) && c.inputs.size() == 1 &&
                        c.i("swapped", 0) == 0 && N % 64 == 0 && xin.nrows() == Mrun)
                        swi_op = ci;
                }
                if (swi_op >= 0) dec = true;
                if (dec) {
                    GemvArgs ga;
                    ga.w = *qw;
                    ga.M = (int)Mrun;
                    BufRef xr, qb, qdb;
                    int64_t xs = 0;
                    const float* gamma = nullptr;
                    float eps = 0.0f;
                    const bool qpro = !xin.virt_rms && xin.q_in_prologue && !xin.has_q &&
                                      Mrun <= kGemvRouteRows && xin.nb[0] == 4 &&
                                      xin.rows_uniform() && xin.nb[1] % 16 == 0;
                    if (xin.virt_rms) {
                        xr = xin.rms_x;
                        xs = xin.rms_stride;
                        gamma = xin.rms_gamma;
                        eps = xin.rms_eps;
                        pg.use(xr, oi);
                    } else if (qpro) {
                        xr = xin.ref;
                        xs = xin.nb[1] / 4;
                        pg.use(xr, oi);
                    } else {
                        ensure_q(xin, oi);
                        qb = xin.q;
                        qdb = xin.qd;
                    }
                    const bool virt = xin.virt_rms || qpro;
                    const bool xrms = xin.virt_rms;
                    const double bytes = mm_bytes(qw, Mrun, add_op >= 0);
                    if (swi_op >= 0) {
                        const uint32_t sout = G.ops[swi_op].outputs[0];
                        Val h;
                        h.type = T_F32;
                        for (int d = 0; d < 4; ++d) h.ne[d] = shape[sout][d];
                        const int64_t F = N / 2;
                        GB_CHECK(h.ne[0] == F, "SwiGLU output width mismatch");
                        bool nf, nq;
                        needs(sout, nf, nq);
                        if (nq && !nf && Mrun <= kGemvRouteRows) {
                            // 1-2 rows: the down GEMV quantizes the f32 rows in its prologue, so
                            // the gate_up GEMV can split its rows at any pair (no Q8_0 block
                            // of the output has to come from one CTA)
                            nf = true;
                            nq = false;
                            h.q_in_prologue = true;
                        }
                        if (nf) alloc(h, oi);
                        else h.has_f = false;
                        if (nq) {
                            h.q.buf = pg.new_buf(Mrun * F, oi);
                            h.qd.buf = pg.new_buf(Mrun * (F / QK) * 4, oi);
                            h.has_q = true;
                        }
                        const BufRef hr = h.ref, hq = h.q, hqd = h.qd;
                        const bool hf = h.has_f, hhq = h.has_q;
                        const size_t li = pg.launches.size();  // this launch's index
                        auto mk = [=](const Program& p) {
                            GemvArgs a = ga;
                            if (li < p.launch_pf.size()) a.pf = p.launch_pf[li];
                            if (virt) {
                                a.xf = (const float*)p.ptr(xr);
                                a.xf_stride = xs;
                                a.xf_rms = xrms;
                                a.eps = eps;
                                a.gamma = gamma;
                            } else {
                                a.xq = (const int8_t*)p.ptr(qb);
                                a.xd = (const float*)p.ptr(qdb);
                            }
                            a.swiglu = true;
                            a.F = F;
                            if (hf) {
                                a.y = (float*)p.ptr(hr);
                                a.y_stride = F;
                            }
                            if (hhq) {
                                a.yq = (int8_t*)p.ptr(hq);
                                a.yd = (float*)p.ptr(hqd);
                            }
                            return a;
                        };
                        add(xrms ? "gemv_rms_swiglu"
                                 : (Mrun <= kGemvRouteRows ? "gemv_swiglu"
                                                         : (Mrun <= kMmvMaxRows ? "mmv_swiglu" : "gemm_swiglu")), [=](Program& p, cudaStream_t st) {
                            launch_gemv_fused(mk(p), st);
                        }, bytes);
                        streams(qw, F);
                        chainable([=](const Program& p, ChainOp& c) { return chain_gemv_op(mk(p), c); });
                        vals[sout] = h;
                        skip.insert(swi_op);
                        vals[out] = Val();  // never materialized
                        vals[out].has_f = false;
                        continue;
                    }
                    Val y = o;
                    const uint32_t out_id = add_op >= 0 ? G.ops[add_op].outputs[0] : out;
                    if (add_op >= 0)
                        for (int d = 0; d < 4; ++d) y.ne[d] = shape[out_id][d];
                    alloc(y, oi);
                    BufRef rref;
                    if (add_op >= 0 && !tp_skip_add) {
                        rref = res.ref;
                        pg.use(res.ref, add_op);
                    }
                    const BufRef yr = y.ref;
                    const size_t li = pg.launches.size();  // this launch's index
                    // one decode row of a K-split projection: the all-reduce rides in the
                    // GEMV's epilogue (no separate launch)
                    GemvAllReduce gar;
                    const bool ar_fused = tp_partial && Mrun == 1 && !pg.batch && gemv_ar_ &&
                                          N <= ar_cap && (qw->type == T_Q4_0 || qw->type == T_Q8_0);
                    if (ar_fused) {
                        gar.peers = peers;
                        gar.rank = tp_rank;
                        gar.T = tp_.size;
                        gar.epochs = ar_epochs + kArCtas;
                        gar.cap = ar_cap;
                        gar.err = ar_err;
                    }
                    auto mk = [=](const Program& p) {
                        GemvArgs a = ga;
                        a.ar = gar;
                        if (li < p.launch_pf.size()) a.pf = p.launch_pf[li];
                        if (virt) {
                            a.xf = (const float*)p.ptr(xr);
                            a.xf_stride = xs;
                            a.xf_rms = xrms;
                            a.eps = eps;
                            a.gamma = gamma;
                        } else {
                            a.xq = (const int8_t*)p.ptr(qb);
                            a.xd = (const float*)p.ptr(qdb);
                        }
                        a.y = (float*)p.ptr(yr);
                        a.y_stride = N;
                        a.bias = bias;
                        if (rref.fixed || rref.buf >= 0) {
                            a.residual = (const float*)p.ptr(rref);
                            a.res_stride = N;
                        }
                        return a;
                    };
                    add(xrms ? "gemv_rms" : (Mrun <= kGemvRouteRows ? (add_op >= 0 ? "gemv_res" : "gemv") : (add_op >= 0 ? "mmv_res" : "mmv")), [=](Program& p, cudaStream_t st) {
                        launch_gemv_fused(mk(p), st);
                    }, bytes);
                    streams(qw, 0);
                    chainable([=](const Program& p, ChainOp& c) { return chain_gemv_op(mk(p), c); });
                    if (tp_partial && !ar_fused) tp_allreduce(y);
                    if (tp_vocab) y = tp_gather(y, oi);
                    if (add_op >= 0) {
                        vals[out_id] = y;
                        skip.insert(add_op);
                    } else {
                        vals[out] = y;
                    }
                    continue;
                }
                Val y = o;
                const uint32_t out_id = add_op >= 0 ? G.ops[add_op].outputs[0] : out;
                if (add_op >= 0)
                    for (int d = 0; d < 4; ++d) y.ne[d] = shape[out_id][d];
                alloc(y, oi);
                MatmulEpilogue ep;
                ep.bias = bias;
                BufRef rref;
                if (add_op >= 0 && !tp_skip_add) {
                    rref = res.ref;
                    pg.use(res.ref, add_op);
                    ep.res_stride = N;
                }
                const BufRef yr = y.ref;
                const int64_t ystride = N;
                // the selected rows gathered into a compact f32 block first
                Val xsel;
                if (sel_rows) {
                    pg.out_rows_of = pg.out_rows_of ? std::min(pg.out_rows_of, M) : M;
                    GB_CHECK(xin.has_f, "output-row matmul needs f32 input");
                    Val x = xin;
                    if (!(x.nb[0] == 4 && x.rows_uniform())) x = cont(x, oi);
                    xsel.type = T_F32;
                    xsel.ne[0] = K;
                    xsel.ne[1] = n_sel;
                    alloc(xsel, oi);
                    pg.use(x.ref, oi);
                    const BufRef src = x.ref, dst = xsel.ref;
                    const int64_t xs = x.nb[1] / 4;
                    const int n = (int)n_sel;
                    StepParams* const dstep = d_step_;
                    add("gather_rows", [=](Program& p, cudaStream_t st) {
                        launch_gather_rows((const float*)p.ptr(src), xs, dstep, n, K,
                                           (float*)p.ptr(dst), st);
                    });
                }
                if (is_quant(qw->type)) {
                    if (sel_rows) {
                        ensure_q(xsel, oi);
                        const BufRef qb = xsel.q, qdb = xsel.qd;
                        add("gemm_q", [=](Program& p, cudaStream_t st) {
                            MatmulEpilogue e = ep;
                            launch_matmul_q(*qw, (const int8_t*)p.ptr(qb),
                                            (const float*)p.ptr(qdb), Mrun, (float*)p.ptr(yr),
                                            ystride, e, st);
                        }, mm_bytes(qw, Mrun, false));
                    } else if (last_only) {
                        // quantize only the last row (the CPU path quantizes the gathered row)
                        GB_CHECK(xin.has_f, "last-token matmul needs f32 input");
                        Val xl = xin;
                        xl.ref.off += row0 * xin.nb[1];
                        xl.ne[1] = 1;
                        xl.ne[2] = 1;
                        xl.ne[3] = 1;
                        xl.nb[2] = xl.nb[1];
                        xl.nb[3] = xl.nb[1];
                        xl.has_q = false;
                        ensure_q(xl, oi);
                        const BufRef qb = xl.q, qdb = xl.qd;
                        add("gemm_q", [=](Program& p, cudaStream_t st) {
                            MatmulEpilogue e = ep;
                            launch_matmul_q(*qw, (const int8_t*)p.ptr(qb),
                                                  (const float*)p.ptr(qdb), 1, (float*)p.ptr(yr),
                                                  ystride, e, st);
                        }, mm_bytes(qw, 1, false));
                    } else {
                        ensure_q(xin, oi);
                        const BufRef qb = xin.q, qdb = xin.qd;
                        add("gemm_q", [=](Program& p, cudaStream_t st) {
                            MatmulEpilogue e = ep;
                            if (rref.fixed || rref.buf >= 0) e.residual = (const float*)p.ptr(rref);
                            launch_matmul_q(*qw, (const int8_t*)p.ptr(qb),
                                                  (const float*)p.ptr(qdb), Mrun, (float*)p.ptr(yr),
                                                  ystride, e, st);
                        }, mm_bytes(qw, Mrun, add_op >= 0));
                    }
                } else {
                    Val x = sel_rows ? xsel : xin;
                    if (!(x.nb[0] == 4 && x.rows_uniform())) x = cont(x, oi);
                    const BufRef xr = x.ref;
                    const int64_t xs = x.nb[1] / 4;
                    const int64_t off = last_only ? row0 * x.nb[1] : 0;
                    add("matmul_f", [=](Program& p, cudaStream_t st) {
                        MatmulEpilogue e = ep;
                        if (rref.fixed || rref.buf >= 0) e.residual = (const float*)p.ptr(rref);
                        launch_matmul_f(*qw, (const float*)(p.ptr(xr) + off), xs, Mrun,
                                        (float*)p.ptr(yr), ystride, e, st);
                    });
                }
                if (tp_partial) tp_allreduce(y);
                if (tp_vocab) y = tp_gather(y, oi);
                if (add_op >= 0) {
                    vals[out_id] = y;
                    skip.insert(add_op);
                    continue;
                }
                vals[out] = y;
                continue;
            }
            case OP_VIEW: {
                Val x = in(0);
                if (!x.contiguous() && x.ref.buf >= 0 && false) x = cont(x, oi);
                const int g = (int)op.i("ggml_dim", 0);
                const int64_t start = op.i("start", 0), step = op.i("step", 1),
                              mult = op.i("offset_mult", 1);
                o = x;
                o.has_q = false;
                o.w = nullptr;
                for (int d = 0; d < 4; ++d) o.ne[d] = one[d];
                o.ref.off += start * mult * x.nb[g];
                if (g >= 1) o.nb[g] = x.nb[g] * step;
                if (g == 0) GB_CHECK(step == 1, "VIEW with a step along dim 0 is not supported");
                if (outputs.count(out) && !o.contiguous()) o = cont(o, oi);
                break;
            }
            case OP_RESHAPE: {
                Val x = in(0);
                o = x;
                o.has_q = false;
                o.w = nullptr;
                for (int d = 0; d < 4; ++d) o.ne[d] = one[d];
                GB_CHECK(nelem(o.ne) == nelem(x.ne), "RESHAPE: element count mismatch");
                if (x.contiguous()) {
                    set_contig(o);
                    // Q8_0 rows are 32-element blocks of the contiguous data: any reshape that
                    // keeps rows a multiple of 32 reuses them
                    if (x.has_q && x.ne[0] % QK == 0 && o.ne[0] % QK == 0) {
                        o.has_q = true;
                        o.q = x.q;
                        o.qd = x.qd;
                    }
                    o.has_f = x.has_f;
                    if (!o.has_f) {  // only Q8_0 rows exist: keep them
                        o.ref = x.ref;
                    }
                } else if (x.nb[0] == 4 && x.ne[0] == one[0] * one[1] && x.ne[1] == one[2] &&
                           x.ne[2] == 1 && x.ne[3] == 1 && one[3] == 1) {
                    // strided split of a fused-QKV slice (executor.cpp:80-113)
                    o.nb[0] = x.nb[0];
                    o.nb[1] = x.nb[0] * one[0];
                    o.nb[2] = x.nb[1];
                    o.nb[3] = x.nb[1] * one[2];
                } else {
                    Val c = cont(x, oi);
                    o = c;
                    for (int d = 0; d < 4; ++d) o.ne[d] = one[d];
                    set_contig(o);
                }
                break;
            }
            case OP_PERMUTE:
            case OP_TRANSPOSE: {
                Val x = in(0);
                int ax[4] = {1, 0, 2, 3};
                if (op.opcode == OP_PERMUTE) {
                    ax[0] = (int)op.i("axis0", 1);
                    ax[1] = (int)op.i("axis1", 0);
                    ax[2] = (int)op.i("axis2", 2);
                    ax[3] = (int)op.i("axis3", 3);
                }
                if (x.virt_rope) {  // only (0,2,1,3) permutes reach here (see OP_ROPE)
                    o = x;
                    o.rope_perm = !x.rope_perm;
                    for (int d = 0; d < 4; ++d) o.ne[d] = one[d];
                    break;
                }
                o = x;
                o.has_q = false;
                o.w = nullptr;
                for (int d = 0; d < 4; ++d) {
                    o.ne[ax[d]] = x.ne[d];
                    o.nb[ax[d]] = x.nb[d];
                }
                if (outputs.count(out)) o = cont(o, oi);
                break;
            }
            case OP_CONT:
            case OP_CPY: {
                o = cont(in(0), oi);
                for (int d = 0; d < 4; ++d) o.ne[d] = one[d];
                set_contig(o);
                break;
            }
            case OP_ROPE: {
                Val x = in(0);
                const int mode = (int)op.i("mode", 2);
                GB_CHECK(mode == 2, "ROPE: only NEOX mode (2) is supported");
                GB_CHECK(op.inputs.size() < 3, "ROPE: frequency factors are not supported");
                GB_CHECK(op.f("ext_factor", 0.0) == 0.0, "ROPE: YaRN ext_factor is not supported");
                const int n_dims = (int)op.i("n_dims", x.ne[0]);
                const float fb = (float)op.f("freq_base", 10000.0);
                const float fs = (float)op.f("freq_scale", 1.0);
                const uint32_t pid = op.inputs.at(1);
                Val pv = get(pid);
                GB_CHECK(pv.type == T_I32, "ROPE positions must be int32");
                if (!pv.contiguous()) pv = cont(pv, oi);
                const GTensor& pt = G.t(pid);
                const bool arange = pt.data && pt.name.find("arange") != std::string::npos;
                const bool use_step = arange && env.count("pos");
                // an identity arange (0, 1, 2, ...) is replaced by base + i on the device, so
                // positions past the stored constant's length stay valid
                bool identity = false;
                if (arange && pt.type == T_I32) {
                    identity = true;
                    const int32_t* a = (const int32_t*)pt.data;
                    for (uint64_t i = 0; i < pt.data_size / 4; ++i)
                        if (a[i] != (int32_t)i) { identity = false; break; }
                }
                const int64_t npos = nelem(pv.ne);
                bool permuted = false;
                if (x.ne[2] != npos && x.ne[1] == npos) {  // [hd, s, H] input (executor.cpp:2076)
                    permuted = true;
                    std::swap(x.ne[1], x.ne[2]);
                    std::swap(x.nb[1], x.nb[2]);
                }
                int64_t tab_n = 0;
                float ts = 1.0f;
                const float2* tab = rope_table(n_dims, fb, fs, &tab_n, &ts);
                RopeTable rt;
                rt.cs = tab;
                rt.n_pos = tab_n;
                rt.n_dims = n_dims;
                rt.theta_scale = ts;
                // Leave the rotation to the attention kernels when every consumer is a
                // (0,2,1,3) PERMUTE feeding FLASH_ATTN_EXT as q or k, the source rows are
                // head-contiguous and the positions are the identity arange.
                bool virt = identity && !permuted && x.nb[0] == 4 && x.nb[1] == x.ne[0] * 4 &&
                            x.type == T_F32 && !outputs.count(out) && !consumers[out].empty();
                for (int ci : consumers[out]) {
                    const GOp& c = G.ops[ci];
                    const bool perm = c.opcode == OP_PERMUTE && c.i("axis0", 1) == 0 &&
                                      c.i("axis1", 0) == 2 && c.i("axis2", 2) == 1 &&
                                      c.i("axis3", 3) == 3;
                    if (!perm || outputs.count(c.outputs[0])) {
                        virt = false;
                        break;
                    }
                    for (int cj : consumers[c.outputs[0]]) {
                        const GOp& f = G.ops[cj];
                        if (f.opcode != OP_FLASH_ATTN_EXT || f.inputs.size() < 2 ||
                            (f.inputs[0] != c.outputs[0] && f.inputs[1] != c.outputs[0]))
                            virt = false;
                    }
                }
                if (virt) {
                    o = Val();
                    o.has_f = false;
                    o.virt_rope = true;
                    o.rsrc = x.ref;
                    for (int d = 0; d < 4; ++d) {
                        o.rsrc_ne[d] = x.ne[d];
                        o.rsrc_nb[d] = x.nb[d];
                        o.ne[d] = one[d];
                    }
                    o.rtab = rt;
                    o.r_use_step = use_step;
                    break;
                }
                Val y;
                y.type = T_F32;
                for (int d = 0; d < 4; ++d) y.ne[d] = x.ne[d];
                alloc(y, oi);
                const Val xs = x, ys = y;
                const BufRef pr = pv.ref;
                const bool ident = identity;
                const StepParams* dstep = d_step_;
                add("rope", [=](Program& p, cudaStream_t st) {
                    TView yv = p.view(ys);
                    launch_rope_neox(p.view(xs), ident ? nullptr : (const int32_t*)p.ptr(pr),
                                     use_step, dstep, rt, &yv, nullptr, st);
                });
                o = y;
                if (permuted) {
                    std::swap(o.ne[1], o.ne[2]);
                    std::swap(o.nb[1], o.nb[2]);
                }
                break;
            }
            case OP_FLASH_ATTN_EXT: {
                Val q = in(0), k = in(1);
                Val v = op.inputs.size() > 2 ? in(2) : in(1);
                GB_CHECK(op.inputs.size() <= 3, "FLASH_ATTN_EXT with an explicit mask is not supported");
                const int64_t hd = q.ne[0], s = q.ne[1], Hq = q.ne[2];
                const int64_t Hkv = k.ne[2];
                GB_CHECK(q.ne[3] == 1 && k.ne[3] == 1, "batched attention (ne3 > 1) is not supported");
                float scale = 1.0f / sqrtf((float)hd);
                if (op.has("scale")) scale = (float)op.f("scale", scale);
                const bool causal = op.i("is_causal", 0) != 0;
                const bool fused_t = op.i("fused_transpose", 0) != 0;
                const bool use_cache = kv && kv_.count(op.id);
                // K/V destination: the persistent cache, or a per-call f16 scratch
                __half* kc;
                __half* vc;
                int64_t ctx;
                BufRef kref, vref;
                int64_t slot_elems = 0;
                int64_t sb = 0;  // bytes per slot window: single-sequence launches add kv_slot * sb
                const int32_t* ptab = nullptr;  // paged cache: the page table (slot 0's row)
                int64_t pstride = 0;
                int pshift = 0;
                if (use_cache) {
                    const KVCache& c = kv_.at(op.id);
                    GB_CHECK(c.hd == hd && c.Hkv == Hkv, "KV cache shape mismatch");
                    kc = c.k;
                    vc = c.v;
                    ctx = c.ctx;
                    slot_elems = c.slot_elems();
                    sb = pg.batch ? 0 : slot_elems * 2;
                    kref.fixed = (char*)kc;
                    vref.fixed = (char*)vc;
                    if (paged_) {  // kc / vc are page pools; the slot is chosen by its page list
                        ptab = d_ptab_;
                        pstride = ptab_stride_;
                        pshift = page_shift_;
                        sb = 0;
                    }
                } else {
                    ctx = k.ne[1];
                    kref.buf = pg.new_buf(Hkv * ctx * hd * 2, oi);
                    vref.buf = pg.new_buf(Hkv * ctx * hd * 2, oi);
                    kc = vc = nullptr;
                }
                // k/v arrive as [hd, s, Hkv]; the cache writer walks [hd, Hkv, s]
                auto heads_then_rows = [](Val t) {
                    std::swap(t.ne[1], t.ne[2]);
                    std::swap(t.nb[1], t.nb[2]);
                    return t;
                };
                GB_CHECK(k.ne[1] == s && v.ne[1] == s && v.ne[2] == Hkv,
                         "FLASH_ATTN_EXT: K/V rows must match the query rows");
                // with the KV cache the reference always applies the causal window mask
                // (executor.cpp:2143-2157); without it only is_causal graphs are served
                GB_CHECK(use_cache || causal || s == 1,
                         "non-causal FLASH_ATTN_EXT over several query rows is not supported");
                const StepParams* dstep = use_cache ? d_step_ : nullptr;
                // ---- fused path: q, k, v are heads of one projection row buffer ----------------
                struct Src {
                    BufRef ref;
                    int64_t head_nb = 0, row_nb = 0;
                    bool rot = false;
                    bool ok = false;
                };
                auto src_of = [&](const Val& t) {
                    Src r;
                    if (t.virt_rope) {
                        r.ok = t.rope_perm && t.rsrc_nb[0] == 4;
                        r.ref = t.rsrc;
                        r.head_nb = t.rsrc_nb[1];
                        r.row_nb = t.rsrc_nb[2];
                        r.rot = true;
                    } else {
                        r.ok = t.has_f && t.type == T_F32 && t.nb[0] == 4;
                        r.ref = t.ref;
                        r.head_nb = t.nb[2];
                        r.row_nb = t.nb[1];
                    }
                    return r;
                };
                Src sq = src_of(q), sk = src_of(k), sv = src_of(v);
                if (s == 1) sq.row_nb = sk.row_nb = sv.row_nb = 0;  // one row: stride unused
                GB_CHECK(!pg.batch || (use_cache && sq.ok && sk.ok && sv.ok),
                         "batched decode needs the fused attention path over the KV cache");
                bool fuse = sq.ok && sk.ok && sv.ok && !sv.rot && sq.rot == sk.rot &&
                            sq.ref.buf == sk.ref.buf && sk.ref.buf == sv.ref.buf &&
                            sq.ref.fixed == sk.ref.fixed && sk.ref.fixed == sv.ref.fixed &&
                            sq.head_nb == hd * 4 && sk.head_nb == hd * 4 && sv.head_nb == hd * 4 &&
                            sq.row_nb == sk.row_nb && sk.row_nb == sv.row_nb && hd % 32 == 0;
                if (fuse && sq.rot)
                    fuse = q.rtab.cs == k.rtab.cs && q.rtab.n_dims == k.rtab.n_dims &&
                           q.r_use_step == use_cache && k.r_use_step == use_cache;
                if (fuse) {
                    BufRef base = sq.ref;
                    base.off = 0;
                    const int64_t q_off = sq.ref.off / 4, k_off = sk.ref.off / 4, v_off = sv.ref.off / 4;
                    const int64_t row_f = sq.row_nb / 4;
                    RopeTable rt;
                    if (sq.rot) rt = q.rtab;  // else n_dims 0: no rotation
                    Val y;
                    y.type = T_F32;
                    y.ne[0] = hd;
                    y.ne[1] = Hq;
                    y.ne[2] = s;
                    y.ne[3] = 1;
                    if (use_cache && (s == 1 || pg.batch)) {
                        // which outputs the consumer chain needs (through a RESHAPE)
                        uint32_t look = out;
                        if (!outputs.count(out) && consumers[out].size() == 1 &&
                            G.ops[consumers[out][0]].opcode == OP_RESHAPE && fused_t)
                            look = G.ops[consumers[out][0]].outputs[0];
                        bool nf, nq;
                        needs(look, nf, nq);
                        if (look == out) nf = true;
                        if (nf) alloc(y, oi);
                        else {
                            set_contig(y);
                            y.has_f = false;
                        }
                        if (nq) {
                            y.q.buf = pg.new_buf(s * Hq * hd, oi);
                            y.qd.buf = pg.new_buf(s * Hq * hd / QK * 4, oi);
                            y.has_q = true;
                        }
                        AttnDecArgs da;
                        da.rows = (int)s;
                        da.batched = pg.batch;
                        da.qkv_stride = sq.row_nb / 4;
                        da.slot_elems = slot_elems;
                        da.q_off = q_off;
                        da.k_off = k_off;
                        da.v_off = v_off;
                        da.Hq = (int)Hq;
                        da.Hkv = (int)Hkv;
                        da.hd = (int)hd;
                        da.tab = rt;
                        da.step = d_step_;
                        da.kc = kc;
                        da.vc = vc;
                        da.ctx = ctx;
                        da.scale = scale;
                        da.max_kv = kv_max_ctx_;
                        da.splits = attn_decode_splits(Hkv, kv_max_ctx_, (int)s);
                        BufRef wref;
                        wref.buf = pg.new_buf((int64_t)attn_decode_workspace(Hq, hd, da.splits) * s, oi);
                        const BufRef yr = y.ref, yq = y.q, yqd = y.qd;
                        const bool hf = y.has_f, hq = y.has_q;
                        const double kvb = (double)Hkv * hd * 2 * 2;  // K+V bytes per position
                        const bool batched = pg.batch;
                        auto mk = [=](const Program& p) {
                            AttnDecArgs a = da;
                            a.kc = (__half*)((char*)da.kc + p.kv_slot * sb);
                            a.vc = (__half*)((char*)da.vc + p.kv_slot * sb);
                            if (ptab) {  // batched rows add row_slot * stride in the kernel
                                a.pg.pages = ptab + (batched ? 0 : p.kv_slot * pstride);
                                a.pg.stride = (int32_t)pstride;
                                a.pg.shift = pshift;
                            }
                            a.qkv = (const float*)p.ptr(base);
                            a.part = (float*)p.ptr(wref);
                            if (hf) a.o = (float*)p.ptr(yr);
                            if (hq) {
                                a.oq = (int8_t*)p.ptr(yq);
                                a.od = (float*)p.ptr(yqd);
                            }
                            return a;
                        };
                        add("attn_decode", [=](Program& p, cudaStream_t st) {
                            launch_attn_decode(mk(p), st);
                        }, kvb);
                        chainable([=](const Program& p, ChainOp& c) {
                            c.kind = CH_ATTN;
                            c.at = mk(p);
                            return chain_attn_ok(c.at);
                        });
                        (void)row_f;
                    } else {
                        // RoPE + KV write in one launch, then attention over the cache
                        Val qt;
                        qt.type = T_F32;
                        qt.ne[0] = hd;
                        qt.ne[1] = Hq;
                        qt.ne[2] = s;
                        alloc(qt, oi);  // [s][Hq][hd]
                        QkvRopeArgs ra;
                        ra.qkv_stride = row_f;
                        ra.q_off = q_off;
                        ra.k_off = k_off;
                        ra.v_off = v_off;
                        ra.Hq = (int)Hq;
                        ra.Hkv = (int)Hkv;
                        ra.hd = (int)hd;
                        ra.s = s;
                        ra.tab = rt;
                        ra.step = dstep;
                        ra.ctx = ctx;
                        const BufRef qtr = qt.ref;
                        add("rope_kv", [=](Program& p, cudaStream_t st) {
                            QkvRopeArgs a = ra;
                            a.qkv = (const float*)p.ptr(base);
                            a.q_out = (float*)p.ptr(qtr);
                            a.kc = (__half*)(p.ptr(kref) + p.kv_slot * sb);
                            a.vc = (__half*)(p.ptr(vref) + p.kv_slot * sb);
                            a.pages = ptab ? ptab + p.kv_slot * pstride : nullptr;
                            a.page_shift = pshift;
                            launch_rope_qkv(a, st);
                        });
                        Val qv = qt;  // view [hd, s, Hq] of the [s][Hq][hd] buffer
                        qv.ne[1] = s;
                        qv.ne[2] = Hq;
                        qv.nb[1] = Hq * hd * 4;
                        qv.nb[2] = hd * 4;
                        alloc(y, oi);
                        const int64_t max_kv = use_cache ? kv_max_ctx_ : s;
                        const size_t wbytes = attn_workspace_bytes(s, Hq, hd, max_kv);
                        BufRef wref;
                        if (wbytes) wref.buf = pg.new_buf((int64_t)wbytes, oi);
                        const BufRef yr = y.ref;
                        const bool step_on = use_cache;
                        pg.use(qt.ref, oi);
                        add("attention", [=](Program& p, cudaStream_t st) {
                            launch_attention(p.view(qv), (const __half*)(p.ptr(kref) + p.kv_slot * sb),
                                             (const __half*)(p.ptr(vref) + p.kv_slot * sb), ctx, Hkv, dstep, step_on, 0,
                                             scale, (float*)p.ptr(yr),
                                             wbytes ? p.ptr(wref) : nullptr, max_kv, st,
                                             ptab ? ptab + p.kv_slot * pstride : nullptr, pshift);
                        });
                    }
                    o = y;
                    if (!fused_t) {
                        std::swap(o.ne[1], o.ne[2]);
                        std::swap(o.nb[1], o.nb[2]);
                        o.has_q = false;
                    }
                    for (int d = 0; d < 4; ++d)
                        GB_CHECK(o.ne[d] == one[d], "FLASH_ATTN_EXT output shape mismatch");
                    break;
                }
                // ---- generic path ----------------------------------------------------------------
                auto materialize = [&](Val& t) {  // emit a deferred RoPE into its own buffer
                    if (!t.virt_rope) return;
                    Val xs;
                    xs.ref = t.rsrc;
                    xs.type = T_F32;
                    for (int d = 0; d < 4; ++d) {
                        xs.ne[d] = t.rsrc_ne[d];
                        xs.nb[d] = t.rsrc_nb[d];
                    }
                    Val y;
                    y.type = T_F32;
                    for (int d = 0; d < 4; ++d) y.ne[d] = xs.ne[d];
                    alloc(y, oi);
                    const RopeTable rt = t.rtab;
                    const bool us = t.r_use_step;
                    const StepParams* ds = d_step_;
                    add("rope", [=](Program& p, cudaStream_t st) {
                        TView yv = p.view(y);
                        launch_rope_neox(p.view(xs), nullptr, us, ds, rt, &yv, nullptr, st);
                    });
                    const bool perm = t.rope_perm;
                    t = y;
                    if (perm) {
                        std::swap(t.ne[1], t.ne[2]);
                        std::swap(t.nb[1], t.nb[2]);
                    }
                };
                materialize(q);
                materialize(k);
                const Val ks = heads_then_rows(k), vs = heads_then_rows(v), qs = q;
                add("kv_write", [=](Program& p, cudaStream_t st) {
                    const int32_t* pl = ptab ? ptab + p.kv_slot * pstride : nullptr;
                    KVDst kd{(__half*)(p.ptr(kref) + p.kv_slot * sb), ctx, pl, pshift};
                    KVDst vd{(__half*)(p.ptr(vref) + p.kv_slot * sb), ctx, pl, pshift};
                    launch_kv_write(p.view(ks), dstep, kd, st);
                    launch_kv_write(p.view(vs), dstep, vd, st);
                });
                Val y;
                y.type = T_F32;
                y.ne[0] = hd;
                y.ne[1] = Hq;
                y.ne[2] = s;
                y.ne[3] = 1;
                alloc(y, oi);
                const int64_t max_kv = use_cache ? kv_max_ctx_ : s;
                const size_t wbytes = attn_workspace_bytes(s, Hq, hd, max_kv);
                BufRef wref;
                if (wbytes) wref.buf = pg.new_buf((int64_t)wbytes, oi);
                const BufRef yr = y.ref;
                const bool step_on = use_cache;
                add("attention", [=](Program& p, cudaStream_t st) {
                    launch_attention(p.view(qs), (const __half*)(p.ptr(kref) + p.kv_slot * sb),
                                     (const __half*)(p.ptr(vref) + p.kv_slot * sb),
                                     ctx, Hkv, dstep, step_on, 0, scale, (float*)p.ptr(yr),
                                     wbytes ? p.ptr(wref) : nullptr, max_kv, st,
                                     ptab ? ptab + p.kv_slot * pstride : nullptr, pshift);
                });
                (void)causal;
                o = y;
                if (!fused_t) {
                    std::swap(o.ne[1], o.ne[2]);
                    std::swap(o.nb[1], o.nb[2]);
                }
                for (int d = 0; d < 4; ++d)
                    GB_CHECK(o.ne[d] == one[d], "FLASH_ATTN_EXT output shape mismatch");
                break;
            }
            case OP_ADD:
            case OP_MUL: {
                Val a = in(0), b = in(1);
                alloc(o, oi);
                const Val as = a, bs = b, os = o;
                const int bop = op.opcode == OP_ADD ? 0 : 1;
                add(bop ? "mul" : "add",
                    [=](Program& p, cudaStream_t st) { launch_binary(p.view(as), p.view(bs), p.view(os), bop, st); });
                break;
            }
            case OP_SWIGLU:
            case OP_GLU: {
                GB_CHECK(op.inputs.size() == 1, "split SWIGLU (gate, up) is not supported");
                Val x = in(0);
                if (!(x.nb[0] == 4 && x.rows_uniform())) x = cont(x, oi);
                const int64_t F = x.ne[0] / 2, M = x.nrows();
                const bool swapped = op.i("swapped", 0) != 0;
                bool nf, nq;
                needs(out, nf, nq);
                if (nf) alloc(o, oi);
                else o.has_f = false;
                if (nq) {
                    o.q.buf = pg.new_buf(M * F, oi);
                    o.qd.buf = pg.new_buf(M * (F / QK) * 4, oi);
                    o.has_q = true;
                }
                const BufRef xr = x.ref, orf = o.ref, qr = o.q, qdr = o.qd;
                const int64_t xs = x.nb[1] / 4;
                const bool hf = o.has_f, hq = o.has_q;
                add("swiglu", [=](Program& p, cudaStream_t st) {
                    launch_swiglu((const float*)p.ptr(xr), xs, M, F, swapped,
                                  hf ? (float*)p.ptr(orf) : nullptr, F,
                                  hq ? (int8_t*)p.ptr(qr) : nullptr, hq ? (float*)p.ptr(qdr) : nullptr,
                                  st);
                });
                break;
            }
            case OP_BIAS_GELU: {
                Val x = in(0);
                if (!(x.nb[0] == 4 && x.rows_uniform())) x = cont(x, oi);
                const float* bias = op.inputs.size() > 1 ? (const float*)get(op.inputs[1]).ref.fixed : nullptr;
                const int64_t F = x.ne[0], M = x.nrows();
                bool nf, nq;
                needs(out, nf, nq);
                if (nf) alloc(o, oi);
                else o.has_f = false;
                if (nq) {
                    o.q.buf = pg.new_buf(M * F, oi);
                    o.qd.buf = pg.new_buf(M * (F / QK) * 4, oi);
                    o.has_q = true;
                }
                const BufRef xr = x.ref, orf = o.ref, qr = o.q, qdr = o.qd;
                const int64_t xs = x.nb[1] / 4;
                const bool hf = o.has_f, hq = o.has_q;
                add("bias_gelu", [=](Program& p, cudaStream_t st) {
                    launch_bias_gelu((const float*)p.ptr(xr), xs, bias, M, F,
                                     hf ? (float*)p.ptr(orf) : nullptr, F,
                                     hq ? (int8_t*)p.ptr(qr) : nullptr,
                                     hq ? (float*)p.ptr(qdr) : nullptr, st);
                });
                break;
            }
            default:
                GB_CHECK(false, "opcode " + std::to_string(op.opcode) + " ('" + op.name +
                                    "') is not supported by the B200 engine");
        }
        vals[out] = o;
    }

    // outputs stay live to the end
    for (uint32_t id : G.outputs) {
        auto it = vals.find(id);
        GB_CHECK(it != vals.end(), "graph output was not produced");
        GB_CHECK(it->second.has_f && it->second.contiguous(), "graph output is not contiguous");
        pg.use(it->second.ref, nops + 1);
    }

    // assign arena offsets: greedy placement of buffers by size over their live ranges
    const int nb = (int)pg.buf_size.size();
    std::vector<int> order(nb);
    for (int i = 0; i < nb; ++i) order[i] = i;
    std::sort(order.begin(), order.end(), [&](int a, int b) { return pg.buf_size[a] > pg.buf_size[b]; });
    pg.buf_off.assign(nb, 0);
    std::vector<int> placed;
    int64_t total = 0;
    for (int b : order) {
        std::vector<std::pair<int64_t, int64_t>> busy;
        for (int o2 : placed)
            if (!(pg.buf_last[o2] < pg.buf_first[b] || pg.buf_last[b] < pg.buf_first[o2]))
                busy.push_back({pg.buf_off[o2], pg.buf_off[o2] + pg.buf_size[o2]});
        std::sort(busy.begin(), busy.end());
        int64_t off = 0;
        for (auto& r : busy) {
            if (off + pg.buf_size[b] <= r.first) break;
            off = std::max(off, r.second);
        }
        pg.buf_off[b] = off;
        total = std::max(total, off + pg.buf_size[b]);
        placed.push_back(b);
    }
    pg.arena_bytes = (size_t)total;
    ensure_arena((size_t)total);
    pg.arena = &arena_;
    // each launch's L2 prefetch: the weights of the next launch that streams any
    pg.launch_pf.assign(pg.launches.size(), PfNext{});
    for (size_t i = pg.launches.size(), nxt = SIZE_MAX; i-- > 0;) {
        if (nxt != SIZE_MAX) pg.launch_pf[i] = pg.launch_w[nxt];
        if (pg.launch_w[i].qs) nxt = i;
    }
    // single-sequence decode on one GPU: runs of chainable launches become decode chains
    if (kv && !pg.batch && tp_.size == 1 && chain_enabled_ && !paged_) fuse_chains(pg);
    pg.chain_descs.clear();
    return P;
}

// Replace every run of at least three consecutive chainable launches, one of them a GEMV, by one
// chain launch (k_chain.cu).  The run's table, barrier counters and attention scratch belong to
// the program.
void Executor::fuse_chains(Program& pg) {
    const size_t n = pg.launches.size();
    std::vector<Launch> launches;
    std::vector<std::string> names;
    std::vector<double> bytes;
    size_t i = 0;
    while (i < n) {
        size_t j = i;
        std::vector<ChainOp> ops;
        bool gemv = false;
        while (j < n && pg.chain_descs[j] && (!chain_max_ops_ || j - i < chain_max_ops_)) {
            ChainOp op;
            if (!pg.chain_descs[j](pg, op)) break;
            gemv = gemv || op.kind == CH_GEMV;
            ops.push_back(op);
            ++j;
        }
        // a bounded chain length takes every chainable run, single ops included
        if (j == i || (!chain_max_ops_ && (j - i < 3 || !gemv))) {
            launches.push_back(pg.launches[i]);
            names.push_back(pg.launch_names[i]);
            bytes.push_back(pg.launch_bytes[i]);
            ++i;
            continue;
        }
        auto run = std::make_shared<ChainRun>();
        run->descs.assign(pg.chain_descs.begin() + i, pg.chain_descs.begin() + j);
        const int64_t part = chain_prepare(ops.data(), (int)ops.size(), dev_);
        GB_CUDA(cudaMalloc(&run->d_ops, ops.size() * sizeof(ChainOp)));
        pg.owned.push_back(run->d_ops);
        GB_CUDA(cudaMalloc(&run->sync, sizeof(ChainSync)));
        pg.owned.push_back(run->sync);
        GB_CUDA(cudaMemset(run->sync, 0, sizeof(ChainSync)));
        GB_CUDA(cudaMalloc(&run->part, std::max<int64_t>(part, 1) * sizeof(float)));
        pg.owned.push_back(run->part);
        double b = 0.0;
        for (size_t k = i; k < j; ++k) b += pg.launch_bytes[k];
        if (!chain_err_host_) {
            GB_CUDA(cudaHostAlloc(&chain_err_host_, sizeof(int), cudaHostAllocMapped));
            *chain_err_host_ = 0;
            GB_CUDA(cudaHostGetDevicePointer((void**)&chain_err_dev_, chain_err_host_, 0));
        }
        int* err = chain_err_dev_;
        launches.push_back([run, err](Program&, cudaStream_t st) {
            launch_chain(run->d_ops, run->h_ops.data(), (int)run->h_ops.size(), run->sync,
                         run->part, err, st);
        });
        std::string nm = "chain";
        if (j - i <= 4) {  // short chains by their ops (per-op timing with a bounded length)
            nm += ":";
            for (size_t k = i; k < j; ++k) nm += (k > i ? "+" : "") + pg.launch_names[k];
        }
        names.push_back(nm);
        bytes.push_back(b);
        pg.chains.push_back(run);
        i = j;
    }
    pg.launches = std::move(launches);
    pg.launch_names = std::move(names);
    pg.launch_bytes = std::move(bytes);
}

// Rewrite a chain's device table when the buffers it points at moved (outside any capture).
void Executor::refresh_chain(Program& p, ChainRun& c) {
    if (!c.h_ops.empty() && c.key_arena == *p.arena && c.key_slot == p.kv_slot) return;
    std::vector<ChainOp> ops(c.descs.size());
    for (size_t k = 0; k < ops.size(); ++k)
        GB_CHECK(c.descs[k](p, ops[k]), "chain: an op no longer fits the chain");
    chain_prepare(ops.data(), (int)ops.size(), dev_);
    GB_CUDA(cudaStreamSynchronize(stream_));  // no launch in flight reads the old table
    GB_CUDA(cudaMemcpy(c.d_ops, ops.data(), ops.size() * sizeof(ChainOp), cudaMemcpyHostToDevice));
    c.h_ops = std::move(ops);
    c.key_arena = *p.arena;
    c.key_slot = p.kv_slot;
}

// ------------------------------------------------------------------------------ execution

void Executor::prepare(const SymEnv& env_in, bool /*arena_reuse*/) {
    const double t0 = profile_on_ ? now_ms() : 0;
    GB_CUDA(cudaSetDevice(dev_));
    SymEnv env = env_in;
    const bool kv = kv_enabled_ && env.count("pos");
    int64_t pos = kv ? env.at("pos") : 0;
    // the program key: every symbol except pos (kernels read pos from StepParams)
    std::string key = kv ? "kv" : "plain";
    if (logits_last_only_) key += "/last";
    if (!out_rows_.empty()) key += "/rows=" + std::to_string(out_rows_.size());
    SymEnv shape_env;
    for (auto& [k, v] : env)
        if (k != "pos" && k != "slot") shape_env[k] = v;
    std::vector<std::pair<std::string, int64_t>> items(shape_env.begin(), shape_env.end());
    std::sort(items.begin(), items.end());
    for (auto& [k, v] : items) key += "/" + k + "=" + std::to_string(v);
    const bool batch = env.count("__rows") != 0;
    if (kv && !batch) {
        int64_t s = env.count("s") ? env.at("s") : 1;
        GB_CHECK(pos >= 0 && pos + s <= kv_max_ctx_,
                 "KV cache overflow: pos " + std::to_string(pos) + " + s " + std::to_string(s) +
                     " > max_ctx " + std::to_string(kv_max_ctx_));
        const int64_t slot = env.count("slot") ? env.at("slot") : 0;
        const int64_t slots = kv_.empty() ? 1 : kv_.begin()->second.slots;
        GB_CHECK(slot >= 0 && slot < slots, "KV slot " + std::to_string(slot) + " out of range");
        if (paged_)
            GB_CHECK(slot < paged_max_batch_ && slot_live_[(size_t)slot] &&
                         pos + s <= (int64_t)slot_pages_[(size_t)slot].size() * tokens_per_page_,
                     "paged KV: positions up to " + std::to_string(pos + s) + " of slot " +
                         std::to_string(slot) + " have no pages (paged_kv_ensure_tokens)");
    }
    GB_CHECK(!batch || kv, "batched decode needs the KV cache");
    auto it = programs_.find(key);
    if (it == programs_.end()) {
        SymEnv benv = shape_env;
        if (kv) benv["pos"] = pos;
        auto p = build(benv, kv);
        p->key = key;
        p->s = env.count("s") ? env.at("s") : 0;
        p->decode = kv && (p->s == 1 || batch);
        programs_[key] = p;
        active_ = p;
    } else {
        active_ = it->second;
    }
    h_step_->pos = pos;
    if (!out_rows_.empty() && active_->out_rows_of > 0) {
        const int64_t s = active_->out_rows_of;
        for (size_t r = 0; r < out_rows_.size(); ++r) {
            GB_CHECK(out_rows_[r] >= 0 && out_rows_[r] < s,
                     "output row " + std::to_string(out_rows_[r]) + " is not among the call's " +
                         std::to_string(s) + " tokens");
            h_step_->out_rows[r] = out_rows_[r];
        }
    }
    active_->kv_slot = env.count("slot") ? env.at("slot") : 0;
    if (profile_on_) {
        profile_.prepare_ms += now_ms() - t0;
        profile_.n_prepare++;
    }
}

void Executor::set_input(uint32_t tid, const void* data, size_t bytes) {
    GB_CHECK(active_, "set_input before prepare");
    auto it = active_->input_bufs.find(tid);
    GB_CHECK(it != active_->input_bufs.end(), "tensor " + std::to_string(tid) + " is not a graph input");
    const Val& v = active_->vals.at(tid);
    const size_t need = (size_t)(nelem(v.ne) * v.nb[0]);
    GB_CHECK(bytes == need, "set_input size mismatch for tensor " + std::to_string(tid) + ": got " +
                                std::to_string(bytes) + " bytes, expected " + std::to_string(need));
    GB_CUDA(cudaMemcpyAsync(it->second, data, bytes, cudaMemcpyHostToDevice, stream_));
}

void Executor::set_input_by_name(const std::string& name, const void* data, size_t bytes) {
    for (uint32_t id : g_->inputs)
        if (g_->t(id).name == name) return set_input(id, data, bytes);
    GB_CHECK(false, "no graph input named '" + name + "'");
}

void Executor::run() {
    GB_CHECK(active_, "run before prepare");
    const double t0 = profile_on_ ? now_ms() : 0;
    Program& p = *active_;
    sync_page_table();
    for (auto& c : p.chains) refresh_chain(p, *c);
    // this step's parameters from a ring entry no queued copy still reads (the working copy is
    // rewritten by the next prepare while this copy may still wait in the stream)
    StepParams* stage = step_ring_ + step_next_;
    GB_CUDA(cudaEventSynchronize(step_ev_[step_next_]));
    *stage = *h_step_;
    GB_CUDA(cudaMemcpyAsync(d_step_, stage, sizeof(StepParams), cudaMemcpyHostToDevice, stream_));
    GB_CUDA(cudaEventRecord(step_ev_[step_next_], stream_));
    step_next_ = (step_next_ + 1) % kStepRing;
    if (ktiming_) {
        const size_t n = p.launches.size();
        while (kevents_.size() < n + 1) {
            cudaEvent_t ev;
            GB_CUDA(cudaEventCreate(&ev));
            kevents_.push_back(ev);
        }
        GB_CUDA(cudaEventRecord(kevents_[0], stream_));
        for (size_t i = 0; i < n; ++i) {
            p.launches[i](p, stream_);
            GB_CUDA(cudaEventRecord(kevents_[i + 1], stream_));
        }
        GB_CUDA(cudaStreamSynchronize(stream_));
        for (size_t i = 0; i < n; ++i) {
            float ms = 0;
            GB_CUDA(cudaEventElapsedTime(&ms, kevents_[i], kevents_[i + 1]));
            KTime& k = ktimes_[p.launch_names[i]];
            k.ms += ms;
            k.n += 1;
            k.bytes += p.launch_bytes[i];
        }
    } else if (cuda_graph_ && p.decode) {
        if (p.graph_exec && p.graph_slot != p.kv_slot) {
            cudaGraphExecDestroy(p.graph_exec);
            p.graph_exec = nullptr;
        }
        if (!p.graph_exec) {
            p.graph_slot = p.kv_slot;
            cudaGraph_t graph;
            GB_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
            try {
                for (auto& l : p.launches) l(p, stream_);
            } catch (...) {
                cudaStreamEndCapture(stream_, &graph);
                throw;
            }
            GB_CUDA(cudaStreamEndCapture(stream_, &graph));
            GB_CUDA(cudaGraphInstantiate(&p.graph_exec, graph, 0));
            cudaGraphDestroy(graph);
        }
        GB_CUDA(cudaGraphLaunch(p.graph_exec, stream_));
    } else {
        for (auto& l : p.launches) l(p, stream_);
    }
    if (profile_on_) {
        GB_CUDA(cudaStreamSynchronize(stream_));
        profile_.run_ms += now_ms() - t0;
        profile_.n_run++;
    }
}

void Executor::synchronize() {
    GB_CUDA(cudaStreamSynchronize(stream_));
    check_tp_error();
}

bool Executor::cuda_graph_captured() const {
    for (auto& [k, p] : programs_)
        if (p->graph_exec) return true;
    return false;
}

const void* Executor::get_output(uint32_t tid, size_t* bytes) {
    GB_CHECK(active_, "get_output before prepare");
    auto it = active_->vals.find(tid);
    GB_CHECK(it != active_->vals.end(), "unknown output tensor " + std::to_string(tid));
    const Val& v = it->second;
    GB_CHECK(v.has_f && v.contiguous(), "output tensor is not contiguous");
    const size_t n = (size_t)(nelem(v.ne) * v.nb[0]);
    if (pinned_out_bytes_ < n) {
        if (pinned_out_) cudaFreeHost(pinned_out_);
        GB_CUDA(cudaMallocHost(&pinned_out_, n));
        pinned_out_bytes_ = n;
    }
    GB_CUDA(cudaMemcpyAsync(pinned_out_, active_->ptr(v.ref), n, cudaMemcpyDeviceToHost, stream_));
    synchronize();
    auto& host = out_host_[tid];
    host.resize(n);
    std::memcpy(host.data(), pinned_out_, n);
    *bytes = n;
    return host.data();
}

void Executor::output_argmax(uint32_t tid, int rows, int32_t* out) {
    GB_CHECK(active_, "output_argmax before prepare");
    GB_CHECK(rows >= 1 && rows <= kMaxRows, "output_argmax: 1..16 rows");
    auto it = active_->vals.find(tid);
    GB_CHECK(it != active_->vals.end(), "unknown output tensor " + std::to_string(tid));
    const Val& v = it->second;
    GB_CHECK(v.has_f && v.type == T_F32 && v.contiguous(), "output_argmax: needs a contiguous f32 output");
    const int64_t total = nelem(v.ne);
    GB_CHECK(total % rows == 0, "output_argmax: output does not split into the rows");
    if (!d_argmax_) {
        GB_CUDA(cudaMalloc(&d_argmax_, kMaxRows * sizeof(int32_t)));
        GB_CUDA(cudaMallocHost(&h_argmax_, kMaxRows * sizeof(int32_t)));
    }
    launch_argmax_rows((const float*)active_->ptr(v.ref), rows, total / rows, d_argmax_, stream_);
    GB_CUDA(cudaMemcpyAsync(h_argmax_, d_argmax_, rows * sizeof(int32_t), cudaMemcpyDeviceToHost,
                            stream_));
    synchronize();
    std::memcpy(out, h_argmax_, rows * sizeof(int32_t));
}

std::array<int64_t, 4> Executor::tensor_shape(uint32_t tid) const {
    if (active_) {
        auto it = active_->vals.find(tid);
        if (it != active_->vals.end())
            return {it->second.ne[0], it->second.ne[1], it->second.ne[2], it->second.ne[3]};
    }
    const GTensor& t = g_->t(tid);
    SymEnv env = active_ ? active_->env : SymEnv{};
    std::array<int64_t, 4> ne{1, 1, 1, 1};
    for (int d = 0; d < 4; ++d) {
        try {
            ne[d] = t.ne[d]->eval(env);
        } catch (...) {
            ne[d] = t.file_ne[d];
        }
    }
    return ne;
}

size_t Executor::tensor_size_bytes(uint32_t tid) const {
    auto ne = tensor_shape(tid);
    const GTensor& t = g_->t(tid);
    return (size_t)(row_bytes(t.type, ne[0]) * ne[1] * ne[2] * ne[3]);
}

void Executor::set_state(uint32_t tid, const void* data, size_t bytes) {
    auto& p = state_dev_[tid];
    if (!p) GB_CUDA(cudaMalloc(&p, bytes));
    GB_CUDA(cudaMemcpy(p, data, bytes, cudaMemcpyHostToDevice));
}

const void* Executor::get_state(uint32_t tid, size_t* bytes) {
    auto it = state_dev_.find(tid);
    GB_CHECK(it != state_dev_.end(), "no state tensor " + std::to_string(tid));
    size_t n = tensor_size_bytes(tid);
    auto& host = out_host_[tid];
    host.resize(n);
    GB_CUDA(cudaMemcpy(host.data(), it->second, n, cudaMemcpyDeviceToHost));
    *bytes = n;
    return host.data();
}

void Executor::reset_state() {
    for (auto& [id, p] : state_dev_) GB_CUDA(cudaMemset(p, 0, tensor_size_bytes(id)));
}

int64_t Executor::launches_per_run() const {
    if (!active_) return 0;
    int64_t n = 0;  // the engine's kernel launches (NCCL collectives are NCCL's kernels)
    for (auto& name : active_->launch_names) n += name != "allreduce" && name != "allgather";
    return n;
}

std::string Executor::graph_summary() const {
    std::map<std::string, int> hist;
    if (active_)
        for (auto& n : active_->launch_names) hist[n]++;
    std::ostringstream os;
    os << "{\"engine\":\"ggmlc_b200\",\"launch_steps\":" << (active_ ? active_->launches.size() : 0)
       << ",\"arena_bytes\":" << (active_ ? active_->arena_bytes : 0) << ",\"steps\":{";
    bool first = true;
    for (auto& [k, v] : hist) {
        os << (first ? "" : ",") << "\"" << k << "\":" << v;
        first = false;
    }
    os << "}}";
    return os.str();
}

std::string Executor::kernel_times_json() const {
    std::ostringstream os;
    os.precision(9);
    os << "{";
    bool first = true;
    for (auto& [k, v] : ktimes_) {
        os << (first ? "" : ",") << "\"" << k << "\":[" << v.ms << "," << v.n << "," << v.bytes
           << "]";
        first = false;
    }
    os << "}";
    return os.str();
}

std::string Executor::mul_mat_shape_summary() const {
    std::map<std::string, int> hist;
    for (auto& op : g_->ops) {
        if (op.opcode != OP_MUL_MAT) continue;
        const GTensor& w = g_->t(op.inputs[0]);
        std::ostringstream k;
        k << "type" << w.type << ":" << w.file_ne[0] << "x" << w.file_ne[1];
        hist[k.str()]++;
    }
    std::ostringstream os;
    os << "{\"mul_mat\":{";
    bool first = true;
    for (auto& [k, v] : hist) {
        os << (first ? "" : ",") << "\"" << k << "\":" << v;
        first = false;
    }
    os << "}}";
    return os.str();
}

}  // namespace gb
