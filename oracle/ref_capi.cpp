// Test infrastructure only: a C ABI over the reference's own CPU code (vendored ggml 0.20.2 CPU
// backend and the ggmlc runtime), compiled from the reference sources by oracle/Makefile into
// oracle/_ref/libggmlc_ref.so.  Python tests load it with ctypes to pin the C restatement in
// oracle/oracle.c against the real reference, and tests/golden/make_golden.py uses it to write
// the golden vectors.  Nothing in the product links or loads this file.
//
// Op-level entry points build a one-op ggml graph and run it with ggml_graph_compute_with_ctx,
// i.e. the same ggml-cpu kernels the reference runtime dispatches (ggml-cpu.c:1254-1457 for
// MUL_MAT, ops.cpp for the rest).  Model-level entry points drive ggmlc::ModelExecutor exactly as
// ggmlc_bench.cpp / generator.py do: prepare({s,pos}) -> set_input -> run -> get_output_data.
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>
#include <memory>
#include <unordered_map>
#include <stdexcept>

#include "ggml.h"
#include "ggml-cpu.h"
#include "ggmlc/executor.h"
#include "ggmlc/loader.h"

extern "C" {
void quantize_row_q8_0(const float* x, void* y, int64_t k);
void ggml_vec_dot_q4_0_q8_0(int n, float* s, size_t bs, const void* vx, size_t bx, const void* vy,
                            size_t by, int nrc);
void ggml_vec_dot_q8_0_q8_0(int n, float* s, size_t bs, const void* vx, size_t bx, const void* vy,
                            size_t by, int nrc);
}

namespace {
thread_local std::string g_err;

struct Ctx {
    ggml_context* ctx = nullptr;
    explicit Ctx(size_t bytes) {
        ggml_init_params p = {bytes, nullptr, false};
        ctx = ggml_init(p);
        if (!ctx) throw std::runtime_error("ggml_init failed");
    }
    ~Ctx() { if (ctx) ggml_free(ctx); }
};

int run_graph(ggml_context* ctx, ggml_tensor* out, int n_threads) {
    ggml_cgraph* gf = ggml_new_graph(ctx);
    ggml_build_forward_expand(gf, out);
    return ggml_graph_compute_with_ctx(ctx, gf, n_threads) == GGML_STATUS_SUCCESS ? 0 : -1;
}

struct RefModel {
    ggmlc::SerializedModelGraph graph;
    std::unique_ptr<ggmlc::ModelExecutor> exec;
    int n_threads = 1;
};
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

// --- op level ---------------------------------------------------------------------------------

// x86 AVX2 activation quantizer (ggml-cpu/arch/x86/quants.c:302-392).
void ref_quantize_row_q8_0(const float* x, void* y, int64_t k) {
    ggml_cpu_init();  // fills the fp16 lookup tables the CPU kernels read
    quantize_row_q8_0(x, y, k);
}

// Row dequantizer (ggml-quants.c:459-477 / :553-567) via the type traits.
int ref_dequantize_row(int type, const void* x, float* y, int64_t k) {
    ggml_cpu_init();
    const ggml_type_traits* tt = ggml_get_type_traits((ggml_type)type);
    if (!tt || !tt->to_float) { g_err = "no to_float"; return -1; }
    tt->to_float(x, y, k);
    return 0;
}

// One weight row (Q8_0 or Q4_0, n elements) dotted with one Q8_0 activation row.
int ref_vec_dot(int wtype, int n, float* s, const void* w, const void* xq) {
    ggml_cpu_init();
    if (wtype == GGML_TYPE_Q8_0) ggml_vec_dot_q8_0_q8_0(n, s, 0, w, 0, xq, 0, 1);
    else if (wtype == GGML_TYPE_Q4_0) ggml_vec_dot_q4_0_q8_0(n, s, 0, w, 0, xq, 0, 1);
    else { g_err = "unsupported wtype"; return -1; }
    return 0;
}

// Y[M,N] = X[M,K] . W[N,K]^T with W quantized (row-major GGUF block rows), X f32.
int ref_mul_mat(int wtype, const void* w, int64_t N, int64_t K, const float* x, int64_t M,
                float* y, int n_threads) {
    try {
        size_t wbytes = ggml_row_size((ggml_type)wtype, K) * N;
        Ctx c(wbytes + (size_t)(M * K + M * N) * 4 + (size_t)M * K * 2 + (64u << 20));
        ggml_tensor* tw = ggml_new_tensor_2d(c.ctx, (ggml_type)wtype, K, N);
        ggml_tensor* tx = ggml_new_tensor_2d(c.ctx, GGML_TYPE_F32, K, M);
        std::memcpy(tw->data, w, wbytes);
        std::memcpy(tx->data, x, (size_t)M * K * 4);
        ggml_tensor* ty = ggml_mul_mat(c.ctx, tw, tx);
        if (run_graph(c.ctx, ty, n_threads)) { g_err = "compute failed"; return -1; }
        std::memcpy(y, ty->data, (size_t)M * N * 4);
        return 0;
    } catch (const std::exception& e) { g_err = e.what(); return -1; }
}

// y = rms_norm(x) [* gamma] over rows of length d (ops.cpp:3859-3920).
int ref_rms_norm(const float* x, int64_t d, int64_t rows, float eps, const float* gamma, float* y,
                 int n_threads) {
    try {
        Ctx c((size_t)(rows * d * 3 + d) * 4 + (16u << 20));
        ggml_tensor* tx = ggml_new_tensor_2d(c.ctx, GGML_TYPE_F32, d, rows);
        std::memcpy(tx->data, x, (size_t)rows * d * 4);
        ggml_tensor* t = ggml_rms_norm(c.ctx, tx, eps);
        if (gamma) {
            ggml_tensor* tg = ggml_new_tensor_1d(c.ctx, GGML_TYPE_F32, d);
            std::memcpy(tg->data, gamma, (size_t)d * 4);
            t = ggml_mul(c.ctx, t, tg);
        }
        if (run_graph(c.ctx, t, n_threads)) { g_err = "compute failed"; return -1; }
        std::memcpy(y, t->data, (size_t)rows * d * 4);
        return 0;
    } catch (const std::exception& e) { g_err = e.what(); return -1; }
}

// NEOX RoPE over x[s, H, hd] (ggml ne = [hd, H, s]) with positions pos[s] (ops.cpp:5893-6016).
int ref_rope_neox(const float* x, int64_t hd, int64_t H, int64_t s, const int32_t* pos,
                  int n_dims, float freq_base, float* y, int n_threads) {
    try {
        Ctx c((size_t)(s * H * hd * 3) * 4 + (16u << 20));
        ggml_tensor* tx = ggml_new_tensor_3d(c.ctx, GGML_TYPE_F32, hd, H, s);
        ggml_tensor* tp = ggml_new_tensor_1d(c.ctx, GGML_TYPE_I32, s);
        std::memcpy(tx->data, x, (size_t)s * H * hd * 4);
        std::memcpy(tp->data, pos, (size_t)s * 4);
        ggml_tensor* t = ggml_rope_ext(c.ctx, tx, tp, nullptr, n_dims, 2 /*NEOX*/, 0, freq_base, 1.0f,
                                       0.0f, 1.0f, 0.0f, 0.0f);
        if (run_graph(c.ctx, t, n_threads)) { g_err = "compute failed"; return -1; }
        std::memcpy(y, t->data, (size_t)s * H * hd * 4);
        return 0;
    } catch (const std::exception& e) { g_err = e.what(); return -1; }
}

// silu(gate)*up over rows of [gate(ffn) ; up(ffn)] (ops.cpp:3246-3303).
int ref_swiglu(const float* x, int64_t ffn, int64_t rows, float* y, int n_threads) {
    try {
        Ctx c((size_t)(rows * ffn * 4) * 4 + (16u << 20));
        ggml_tensor* tx = ggml_new_tensor_2d(c.ctx, GGML_TYPE_F32, 2 * ffn, rows);
        std::memcpy(tx->data, x, (size_t)rows * 2 * ffn * 4);
        ggml_tensor* t = ggml_swiglu(c.ctx, tx);
        if (run_graph(c.ctx, t, n_threads)) { g_err = "compute failed"; return -1; }
        std::memcpy(y, t->data, (size_t)rows * ffn * 4);
        return 0;
    } catch (const std::exception& e) { g_err = e.what(); return -1; }
}

// Flash attention over an F16 cache, exactly as the executor's padded-KV path builds it
// (executor.cpp:2160-2197): q f32 [s, Hq, hd] (ggml ne [hd, s, Hq]), k/v f16 [Hkv, n_kv, hd]
// (ggml ne [hd, n_kv, Hkv]), mask f16 [s, n_kv] (0 or -32768) or null.  Output y[s, Hq, hd]
// (the op's permuted result, ne [hd, Hq, s]).
int ref_flash_attn(const float* q, const uint16_t* k, const uint16_t* v, const uint16_t* mask,
                   int64_t hd, int64_t s, int64_t Hq, int64_t Hkv, int64_t n_kv, float scale,
                   float* y, int n_threads) {
    try {
        Ctx c((size_t)(s * Hq * hd * 2) * 4 + (size_t)(2 * n_kv * Hkv * hd + s * n_kv) * 2 +
              (64u << 20));
        ggml_tensor* tq = ggml_new_tensor_3d(c.ctx, GGML_TYPE_F32, hd, s, Hq);
        ggml_tensor* tk = ggml_new_tensor_3d(c.ctx, GGML_TYPE_F16, hd, n_kv, Hkv);
        ggml_tensor* tv = ggml_new_tensor_3d(c.ctx, GGML_TYPE_F16, hd, n_kv, Hkv);
        std::memcpy(tq->data, q, (size_t)s * Hq * hd * 4);
        std::memcpy(tk->data, k, (size_t)n_kv * Hkv * hd * 2);
        std::memcpy(tv->data, v, (size_t)n_kv * Hkv * hd * 2);
        ggml_tensor* tm = nullptr;
        if (mask) {
            tm = ggml_new_tensor_2d(c.ctx, GGML_TYPE_F16, n_kv, s);
            std::memcpy(tm->data, mask, (size_t)s * n_kv * 2);
        }
        ggml_tensor* t = ggml_flash_attn_ext(c.ctx, tq, tk, tv, tm, scale, 0.0f, 0.0f);
        if (run_graph(c.ctx, t, n_threads)) { g_err = "compute failed"; return -1; }
        std::memcpy(y, t->data, (size_t)s * Hq * hd * 4);
        return 0;
    } catch (const std::exception& e) { g_err = e.what(); return -1; }
}

// --- model level (ggmlc::ModelExecutor on device "cpu") ---------------------------------------

void* ref_model_open(const char* path, int n_threads) {
    try {
        auto* m = new RefModel();
        m->graph = ggmlc::ModelLoader::load_from_file(path);
        m->exec.reset(new ggmlc::ModelExecutor(m->graph, "cpu"));
        m->n_threads = n_threads;
        return m;
    } catch (const std::exception& e) { g_err = e.what(); return nullptr; }
}

void ref_model_close(void* h) { delete static_cast<RefModel*>(h); }

int ref_model_init_kv(void* h, int64_t max_ctx) {
    try {
        auto* m = static_cast<RefModel*>(h);
        m->exec->init_kv_cache(max_ctx);
        return m->exec->has_kv_cache() ? 1 : 0;
    } catch (const std::exception& e) { g_err = e.what(); return -1; }
}

int ref_model_reset_kv(void* h) {
    try { static_cast<RefModel*>(h)->exec->reset_kv_cache(); return 0; }
    catch (const std::exception& e) { g_err = e.what(); return -1; }
}

void ref_model_set_logits_last_only(void* h, int on) {
    static_cast<RefModel*>(h)->exec->set_logits_last_only(on != 0);
}

// One forward over tokens[0..s) at position pos (pos < 0: no "pos" symbol, plain forward).
// Binds every graph symbol to s and the first input to the tokens; a second input (GPT-2
// position_ids) gets pos..pos+s-1.  Copies the single output's f32 payload into out (capacity
// out_cap floats) and returns the element count, or -1 on error.
int64_t ref_model_forward(void* h, const int32_t* tokens, int64_t s, int64_t pos, float* out,
                          int64_t out_cap) {
    try {
        auto* m = static_cast<RefModel*>(h);
        std::unordered_map<std::string, int64_t> env;
        for (const auto& sym : m->graph.symbol_table) env[sym] = s;
        env["s"] = s;
        if (pos >= 0) env["pos"] = pos;
        m->exec->prepare(env, true);
        const auto& ins = m->graph.inputs;
        if (ins.empty()) throw std::runtime_error("graph has no inputs");
        m->exec->set_input(ins[0], tokens, (size_t)s * 4);
        if (ins.size() > 1) {
            std::vector<int32_t> p((size_t)s);
            for (int64_t i = 0; i < s; ++i) p[(size_t)i] = (int32_t)((pos < 0 ? 0 : pos) + i);
            m->exec->set_input(ins[1], p.data(), (size_t)s * 4);
        }
        m->exec->run(m->n_threads);
        uint32_t oid = m->graph.outputs.at(0);
        size_t nb = m->exec->get_tensor_size_bytes(oid);
        const void* src = m->exec->get_output_data(oid);
        int64_t n = (int64_t)(nb / 4);
        if (n > out_cap) throw std::runtime_error("output buffer too small");
        std::memcpy(out, src, nb);
        return n;
    } catch (const std::exception& e) { g_err = e.what(); return -1; }
}

}  // extern "C"
