// Host-side declarations of the engine's CUDA kernels (launchers).  Every launcher takes the
// stream explicitly; none allocates memory.  Layout conventions (all device memory):
//   quantized weight  W[N][K] ("split-row layout"): a row holds the quants of its nb = K/32
//                     blocks in block order, then the fp16 block scales.  A block's quants are
//                     32-bit words: Q8_0 has 8 (word w = elements 4w..4w+3), Q4_0 has 4 (word w
//                     = GGUF bytes 4w..4w+3: low nibbles are elements 4w.., high 16+4w..).
//                     Q4_0 row: [nb][16 B] quants.  Q8_0 row: [nb][16 B] words 0-3, then
//                     [nb][16 B] words 4-7.  A warp whose lanes take consecutive blocks reads 512
//                     contiguous bytes per 16-byte load.  Scales come in groups of 64 blocks,
//                     ordered [lane l 0..31][i 0..1] for block 64g + 32i + l, so the lane that
//                     owns blocks l and l+32 of a group reads both scales with one 4-byte load;
//                     the scale region is padded to whole groups (zero scales).
//   Q8_0 activations  X[M][K]: xq = M rows of K int8, xd = M rows of K/32 fp32 scales (the fp16
//                     scale widened, exactly as the CPU reads it).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace gb {

// Per-step values read by kernels inside captured graphs (decode replays change only these).
constexpr int kMaxRows = 16;  // rows of a batched decode step (sequences decoded together)
constexpr int kMaxOutRows = 64;  // rows an output projection can be restricted to (out_rows)
struct StepParams {
    int64_t pos;                  // first position of this call's tokens in the KV cache
    int32_t row_pos[kMaxRows];    // batched decode: position of each row's token
    int32_t row_slot[kMaxRows];   // batched decode: KV-cache slot of each row's sequence
    int32_t out_rows[kMaxOutRows];  // rows of this call whose outputs are computed (out_rows)
};

__host__ __device__ inline int64_t quant_bytes(int type) { return type == 8 ? 32 : 16; }
__host__ __device__ inline int64_t scale_region(int64_t nb) { return ((nb + 63) / 64) * 128; }
__host__ __device__ inline int64_t qrow_bytes(int type, int64_t K) {
    const int64_t nb = K / 32;
    return nb * quant_bytes(type) + scale_region(nb);
}
// byte offset, inside a weight row of nb blocks, of 32-bit word w of block b / of b's scale
__host__ __device__ inline int64_t w_word_off(int type, int64_t nb, int64_t b, int w) {
    if (type == 8) return (w >> 2) * nb * 16 + b * 16 + (w & 3) * 4;
    return b * 16 + w * 4;
}
__host__ __device__ inline int64_t w_scale_off(int type, int64_t nb, int64_t b) {
    return nb * quant_bytes(type) + (b >> 6) * 128 + (b & 31) * 4 + ((b >> 5) & 1) * 2;
}

struct QWeight {
    int type = 0;               // T_Q8_0 or T_Q4_0 (or T_F32 / T_F16 for float weights)
    int64_t N = 0, K = 0;       // rows, columns
    const void* qs = nullptr;   // split-row layout rows (or float data for T_F32 / T_F16)
};

// ---- quantization ----------------------------------------------------------------------------
// Q8_0 activation quantization with the x86 AVX2 CPU semantics (amax/127 -> fp16 scale,
// q = rint(x * 127/amax)).  x rows are `x_stride` floats apart.
void launch_quantize_q8_0(const float* x, int64_t x_stride, int64_t M, int64_t K, int8_t* xq,
                          float* xd, cudaStream_t st);

// Repack a GGUF block tensor (N rows of K elements, 34/18-byte blocks) into the split-row
// layout.  qs must hold N * qrow_bytes(type, K) bytes; padding is zeroed.
void launch_repack_blocks(const uint8_t* gguf, int type, int64_t N, int64_t K, void* qs,
                          cudaStream_t st);

// Index of the first maximum of each of `rows` f32 rows of length n (greedy sampling).
void launch_argmax_rows(const float* x, int64_t rows, int64_t n, int32_t* out, cudaStream_t st);

// GET_ROWS: rows ids[i] of a quantized / f16 / f32 table [V][K] dequantized to f32 out[i][K].
void launch_get_rows(const QWeight& w, const int32_t* ids, int64_t n, float* out,
                     int64_t out_stride, cudaStream_t st);

// ---- matmul -----------------------------------------------------------------------------------
// Y[m][n] = sum_k X[m][k] W[n][k] (+ bias[n]) (+ residual[m][n]) for Q8_0/Q4_0 W and Q8_0 X.
// Per 32-element block the int32 dot is exact; block terms sumi * (d_w * d_x) accumulate in fp32
// (the reference's generic block formula; the x86 lane order differs only in rounding).
// M <= 2 runs the decode GEMV, M <= 16 the tensor-core decode kernel, larger M the block GEMM.
struct MatmulEpilogue {
    const float* bias = nullptr;      // [N] or null
    const float* residual = nullptr;  // [M][res_stride] or null
    int64_t res_stride = 0;
};
void launch_matmul_q(const QWeight& w, const int8_t* xq, const float* xd, int64_t M, float* y,
                     int64_t y_stride, const MatmulEpilogue& ep, cudaStream_t st);
// Decode GEMV with fused prologue / epilogue (M <= kGemvMaxRows).  Q8_0 input with more than
// kGemvRouteRows rows goes to launch_mmv, and past 16 rows to the block GEMM, with the same
// epilogues.  Lanes run along K, so each row costs a fixed number of instructions per weight
// byte; for 1-2 rows this beats the tensor-core kernel, whose 16x8 tiles are mostly idle there
// (at 3-4 rows the tensor-core kernel fed by the standalone RMSNorm is the faster step).
// Launched as a programmatic dependent launch: its weight loads start before the previous kernel
// on the stream has finished.
//   input : Q8_0 rows (xq, xd; xq 16-byte aligned), or f32 rows xf quantized to Q8_0 in shared
//           memory, after RMSNorm with eps and optional gamma when xf_rms (exactly as
//           launch_rms_norm) — the standalone norm and quantize launches disappear;
//   output: f32 rows y (+bias, +residual), or SwiGLU of row pairs (gate n, up n+F) emitted as
//           Q8_0 rows (yq, yd) and/or f32 rows (y) of length F — exactly launch_swiglu.
constexpr int kGemvMaxRows = 4;
constexpr int kGemvRouteRows = 2;  // rows the engine sends to the GEMV (fused RMSNorm included)
// Tensor-parallel peer buffers (k_allreduce.cu, k_dgemv.cu).
constexpr int kMaxTp = 8;
constexpr int kArCtas = 4;
constexpr int kGemvArCtas = 160;  // CTAs of a decode GEMV with the all-reduce in its epilogue
struct TpPeers {
    float* recv[kMaxTp];       // rank r's receive slots [2][T][cap]
    uint32_t* flags[kMaxTp];   // rank r's flags [2][T][kArCtas]
    float* grecv[kMaxTp];      // the same for the GEMV epilogue's all-reduce: [2][T][cap]
    uint32_t* gflags[kMaxTp];  // [2][T][kGemvArCtas]
};
// All-reduce folded into the epilogue of the single-row decode GEMV (k_dgemv.cu): every CTA,
// once its rows of y are final, stores them into slot [parity][rank] of every rank (NVLink
// stores), raises its flag there (system-scope release), waits (bounded) for the same CTA of
// every rank and sums its rows over the ranks in rank order, so every rank holds the same bits.
// The slots, flags and per-CTA epochs are its own (not the standalone kernel's).  T == 0: none.
struct GemvAllReduce {
    TpPeers peers;
    int rank = 0, T = 0;
    uint32_t* epochs = nullptr;  // kGemvArCtas per-CTA counters of this rank
    int64_t cap = 0;             // floats per slot
    int* err = nullptr;          // set when a wait for a peer ran out
};

// The weights a GEMV launch streams, described for the launch before it (L2 prefetch)
struct PfNext {
    const void* qs = nullptr;  // split-row rows; null: nothing to prefetch
    int type = 0;
    int64_t N = 0, K = 0;
    int64_t F = 0;             // SwiGLU: the up rows start F rows after the gate rows (0: plain)
};
struct GemvArgs {
    QWeight w;
    int M = 1;
    const int8_t* xq = nullptr;  // Q8_0 input
    const float* xd = nullptr;
    const float* xf = nullptr;   // f32 input, quantized in the prologue
    int64_t xf_stride = 0;
    bool xf_rms = true;          // RMSNorm the f32 input first
    float eps = 0.0f;
    const float* gamma = nullptr;
    bool swiglu = false;         // output mode
    int64_t F = 0;               // SwiGLU half width (w.N == 2F)
    float* y = nullptr;
    int64_t y_stride = 0;
    const float* bias = nullptr;
    const float* residual = nullptr;
    int64_t res_stride = 0;
    int8_t* yq = nullptr;
    float* yd = nullptr;
    // L2 prefetch (launch_dgemv only): the weights of the next GEMV launch; each CTA requests,
    // at its start, the rows that the same CTA index of that launch streams first
    PfNext pf;
    // tensor parallelism: y summed over the ranks in the epilogue (launch_dgemv, one row)
    GemvAllReduce ar;
};
void launch_gemv_fused(const GemvArgs& a, cudaStream_t st);
// whether the GEMV's shared-memory stage fits: gemv_fits for one configuration (staged = f32
// input, gamma = with gamma), gemv_fused_fits for Q8_0 input with either weight type
bool gemv_fits(int type, int64_t K, int M, bool staged, bool gamma);
bool gemv_fused_fits(int64_t K, int M);
// Decode / small-batch matmul on int8 tensor cores (k_mmv.cu): Q8_0 input only (xq, xd), M <= 16,
// the GemvArgs epilogues (bias / residual, or SwiGLU to f32 and/or Q8_0).  Any K.  A row's
// result does not depend on M (nor on the epilogue mode).  Programmatic dependent launch.
constexpr int kMmvMaxRows = 16;
void launch_mmv(const GemvArgs& a, cudaStream_t st);
// Single-row decode GEMV with bulk-copy weight rings (k_dgemv.cu): M == 1, Q8_0 or f32 input (the
// GemvArgs prologues), f32 output (+bias, +residual) or SwiGLU to f32 (no Q8_0 output).
// launch_gemv_fused sends every eligible single-row call here.  dgemv_error() reads its sticky
// error word (non-zero after one of its bounded waits ran out).
bool dgemv_eligible(const GemvArgs& a);
void launch_dgemv(const GemvArgs& a, cudaStream_t st);
int dgemv_error();
// Prefill gate_up matmul (M > 16) with the SwiGLU epilogue of GemvArgs (k_matmul.cu): Q8_0 input,
// N == 2F, F % 64 == 0, no bias / residual; outputs f32 y and/or Q8_0 yq, yd.
void launch_gemm_swiglu(const GemvArgs& a, cudaStream_t st);
// Prefill matmul on the 5th-generation tensor cores (k_gemm_tc.cu): tcgen05 int8 MMA into
// tensor memory, per-block scales in the epilogue; any M.  gemm_tc_error() reads the kernel's
// sticky error word (non-zero after one of its bounded waits ran out).
void launch_gemm_tc(const QWeight& w, const int8_t* xq, const float* xd, int64_t M, float* y,
                    int64_t y_stride, const MatmulEpilogue& ep, cudaStream_t st);
// The same with the SwiGLU epilogue of launch_gemm_swiglu (N == 2F, F % 64 == 0).
void launch_gemm_tc_swiglu(const GemvArgs& a, cudaStream_t st);
// whether the tcgen05 GEMM takes this K (its TMA stages are 4 blocks: K % 128 == 0)
bool gemm_tc_fits(int64_t K);
// Split K of the prefill GEMMs (k_matmul.cu, k_gemm_tc.cu): plain GEMMs whose tiles fill at most
// half the SMs cut K into gridDim.z ranges whose partial sums [z][M][N] (stream-ordered scratch)
// launch_splitk_sum adds in split order before bias and residual.  GGMLC_B200_SPLITK=0: off.
bool splitk_enabled();
void launch_splitk_sum(const float* part, int splits, int M, int N, float* y, int64_t y_stride,
                       const MatmulEpilogue& ep, cudaStream_t st);
int gemm_tc_error();

// Tensor-parallel one-shot all-reduce (k_allreduce.cu): y[0..n) summed over T ranks through
// peer-mapped buffers of `cap` floats per slot (n <= cap); identical bits on every rank.
// `epochs` holds kArCtas per-rank counters (zero at set-up), `err` is set non-zero when a bounded
// wait for a peer ran out.  Every rank must make the same sequence of calls.
void launch_tp_allreduce(float* y, int64_t n, const TpPeers& peers, int rank, int T,
                         uint32_t* epochs, int64_t cap, int* err, cudaStream_t st);

// Float-weight matmul (F32/F16 W, f32 X), used for non-quantized linears.
void launch_matmul_f(const QWeight& w, const float* x, int64_t x_stride, int64_t M, float* y,
                     int64_t y_stride, const MatmulEpilogue& ep, cudaStream_t st);

// ---- norms / activations --------------------------------------------------------------------
// RMSNorm (fp32 squares summed in double, scale = 1/sqrtf(mean+eps)), optional gamma; writes f32
// rows (y) and/or Q8_0 rows (yq, yd).
void launch_rms_norm(const float* x, int64_t x_stride, int64_t M, int64_t D, float eps,
                     const float* gamma, float* y, int64_t y_stride, int8_t* yq, float* yd,
                     cudaStream_t st);
// LayerNorm (NORM op semantics of the x86 CPU build), optional gamma / beta.
void launch_layer_norm(const float* x, int64_t x_stride, int64_t M, int64_t D, float eps,
                       const float* gamma, const float* beta, float* y, int64_t y_stride,
                       int8_t* yq, float* yd, cudaStream_t st);
// SwiGLU over rows [gate(F) ; up(F)] (x row stride x_stride) -> F outputs, f32 and/or Q8_0.
void launch_swiglu(const float* x, int64_t x_stride, int64_t M, int64_t F, bool swapped,
                   float* y, int64_t y_stride, int8_t* yq, float* yd, cudaStream_t st);
// bias + tanh-GELU (fast_gelu_f32 of the reference's CPU custom op), f32 and/or Q8_0.
void launch_bias_gelu(const float* x, int64_t x_stride, const float* bias, int64_t M, int64_t F,
                      float* y, int64_t y_stride, int8_t* yq, float* yd, cudaStream_t st);

// ---- generic strided tensors ------------------------------------------------------------------
struct TView {
    char* data = nullptr;
    int type = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    int64_t nb[4] = {0, 0, 0, 0};  // byte strides
};
// dst = a (op) b with ggml broadcasting of b over a; op: 0 add, 1 mul.  f32 only.
void launch_binary(const TView& a, const TView& b, const TView& dst, int op, cudaStream_t st);
// dst = src (any strides, f32/f16/i32 with conversion to dst type).
void launch_copy(const TView& src, const TView& dst, cudaStream_t st);
// y[r][:] = x[step->out_rows[r]][:] for r < n (f32 rows of K, x rows x_stride floats apart)
void launch_gather_rows(const float* x, int64_t x_stride, const StepParams* step, int n, int64_t K,
                        float* y, cudaStream_t st);

// ---- RoPE / KV cache / attention ---------------------------------------------------------------
// NEOX RoPE.  x: f32 view [hd, H, s] (ne0 contiguous); positions = pos_src[pos_off + i] where
// pos_off = step->pos when use_step_pos else 0.  cos/sin come from `table` (n_pos x n_dims/2
// pairs computed on the host with the CPU's theta recurrence) when the position is inside it.
// Output either f32 view y, or (kv != null) f16 rows into a KV cache at row step->pos + i.
struct RopeTable {
    const float2* cs = nullptr;  // [n_pos][n_dims/2] (cos, sin)
    int64_t n_pos = 0;
    int n_dims = 0;
    float theta_scale = 1.0f;
};
// Where one sequence's K (or V) rows live in a KV cache.
//   contiguous (pages == nullptr): the sequence's window [H][ctx][hd] starts at the base pointer;
//   paged: the base pointer is a layer's page pool [page][H][1 << shift][hd], and pages[i] names
//     the pool page holding the sequence's positions [i << shift, (i + 1) << shift) in every
//     layer (one page table serves all layers).  Batched launches pass slot 0's list; slot s's
//     list starts `stride` entries further on.
struct KvPages {
    const int32_t* pages = nullptr;
    int32_t stride = 0;
    int32_t shift = 0;
};
// element offset of row (h, t) of a sequence whose page list is `pages` (see KvPages)
__host__ __device__ __forceinline__ int64_t kv_row_off(const int32_t* pages, int shift, int64_t H,
                                                       int64_t ctx, int64_t h, int64_t t,
                                                       int64_t hd) {
    if (!pages) return (h * ctx + t) * hd;
    const int64_t pg = pages[t >> shift];
    return (((pg * H + h) << shift) + (t & ((int64_t(1) << shift) - 1))) * hd;
}
struct KVDst {
    __half* base = nullptr;  // [H][ctx][hd], or a page pool (pages != nullptr)
    int64_t ctx = 0;         // rows per head
    const int32_t* pages = nullptr;
    int32_t shift = 0;
};
void launch_rope_neox(const TView& x, const int32_t* pos_src, bool use_step_pos,
                      const StepParams* step, const RopeTable& tab, const TView* y,
                      const KVDst* kv, cudaStream_t st);
// Write s rows of a f32 view [hd, H, s] into a f16 KV cache at rows step->pos + i.
void launch_kv_write(const TView& src, const StepParams* step, const KVDst& kv, cudaStream_t st);

// Fused RoPE + KV write straight from the QKV projection output (rows of qkv_stride floats,
// q/k/v heads at float offsets q_off/k_off/v_off): rotated q -> q_out [s][Hq][hd] f32, rotated k
// and v -> cache rows base+t, base = step->pos (if step) + pos_off.  tab.n_dims == 0 disables
// the rotation (models without RoPE).
struct QkvRopeArgs {
    const float* qkv = nullptr;
    int64_t qkv_stride = 0, q_off = 0, k_off = 0, v_off = 0;
    int Hq = 0, Hkv = 0, hd = 0;
    int64_t s = 0;
    RopeTable tab;
    const StepParams* step = nullptr;
    int64_t pos_off = 0;
    float* q_out = nullptr;
    __half* kc = nullptr;
    __half* vc = nullptr;
    int64_t ctx = 0;
    const int32_t* pages = nullptr;  // paged cache: this sequence's page list (KvPages)
    int32_t page_shift = 0;
};
void launch_rope_qkv(const QkvRopeArgs& a, cudaStream_t st);

// Decode attention (one new token) fused with its RoPE and KV write: split-KV over the cache
// (splits CTAs per KV head) and a combine that writes o (f32 [Hq][hd]) and/or the Q8_0 rows of
// the output projection's input (oq [Hq*hd], od [Hq*hd/32]).  part: attn_decode_workspace().
struct AttnDecArgs {
    const float* qkv = nullptr;
    int64_t q_off = 0, k_off = 0, v_off = 0;
    int Hq = 0, Hkv = 0, hd = 0;
    RopeTable tab;
    const StepParams* step = nullptr;
    int64_t pos_off = 0;
    __half* kc = nullptr;
    __half* vc = nullptr;
    int64_t ctx = 0;
    float scale = 1.0f;
    int splits = 1;
    int64_t max_kv = 0;
    float* part = nullptr;
    float* o = nullptr;
    int8_t* oq = nullptr;
    float* od = nullptr;
    // batched decode (rows > 1 or batched): row r of qkv (qkv_stride floats apart) is the new
    // token of a sequence at position step->row_pos[r] in KV slot step->row_slot[r]; slots are
    // slot_elems elements apart in kc / vc; outputs and partials are per row
    int rows = 1;
    bool batched = false;
    int64_t qkv_stride = 0;
    int64_t slot_elems = 0;
    // paged cache (KvPages): kc / vc are the layer's page pools; a single sequence's page list,
    // or for batched launches slot 0's list with row r's at pg.pages + row_slot[r] * pg.stride
    KvPages pg;
};
// splits per (row, KV head): about two CTAs per SM over all rows and heads of the launch
int attn_decode_splits(int64_t Hkv, int64_t max_kv, int rows = 1);
size_t attn_decode_workspace(int64_t Hq, int64_t hd, int splits);  // per row
// CTAs per (row, KV head) when decode attention runs as one launch whose thread-block clusters
// merge their partials in distributed shared memory (head_dim 64 / 128, caches up to a few
// thousand positions); 0 when it takes the split workspace and the merge launch.  The workspace
// argument is not read in the first case.
int attn_decode_cluster(int64_t Hkv, int64_t hd, int64_t ctx, int rows = 1);
void launch_attn_decode(const AttnDecArgs& a, cudaStream_t st);
// Size of the per-device static split scratch behind gb_attn_decode_noalloc.
constexpr size_t kAttnDecStaticWorkBytes = size_t(4) << 20;
// Device address of that scratch on the current device (looked up once per device); throws when
// need exceeds kAttnDecStaticWorkBytes.
float* attn_decode_static_work(size_t need);

// Attention of q (f32 view [hd, s, Hq]) over KV caches [Hkv][ctx][hd] f16, causal at absolute
// positions: query i sees cache rows 0 .. kv_base + i where kv_base = step->pos (use_step) or 0.
// Output o: f32 [s][Hq][hd] contiguous (the FLASH_ATTN_EXT permuted result) .  Q is rounded to
// fp16 like the CPU kernel.  work: scratch of attn_workspace_bytes().
size_t attn_workspace_bytes(int64_t s, int64_t Hq, int64_t hd, int64_t max_kv);
// A paged cache passes its page pools as kc / vc and the sequence's page list (KvPages).
void launch_attention(const TView& q, const __half* kc, const __half* vc, int64_t ctx,
                      int64_t Hkv, const StepParams* step, bool use_step, int64_t kv_off,
                      float scale, float* o, void* work, int64_t max_kv, cudaStream_t st,
                      const int32_t* pages = nullptr, int page_shift = 0);

// ---- decode chain (k_chain.cu) ---------------------------------------------------------------
// The launches of one single-sequence decode step — quantized GEMVs with their RMSNorm / quantize
// prologues and residual / SwiGLU epilogues, decode attention with its RoPE and K/V write, row
// norms — run as ONE persistent launch: one CTA per SM, the ops in order with a grid-wide barrier
// between them, and per-warp bulk-copy rings that keep requesting the weights of the next GEMVs
// while the CTA waits at a barrier or works on attention, so HBM streams across op boundaries.
// Results: every GEMV bit-identical to launch_dgemv on the same input (same block order, lane
// butterfly and chunk order); attention within the attention tests' tolerance (fp32 online
// softmax, another summation order than launch_attn_decode).
enum ChainKind : int { CH_GEMV = 0, CH_ATTN = 1, CH_ROW = 2 };
struct ChainOp {
    int kind = CH_GEMV;
    // CH_GEMV (one row): y = W x; W in the split-row layout, rb bytes per row
    const uint8_t* w = nullptr;
    int wtype = 0;
    int64_t N = 0, K = 0, rb = 0;
    int swiglu = 0;              // y[n] = silu(row n) * row n + F, n < F
    int64_t F = 0;
    const int8_t* xq = nullptr;  // Q8_0 input, or
    const float* xd = nullptr;
    const float* xf = nullptr;   // f32 input quantized in the prologue (CH_ROW: the row)
    int rms = 0;                 // RMSNorm the f32 input first (eps, optional gamma)
    float eps = 0.0f;
    const float* gamma = nullptr;
    float* y = nullptr;          // f32 output (+bias, +residual)
    const float* bias = nullptr;
    const float* residual = nullptr;
    // CH_ATTN: one decode row over the KV cache (rows == 1, not batched); splits per KV head
    AttnDecArgs at;
    int splits = 1;
    // CH_ROW: D elements of xf (RMSNorm when rms) to f32 y and/or Q8_0 (yq, yd)
    int64_t D = 0;
    int8_t* yq = nullptr;
    float* yd = nullptr;
};
// grid-barrier and attention-merge counters of the chain (zero-initialised once; every launch
// leaves them as it found them)
constexpr int kChainMaxKvHeads = 64;
struct ChainSync {
    unsigned count;
    unsigned gen;
    unsigned attn_cnt[kChainMaxKvHeads];
};
// whether one op can run inside the chain (alignment, shapes, kinds the chain implements)
bool chain_gemv_ok(const GemvArgs& a);
bool chain_attn_ok(const AttnDecArgs& a);
bool chain_row_ok(int64_t M, int64_t D);
// a CH_GEMV op from the arguments of launch_gemv_fused; false when the chain does not take them
bool chain_gemv_op(const GemvArgs& a, ChainOp& c);
// fills the derived fields of the ops (row bytes, attention splits for this GPU) and returns the
// f32 elements of the attention-partials scratch the chain needs; throws when an op cannot run
int64_t chain_prepare(ChainOp* ops, int n, int dev);
// ops: device copy of n prepared ops (host_ops: the same on the host); part: chain_prepare's
// floats; sync: zeroed ChainSync; err: device-visible int set to 1 when the launch fails (or null)
void launch_chain(const ChainOp* ops, const ChainOp* host_ops, int n, ChainSync* sync, float* part,
                  int* err, cudaStream_t st);
// sticky error word (non-zero after one of the chain's bounded waits ran out; the sync counters
// are then not trusted and later launches return at once)
int chain_error();

}  // namespace gb
