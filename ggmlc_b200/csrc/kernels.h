// Host-side declarations of the engine's CUDA kernels (launchers).  Every launcher takes the
// stream explicitly; none allocates memory.  Layout conventions (all device memory):
//   quantized weight  W[N][K] ("super-group layout"): a row is one contiguous stream of
//                     super-groups (SG) of 8 blocks, each SG = the quants of two groups of 4
//                     blocks followed by the 8 fp16 block scales (16 B): Q8_0 SG = 2x128 + 16 =
//                     272 B, Q4_0 SG = 2x64 + 16 = 144 B.  A block's quants are read as 32-bit
//                     words: Q8_0 has 8 (word w = elements 4w..4w+3), Q4_0 has 4 (word w = GGUF
//                     bytes 4w..4w+3: low nibbles elements 4w.., high nibbles 16+4w..).
//                     Q8_0 group (128 B): [t 0..3][block j 0..3][word t, word t+4];
//                     Q4_0 group (64 B):  [t 0..3][block j 0..3][word t] —
//                     thread t of a row's quad reads its words of 4 blocks in 16-byte loads.
//                     Padding blocks (K/32 rounded up to 8) are zero.
//   Q8_0 activations  X[M][K]: xq = M rows of K int8, xd = M rows of K/32 fp32 scales (the fp16
//                     scale widened, exactly as the CPU reads it).
__host__ __device__ inline int64_t n_sg(int64_t K) { return ((K / 32) + 7) / 8; }
__host__ __device__ inline int64_t sg_bytes(int type) { return type == 8 ? 272 : 144; }
__host__ __device__ inline int64_t qrow_bytes(int type, int64_t K) { return n_sg(K) * sg_bytes(type); }
// byte offset, inside a weight row, of 32-bit word w of block b / of block b's fp16 scale
__host__ __device__ inline int64_t w_word_off(int type, int64_t b, int w) {
    const int64_t sg = b >> 3, bb = b & 7;
    if (type == 8)
        return sg * 272 + (bb >> 2) * 128 + (w & 3) * 32 + (bb & 3) * 8 + (w >> 2) * 4;
    return sg * 144 + (bb >> 2) * 64 + w * 16 + (bb & 3) * 4;
}
__host__ __device__ inline int64_t w_scale_off(int type, int64_t b) {
    return (b >> 3) * sg_bytes(type) + (type == 8 ? 256 : 128) + (b & 7) * 2;
}
// activation staging (shared memory): Q8_0 words in 4-block groups, same order as a Q8_0
// weight group: [group][t 0..3][block j][word t, word t+4]
__host__ __device__ inline int64_t x_word_off(int64_t b, int w) {
    return (b >> 2) * 128 + (w & 3) * 32 + (b & 3) * 8 + (w >> 2) * 4;
}
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace gb {

// Per-step values read by kernels inside captured graphs (decode replays change only these).
struct StepParams {
    int64_t pos;  // first position of this call's tokens in the KV cache
};

struct QWeight {
    int type = 0;               // T_Q8_0 or T_Q4_0 (or T_F32 / T_F16 for float weights)
    int64_t N = 0, K = 0;       // rows, columns
    const void* qs = nullptr;   // super-group rows (or float data for T_F32 / T_F16)
};

// ---- quantization ----------------------------------------------------------------------------
// Q8_0 activation quantization with the x86 AVX2 CPU semantics (amax/127 -> fp16 scale,
// q = rint(x * 127/amax)).  x rows are `x_stride` floats apart.
void launch_quantize_q8_0(const float* x, int64_t x_stride, int64_t M, int64_t K, int8_t* xq,
                          float* xd, cudaStream_t st);

// Repack a GGUF block tensor (N rows of K elements, 34/18-byte blocks) into the super-group
// layout.  qs must hold N * qrow_bytes(type, K) bytes; padding is zeroed.
void launch_repack_blocks(const uint8_t* gguf, int type, int64_t N, int64_t K, void* qs,
                          cudaStream_t st);

// GET_ROWS: rows ids[i] of a quantized / f16 / f32 table [V][K] dequantized to f32 out[i][K].
void launch_get_rows(const QWeight& w, const int32_t* ids, int64_t n, float* out,
                     int64_t out_stride, cudaStream_t st);

// ---- matmul -----------------------------------------------------------------------------------
// Y[m][n] = sum_k X[m][k] W[n][k] (+ bias[n]) (+ residual[m][n]) for Q8_0/Q4_0 W and Q8_0 X.
// Bit-exact with the reference x86 CPU kernels: 8 fp32 lane accumulators per output, lane i
// holding the int32 dot of elements 4i..4i+3 of each block, fma(d_w*d_x, lane, acc) block by
// block, lanes reduced ((a0+a4)+(a2+a6))+((a1+a5)+(a3+a7)).
struct MatmulEpilogue {
    const float* bias = nullptr;      // [N] or null
    const float* residual = nullptr;  // [M][res_stride] or null
    int64_t res_stride = 0;
};
void launch_matmul_q_exact(const QWeight& w, const int8_t* xq, const float* xd, int64_t M,
                           float* y, int64_t y_stride, const MatmulEpilogue& ep,
                           cudaStream_t st);
// Decode GEMV with fused prologue / epilogue (M <= 8, bit-exact like launch_matmul_q_exact).
//   input : Q8_0 rows (xq, xd), or f32 rows xf normalized in the prologue — RMSNorm with eps
//           and optional gamma, exactly as launch_rms_norm — and quantized to Q8_0 in shared
//           memory (the standalone norm and quantize launches disappear);
//   output: f32 rows y (+bias, +residual), or SwiGLU of row pairs (gate n, up n+F) emitted as
//           Q8_0 rows (yq, yd) and/or f32 rows (y) of length F — exactly launch_swiglu.
struct GemvArgs {
    QWeight w;
    int M = 1;
    const int8_t* xq = nullptr;  // input mode 0
    const float* xd = nullptr;
    const float* xf = nullptr;   // input mode 1 (RMSNorm prologue)
    int64_t xf_stride = 0;
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
};
void launch_gemv_fused(const GemvArgs& a, cudaStream_t st);
bool gemv_fused_fits(int64_t K, int M);
// The GEMV's pipeline waits are bounded; a timeout is recorded in a per-device error word
// (1: producer, 2: consumer) instead of hanging.  gemv_prepare_device allocates that word
// (call before graph capture); gemv_error_code reads it (0 = none).
void gemv_prepare_device(int dev);
int gemv_error_code(int dev);

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
struct KVDst {
    __half* base = nullptr;  // [H][ctx][hd]
    int64_t ctx = 0;         // rows per head
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
};
int attn_decode_splits(int64_t Hkv, int64_t max_kv);
size_t attn_decode_workspace(int64_t Hq, int64_t hd, int splits);
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
void launch_attention(const TView& q, const __half* kc, const __half* vc, int64_t ctx,
                      int64_t Hkv, const StepParams* step, bool use_step, int64_t kv_off,
                      float scale, float* o, void* work, int64_t max_kv, cudaStream_t st);

}  // namespace gb
