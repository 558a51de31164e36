/*
 * CPU ORACLE — test infrastructure, not product code.
 *
 * A plain-C restatement of the reference's CPU arithmetic for the ggmlc decoder hot path
 * (vendored ggml 0.20.2 CPU backend + ggmlc runtime).  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / reference legs may load it, and only as the checker; the
 * product (ggmlc_b200/) never links or calls it.
 *
 * Parity pinning: tests/test_oracle_golden.py checks every function here against golden
 * vectors written by tests/golden/make_golden.py from the reference itself (oracle/_ref,
 * built from the reference sources by oracle/Makefile).
 *
 * Reference files are cited as <path inside the ggmlc project>:<line>.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QK 32
#define GGML_TYPE_F32 0
#define GGML_TYPE_F16 1
#define GGML_TYPE_Q4_0 2
#define GGML_TYPE_Q8_0 8

/* ---------------------------------------------------------------- fp16 (IEEE binary16, RNE) */

/* float -> half with round-to-nearest-even, the conversion F16C's vcvtps2ph performs for
 * GGML_CPU_FP32_TO_FP16 (ggml-cpu/simd-mappings.h) and that ggml_fp32_to_fp16 performs. */
uint16_t oracle_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520 -> inf */
    if (ax < 0x38800000u) {                                    /* subnormal half or zero */
        /* value = ax_float; half subnormal unit = 2^-24 */
        float af;
        memcpy(&af, &ax, 4);
        float scaled = af * 16777216.0f; /* exact: power-of-two scaling */
        /* round to nearest even integer */
        float r = nearbyintf(scaled);    /* default rounding mode is RNE */
        return (uint16_t)(sign | (uint32_t)r);
    }
    uint32_t exp = ((ax >> 23) - 127 + 15);
    uint32_t mant = ax & 0x7fffffu;
    uint32_t h = (exp << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1; /* carries into exp correctly */
    return (uint16_t)(sign | h);
}

float oracle_fp16_to_fp32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (mant == 0) {
            x = sign;
        } else { /* subnormal: mant * 2^-24 */
            float v = (float)mant * (1.0f / 16777216.0f);
            memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (exp == 31) {
        x = sign | 0x7f800000u | (mant << 13);
    } else {
        x = sign | ((exp - 15 + 127) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ------------------------------------------------------------------------- block formats */
/* block_q8_0 = { fp16 d; int8 qs[32]; } (34 B), block_q4_0 = { fp16 d; uint8 qs[16]; } (18 B):
 * ggml-common.h:194-198, :251-255.  Q4_0 byte j holds element j (low nibble) and element j+16
 * (high nibble), value (q - 8) * d. */

static inline float blk_d(const uint8_t* b) {
    uint16_t h;
    memcpy(&h, b, 2);
    return oracle_fp16_to_fp32(h);
}

/* dequantize_row_q4_0 ggml-quants.c:459-477, dequantize_row_q8_0 ggml-quants.c:553-567 */
void oracle_dequantize_row(int type, const uint8_t* x, float* y, int64_t k) {
    const int64_t nb = k / QK;
    for (int64_t i = 0; i < nb; i++) {
        if (type == GGML_TYPE_Q8_0) {
            const uint8_t* b = x + i * 34;
            const float d = blk_d(b);
            for (int j = 0; j < QK; j++) y[i * QK + j] = (float)(int8_t)b[2 + j] * d;
        } else if (type == GGML_TYPE_Q4_0) {
            const uint8_t* b = x + i * 18;
            const float d = blk_d(b);
            for (int j = 0; j < QK / 2; j++) {
                const int x0 = (b[2 + j] & 0x0F) - 8;
                const int x1 = (b[2 + j] >> 4) - 8;
                y[i * QK + j] = x0 * d;
                y[i * QK + j + QK / 2] = x1 * d;
            }
        }
    }
    if (type == GGML_TYPE_F32) memcpy(y, x, (size_t)k * 4);
    if (type == GGML_TYPE_F16) {
        for (int64_t j = 0; j < k; j++) {
            uint16_t h;
            memcpy(&h, x + 2 * j, 2);
            y[j] = oracle_fp16_to_fp32(h);
        }
    }
}

/* Activation quantizer as it runs on x86 hosts with AVX2 (ggml-cpu/arch/x86/quants.c:302-392):
 * amax over the block, d = amax/127 (fp32 division, stored fp16), id = 127/amax (0 when amax
 * is 0), q = round-half-even(x*id) (_mm256_round_ps(_MM_ROUND_NEAREST)). */
void oracle_quantize_row_q8_0(const float* x, uint8_t* y, int64_t k) {
    const int64_t nb = k / QK;
    for (int64_t i = 0; i < nb; i++) {
        const float* xb = x + i * QK;
        uint8_t* b = y + i * 34;
        float amax = 0.0f;
        for (int j = 0; j < QK; j++) {
            const float a = fabsf(xb[j]);
            amax = a > amax ? a : amax;
        }
        const float d = amax / 127.f;
        const uint16_t dh = oracle_fp32_to_fp16(d);
        memcpy(b, &dh, 2);
        const float id = (amax != 0.0f) ? 127.f / amax : 0.0f;
        for (int j = 0; j < QK; j++) {
            volatile float p = xb[j] * id; /* one rounded fp32 product, no contraction */
            float r = nearbyintf(p);       /* RNE in the default rounding mode */
            int v = (int)r;
            if (v > 127) v = 127;          /* _mm256_packs saturation (never reached) */
            if (v < -128) v = -128;
            b[2 + j] = (uint8_t)(int8_t)v;
        }
    }
}

/* Portable scalar quantizer quantize_row_q8_0_ref (ggml-quants.c:276-297): id = 1/d and
 * roundf (half away from zero).  Used by non-x86 hosts; kept to document the tie difference. */
void oracle_quantize_row_q8_0_ref(const float* x, uint8_t* y, int64_t k) {
    const int64_t nb = k / QK;
    for (int64_t i = 0; i < nb; i++) {
        const float* xb = x + i * QK;
        uint8_t* b = y + i * 34;
        float amax = 0.0f;
        for (int j = 0; j < QK; j++) {
            const float a = fabsf(xb[j]);
            amax = a > amax ? a : amax;
        }
        const float d = amax / ((1 << 7) - 1);
        const float id = d ? 1.0f / d : 0.0f;
        const uint16_t dh = oracle_fp32_to_fp16(d);
        memcpy(b, &dh, 2);
        for (int j = 0; j < QK; j++) {
            volatile float p = xb[j] * id;
            b[2 + j] = (uint8_t)(int8_t)roundf(p);
        }
    }
}

/* Exact int32 dot of one weight block with one Q8_0 activation block: the sumi of
 * ggml_vec_dot_q8_0_q8_0 / ggml_vec_dot_q4_0_q8_0 (ggml-cpu/quants.c:225-256, :451-477). */
int32_t oracle_block_dot(int wtype, const uint8_t* wb, const uint8_t* xb) {
    int32_t sumi = 0;
    const int8_t* xq = (const int8_t*)(xb + 2);
    if (wtype == GGML_TYPE_Q8_0) {
        const int8_t* wq = (const int8_t*)(wb + 2);
        for (int j = 0; j < QK; j++) sumi += (int32_t)wq[j] * xq[j];
    } else {
        for (int j = 0; j < QK / 2; j++) {
            const int v0 = (wb[2 + j] & 0x0F) - 8;
            const int v1 = (wb[2 + j] >> 4) - 8;
            sumi += v0 * xq[j] + v1 * xq[j + QK / 2];
        }
    }
    return sumi;
}

static inline int64_t wblock_bytes(int wtype) { return wtype == GGML_TYPE_Q8_0 ? 34 : 18; }

/* sum over blocks of sumi * (d_w * d_x) in fp32 (ggml-cpu/quants.c:225-256).  The SIMD and
 * tinyBLAS variants (arch/x86/quants.c:1308-1370, llamafile/sgemm.cpp:1353) only reorder this
 * fp32 sum. */
float oracle_vec_dot(int wtype, int64_t k, const uint8_t* w, const uint8_t* xq) {
    /* The x86 AVX2 kernels (arch/x86/quants.c:1308-1342 ggml_vec_dot_q8_0_q8_0, the Q4_0 twin,
     * and llamafile tinyBLAS_Q0_AVX sgemm.cpp:1353) all keep 8 fp32 lanes: lane i holds the int32
     * sum of elements 4i..4i+3 of each block (maddubs + madd), accumulated block after block as
     * fma(d_w*d_x, float(lane), acc_i); the lanes are then reduced as
     * ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)) (hsum_float_8).  Restating that order makes this
     * function bit-exact with the reference. */
    const int64_t nb = k / QK;
    const int64_t wbb = wblock_bytes(wtype);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t i = 0; i < nb; i++) {
        const uint8_t* wb = w + i * wbb;
        const uint8_t* xb = xq + i * 34;
        const int8_t* xs = (const int8_t*)(xb + 2);
        int wv[QK];
        if (wtype == GGML_TYPE_Q8_0) {
            for (int j = 0; j < QK; j++) wv[j] = (int8_t)wb[2 + j];
        } else {
            for (int j = 0; j < QK / 2; j++) {
                wv[j] = (wb[2 + j] & 0x0F) - 8;
                wv[j + QK / 2] = (wb[2 + j] >> 4) - 8;
            }
        }
        const float s = blk_d(wb) * blk_d(xb);
        for (int l = 0; l < 8; l++) {
            int32_t p = 0;
            for (int j = 0; j < 4; j++) p += wv[4 * l + j] * xs[4 * l + j];
            acc[l] = fmaf(s, (float)p, acc[l]);
        }
    }
    const float t0 = acc[0] + acc[4], t1 = acc[1] + acc[5], t2 = acc[2] + acc[6],
                t3 = acc[3] + acc[7];
    return (t0 + t2) + (t1 + t3);
}

/* MUL_MAT(W[N,K] quantized, X[M,K] f32) -> Y[M,N] f32 (ggml-cpu.c:1254-1457): every activation
 * row is quantized to Q8_0 (vec_dot_type of Q8_0/Q4_0, ggml-cpu.c:239-279), then dotted. */
void oracle_mul_mat(int wtype, const uint8_t* w, int64_t N, int64_t K, const float* x, int64_t M,
                    float* y) {
    const int64_t rowb = K / QK * wblock_bytes(wtype);
    uint8_t* xq = (uint8_t*)malloc((size_t)(K / QK * 34));
    for (int64_t m = 0; m < M; m++) {
        oracle_quantize_row_q8_0(x + m * K, xq, K);
        for (int64_t n = 0; n < N; n++) y[m * N + n] = oracle_vec_dot(wtype, K, w + n * rowb, xq);
    }
    free(xq);
}

/* F32 weight MUL_MAT (biases-only models never quantize some small linears). */
void oracle_mul_mat_f32(const float* w, int64_t N, int64_t K, const float* x, int64_t M, float* y) {
    for (int64_t m = 0; m < M; m++)
        for (int64_t n = 0; n < N; n++) {
            double s = 0.0;
            for (int64_t k = 0; k < K; k++) s += (double)w[n * K + k] * x[m * K + k];
            y[m * N + n] = (float)s;
        }
}

/* GET_ROWS with dequantization (ggml-cpu/ops.cpp:4914). */
void oracle_get_rows(int type, const uint8_t* table, int64_t d, const int32_t* ids, int64_t n,
                     float* y) {
    int64_t rowb;
    if (type == GGML_TYPE_Q8_0) rowb = d / QK * 34;
    else if (type == GGML_TYPE_Q4_0) rowb = d / QK * 18;
    else if (type == GGML_TYPE_F16) rowb = d * 2;
    else rowb = d * 4;
    for (int64_t i = 0; i < n; i++) oracle_dequantize_row(type, table + ids[i] * rowb, y + i * d, d);
}

/* RMS_NORM (ggml-cpu/ops.cpp:3859-3920): squares rounded in fp32, summed in double, then
 * scale = 1/sqrtf(mean+eps) in fp32; y = x*scale [* gamma]. */
void oracle_rms_norm(const float* x, int64_t d, int64_t rows, float eps, const float* gamma,
                     float* y) {
    for (int64_t r = 0; r < rows; r++) {
        const float* xr = x + r * d;
        double sum = 0.0;
        for (int64_t i = 0; i < d; i++) {
            volatile float sq = xr[i] * xr[i];
            sum += (double)sq;
        }
        const float mean = (float)(sum / d);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (int64_t i = 0; i < d; i++) {
            volatile float t = xr[i] * scale;
            y[r * d + i] = gamma ? t * gamma[i] : t;
        }
    }
}

/* NORM (ggml-cpu/ops.cpp:3762-3815, vec.cpp:455 ggml_vec_cvar_f32): mean in fp32, centred
 * variance accumulated in double, scale = 1/sqrtf(var+eps); then optional *gamma, +beta
 * (executor.cpp:2716-2730). */
void oracle_layer_norm(const float* x, int64_t d, int64_t rows, float eps, const float* gamma,
                       const float* beta, float* y) {
    for (int64_t r = 0; r < rows; r++) {
        const float* xr = x + r * d;
        double s = 0.0;
        for (int64_t i = 0; i < d; i++) s += xr[i];
        const float mean = (float)(s / d);
        double v = 0.0;
        for (int64_t i = 0; i < d; i++) {
            volatile float c = xr[i] - mean;
            volatile float c2 = c * c;
            v += (double)c2;
        }
        const float var = (float)(v / d);
        const float scale = 1.0f / sqrtf(var + eps);
        for (int64_t i = 0; i < d; i++) {
            volatile float t = (xr[i] - mean) * scale;
            float o = t;
            if (gamma) o = o * gamma[i];
            if (beta) o = o + beta[i];
            y[r * d + i] = o;
        }
    }
}

/* NEOX RoPE (ggml-cpu/ops.cpp:5910-5923 cache init, :5998-6015 rotate_pairs, :6072
 * theta_scale): theta starts at the position and is multiplied by theta_scale once per pair in
 * fp32; cos/sin of the fp32 theta; pairs (i, i + n_dims/2).  x and y are [s][H][hd]. */
void oracle_rope_neox(const float* x, int64_t hd, int64_t H, int64_t s, const int32_t* pos,
                      int n_dims, float freq_base, float* y) {
    const float theta_scale = powf(freq_base, -2.0f / n_dims);
    float* cache = (float*)malloc((size_t)n_dims * sizeof(float));
    for (int64_t t = 0; t < s; t++) {
        float theta = (float)(int64_t)pos[t];
        for (int i0 = 0; i0 < n_dims; i0 += 2) {
            cache[i0 + 0] = cosf(theta);
            cache[i0 + 1] = sinf(theta);
            theta *= theta_scale;
        }
        for (int64_t h = 0; h < H; h++) {
            const float* src = x + (t * H + h) * hd;
            float* dst = y + (t * H + h) * hd;
            memcpy(dst, src, (size_t)hd * 4);
            for (int i0 = 0; i0 < n_dims; i0 += 2) {
                const int ic = i0 / 2;
                const float c = cache[i0], sn = cache[i0 + 1];
                const float x0 = src[ic], x1 = src[ic + n_dims / 2];
                /* The reference is built with GNU floating-point contraction, which turns
                 * x0*cos - x1*sin and x0*sin + x1*cos into one FMA each around the second
                 * product; these two forms reproduce its results bit for bit. */
                volatile float b = x1 * sn, f = x1 * c;
                dst[ic] = fmaf(x0, c, -b);
                dst[ic + n_dims / 2] = fmaf(x0, sn, f);
            }
        }
    }
    free(cache);
}

static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* Vector exp of the AVX2+FMA build, ggml_v_expf (ggml-cpu/vec.h:1209-1253): the published Arm
 * optimized-routines single-precision exp (range reduction x = n*ln2 + b with a two-constant
 * ln2, degree-5 polynomial in b, scale by 2^n with a special path for |n| > 126).  Every step
 * is an IEEE fma/mul/add or an integer op, so this scalar form reproduces each lane exactly. */
float oracle_v_expf(float x) {
    const float r = 0x1.8p23f;
    const float z = fmaf(x, 0x1.715476p+0f, r);
    const float n = z - r;
    const float b = fmaf(-n, 0x1.7f7d1cp-20f, fmaf(-n, 0x1.62e4p-1f, x));
    const uint32_t e = f2u(z) << 23;
    const float k = u2f(e + f2u(1.0f));
    const int c = fabsf(n) > 126.0f;
    const float u = b * b;
    const float j = fmaf(fmaf(fmaf(0x1.0e4020p-7f, b, 0x1.573e2ep-5f), u,
                              fmaf(0x1.555e66p-3f, b, 0x1.fffdb6p-2f)),
                         u, 0x1.ffffecp-1f * b);
    if (!c) return fmaf(j, k, k);
    const uint32_t g = (n <= 0.0f) ? 0x82000000u : 0u;
    const float s1 = u2f(g + 0x7f000000u);
    const float s2 = u2f(e - g);
    if (fabsf(n) > 192.0f) return s1 * s1;
    return fmaf(s2, j, s2) * s1;
}

/* ggml_v_silu (vec.h:1255-1262): x / (1 + exp(-x)) with the vector exp above. */
float oracle_v_silu(float x) {
    const float e = oracle_v_expf(0.0f - x);
    return x / (1.0f + e);
}

/* SWIGLU over [gate(ffn) ; up(ffn)] rows (ggml-cpu/ops.cpp:3246-3303 -> ggml_vec_swiglu_f32
 * vec.cpp:417-426): silu(g) * up on 8-wide vectors; a tail shorter than 8 uses the scalar
 * ggml_silu_f32 (vec.h:1046, libm expf). */
void oracle_swiglu(const float* x, int64_t ffn, int64_t rows, float* y) {
    const int64_t nv = ffn & ~(int64_t)7;
    for (int64_t r = 0; r < rows; r++) {
        const float* g = x + r * 2 * ffn;
        const float* u = g + ffn;
        for (int64_t i = 0; i < ffn; i++) {
            const float s = i < nv ? oracle_v_silu(g[i]) : g[i] / (1.0f + expf(-g[i]));
            y[r * ffn + i] = s * u[i];
        }
    }
}

/* Bias + tanh-GELU, fast_gelu_f32 (runtime/src/stdlib_kernels.cpp:9-19), the CPU custom op the
 * GPT-2 graph runs (executor.cpp:2703-2715). */
void oracle_bias_gelu(const float* x, const float* b, int64_t d, int64_t rows, float* y) {
    const float SQRT_2_OVER_PI = 0.79788456080286535587989211986876f;
    const float GELU_COEF_A = 0.044715f;
    for (int64_t r = 0; r < rows; r++)
        for (int64_t i = 0; i < d; i++) {
            const float v = x[r * d + i] + (b ? b[i] : 0.0f);
            const float v3 = v * v * v;
            float inner = SQRT_2_OVER_PI * (v + GELU_COEF_A * v3);
            inner = inner < -9.0f ? -9.0f : (inner > 9.0f ? 9.0f : inner);
            const float e2 = expf(2.0f * inner);
            const float th = (e2 - 1.0f) / (e2 + 1.0f);
            y[r * d + i] = 0.5f * v * (1.0f + th);
        }
}

/* FLASH_ATTN_EXT over an F16 cache, one_chunk semantics (ggml-cpu/ops.cpp:8532-8768): Q is
 * rounded to F16 (q_to_vec_dot, :8650), scores s = dot(k,q)*scale + mask, online softmax with
 * an F16 V accumulator (VKQ16, :8630, :8689-8696): on a new maximum VKQ16 *= exp(Mold-M), then
 * VKQ16 += v*exp(s-M) rounding to F16 each time; result VKQ/S.  Positions whose mask is -inf
 * are skipped.  q: [s][Hq][hd]; k, v: [Hkv][n_kv][hd] fp16; mask [s][n_kv] fp16 or NULL;
 * y: [s][Hq][hd]. */
void oracle_flash_attn(const float* q, const uint16_t* k, const uint16_t* v, const uint16_t* mask,
                       int64_t hd, int64_t s, int64_t Hq, int64_t Hkv, int64_t n_kv, float scale,
                       float* y) {
    const int64_t rk = Hq / Hkv;
    uint16_t* qh = (uint16_t*)malloc((size_t)hd * 2);
    uint16_t* acc = (uint16_t*)malloc((size_t)hd * 2);
    for (int64_t t = 0; t < s; t++)
        for (int64_t h = 0; h < Hq; h++) {
            const float* qr = q + (t * Hq + h) * hd;
            const int64_t hk = h / rk;
            for (int64_t i = 0; i < hd; i++) qh[i] = oracle_fp32_to_fp16(qr[i]);
            memset(acc, 0, (size_t)hd * 2);
            float S = 0.0f, M = -INFINITY;
            for (int64_t c = 0; c < n_kv; c++) {
                const float mv = mask ? oracle_fp16_to_fp32(mask[t * n_kv + c]) : 0.0f;
                if (mv == -INFINITY) continue;
                const uint16_t* kr = k + (hk * n_kv + c) * hd;
                /* ggml_vec_dot_f16 on AVX2/F16C (ggml-cpu/vec.cpp:345-366, simd-mappings.h
                 * GGML_F16_STEP 32 / EPR 8 / GGML_F32x8_REDUCE): 32 fp32 lanes, lane 8j+l
                 * accumulates elements i+8j+l; reduce (j0+j2)+(j1+j3) lane-wise, then
                 * (l_i + l_{i+4}), then ((t0+t1)+(t2+t3)).  Products of halves are exact, so
                 * FMA and multiply-add agree. */
                float lane[32];
                for (int l = 0; l < 32; l++) lane[l] = 0.0f;
                const int64_t np = hd & ~(int64_t)31;
                for (int64_t i = 0; i < np; i += 32)
                    for (int l = 0; l < 32; l++)
                        lane[l] += oracle_fp16_to_fp32(kr[i + l]) * oracle_fp16_to_fp32(qh[i + l]);
                float x8[8];
                for (int l = 0; l < 8; l++) x8[l] = (lane[l] + lane[16 + l]) + (lane[8 + l] + lane[24 + l]);
                const float t0 = x8[0] + x8[4], t1 = x8[1] + x8[5], t2 = x8[2] + x8[6],
                            t3 = x8[3] + x8[7];
                double dot = (double)((t0 + t1) + (t2 + t3));
                for (int64_t i = np; i < hd; i++)
                    dot += (double)(oracle_fp16_to_fp32(kr[i]) * oracle_fp16_to_fp32(qh[i]));
                float sc = (float)dot;
                sc = sc * scale;
                sc += mv;
                const float Mold = M;
                float ms = 1.0f, vs = 1.0f;
                if (sc > M) {
                    M = sc;
                    ms = expf(Mold - M);
                    for (int64_t i = 0; i < hd; i++)
                        acc[i] = oracle_fp32_to_fp16(oracle_fp16_to_fp32(acc[i]) * ms);
                } else {
                    vs = expf(sc - M);
                }
                const uint16_t* vr = v + (hk * n_kv + c) * hd;
                /* ggml_vec_mad_f16 SIMD form (vec.h): y = f16(fma(x, v, y)) */
                for (int64_t i = 0; i < hd; i++)
                    acc[i] = oracle_fp32_to_fp16(
                        fmaf(oracle_fp16_to_fp32(vr[i]), vs, oracle_fp16_to_fp32(acc[i])));
                S = fmaf(S, ms, vs); /* contracted by the reference build */
            }
            const float inv = S == 0.0f ? 0.0f : 1.0f / S;
            float* yr = y + (t * Hq + h) * hd;
            for (int64_t i = 0; i < hd; i++) yr[i] = oracle_fp16_to_fp32(acc[i]) * inv;
        }
    free(qh);
    free(acc);
}
