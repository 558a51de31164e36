// Shared definitions for the B200 engine: ggml type ids and sizes, error handling.
#pragma once

#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

namespace gb {

// ggml type ids as serialized in GGUF tensor infos and the ggmlc graph spec
// (third_party/ggml/include/ggml.h enum ggml_type; python/ggmlc/dialect/ggml/ops.py GGMLType).
enum GgmlType : int32_t {
    T_F32 = 0,
    T_F16 = 1,
    T_Q4_0 = 2,
    T_Q8_0 = 8,
    T_I8 = 24,
    T_I16 = 25,
    T_I32 = 26,
    T_I64 = 27,
    T_F64 = 28,
};

// ggml opcodes that appear on the decoder hot path (ggml.h enum ggml_op; ggmlc custom ops
// 200-203 from python/ggmlc/dialect/ggml/ops.py:68-72).
enum OpCode : int32_t {
    OP_ADD = 2,
    OP_MUL = 7,
    OP_NORM = 24,
    OP_RMS_NORM = 25,
    OP_MUL_MAT = 29,
    OP_SCALE = 32,
    OP_CPY = 34,
    OP_CONT = 35,
    OP_RESHAPE = 36,
    OP_VIEW = 37,
    OP_PERMUTE = 38,
    OP_TRANSPOSE = 39,
    OP_GET_ROWS = 40,
    OP_ROPE = 48,
    OP_FLASH_ATTN_EXT = 74,
    OP_GLU = 100,
    OP_BIAS_GELU = 200,
    OP_LAYER_NORM = 201,
    OP_RMS_NORM_C = 202,
    OP_SWIGLU = 203,
};

constexpr int QK = 32;  // block length of Q8_0 / Q4_0

inline bool is_quant(int t) { return t == T_Q8_0 || t == T_Q4_0; }

// bytes of one row of k elements in the GGUF (block) layout
inline int64_t row_bytes(int t, int64_t k) {
    switch (t) {
        case T_F32: case T_I32: return 4 * k;
        case T_F16: case T_I16: return 2 * k;
        case T_Q8_0: return k / QK * 34;
        case T_Q4_0: return k / QK * 18;
        case T_I8: return k;
        case T_I64: case T_F64: return 8 * k;
        default: throw std::runtime_error("unsupported ggml type " + std::to_string(t));
    }
}

// size of one element for non-block types (ggml nb[0])
inline int64_t elem_bytes(int t) {
    switch (t) {
        case T_F32: case T_I32: return 4;
        case T_F16: case T_I16: return 2;
        case T_I8: return 1;
        case T_I64: case T_F64: return 8;
        default: return 0;
    }
}

struct Error : std::runtime_error {
    using std::runtime_error::runtime_error;
};

}  // namespace gb

#define GB_CHECK(cond, msg)                                                              \
    do {                                                                                 \
        if (!(cond)) throw ::gb::Error(std::string("ggmlc_b200: ") + (msg));             \
    } while (0)
