// Tensor parallelism over the decoder graphs ggmlc compiles (Megatron-style, one exchange step
// per block).  The reference runtime has no tensor parallelism; the partition follows the
// structure its fusion passes emit (fused QKV projection, fused gate_up projection with the gate
// half first, python/ggmlc/compiler/fusion.py:1310-1312, :1528-1534):
//   - fused QKV [d -> (Hq + 2 Hkv) hd]: each of its q / k / v slices is cut by heads, a rank keeps
//     its Hq/T query and Hkv/T key/value heads (and the matching KV cache);
//   - fused gate_up [d -> 2F]: gate and up halves cut alike, SwiGLU stays local;
//   - O [Hq hd -> d] and down [F -> d]: cut along K; their outputs are partial sums, all-reduced
//     (NCCL) before the residual add, which only rank 0 contributes;
//   - the output projection [d -> V]: cut by vocabulary rows, the logits all-gathered;
//   - everything else (embedding, norms, residual stream) replicated.
// plan_tensor_parallel rewrites one rank's copy of the graph: the head / FFN dimensions of the
// sharded activations and the offsets of the q / k / v slices.
#pragma once

#include <cstdint>
#include <map>
#include <set>
#include <string>
#include <utility>
#include <vector>

#include "graph.h"

namespace gb {

struct TpSlice {
    bool cols = false;                              // false: keep row ranges; true: columns
    std::vector<std::pair<int64_t, int64_t>> rows;  // [begin, end) row ranges, concatenated
    int64_t c0 = 0, c1 = 0;                         // kept column range (element units)
};

struct TpPlan {
    int rank = 0, size = 1;
    std::map<uint32_t, TpSlice> slices;  // weight / bias tensor id -> the part this rank holds
    std::set<uint32_t> partial;          // MUL_MAT outputs holding partial sums (all-reduced)
    uint32_t vocab_out = UINT32_MAX;     // output of the vocabulary-split projection
    uint32_t vocab_w = UINT32_MAX;       // its weight (kept whole: a tied embedding reads it)
    int64_t vocab_rows = 0;              // vocabulary rows per rank
    int n_attention = 0, n_mlp = 0;      // blocks sharded
};

// Plan and rewrite g (this rank's copy) for `size` ranks.  Throws on graphs whose attention or
// MLP blocks do not have the fused-projection structure, or whose heads / FFN width do not
// divide by size in whole 32-element blocks.
TpPlan plan_tensor_parallel(Graph& g, int rank, int size);

// The plan and the rewritten shapes as JSON (host-side tests).
std::string tp_plan_json(const TpPlan& p, const Graph& g);

}  // namespace gb
