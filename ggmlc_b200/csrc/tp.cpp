// Tensor-parallel planning (see tp.h).
#include "tp.h"

#include <algorithm>
#include <array>
#include <sstream>

#include "common.h"

namespace gb {

namespace {

using Dims = std::array<int64_t, 4>;

struct Ctx {
    Graph& g;
    SymEnv env;
    std::map<uint32_t, int> prod;               // tensor -> producing op index
    std::map<uint32_t, std::vector<int>> cons;  // tensor -> consuming op indices
    std::map<uint32_t, int> shard;              // tensor -> dimension divided by the rank count
    std::set<int> views;                        // q / k / v slice ops whose offsets are divided
    std::set<int> allowed;                      // ops that may consume a sharded activation

    explicit Ctx(Graph& gr) : g(gr) {}
    Dims dims(uint32_t id) const {
        Dims d{1, 1, 1, 1};
        const GTensor& t = g.t(id);
        for (int k = 0; k < 4; ++k) d[k] = t.ne[k] ? t.ne[k]->eval(env) : 1;
        return d;
    }
};

void fail(const std::string& m) { GB_CHECK(false, "tensor parallelism: " + m); }

// Output dimension holding the cut of a reshape whose input is cut along dimension di: the cut
// is the outer part of the prefix of dims 0..di, which must end at an output prefix boundary.
int reshape_dim(const Dims& in, int di, const Dims& out) {
    int64_t S = 1;
    for (int k = 0; k <= di; ++k) S *= in[(size_t)k];
    int64_t p = 1;
    for (int k = 0; k < 4; ++k) {
        const int64_t q = p * out[(size_t)k];
        if (p < S && q >= S) {
            if (q != S) fail("a reshape splits the sharded dimension");
            return k;
        }
        p = q;
    }
    fail("reshape of a sharded tensor has no matching dimension");
    return -1;
}

bool is_shape_op(int opc) {
    return opc == OP_RESHAPE || opc == OP_PERMUTE || opc == OP_TRANSPOSE || opc == OP_ROPE ||
           opc == OP_CONT || opc == OP_CPY;
}

// the cut dimension after one shape op (input 0 -> output)
int map_dim(const Ctx& c, const GOp& op, int din) {
    switch (op.opcode) {
        case OP_RESHAPE: return reshape_dim(c.dims(op.inputs[0]), din, c.dims(op.outputs[0]));
        case OP_PERMUTE: {
            const int ax[4] = {(int)op.i("axis0", 1), (int)op.i("axis1", 0), (int)op.i("axis2", 2),
                               (int)op.i("axis3", 3)};
            return ax[din];
        }
        case OP_TRANSPOSE: return din == 0 ? 1 : (din == 1 ? 0 : din);
        default: return din;  // ROPE, CONT, CPY keep the shape
    }
}

void set_num(JValue& v, int64_t x) {
    v.kind = JValue::NUM;
    v.is_int = true;
    v.inum = x;
    v.num = (double)x;
}

// Follow the consumers of t through shape ops to the MUL_MAT that reads it as activations; the
// cut must arrive on dimension 0 (K).  Returns the op index.
int forward_to_matmul(Ctx& c, uint32_t t, int d) {
    for (int guard = 0; guard < 64; ++guard) {
        auto it = c.cons.find(t);
        if (it == c.cons.end() || it->second.size() != 1)
            fail("a sharded activation must have exactly one consumer");
        const int oi = it->second[0];
        const GOp& op = c.g.ops[(size_t)oi];
        c.allowed.insert(oi);
        if (op.opcode == OP_MUL_MAT) {
            if (op.inputs.size() < 2 || op.inputs[1] != t || d != 0)
                fail("a sharded activation reaches a matmul other than along K");
            return oi;
        }
        if (!is_shape_op(op.opcode)) fail("unsupported op '" + op.name + "' on a sharded path");
        d = map_dim(c, op, d);
        t = op.outputs[0];
        c.shard[t] = d;
    }
    fail("sharded path too long");
    return -1;
}

// K-split weight of a row-parallel matmul (O / down); its output becomes a partial sum
void split_k(Ctx& c, TpPlan& P, int oi) {
    const GOp& op = c.g.ops[(size_t)oi];
    const uint32_t w = op.inputs[0];
    const int64_t K = c.dims(w)[0];
    if (K % P.size != 0 || (K / P.size) % QK != 0)
        fail("K = " + std::to_string(K) + " of '" + c.g.t(w).name +
             "' does not split into whole 32-element blocks");
    TpSlice s;
    s.cols = true;
    s.c0 = K / P.size * P.rank;
    s.c1 = s.c0 + K / P.size;
    P.slices[w] = s;
    c.shard[w] = 0;
    P.partial.insert(op.outputs[0]);
}

// row ranges [start + r*len/T, start + (r+1)*len/T) of a column-parallel projection
void split_rows(Ctx& c, TpPlan& P, int mm, const std::vector<std::pair<int64_t, int64_t>>& parts) {
    const GOp& op = c.g.ops[(size_t)mm];
    TpSlice s;
    for (auto& [a, b] : parts) {
        const int64_t len = (b - a) / P.size;
        s.rows.push_back({a + len * P.rank, a + len * (P.rank + 1)});
    }
    for (size_t k = 0; k < op.inputs.size(); ++k) {
        if (k == 1) continue;  // activations
        const uint32_t id = op.inputs[k];
        if (P.slices.count(id)) fail("weight '" + c.g.t(id).name + "' is used by two blocks");
        P.slices[id] = s;
        c.shard[id] = k == 0 ? 1 : 0;  // weight rows (ne[1]) / bias elements (ne[0])
    }
    c.shard[op.outputs[0]] = 0;
}

void plan_attention(Ctx& c, TpPlan& P, int fa_i) {
    const GOp& fa = c.g.ops[(size_t)fa_i];
    if (fa.inputs.size() < 3) fail("attention without q, k, v inputs");
    int proj = -1;
    int64_t heads[3] = {0, 0, 0};
    std::vector<int> view_ops;
    for (int j = 0; j < 3; ++j) {
        std::vector<int> path;
        uint32_t t = fa.inputs[(size_t)j];
        int view = -1;
        for (int guard = 0; guard < 64 && view < 0; ++guard) {
            const int oi = c.prod.count(t) ? c.prod.at(t) : -1;
            if (oi < 0) fail("attention input is not produced by an op");
            const GOp& op = c.g.ops[(size_t)oi];
            if (op.opcode == OP_VIEW) {
                view = oi;
                break;
            }
            if (!is_shape_op(op.opcode))
                fail("unsupported op '" + op.name + "' between the QKV projection and attention");
            path.push_back(oi);
            t = op.inputs[0];
        }
        if (view < 0) fail("attention input does not come from a slice of a projection");
        const GOp& v = c.g.ops[(size_t)view];
        if (v.i("ggml_dim", 0) != 0 || v.i("step", 1) != 1)
            fail("q / k / v must be slices of the projection rows");
        const int mm = c.prod.count(v.inputs[0]) ? c.prod.at(v.inputs[0]) : -1;
        if (mm < 0 || c.g.ops[(size_t)mm].opcode != OP_MUL_MAT)
            fail("q / k / v slices must come from one MUL_MAT");
        if (proj >= 0 && proj != mm) fail("q, k and v come from different projections");
        proj = mm;
        view_ops.push_back(view);
        std::reverse(path.begin(), path.end());
        int d = 0;
        c.shard[v.outputs[0]] = 0;
        c.allowed.insert(view);
        for (int oi : path) {
            const GOp& op = c.g.ops[(size_t)oi];
            d = map_dim(c, op, d);
            c.shard[op.outputs[0]] = d;
            c.allowed.insert(oi);
        }
        heads[j] = c.dims(fa.inputs[(size_t)j])[(size_t)d];
    }
    c.allowed.insert(fa_i);
    for (int j = 0; j < 3; ++j)
        if (heads[j] % P.size != 0)
            fail("attention heads (" + std::to_string(heads[j]) + ") do not divide by " +
                 std::to_string(P.size) + " ranks");
    // the slices of the projection: exactly the q / k / v slices, tiling its rows
    const GOp& mm = c.g.ops[(size_t)proj];
    const uint32_t pout = mm.outputs[0];
    std::vector<std::pair<int64_t, int64_t>> parts;
    for (int oi : c.cons[pout]) {
        const GOp& v = c.g.ops[(size_t)oi];
        if (v.opcode != OP_VIEW || std::find(view_ops.begin(), view_ops.end(), oi) == view_ops.end())
            fail("the QKV projection output has a consumer other than its q / k / v slices");
        const int64_t a = v.i("start", 0);
        parts.push_back({a, a + c.dims(v.outputs[0])[0]});
        c.views.insert(oi);
    }
    std::sort(parts.begin(), parts.end());
    int64_t at = 0;
    for (auto& [a, b] : parts) {
        if (a != at || (b - a) % P.size != 0) fail("q / k / v slices do not tile the projection");
        at = b;
    }
    if (at != c.dims(pout)[0]) fail("q / k / v slices do not cover the projection");
    split_rows(c, P, proj, parts);
    // attention output [hd, Hq, s] -> ... -> O projection along K
    c.shard[fa.outputs[0]] = 1;
    if (c.dims(fa.outputs[0])[1] != heads[0]) fail("unexpected attention output layout");
    split_k(c, P, forward_to_matmul(c, fa.outputs[0], 1));
    P.n_attention++;
}

void plan_mlp(Ctx& c, TpPlan& P, int gi) {
    const GOp& glu = c.g.ops[(size_t)gi];
    if (glu.inputs.size() != 1) fail("only the fused gate_up SwiGLU form is supported");
    const uint32_t gu = glu.inputs[0];
    const int mm = c.prod.count(gu) ? c.prod.at(gu) : -1;
    if (mm < 0 || c.g.ops[(size_t)mm].opcode != OP_MUL_MAT)
        fail("SwiGLU input is not a projection");
    if (c.cons[gu].size() != 1) fail("the gate_up projection has several consumers");
    const int64_t N = c.dims(gu)[0], F = N / 2;
    if (N % 2 != 0 || F % P.size != 0 || (F / P.size) % QK != 0)
        fail("FFN width " + std::to_string(F) + " does not split into whole blocks");
    split_rows(c, P, mm, {{0, F}, {F, N}});
    c.allowed.insert(gi);
    c.shard[glu.outputs[0]] = 0;
    split_k(c, P, forward_to_matmul(c, glu.outputs[0], 0));
    P.n_mlp++;
}

}  // namespace

TpPlan plan_tensor_parallel(Graph& g, int rank, int size) {
    GB_CHECK(size >= 1 && rank >= 0 && rank < size, "tensor parallelism: bad rank / size");
    TpPlan P;
    P.rank = rank;
    P.size = size;
    if (size == 1) return P;
    Ctx c(g);
    c.env["s"] = 3;
    for (auto& s : g.symbol_table) c.env[s] = 3;
    for (size_t i = 0; i < g.ops.size(); ++i) {
        for (uint32_t o : g.ops[i].outputs) c.prod[o] = (int)i;
        for (uint32_t in : g.ops[i].inputs) c.cons[in].push_back((int)i);
    }
    for (size_t i = 0; i < g.ops.size(); ++i) {
        const int opc = g.ops[i].opcode;
        if (opc == OP_FLASH_ATTN_EXT) plan_attention(c, P, (int)i);
        else if (opc == OP_SWIGLU || opc == OP_GLU) plan_mlp(c, P, (int)i);
    }
    if (P.n_attention == 0) fail("the graph has no attention block to shard");
    // every consumer of a sharded activation is part of a planned block
    for (auto& [id, d] : c.shard) {
        if (g.t(id).data) continue;  // weights
        for (int oi : c.cons[id])
            if (!c.allowed.count(oi))
                fail("sharded tensor '" + g.t(id).name + "' feeds '" + g.ops[(size_t)oi].name + "'");
    }
    // vocabulary-split output projection
    if (!g.outputs.empty() && c.prod.count(g.outputs[0])) {
        const GOp& op = g.ops[(size_t)c.prod.at(g.outputs[0])];
        if (op.opcode == OP_MUL_MAT && op.inputs.size() == 2 && is_quant(g.t(op.inputs[0]).type) &&
            !P.slices.count(op.inputs[0])) {
            const int64_t V = c.dims(op.inputs[0])[1];
            if (V % size == 0) {
                P.vocab_out = g.outputs[0];
                P.vocab_w = op.inputs[0];
                P.vocab_rows = V / size;
            }
        }
    }
    // rewrite this rank's shapes and slice offsets
    for (auto& [id, d] : c.shard) {
        GTensor& t = g.tensors.at(id);
        auto& e = t.ne[d];
        if (!e || !e->is_static()) fail("sharded dimension of '" + t.name + "' is symbolic");
        const int64_t v = e->eval(c.env);
        if (v % size != 0) fail("dimension " + std::to_string(v) + " of '" + t.name + "' does not divide");
        auto ne = std::make_shared<DimExpr>();
        ne->kind = DimExpr::STATIC;
        ne->val = v / size;
        e = ne;
    }
    for (int oi : c.views) {
        GOp& v = g.ops[(size_t)oi];
        const int64_t a = v.i("start", 0);
        set_num(v.attrs["start"], a / size);
        if (v.has("end")) set_num(v.attrs["end"], v.i("end", 0) / size);
    }
    return P;
}

std::string tp_plan_json(const TpPlan& p, const Graph& g) {
    std::ostringstream o;
    SymEnv env;
    env["s"] = 1;
    for (auto& s : g.symbol_table) env[s] = 1;
    o << "{\"rank\":" << p.rank << ",\"size\":" << p.size << ",\"n_attention\":" << p.n_attention
      << ",\"n_mlp\":" << p.n_mlp << ",\"vocab_rows\":" << p.vocab_rows << ",\"vocab_weight\":\""
      << (p.vocab_w == UINT32_MAX ? "" : g.t(p.vocab_w).name) << "\",\"slices\":{";
    bool first = true;
    for (auto& [id, s] : p.slices) {
        o << (first ? "" : ",") << "\"" << g.t(id).name << "\":{";
        first = false;
        if (s.cols) {
            o << "\"cols\":[" << s.c0 << "," << s.c1 << "]";
        } else {
            o << "\"rows\":[";
            for (size_t i = 0; i < s.rows.size(); ++i)
                o << (i ? "," : "") << "[" << s.rows[i].first << "," << s.rows[i].second << "]";
            o << "]";
        }
        o << "}";
    }
    o << "},\"partial\":[";
    first = true;
    for (uint32_t id : p.partial) {
        o << (first ? "" : ",") << "\"" << g.t(id).name << "\"";
        first = false;
    }
    o << "],\"shapes\":{";
    first = true;
    for (auto& [id, t] : g.tensors) {
        o << (first ? "" : ",") << "\"" << t.name << "\":[";
        first = false;
        for (int d = 0; d < 4; ++d) o << (d ? "," : "") << (t.ne[d] ? t.ne[d]->eval(env) : 1);
        o << "]";
    }
    o << "}}";
    return o.str();
}

}  // namespace gb
