// In-memory form of a ggmlc-compiled model: the GGUF v3 container plus its "ggmlc.graph_spec"
// JSON graph.  Mirrors the reference's SerializedModelGraph (runtime/include/ggmlc/types.h:
// 114-233) closely enough that the Python boundary can expose the same attributes.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "json.h"

namespace gb {

using SymEnv = std::unordered_map<std::string, int64_t>;

// Symbolic dimension (types.h:14-75 DimExpr): static | symbol | add/sub/mul/floordiv/ceildiv.
struct DimExpr {
    enum Kind { STATIC, SYMBOL, ADD, SUB, MUL, FLOORDIV, CEILDIV } kind = STATIC;
    int64_t val = 1;
    std::string sym;
    std::shared_ptr<DimExpr> l, r;

    int64_t eval(const SymEnv& env) const;
    bool is_static() const;
    // index into the graph symbol table of the single symbol this dim names, or -1
    int symbol_index(const std::vector<std::string>& table) const;
    static std::shared_ptr<DimExpr> from_json(const JValue& j);
};

// storage classes (types.h:77-84)
enum Storage { ST_INPUT = 0, ST_PARAMETER = 1, ST_CONSTANT = 2, ST_ACTIVATION = 3, ST_STATE = 4,
               ST_OUTPUT = 5 };

struct GTensor {
    uint32_t id = 0;
    std::string name;
    int type = 0;
    std::shared_ptr<DimExpr> ne[4];
    int storage = ST_ACTIVATION;
    std::string role;
    const uint8_t* data = nullptr;  // GGUF payload, or null
    uint64_t data_size = 0;
    int64_t file_ne[4] = {1, 1, 1, 1};  // dims recorded in the GGUF tensor info
};

struct GOp {
    uint32_t id = 0;
    int opcode = 0;
    std::string name;
    std::vector<uint32_t> inputs;
    std::vector<uint32_t> outputs;
    std::map<std::string, JValue> attrs;

    bool has(const std::string& k) const { return attrs.count(k) != 0; }
    int64_t i(const std::string& k, int64_t d) const {
        auto it = attrs.find(k);
        return it == attrs.end() ? d : it->second.as_int(d);
    }
    double f(const std::string& k, double d) const {
        auto it = attrs.find(k);
        return it == attrs.end() ? d : it->second.as_num(d);
    }
};

struct Graph {
    std::string name;
    std::vector<std::string> symbol_table;
    std::vector<uint32_t> inputs, outputs, parameters;
    std::map<uint32_t, GTensor> tensors;
    std::vector<GOp> ops;
    std::map<std::string, std::string> meta_str;
    std::map<std::string, int64_t> meta_int;
    // backing storage of the GGUF bytes (mmap'd file or owned copy)
    std::shared_ptr<void> storage;
    uint64_t storage_size = 0;

    const GTensor& t(uint32_t id) const;
};

// Parse a GGUF v3 file / buffer (loader.cpp:257-443 equivalent).
std::shared_ptr<Graph> load_gguf_file(const std::string& path);
std::shared_ptr<Graph> load_gguf_bytes(const uint8_t* data, size_t size);

}  // namespace gb
