// Minimal JSON reader for the ggmlc graph spec (the "ggmlc.graph_spec" GGUF string written by
// python/ggmlc/serialization/gguf.py:133-177 _graph_to_json_spec).  Numbers keep both an int64
// and a double view so attributes round-trip like the reference loader (loader.cpp:357-439).
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace gb {

struct JValue {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    double num = 0.0;
    int64_t inum = 0;
    bool is_int = false;
    std::string str;
    std::vector<JValue> arr;
    std::map<std::string, JValue> obj;

    const JValue* get(const std::string& k) const {
        if (kind != OBJ) return nullptr;
        auto it = obj.find(k);
        return it == obj.end() ? nullptr : &it->second;
    }
    int64_t as_int(int64_t dflt = 0) const {
        if (kind == NUM) return is_int ? inum : (int64_t)num;
        if (kind == BOOL) return b ? 1 : 0;
        return dflt;
    }
    double as_num(double dflt = 0.0) const {
        if (kind == NUM) return num;
        if (kind == BOOL) return b ? 1.0 : 0.0;
        return dflt;
    }
    std::string as_str(const std::string& dflt = "") const { return kind == STR ? str : dflt; }
};

JValue json_parse(const std::string& text);

}  // namespace gb
