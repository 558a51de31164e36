// GGUF v3 reader and graph-spec decoder (replaces runtime/src/loader.cpp and the vendored
// gguf.cpp for the engine).  The file is mmap'd read-only; tensor payloads are bound to graph
// tensors by name, as the reference loader does (loader.cpp:357-439).
#include "graph.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

#include "common.h"

namespace gb {

int64_t DimExpr::eval(const SymEnv& env) const {
    switch (kind) {
        case STATIC: return val;
        case SYMBOL: {
            auto it = env.find(sym);
            GB_CHECK(it != env.end(), "symbol not found in environment: " + sym);
            return it->second;
        }
        case ADD: return l->eval(env) + r->eval(env);
        case SUB: return l->eval(env) - r->eval(env);
        case MUL: return l->eval(env) * r->eval(env);
        case FLOORDIV: {
            int64_t d = r->eval(env);
            GB_CHECK(d != 0, "division by zero in dim expression");
            return l->eval(env) / d;
        }
        case CEILDIV: {
            int64_t d = r->eval(env);
            GB_CHECK(d != 0, "division by zero in dim expression");
            return (l->eval(env) + d - 1) / d;
        }
    }
    return 1;
}

bool DimExpr::is_static() const {
    if (kind == STATIC) return true;
    if (kind == SYMBOL) return false;
    return (!l || l->is_static()) && (!r || r->is_static());
}

int DimExpr::symbol_index(const std::vector<std::string>& table) const {
    if (kind != SYMBOL) return -1;
    for (size_t i = 0; i < table.size(); ++i)
        if (table[i] == sym) return (int)i;
    return -1;
}

std::shared_ptr<DimExpr> DimExpr::from_json(const JValue& j) {
    auto d = std::make_shared<DimExpr>();
    std::string ty = j.get("type") ? j.get("type")->as_str("static") : "static";
    if (ty == "static") {
        d->kind = STATIC;
        d->val = j.get("val") ? j.get("val")->as_int(1) : 1;
    } else if (ty == "symbol") {
        d->kind = SYMBOL;
        d->sym = j.get("name") ? j.get("name")->as_str() : "";
    } else {
        static const std::map<std::string, Kind> ops = {
            {"add", ADD}, {"sub", SUB}, {"mul", MUL}, {"floordiv", FLOORDIV}, {"ceildiv", CEILDIV}};
        auto it = ops.find(ty);
        if (it == ops.end()) {
            d->kind = STATIC;
            d->val = 1;
        } else {
            d->kind = it->second;
            d->l = from_json(*j.get("left"));
            d->r = from_json(*j.get("right"));
        }
    }
    return d;
}

const GTensor& Graph::t(uint32_t id) const {
    auto it = tensors.find(id);
    GB_CHECK(it != tensors.end(), "unknown tensor id " + std::to_string(id));
    return it->second;
}

namespace {

struct Reader {
    const uint8_t* p;
    size_t n, off = 0;
    template <class T> T get() {
        GB_CHECK(off + sizeof(T) <= n, "truncated GGUF");
        T v;
        std::memcpy(&v, p + off, sizeof(T));
        off += sizeof(T);
        return v;
    }
    std::string str() {
        uint64_t len = get<uint64_t>();
        GB_CHECK(off + len <= n, "truncated GGUF string");
        std::string s((const char*)p + off, len);
        off += len;
        return s;
    }
};

// GGUF value types (ggml/include/gguf.h enum gguf_type)
struct KV {
    int type = -1;
    std::string s;
    int64_t i = 0;
    double f = 0;
    std::vector<std::string> sarr;
};

void read_value(Reader& r, int type, KV& kv) {
    switch (type) {
        case 0: kv.i = r.get<uint8_t>(); break;
        case 1: kv.i = r.get<int8_t>(); break;
        case 2: kv.i = r.get<uint16_t>(); break;
        case 3: kv.i = r.get<int16_t>(); break;
        case 4: kv.i = r.get<uint32_t>(); break;
        case 5: kv.i = r.get<int32_t>(); break;
        case 6: kv.f = r.get<float>(); break;
        case 7: kv.i = r.get<uint8_t>(); break;
        case 8: kv.s = r.str(); break;
        case 10: kv.i = (int64_t)r.get<uint64_t>(); break;
        case 11: kv.i = r.get<int64_t>(); break;
        case 12: kv.f = r.get<double>(); break;
        case 9: {
            int et = (int)r.get<uint32_t>();
            uint64_t cnt = r.get<uint64_t>();
            for (uint64_t k = 0; k < cnt; ++k) {
                KV e;
                read_value(r, et, e);
                if (et == 8) kv.sarr.push_back(e.s);
            }
            break;
        }
        default: GB_CHECK(false, "unsupported GGUF value type " + std::to_string(type));
    }
    kv.type = type;
}

std::shared_ptr<Graph> parse(const uint8_t* base, size_t size, std::shared_ptr<void> storage) {
    Reader r{base, size};
    GB_CHECK(size >= 4 && std::memcmp(base, "GGUF", 4) == 0, "not a GGUF file (bad magic)");
    r.off = 4;
    uint32_t version = r.get<uint32_t>();
    GB_CHECK(version == 3, "unsupported GGUF version " + std::to_string(version));
    uint64_t n_tensors = r.get<uint64_t>();
    uint64_t n_kv = r.get<uint64_t>();
    std::map<std::string, KV> kvs;
    for (uint64_t k = 0; k < n_kv; ++k) {
        std::string key = r.str();
        int type = (int)r.get<uint32_t>();
        KV kv;
        read_value(r, type, kv);
        kvs[key] = kv;
    }
    struct Info { int64_t ne[4]; int type; uint64_t off; };
    std::map<std::string, Info> infos;
    for (uint64_t k = 0; k < n_tensors; ++k) {
        std::string name = r.str();
        uint32_t nd = r.get<uint32_t>();
        GB_CHECK(nd <= 4, "tensor with more than 4 dims");
        Info in{{1, 1, 1, 1}, 0, 0};
        for (uint32_t d = 0; d < nd; ++d) in.ne[d] = (int64_t)r.get<uint64_t>();
        in.type = (int)r.get<uint32_t>();
        in.off = r.get<uint64_t>();
        infos[name] = in;
    }
    uint64_t align = 32;
    if (kvs.count("general.alignment")) align = (uint64_t)kvs["general.alignment"].i;
    const uint64_t data_start = (r.off + align - 1) / align * align;

    auto g = std::make_shared<Graph>();
    g->storage = storage;
    g->storage_size = size;
    for (auto& [k, v] : kvs) {
        if (v.type == 8) g->meta_str[k] = v.s;
        else if (v.type != 9 && v.type != 6 && v.type != 12) g->meta_int[k] = v.i;
    }
    GB_CHECK(kvs.count("ggmlc.graph_spec"), "GGUF has no ggmlc.graph_spec (not a ggmlc model)");
    JValue spec = json_parse(kvs["ggmlc.graph_spec"].s);
    g->name = spec.get("name") ? spec.get("name")->as_str() : "";
    auto ids = [](const JValue* a, std::vector<uint32_t>& out) {
        if (!a) return;
        for (auto& e : a->arr) out.push_back((uint32_t)e.as_int());
    };
    ids(spec.get("inputs"), g->inputs);
    ids(spec.get("outputs"), g->outputs);
    ids(spec.get("parameters"), g->parameters);
    if (auto st = spec.get("symbol_table"))
        for (auto& e : st->arr) g->symbol_table.push_back(e.as_str());
    if (auto ts = spec.get("tensors")) {
        for (auto& [k, tj] : ts->obj) {
            GTensor t;
            t.id = (uint32_t)tj.get("id")->as_int();
            t.name = tj.get("name") ? tj.get("name")->as_str() : "";
            t.type = (int)(tj.get("type") ? tj.get("type")->as_int() : 0);
            const JValue* ne = tj.get("ne");
            for (int d = 0; d < 4; ++d) {
                if (ne && d < (int)ne->arr.size()) t.ne[d] = DimExpr::from_json(ne->arr[d]);
                else t.ne[d] = std::make_shared<DimExpr>();
            }
            t.storage = (int)(tj.get("storage") ? tj.get("storage")->as_int(3) : 3);
            if (auto role = tj.get("role")) t.role = role->as_str();
            auto it = infos.find(t.name);
            if (it != infos.end()) {
                const Info& in = it->second;
                int64_t n = in.ne[0] * in.ne[1] * in.ne[2] * in.ne[3];
                t.data_size = (uint64_t)(row_bytes(in.type, in.ne[0]) * (n / in.ne[0]));
                GB_CHECK(data_start + in.off + t.data_size <= size,
                         "tensor '" + t.name + "' payload runs past the end of the file");
                t.data = base + data_start + in.off;
                for (int d = 0; d < 4; ++d) t.file_ne[d] = in.ne[d];
            }
            g->tensors[t.id] = std::move(t);
        }
    }
    if (auto ns = spec.get("nodes")) {
        for (auto& nj : ns->arr) {
            GOp op;
            op.id = (uint32_t)nj.get("id")->as_int();
            op.opcode = (int)nj.get("opcode")->as_int();
            op.name = nj.get("name") ? nj.get("name")->as_str() : "";
            ids(nj.get("inputs"), op.inputs);
            ids(nj.get("outputs"), op.outputs);
            if (auto a = nj.get("attributes"))
                for (auto& [k, v] : a->obj) op.attrs[k] = v;
            g->ops.push_back(std::move(op));
        }
    }
    return g;
}

}  // namespace

std::shared_ptr<Graph> load_gguf_file(const std::string& path) {
    int fd = ::open(path.c_str(), O_RDONLY);
    GB_CHECK(fd >= 0, "cannot open model file: " + path);
    struct stat st;
    if (fstat(fd, &st) != 0) {
        ::close(fd);
        GB_CHECK(false, "cannot stat model file: " + path);
    }
    size_t size = (size_t)st.st_size;
    void* m = size ? mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
    ::close(fd);
    GB_CHECK(m != MAP_FAILED, "cannot mmap model file: " + path);
    madvise(m, size, MADV_SEQUENTIAL);
    std::shared_ptr<void> storage(m, [size](void* p) { munmap(p, size); });
    return parse((const uint8_t*)m, size, storage);
}

std::shared_ptr<Graph> load_gguf_bytes(const uint8_t* data, size_t size) {
    auto* copy = new std::vector<uint8_t>(data, data + size);
    std::shared_ptr<void> storage(copy, [](void* p) { delete (std::vector<uint8_t>*)p; });
    return parse(copy->data(), copy->size(), storage);
}

}  // namespace gb
