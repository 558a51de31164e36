// ggmlc-bench for the B200 engine: the flags, test matrix, timing points and output formats of
// the reference's benchmark binary (runtime/tools/ggmlc_bench.cpp:65-98 flags, :296-420 pp,
// :422-560 tg, :562-700 pg, :708-744 JSON, :745-790 CSV / markdown), over this library's C ABI,
// so the reference's comparison scripts (examples/benchmarks/compare_ggmlc_vs_llama_cpp.py) run
// it unchanged.
//
//   pp<P>     prompt of P tokens in ubatch-sized chunks through the KV cache, from an empty cache
//   tg<N>     N single-token decode steps after one untimed token at position 0
//   pp<P>+tg<N> (-pg P,N) prefill then N decode steps, wall clock a user feels
//
// Each test repeats -r times (host wall clock around the work, then a device synchronize, as the
// reference measures); avg_ts / stddev_ts are over the repetitions' tokens per second.
// Differences: the engine is CUDA only (-d defaults to cuda; cpu is refused with an error), and
// the "engine" field reads "ggmlc_b200".
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <map>
#include <numeric>
#include <sstream>
#include <string>
#include <utility>
#include <vector>

#include "ggmlc_b200.h"

namespace {

constexpr int kOpFlashAttnExt = 74;  // ggml_op GGML_OP_FLASH_ATTN_EXT in the serialized graph

struct Result {
    std::string model_filename, model_type, device, test_type;
    uint64_t model_size = 0, model_n_params = 0;
    int n_threads = 1, n_prompt = 0, n_gen = 0, n_depth = 0;
    double avg_ns = 0, stddev_ns = 0, avg_ts = 0, stddev_ts = 0;
    double ttft_ms = 0, decode_ms = 0;
};

struct Fail {
    std::string what;
};

void ok(int rc) {
    if (rc != 0) throw Fail{gb_last_error()};
}

std::vector<int> int_list(const std::string& s) {
    std::vector<int> v;
    std::stringstream ss(s);
    std::string item;
    while (std::getline(ss, item, ','))
        if (!item.empty()) {
            try {
                v.push_back(std::stoi(item));
            } catch (...) {
            }
        }
    return v;
}

std::string json_str(const std::string& s) {
    std::string o;
    for (char c : s) {
        switch (c) {
            case '\\': o += "\\\\"; break;
            case '"': o += "\\\""; break;
            case '\n': o += "\\n"; break;
            case '\r': o += "\\r"; break;
            case '\t': o += "\\t"; break;
            default: o += c;
        }
    }
    return o;
}

std::pair<double, double> mean_sd(const std::vector<double>& v) {
    if (v.empty()) return {0.0, 0.0};
    const double m = std::accumulate(v.begin(), v.end(), 0.0) / (double)v.size();
    double q = 0.0;
    for (double x : v) q += (x - m) * (x - m);
    return {m, v.size() > 1 ? std::sqrt(q / (double)(v.size() - 1)) : 0.0};
}

std::string label(const Result& r) {
    if (r.test_type == "pg" || (r.n_prompt > 0 && r.n_gen > 0))
        return "pp" + std::to_string(r.n_prompt) + "+tg" + std::to_string(r.n_gen);
    if (r.n_prompt > 0) return "pp" + std::to_string(r.n_prompt);
    return "tg" + std::to_string(r.n_gen);
}

// elements of a tensor payload from its GGUF type and byte size
uint64_t payload_elems(int type, uint64_t bytes) {
    switch (type) {
        case 0: return bytes / 4;          // F32
        case 1: return bytes / 2;          // F16
        case 2: return bytes / 18 * 32;    // Q4_0
        case 8: return bytes / 34 * 32;    // Q8_0
        case 24: return bytes;             // I8
        case 25: return bytes / 2;         // I16
        case 26: return bytes / 4;         // I32
        case 27: return bytes / 8;         // I64
        case 28: return bytes / 8;         // F64
        case 30: return bytes / 2;         // BF16
        default: return bytes / 4;
    }
}

void help(const char* prog) {
    std::cout
        << "ggmlc-bench (B200 engine): prompt-processing and generation benchmark\n"
        << "Usage: " << prog << " [options]\n\n"
        << "  -h, --help                    this text\n"
        << "  -m, --model <file>            compiled GGUF model\n"
        << "  -p, --n-prompt <n1,n2,...>    prompt lengths (default 16,64,128,256,512,1024)\n"
        << "  -n, --n-gen <n1,n2,...>       decode step counts (default 0,32,64,128)\n"
        << "  -pg <pp,tg>                   prefill pp then decode tg (repeatable; alone it\n"
        << "                                replaces the separate pp / tg matrix)\n"
        << "  -r, --repetitions <n>         repetitions per test (default 5)\n"
        << "  -o, --output <json|md|csv>    output format (default json)\n"
        << "  -d, --device <cuda|cuda:N>    device (default cuda; cpu is not served)\n"
        << "  -t, --threads <n>             recorded in the output (the GPU ignores it)\n"
        << "  -ub, --ubatch <n>             prefill chunk size through the KV cache (default 512)\n"
        << "  --no-warmup                   skip the warm-up pass of each test\n"
        << "  --cuda-graph                  replay decode steps from captured CUDA graphs\n"
        << "  --unplanned                   prepare without arena reuse\n"
        << "  --profile                     per-test prepare / run times on stderr\n"
        << "  --dump-graph                  op histogram and runtime graph summaries on stderr\n"
        << "  --full-logits                 logits for every prompt row (default: last row)\n"
        << "  --diag-mode <normal|replay|host-only|no-pos-update>   tg isolation modes\n";
}

struct Bench {
    gb_graph* g = nullptr;
    gb_executor* e = nullptr;
    uint32_t in_tid = 0;
    int64_t pos_tid = -1;
    bool kv = false;
    bool planned = true;
    int threads = 4;
    std::vector<std::string> symbols;

    ~Bench() {
        if (e) gb_executor_free(e);
        if (g) gb_graph_free(g);
    }

    // prepare for `s` tokens at position `pos`: every graph symbol takes s (the reference's
    // symbol environment), "pos" the position when the KV cache is on
    void prepare(int64_t s, int64_t pos) {
        std::vector<std::string> names;
        std::vector<int64_t> vals;
        names.push_back("s");
        vals.push_back(s);
        for (auto& sym : symbols)
            if (sym != "s") {
                names.push_back(sym);
                vals.push_back(s);
            }
        if (kv) {
            names.push_back("pos");
            vals.push_back(pos);
        }
        std::vector<const char*> cn;
        for (auto& n : names) cn.push_back(n.c_str());
        ok(gb_executor_prepare(e, cn.data(), vals.data(), (int)cn.size(), planned ? 1 : 0));
    }
    void feed(const int32_t* tok, const int32_t* pos, int64_t n) {
        ok(gb_executor_set_input(e, in_tid, tok, (size_t)n * 4));
        if (pos_tid >= 0) ok(gb_executor_set_input(e, (uint32_t)pos_tid, pos, (size_t)n * 4));
    }
    void run() { ok(gb_executor_run(e, threads)); }
    void sync() { ok(gb_executor_synchronize(e)); }
    void reset() {
        if (kv) ok(gb_executor_reset_kv_cache(e));
    }
    // prompt of P tokens in chunks of `chunk` through the cache
    void prefill(const std::vector<int32_t>& tok, const std::vector<int32_t>& pos, int P, int chunk) {
        for (int c0 = 0; c0 < P; c0 += chunk) {
            const int len = std::min(chunk, P - c0);
            prepare(len, c0);
            feed(tok.data() + c0, pos.data() + c0, len);
            run();
        }
    }
};

double now_ns() {
    return (double)std::chrono::duration_cast<std::chrono::nanoseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) {
        help(argv[0]);
        return 1;
    }
    std::string model, out_fmt = "json", device = "cuda", diag = "normal";
    std::vector<int> pp = {16, 64, 128, 256, 512, 1024}, tg = {0, 32, 64, 128};
    std::vector<std::pair<int, int>> pg;
    bool pp_set = false, tg_set = false, no_warmup = false, cuda_graph = false, unplanned = false;
    bool profile = false, dump = false, full_logits = false;
    int reps = 5, threads = 4, ubatch = 512;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        const bool more = i + 1 < argc;
        if (a == "-h" || a == "--help") {
            help(argv[0]);
            return 0;
        } else if ((a == "-m" || a == "--model") && more) {
            model = argv[++i];
        } else if ((a == "-p" || a == "--n-prompt") && more) {
            pp = int_list(argv[++i]);
            pp_set = true;
        } else if ((a == "-n" || a == "--n-gen") && more) {
            tg = int_list(argv[++i]);
            tg_set = true;
        } else if (a == "-pg" && more) {
            const auto v = int_list(argv[++i]);
            if (v.size() != 2) {
                std::cerr << "[ggmlc-bench ERROR] -pg expects exactly two ints: <pp,tg>\n";
                return 1;
            }
            pg.emplace_back(v[0], v[1]);
        } else if ((a == "-r" || a == "--repetitions") && more) {
            reps = std::max(1, std::atoi(argv[++i]));
        } else if ((a == "-o" || a == "--output") && more) {
            out_fmt = argv[++i];
        } else if ((a == "-d" || a == "--device") && more) {
            device = argv[++i];
        } else if ((a == "-t" || a == "--threads") && more) {
            threads = std::max(1, std::atoi(argv[++i]));
        } else if ((a == "-ub" || a == "--ubatch" || a == "--chunk-size") && more) {
            ubatch = std::max(1, std::atoi(argv[++i]));
        } else if (a == "--no-warmup") {
            no_warmup = true;
        } else if (a == "--cuda-graph") {
            cuda_graph = true;
        } else if (a == "--unplanned") {
            unplanned = true;
        } else if (a == "--profile") {
            profile = true;
        } else if (a == "--dump-graph") {
            dump = true;
        } else if (a == "--full-logits") {
            full_logits = true;
        } else if (a == "--diag-mode" && more) {
            diag = argv[++i];
        } else if (model.empty() && a.rfind("-", 0) != 0) {
            model = a;
        }
    }
    if (!pg.empty() && !pp_set && !tg_set) {  // -pg alone: no separate pp / tg tests
        pp = {0};
        tg = {0};
    }
    if (model.empty()) {
        std::cerr << "[ggmlc-bench ERROR] No model file specified. Use '-m <path.gguf>'.\n";
        return 1;
    }
    if (diag != "normal" && diag != "replay" && diag != "host-only" && diag != "no-pos-update") {
        std::cerr << "[ggmlc-bench ERROR] unknown --diag-mode " << diag << "\n";
        return 1;
    }
    std::ifstream f(model, std::ios::binary | std::ios::ate);
    if (!f.is_open()) {
        std::cerr << "[ggmlc-bench ERROR] Cannot open model file: " << model << "\n";
        return 1;
    }
    const uint64_t file_size = (uint64_t)f.tellg();
    f.close();

    std::vector<Result> results;
    try {
        Bench b;
        b.threads = threads;
        b.planned = !unplanned;
        ok(gb_loader_load_from_file(model.c_str(), &b.g));
        const std::string model_type = gb_graph_name(b.g) ? gb_graph_name(b.g) : "";
        for (int i = 0; i < gb_graph_num_symbols(b.g); ++i) b.symbols.push_back(gb_graph_symbol(b.g, i));
        const int n_in = gb_graph_num_ids(b.g, 0);
        if (n_in < 1) throw Fail{"the graph has no inputs"};
        ok(gb_graph_id(b.g, 0, 0, &b.in_tid));
        for (int i = 1; i < n_in; ++i) {  // a position-id input, when the graph has one
            uint32_t id = 0;
            ok(gb_graph_id(b.g, 0, i, &id));
            const char* name = nullptr;
            int type = 0, storage = 0;
            uint64_t bytes = 0;
            ok(gb_graph_tensor_info(b.g, id, &name, &type, &storage, &bytes));
            const std::string n = name ? name : "";
            if (n == "position_ids" || n.find("pos") != std::string::npos) b.pos_tid = id;
        }
        std::map<std::string, int> op_hist;
        for (int i = 0; i < gb_graph_num_ops(b.g); ++i) {
            uint32_t id = 0;
            int opcode = 0;
            const char* name = nullptr;
            ok(gb_graph_op_info(b.g, i, &id, &opcode, &name));
            if (opcode == kOpFlashAttnExt) b.kv = true;
            ++op_hist[name ? name : std::to_string(opcode)];
        }
        uint64_t n_params = 0;
        for (int i = 0; i < gb_graph_num_tensors(b.g); ++i) {
            uint32_t id = 0;
            ok(gb_graph_tensor_id(b.g, i, &id));
            const char* name = nullptr;
            int type = 0, storage = 0;
            uint64_t bytes = 0;
            ok(gb_graph_tensor_info(b.g, id, &name, &type, &storage, &bytes));
            if (bytes > 0) n_params += payload_elems(type, bytes);
        }
        int max_p = 0, max_g = 0;
        for (int p : pp) max_p = std::max(max_p, p);
        for (int t : tg) max_g = std::max(max_g, t);
        for (auto& c : pg) {
            max_p = std::max(max_p, c.first);
            max_g = std::max(max_g, c.second);
        }
        ok(gb_executor_create(b.g, device.c_str(), &b.e));
        if (cuda_graph) ok(gb_executor_set_enable_cuda_graph(b.e, 1));
        if (profile) ok(gb_executor_set_enable_profile(b.e, 1));
        ok(gb_executor_set_logits_last_only(b.e, full_logits ? 0 : 1));
        if (b.kv) ok(gb_executor_init_kv_cache(b.e, max_p + max_g + 512));
        if (dump) {
            std::cerr << "[ggmlc-bench] serialized_ops n=" << gb_graph_num_ops(b.g)
                      << " diag_mode=" << diag << "\n";
            for (auto& [n, c] : op_hist) std::cerr << "  ser " << n << " " << c << "\n";
        }
        auto base = [&](const std::string& type, int P, int N) {
            Result r;
            r.model_filename = model;
            r.model_type = model_type;
            r.model_size = file_size;
            r.model_n_params = n_params;
            r.device = device;
            r.n_threads = threads;
            r.n_prompt = P;
            r.n_gen = N;
            r.test_type = type;
            return r;
        };
        auto print_profile = [&](const std::string& test) {
            if (!profile) return;
            double prep = 0, run = 0;
            int np = 0, nr = 0;
            ok(gb_executor_get_profile(b.e, &prep, &run, &np, &nr));
            std::cerr << "[ggmlc-bench] profile " << test << " prepare_ms=" << prep
                      << " run_ms=" << run << " n_prepare=" << np << " n_run=" << nr << "\n";
            ok(gb_executor_reset_profile(b.e));
        };

        // ---- pp: prompt in ubatch chunks from an empty cache ----------------------------------
        for (int P : pp) {
            if (P <= 0) continue;
            const int chunk = b.kv ? ubatch : P;
            std::vector<int32_t> tok((size_t)P, 1), pos((size_t)P);
            for (int i = 0; i < P; ++i) pos[(size_t)i] = i;
            if (!no_warmup) {
                b.reset();
                b.prefill(tok, pos, P, chunk);
                b.sync();
            }
            if (dump) {
                b.reset();
                b.prepare(std::min(chunk, P), 0);
                std::cerr << "[ggmlc-bench] runtime prefill graph P=" << P << " chunk="
                          << std::min(chunk, P) << ": " << gb_executor_graph_summary(b.e) << "\n"
                          << "[ggmlc-bench] mul_mat/fa shapes: "
                          << gb_executor_mul_mat_shape_summary(b.e) << "\n";
            }
            std::vector<double> ns, ts;
            for (int r = 0; r < reps; ++r) {
                b.reset();
                const double t0 = now_ns();
                b.prefill(tok, pos, P, chunk);
                b.sync();
                const double dt = now_ns() - t0;
                ns.push_back(dt);
                ts.push_back(P / (dt * 1e-9));
            }
            Result res = base("pp", P, 0);
            std::tie(res.avg_ns, res.stddev_ns) = mean_sd(ns);
            std::tie(res.avg_ts, res.stddev_ts) = mean_sd(ts);
            res.ttft_ms = res.avg_ns * 1e-6;
            results.push_back(res);
            print_profile("pp" + std::to_string(P));
        }

        // ---- tg: N decode steps after an untimed first token ---------------------------------
        for (int N : tg) {
            if (N <= 0) continue;
            int32_t tok = 1, p = 0;
            if (!no_warmup) {
                b.reset();
                b.prepare(1, 0);
                b.feed(&tok, &p, 1);
                b.run();
                b.sync();
            }
            std::vector<double> ns, ts;
            for (int r = 0; r < reps; ++r) {
                b.reset();
                p = 0;
                b.prepare(1, 0);
                if (dump && r == 0) {
                    std::cerr << "[ggmlc-bench] runtime decode graph: "
                              << gb_executor_graph_summary(b.e) << "\n";
                    dump = false;
                }
                b.feed(&tok, &p, 1);
                b.run();
                b.sync();
                if (profile) ok(gb_executor_reset_profile(b.e));
                const double t0 = now_ns();
                if (diag == "replay") {  // one prepared step at position 1, replayed
                    p = 1;
                    b.prepare(1, 1);
                    b.feed(&tok, &p, 1);
                    for (int s = 1; s <= N; ++s) b.run();
                } else if (diag == "no-pos-update") {
                    p = 1;
                    b.prepare(1, 1);
                    for (int s = 1; s <= N; ++s) {
                        b.feed(&tok, &p, 1);
                        b.run();
                    }
                } else {
                    for (int s = 1; s <= N; ++s) {
                        p = s;
                        b.prepare(1, s);
                        b.feed(&tok, &p, 1);
                        if (diag != "host-only") b.run();
                    }
                }
                b.sync();
                const double dt = now_ns() - t0;
                ns.push_back(dt);
                ts.push_back(N / (dt * 1e-9));
            }
            Result res = base("tg", 0, N);
            std::tie(res.avg_ns, res.stddev_ns) = mean_sd(ns);
            std::tie(res.avg_ts, res.stddev_ts) = mean_sd(ts);
            res.decode_ms = res.avg_ns * 1e-6;
            results.push_back(res);
            print_profile("tg" + std::to_string(N) + " diag=" + diag);
        }

        // ---- pg: prefill then decode, time to first token and decode split -------------------
        for (auto& [P, N] : pg) {
            if (P <= 0 && N <= 0) continue;
            const int chunk = b.kv ? ubatch : std::max(P, 1);
            std::vector<int32_t> tok((size_t)std::max(P, 1), 1), pos((size_t)std::max(P, 1));
            for (int i = 0; i < P; ++i) pos[(size_t)i] = i;
            auto decode = [&](int start, int steps) {
                int32_t t = 1;
                for (int s = 0; s < steps; ++s) {
                    int32_t p = start + s;
                    b.prepare(1, p);
                    b.feed(&t, &p, 1);
                    b.run();
                }
            };
            if (!no_warmup) {
                b.reset();
                if (P > 0) b.prefill(tok, pos, P, chunk);
                if (N > 0) decode(P, 1);
                b.sync();
            }
            std::vector<double> ns, ts, ttft, dec;
            for (int r = 0; r < reps; ++r) {
                b.reset();
                const double t0 = now_ns();
                if (P > 0) b.prefill(tok, pos, P, chunk);
                b.sync();
                const double t1 = now_ns();
                if (N > 0) decode(P, N);
                b.sync();
                const double t2 = now_ns();
                ns.push_back(t2 - t0);
                ttft.push_back(t1 - t0);
                dec.push_back(t2 - t1);
                ts.push_back(P + N > 0 ? (P + N) / ((t2 - t0) * 1e-9) : 0.0);
            }
            Result res = base("pg", P, N);
            std::tie(res.avg_ns, res.stddev_ns) = mean_sd(ns);
            std::tie(res.avg_ts, res.stddev_ts) = mean_sd(ts);
            res.ttft_ms = mean_sd(ttft).first * 1e-6;
            res.decode_ms = mean_sd(dec).first * 1e-6;
            results.push_back(res);
            if (profile)
                std::cerr << "[ggmlc-bench] profile pg " << label(res) << " total_ms="
                          << res.avg_ns * 1e-6 << " ttft_ms=" << res.ttft_ms
                          << " decode_ms=" << res.decode_ms << "\n";
        }
    } catch (const Fail& x) {
        std::cerr << "[ggmlc-bench ERROR] " << x.what << "\n";
        return 1;
    }

    std::cout << std::fixed;
    if (out_fmt == "json") {
        std::cout << "[\n";
        for (size_t i = 0; i < results.size(); ++i) {
            const Result& r = results[i];
            std::cout << "  {\n"
                      << "    \"engine\": \"ggmlc_b200\",\n"
                      << "    \"model_filename\": \"" << json_str(r.model_filename) << "\",\n"
                      << "    \"model_type\": \"" << json_str(r.model_type) << "\",\n"
                      << "    \"model_size\": " << r.model_size << ",\n"
                      << "    \"model_n_params\": " << r.model_n_params << ",\n"
                      << "    \"device\": \"" << json_str(r.device) << "\",\n"
                      << "    \"n_threads\": " << r.n_threads << ",\n"
                      << "    \"n_prompt\": " << r.n_prompt << ",\n"
                      << "    \"n_gen\": " << r.n_gen << ",\n"
                      << "    \"n_depth\": " << r.n_depth << ",\n"
                      << "    \"test\": \"" << label(r) << "\",\n"
                      << std::setprecision(0) << "    \"avg_ns\": " << r.avg_ns << ",\n"
                      << "    \"stddev_ns\": " << r.stddev_ns << ",\n"
                      << std::setprecision(2) << "    \"avg_ts\": " << r.avg_ts << ",\n"
                      << "    \"stddev_ts\": " << r.stddev_ts << ",\n"
                      << std::setprecision(3) << "    \"avg_ms\": " << r.avg_ns * 1e-6 << ",\n"
                      << "    \"ttft_ms\": " << r.ttft_ms << ",\n"
                      << "    \"decode_ms\": " << r.decode_ms << "\n"
                      << "  }" << (i + 1 < results.size() ? "," : "") << "\n";
        }
        std::cout << "]\n";
    } else if (out_fmt == "csv") {
        std::cout << "engine,model_filename,model_type,model_size,model_n_params,device,n_threads,"
                     "n_prompt,n_gen,test,avg_ns,stddev_ns,avg_ts,stddev_ts,avg_ms,ttft_ms,"
                     "decode_ms\n";
        for (const Result& r : results)
            std::cout << "ggmlc_b200,\"" << r.model_filename << "\",\"" << r.model_type << "\","
                      << r.model_size << "," << r.model_n_params << ",\"" << r.device << "\","
                      << r.n_threads << "," << r.n_prompt << "," << r.n_gen << ",\"" << label(r)
                      << "\"," << std::setprecision(0) << r.avg_ns << "," << r.stddev_ns << ","
                      << std::setprecision(2) << r.avg_ts << "," << r.stddev_ts << ","
                      << std::setprecision(3) << r.avg_ns * 1e-6 << "," << r.ttft_ms << ","
                      << r.decode_ms << "\n";
    } else {
        std::cout << "| model | size | params | backend | threads | test | t/s | wall ms |\n"
                  << "| :--- | ---: | ---: | :--- | ---: | :--- | ---: | ---: |\n";
        for (const Result& r : results)
            std::cout << "| " << r.model_type << " | " << std::setprecision(2)
                      << r.model_size / (1024.0 * 1024.0 * 1024.0) << " GiB | "
                      << std::setprecision(1) << r.model_n_params / 1e6 << " M | " << r.device
                      << " | " << r.n_threads << " | " << label(r) << " | "
                      << std::setprecision(2) << r.avg_ts << " ± " << r.stddev_ts << " | "
                      << std::setprecision(1) << r.avg_ns * 1e-6 << " |\n";
    }
    return 0;
}
