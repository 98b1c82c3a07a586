// `jalapeno`: the engine's command line (engine/src/main.rs:7-112) over the C ABI.
//
//   jalapeno <cpu|metal|gpu> <model> <new tokens> [--draft <model>] [--gamma <count>]
//            [--mxfp4] [--adaptive] [--max-gamma <count>] [--prefill-backend <b>]
//            [--draft-backend <b>] [--stats] [--time-rows <r1,r2,...>] < prompt.json
//
// Same flags, defaults (gamma 5, max gamma 8), checks and messages, in the
// same order: arguments, then the prompt (a JSON array of token ids on
// stdin), then the models.  Prints the generated ids as a JSON array on
// stdout; with a draft, "accepted A / D draft tokens in R rounds" and (with
// --stats) the statistics object on stderr.  A failure prints
// `Error: <message>` on stderr and exits with status 1, as a Rust main
// returning Err does.
//
// Model names resolve to <weights>/<name> (with "-MXFP4" appended under
// --mxfp4), where <weights> is $JALAPENO_WEIGHTS or, by default, the
// `weights` folder at the repository root (the reference's
// engine/../weights).  Only the gpu backend runs in this build; cpu and
// metal are accepted by the parser, as in the reference, and refused when a
// model would be loaded for them.  --time-rows (Model::time_pass,
// model.rs:242-266) is macOS-only in the reference; here it runs on the GPU.
#include <algorithm>
#include <chrono>
#include <cinttypes>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <iterator>
#include <limits>
#include <string>
#include <vector>

#include <unistd.h>

#include "../../include/jalapeno.h"

namespace {

// An error as a Rust main prints it: `Error: ` and the error's Debug form.
struct Fail {
    std::string debug;
};

// Debug form of a string error (Box<dyn Error> from &str or String).
std::string quoted(const std::string& s) {
    std::string out = "\"";
    for (char c : s) {
        if (c == '"' || c == '\\') out += '\\';
        out += c;
    }
    return out + "\"";
}

[[noreturn]] void fail(const std::string& msg) { throw Fail{quoted(msg)}; }

// usize::from_str (ParseIntError's Debug form on failure).
size_t parse_usize(const std::string& s) {
    if (s.empty()) throw Fail{"ParseIntError { kind: Empty }"};
    size_t i = s[0] == '+' ? 1 : 0;
    if (i == s.size()) throw Fail{"ParseIntError { kind: InvalidDigit }"};
    uint64_t v = 0;
    for (; i < s.size(); ++i) {
        if (s[i] < '0' || s[i] > '9') throw Fail{"ParseIntError { kind: InvalidDigit }"};
        const uint64_t d = (uint64_t)(s[i] - '0');
        if (v > (std::numeric_limits<uint64_t>::max() - d) / 10) throw Fail{"ParseIntError { kind: PosOverflow }"};
        v = v * 10 + d;
    }
    return (size_t)v;
}

enum class Backend { Cpu, Metal, Gpu };

// Backend::from_str (model.rs:298-308).
Backend parse_backend(const std::string& s) {
    if (s == "cpu") return Backend::Cpu;
    if (s == "metal") return Backend::Metal;
    if (s == "gpu") return Backend::Gpu;
    fail("backend must be cpu, metal or gpu");
}

const char* backend_name(Backend b) {  // serde rename_all = "lowercase"
    return b == Backend::Cpu ? "cpu" : (b == Backend::Metal ? "metal" : "gpu");
}

// serde_json::from_reader::<Vec<usize>>: a JSON array of non-negative
// integers, whitespace around tokens, nothing after the array.
std::vector<uint32_t> parse_prompt(const std::string& text) {
    size_t i = 0, line = 1, col = 0;
    auto err = [&](const std::string& what) -> Fail {
        return Fail{"Error(" + quoted(what) + ", line: " + std::to_string(line) + ", column: " + std::to_string(col) + ")"};
    };
    auto skip = [&]() {
        while (i < text.size() && (text[i] == ' ' || text[i] == '\t' || text[i] == '\n' || text[i] == '\r')) {
            if (text[i] == '\n') {
                ++line;
                col = 0;
            } else {
                ++col;
            }
            ++i;
        }
    };
    auto next = [&]() {
        ++col;
        return text[i++];
    };
    std::vector<uint32_t> ids;
    skip();
    if (i == text.size()) throw err("EOF while parsing a value");
    if (text[i] != '[') {
        next();
        throw err("invalid type: expected a sequence");
    }
    next();
    skip();
    if (i < text.size() && text[i] == ']') {
        next();
    } else {
        for (;;) {
            skip();
            if (i == text.size()) throw err("EOF while parsing a list");
            if (text[i] < '0' || text[i] > '9') {
                next();
                throw err(text[i - 1] == '-' ? "invalid value: integer, expected usize" : "expected value");
            }
            uint64_t v = 0;
            while (i < text.size() && text[i] >= '0' && text[i] <= '9') {
                const uint64_t d = (uint64_t)(next() - '0');
                if (v > (std::numeric_limits<uint64_t>::max() - d) / 10) throw err("number out of range");
                v = v * 10 + d;
            }
            if (i < text.size() && (text[i] == '.' || text[i] == 'e' || text[i] == 'E')) {
                next();
                throw err("invalid type: floating point, expected usize");
            }
            // ids index the embedding table; the engine takes them as u32
            if (v > 0xFFFFFFFFull) throw err("token id out of range");
            ids.push_back((uint32_t)v);
            skip();
            if (i == text.size()) throw err("EOF while parsing a list");
            const char c = next();
            if (c == ']') break;
            if (c != ',') throw err("expected `,` or `]`");
        }
    }
    skip();
    if (i != text.size()) {
        next();
        throw err("trailing characters");
    }
    return ids;
}

// serde_json's f64 text: the shortest round-trip digits, ".0" on integers.
std::string json_f64(double v) {
    char buf[64];
    for (int prec = 1; prec <= 17; ++prec) {
        snprintf(buf, sizeof buf, "%.*g", prec, v);
        if (strtod(buf, nullptr) == v) break;
    }
    std::string s = buf;
    if (s.find_first_of(".eEn") == std::string::npos) s += ".0";
    return s;
}

std::string json_ids(const uint32_t* ids, size_t n) {
    std::string s = "[";
    for (size_t i = 0; i < n; ++i) {
        if (i) s += ',';
        s += std::to_string(ids[i]);
    }
    return s + "]";
}

void check(jl_status st) {
    if (st != JL_OK) fail(jl_last_error());
}

std::string weights_root() {
    if (const char* env = getenv("JALAPENO_WEIGHTS")) return env;
    // <repo>/jalapenos-at-home_b200/bin/jalapeno -> <repo>/weights
    char exe[4096];
    const ssize_t n = readlink("/proc/self/exe", exe, sizeof exe - 1);
    if (n <= 0) return "weights";
    exe[n] = 0;
    std::string p = exe;
    for (int up = 0; up < 3; ++up) {
        const size_t cut = p.find_last_of('/');
        if (cut == std::string::npos) return "weights";
        p.erase(cut);
    }
    return p + "/weights";
}

// Model::load_with_prefill (model.rs:59-63): the gpu backend needs a gpu
// prefill; this build has no cpu or metal engine.
jl_model* load(const std::string& name, Backend backend, Backend prefill) {
    const bool gpu = backend == Backend::Gpu || prefill == Backend::Gpu;
    if (gpu && !(backend == Backend::Gpu && prefill == Backend::Gpu))
        fail("the gpu backend keeps the KV cache on the GPU, so prefill must use gpu too");
    if (!gpu) fail(std::string("the ") + backend_name(backend) + " backend is not part of this build: use gpu");
    jl_model* m = nullptr;
    check(jl_model_load((weights_root() + "/" + name).c_str(), nullptr, &m));
    return m;
}

struct Args {
    Backend backend = Backend::Gpu;
    std::string name;
    size_t count = 0;
    bool have_draft = false;
    std::string draft_name;
    size_t gamma = 5, max_gamma = 8;
    bool mxfp4 = false, adaptive = false, stats = false;
    bool have_prefill = false, have_draft_backend = false, have_time_rows = false;
    Backend prefill_backend = Backend::Gpu, draft_backend = Backend::Gpu;
    std::string time_rows;
};

int run(int argc, char** argv) {
    const char* usage =
        "usage: engine <cpu|metal|gpu> <model> <new tokens> [--draft <model>] [--gamma <count>] [--mxfp4] "
        "[--adaptive] [--max-gamma <count>] [--prefill-backend <cpu|metal|gpu>] [--draft-backend "
        "<cpu|metal|gpu>] [--stats] < prompt.json";
    int a = 1;
    auto next = [&]() -> const char* { return a < argc ? argv[a++] : nullptr; };
    Args o;
    const char* b = next();
    if (!b || (strcmp(b, "cpu") && strcmp(b, "metal") && strcmp(b, "gpu"))) fail(usage);
    o.backend = parse_backend(b);
    const char* nm = next();
    if (!nm) fail("missing model");
    o.name = nm;
    const char* cnt = next();
    if (!cnt) fail("missing token count");
    o.count = parse_usize(cnt);
    while (const char* flag = next()) {
        const std::string f = flag;
        auto value = [&](const char* missing) -> std::string {
            const char* v = next();
            if (!v) fail(missing);
            return v;
        };
        if (f == "--adaptive") {
            o.adaptive = true;
        } else if (f == "--max-gamma") {
            o.max_gamma = parse_usize(value("missing max gamma"));
        } else if (f == "--prefill-backend") {
            o.prefill_backend = parse_backend(value("missing prefill backend"));
            o.have_prefill = true;
        } else if (f == "--draft-backend") {
            o.draft_backend = parse_backend(value("missing draft backend"));
            o.have_draft_backend = true;
        } else if (f == "--stats") {
            o.stats = true;
        } else if (f == "--time-rows") {
            o.time_rows = value("missing row counts");
            o.have_time_rows = true;
        } else if (f == "--mxfp4") {
            o.mxfp4 = true;
        } else if (f == "--draft") {
            o.draft_name = value("missing draft model");
            o.have_draft = true;
        } else if (f == "--gamma") {
            o.gamma = parse_usize(value("missing gamma"));
        } else {
            fail("unexpected argument: " + f);
        }
    }
    if (o.gamma == 0) fail("gamma must be positive");
    if ((o.adaptive || o.have_draft_backend || o.stats) && !o.have_draft)
        fail("--adaptive, --draft-backend and --stats require --draft");
    jl_schedule schedule;
    if (o.adaptive) {
        if (o.gamma > 0xFFFFFFFFull || o.max_gamma > 0xFFFFFFFFull ||
            jl_schedule_adaptive((uint32_t)o.gamma, (uint32_t)o.max_gamma, &schedule) != JL_OK)
            fail("adaptive gamma must be positive and no greater than max gamma");
    } else {
        check(jl_schedule_fixed((uint32_t)std::min<size_t>(o.gamma, 0xFFFFFFFFu), &schedule));
    }
    const std::string text((std::istreambuf_iterator<char>(std::cin)), std::istreambuf_iterator<char>());
    const std::vector<uint32_t> prompt = parse_prompt(text);
    if (prompt.empty()) fail("prompt is empty");

    if (o.mxfp4) {
        o.name += "-MXFP4";
        if (o.have_draft) o.draft_name += "-MXFP4";
    }
    const Backend prefill = o.have_prefill ? o.prefill_backend : o.backend;
    jl_model* model = load(o.name, o.backend, prefill);
    struct Free {
        jl_model* m;
        ~Free() { jl_model_free(m); }
    } free_model{model};

    if (o.have_time_rows) {
        // profiling: how long one pass takes for each number of tokens
        size_t start = 0;
        for (;;) {
            const size_t comma = o.time_rows.find(',', start);
            const size_t rows = parse_usize(o.time_rows.substr(start, comma == std::string::npos ? std::string::npos : comma - start));
            double wall = 0, gpu = 0;
            check(jl_time_pass(model, prompt.data(), prompt.size(), rows, 15, &wall, &gpu));
            printf("{\"gpu_ms\":%s,\"rows\":%zu,\"wall_ms\":%s}\n", json_f64(gpu).c_str(), rows, json_f64(wall).c_str());
            if (comma == std::string::npos) break;
            start = comma + 1;
        }
        return 0;
    }

    std::vector<uint32_t> out(prompt.size() + o.count + 1);
    size_t n_out = 0;
    if (o.have_draft) {
        const Backend dback = o.have_draft_backend ? o.draft_backend : o.backend;
        const Backend dprefill = o.have_prefill ? o.prefill_backend : dback;
        jl_model* draft = load(o.draft_name, dback, dprefill);
        Free free_draft{draft};
        std::vector<jl_round_stats> rounds(o.count + 1);
        jl_spec_options so;
        jl_spec_options_default(&so);
        // --stats reports per-phase times, which the host-driven loop measures
        so.mode = o.stats ? JL_SPEC_HOST : JL_SPEC_DEVICE;
        jl_spec_result r = {};
        r.tokens = out.data();
        r.tokens_cap = out.size();
        r.rounds_out = rounds.data();
        r.rounds_cap = rounds.size();
        const auto t0 = std::chrono::steady_clock::now();
        check(jl_generate_speculative(model, draft, prompt.data(), prompt.size(), o.count, &schedule, &so, &r));
        const double elapsed = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        n_out = r.n_tokens;
        if (o.stats) {
            std::string rs = "[";
            for (size_t i = 0; i < std::min(r.rounds, rounds.size()); ++i) {
                if (i) rs += ',';
                const jl_round_stats& s = rounds[i];
                rs += "{\"accepted\":" + std::to_string(s.accepted) + ",\"drafted\":" + std::to_string(s.drafted) +
                      ",\"gamma\":" + std::to_string(s.gamma) + ",\"next_gamma\":" + std::to_string(s.next_gamma) + "}";
            }
            rs += "]";
            auto phase = [](size_t passes, double ms) {
                return "{\"elapsed_ms\":" + json_f64(ms) + ",\"passes\":" + std::to_string(passes) + "}";
            };
            // keys in serde_json's (sorted) order
            fprintf(stderr,
                    "{\"accepted\":%zu,\"adaptive\":%s,\"draft\":%s,\"draft_backend\":\"%s\","
                    "\"draft_prefill_backend\":\"%s\",\"drafted\":%zu,\"elapsed_ms\":%s,\"generated\":%zu,"
                    "\"prefill\":%s,\"round_stats\":%s,\"rounds\":%zu,\"target_prefill_backend\":\"%s\","
                    "\"verify\":%s,\"verify_backend\":\"%s\"}\n",
                    r.accepted, o.adaptive ? "true" : "false", phase(r.draft_passes, r.draft_ms).c_str(),
                    backend_name(dback), backend_name(dprefill), r.drafted, json_f64(elapsed).c_str(),
                    r.n_tokens - prompt.size(), phase(r.prefill_passes, r.prefill_ms).c_str(), rs.c_str(),
                    r.rounds, backend_name(prefill), phase(r.verify_passes, r.verify_ms).c_str(),
                    backend_name(o.backend));
        }
        fprintf(stderr, "accepted %zu / %zu draft tokens in %zu rounds\n", r.accepted, r.drafted, r.rounds);
    } else {
        check(jl_generate(model, prompt.data(), prompt.size(), o.count, out.data(), out.size(), &n_out));
    }
    printf("%s\n", json_ids(out.data() + prompt.size(), n_out - prompt.size()).c_str());
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        return run(argc, argv);
    } catch (const Fail& f) {
        fprintf(stderr, "Error: %s\n", f.debug.c_str());
        return 1;
    }
}
