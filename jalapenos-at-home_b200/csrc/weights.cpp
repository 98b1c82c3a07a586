// Host-side checkpoint loading: the reference's `load` / `try_load`
// (engine/src/lib.rs:85-202) and config.json reading (engine/src/model.rs:
// 19-24, 64-68).  Runs without a GPU.
#include <dirent.h>
#include <sys/stat.h>

#include <algorithm>
#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>

#include "jl_internal.h"

namespace jl {
namespace {

// ---- a small JSON reader: enough for safetensors headers and config.json ----

struct Json {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    double num = 0;
    bool is_int = false;
    long long i = 0;
    unsigned long long u = 0;
    bool neg = false;
    std::string s;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    const Json* get(const char* key) const {
        for (auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

struct Parser {
    const char* p;
    const char* end;
    std::string err;

    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    bool fail(const char* m) {
        if (err.empty()) err = m;
        return false;
    }
    bool lit(const char* w) {
        size_t n = strlen(w);
        if ((size_t)(end - p) < n || memcmp(p, w, n)) return false;
        p += n;
        return true;
    }
    bool str(std::string& out) {
        if (p >= end || *p != '"') return fail("expected string");
        ++p;
        while (p < end && *p != '"') {
            char c = *p++;
            if (c == '\\') {
                if (p >= end) return fail("bad escape");
                char e = *p++;
                switch (e) {
                    case '"': out += '"'; break;
                    case '\\': out += '\\'; break;
                    case '/': out += '/'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'n': out += '\n'; break;
                    case 'r': out += '\r'; break;
                    case 't': out += '\t'; break;
                    case 'u': {
                        if (end - p < 4) return fail("bad unicode escape");
                        unsigned cp = (unsigned)strtoul(std::string(p, 4).c_str(), nullptr, 16);
                        p += 4;
                        if (cp < 0x80) {
                            out += (char)cp;
                        } else if (cp < 0x800) {
                            out += (char)(0xC0 | (cp >> 6));
                            out += (char)(0x80 | (cp & 0x3F));
                        } else {
                            out += (char)(0xE0 | (cp >> 12));
                            out += (char)(0x80 | ((cp >> 6) & 0x3F));
                            out += (char)(0x80 | (cp & 0x3F));
                        }
                        break;
                    }
                    default: return fail("bad escape");
                }
            } else {
                out += c;
            }
        }
        if (p >= end) return fail("unterminated string");
        ++p;
        return true;
    }
    bool value(Json& v, int depth) {
        if (depth > 64) return fail("nesting too deep");
        ws();
        if (p >= end) return fail("unexpected end");
        char c = *p;
        if (c == '{') {
            v.kind = Json::OBJ;
            ++p;
            ws();
            if (p < end && *p == '}') { ++p; return true; }
            for (;;) {
                ws();
                std::string k;
                if (!str(k)) return false;
                ws();
                if (p >= end || *p != ':') return fail("expected ':'");
                ++p;
                Json child;
                if (!value(child, depth + 1)) return false;
                v.obj.emplace_back(std::move(k), std::move(child));
                ws();
                if (p < end && *p == ',') { ++p; continue; }
                if (p < end && *p == '}') { ++p; return true; }
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.kind = Json::ARR;
            ++p;
            ws();
            if (p < end && *p == ']') { ++p; return true; }
            for (;;) {
                Json child;
                if (!value(child, depth + 1)) return false;
                v.arr.push_back(std::move(child));
                ws();
                if (p < end && *p == ',') { ++p; continue; }
                if (p < end && *p == ']') { ++p; return true; }
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = Json::STR;
            return str(v.s);
        }
        if (lit("true")) { v.kind = Json::BOOL; v.b = true; return true; }
        if (lit("false")) { v.kind = Json::BOOL; v.b = false; return true; }
        if (lit("null")) { v.kind = Json::NUL; return true; }
        if (c == '-' || (c >= '0' && c <= '9')) {
            const char* q = p;
            if (*q == '-') ++q;
            bool integral = true;
            while (q < end && (isdigit((unsigned char)*q) || *q == '.' || *q == 'e' || *q == 'E' ||
                               *q == '+' || *q == '-')) {
                if (*q == '.' || *q == 'e' || *q == 'E') integral = false;
                ++q;
            }
            std::string t(p, q);
            v.kind = Json::NUM;
            v.num = strtod(t.c_str(), nullptr);
            v.neg = t[0] == '-';
            if (integral) {
                errno = 0;
                if (v.neg) {
                    v.i = strtoll(t.c_str(), nullptr, 10);
                } else {
                    v.u = strtoull(t.c_str(), nullptr, 10);
                    v.i = (long long)v.u;
                }
                v.is_int = errno == 0;
            }
            p = q;
            return true;
        }
        return fail("unexpected character");
    }
};

bool parse_json(const char* data, size_t len, Json& out, std::string& err) {
    Parser ps{data, data + len, {}};
    if (!ps.value(out, 0)) {
        err = ps.err;
        return false;
    }
    ps.ws();
    if (ps.p != ps.end) {
        err = "trailing characters";
        return false;
    }
    return true;
}

bool as_usize(const Json* v, unsigned long long& out) {
    if (!v || v->kind != Json::NUM || !v->is_int || v->neg) return false;
    out = v->u;
    return true;
}

bool ends_with(const std::string& s, const char* suffix) {
    size_t n = strlen(suffix);
    return s.size() >= n && s.compare(s.size() - n, n, suffix) == 0;
}

jl_status fmt_error(const char* msg, const std::string& name = "") {
    if (name.empty())
        set_error("%s", msg);
    else
        set_error("%s: %s", msg, name.c_str());
    return JL_ERR_FORMAT;
}

}  // namespace

jl_status load_config(const std::string& dir, HostConfig* out) {
    // engine/src/model.rs:64-68: config.json -> Config { num_hidden_layers,
    // max_position_embeddings, eos_token_id }, all usize.
    std::string path = dir + "/config.json";
    std::ifstream f(path, std::ios::binary);
    if (!f) {
        set_error("cannot read %s", path.c_str());
        return JL_ERR_IO;
    }
    std::string text((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    Json j;
    std::string err;
    if (!parse_json(text.data(), text.size(), j, err) || j.kind != Json::OBJ) {
        set_error("config.json: %s", err.empty() ? "not an object" : err.c_str());
        return JL_ERR_FORMAT;
    }
    unsigned long long layers, maxpos, eos;
    if (!as_usize(j.get("num_hidden_layers"), layers) ||
        !as_usize(j.get("max_position_embeddings"), maxpos) ||
        !as_usize(j.get("eos_token_id"), eos)) {
        set_error("config.json: num_hidden_layers, max_position_embeddings and eos_token_id "
                  "must be non-negative integers");
        return JL_ERR_FORMAT;
    }
    if (layers > 4096 || maxpos > (1u << 30) || eos > 0xFFFFFFFFull) {
        set_error("config.json: value out of range");
        return JL_ERR_FORMAT;
    }
    out->layers = (int)layers;
    out->max_positions = (int)maxpos;
    out->eos = (int)eos;
    return JL_OK;
}

jl_status scan_weights(const std::string& dir, WeightIndex* out) {
    // engine/src/lib.rs:89-100: every *.safetensors file, sorted by path.
    DIR* d = opendir(dir.c_str());
    if (!d) {
        set_error("cannot open model directory %s", dir.c_str());
        return JL_ERR_IO;
    }
    std::vector<std::string> paths;
    while (dirent* e = readdir(d)) {
        std::string n = e->d_name;
        if (ends_with(n, ".safetensors")) paths.push_back(dir + "/" + n);
    }
    closedir(d);
    std::sort(paths.begin(), paths.end());
    if (paths.empty()) {
        set_error("model directory has no safetensors files");
        return JL_ERR_FORMAT;
    }
    struct Raw {
        std::vector<size_t> shape;
        FileRange at;
        std::vector<uint8_t> bytes;  // scales only
    };
    std::map<std::string, Raw> packed, scales;
    auto& tensors = out->tensors;
    for (const auto& path : paths) {
        FILE* f = fopen(path.c_str(), "rb");
        if (!f) {
            set_error("cannot open %s", path.c_str());
            return JL_ERR_IO;
        }
        std::unique_ptr<FILE, int (*)(FILE*)> guard(f, fclose);
        struct stat st;
        if (fstat(fileno(f), &st) != 0) {
            set_error("cannot stat %s", path.c_str());
            return JL_ERR_IO;
        }
        const uint64_t file_len = (uint64_t)st.st_size;
        uint8_t first8[8];
        if (fread(first8, 1, 8, f) != 8) {
            set_error("cannot read safetensors header length: %s", path.c_str());
            return JL_ERR_IO;
        }
        uint64_t header_len = 0;
        for (int i = 7; i >= 0; --i) header_len = (header_len << 8) | first8[i];
        // lib.rs:109-111
        if (header_len > 100000000ull || header_len + 8 > file_len)
            return fmt_error("invalid safetensors header length");
        std::string header(header_len, '\0');
        if (fread(&header[0], 1, header_len, f) != header_len) {
            set_error("short read in %s", path.c_str());
            return JL_ERR_IO;
        }
        Json h;
        std::string err;
        if (!parse_json(header.data(), header.size(), h, err) || h.kind != Json::OBJ) {
            set_error("invalid safetensors header in %s: %s", path.c_str(),
                      err.empty() ? "not an object" : err.c_str());
            return JL_ERR_FORMAT;
        }
        // lib.rs:115-120
        bool quantized = false;
        struct Entry {
            std::string name, dtype;
            std::vector<size_t> shape;
            uint64_t start, end;
        };
        std::vector<Entry> entries;
        for (auto& kv : h.obj) {
            if (kv.first == "__metadata__") {
                const Json* fmt = kv.second.kind == Json::OBJ ? kv.second.get("format") : nullptr;
                quantized = fmt && fmt->kind == Json::STR && fmt->s == "jalapenos-mxfp4-v1";
                continue;
            }
            // lib.rs:121-126: each entry must deserialize as HeaderEntry
            const Json& v = kv.second;
            const Json* dt = v.kind == Json::OBJ ? v.get("dtype") : nullptr;
            const Json* sh = v.kind == Json::OBJ ? v.get("shape") : nullptr;
            const Json* off = v.kind == Json::OBJ ? v.get("data_offsets") : nullptr;
            if (!dt || dt->kind != Json::STR || !sh || sh->kind != Json::ARR || !off ||
                off->kind != Json::ARR || off->arr.size() != 2)
                return fmt_error("invalid safetensors header entry", kv.first);
            Entry e;
            e.name = kv.first;
            e.dtype = dt->s;
            for (auto& dim : sh->arr) {
                unsigned long long u;
                if (!as_usize(&dim, u)) return fmt_error("invalid tensor shape", kv.first);
                e.shape.push_back((size_t)u);
            }
            unsigned long long a, b;
            if (!as_usize(&off->arr[0], a) || !as_usize(&off->arr[1], b))
                return fmt_error("invalid tensor offsets", kv.first);
            e.start = a;
            e.end = b;
            entries.push_back(std::move(e));
        }
        std::stable_sort(entries.begin(), entries.end(),
                         [](const Entry& x, const Entry& y) { return x.start < y.start; });
        const uint64_t base = 8 + header_len;
        for (auto& e : entries) {
            // lib.rs:129-133
            if (e.start > e.end || e.end > file_len - base)
                return fmt_error("invalid tensor offsets", e.name);
            const FileRange at{path, base + e.start, e.end - e.start};
            // lib.rs:137-141
            size_t elements = 1;
            for (size_t dim : e.shape) {
                if (dim != 0 && elements > SIZE_MAX / dim) return fmt_error("tensor shape overflow");
                elements *= dim;
            }
            if (quantized && e.dtype == "U8") {
                // lib.rs:142-162
                if (elements != at.bytes) return fmt_error("invalid packed tensor size", e.name);
                if (ends_with(e.name, ".mxfp4_packed")) {
                    std::string n = e.name.substr(0, e.name.size() - strlen(".mxfp4_packed"));
                    if (packed.count(n)) return fmt_error("duplicate packed tensor");
                    packed[n] = Raw{e.shape, at, {}};
                } else if (ends_with(e.name, ".mxfp4_scales")) {
                    std::string n = e.name.substr(0, e.name.size() - strlen(".mxfp4_scales"));
                    if (scales.count(n)) return fmt_error("duplicate scale tensor");
                    Raw r{e.shape, at, std::vector<uint8_t>(at.bytes)};
                    if (fseeko(f, (off_t)at.offset, SEEK_SET) != 0 ||
                        (at.bytes && fread(r.bytes.data(), 1, at.bytes, f) != at.bytes)) {
                        set_error("short read of %s in %s", e.name.c_str(), path.c_str());
                        return JL_ERR_IO;
                    }
                    scales[n] = std::move(r);
                } else {
                    return fmt_error("unexpected U8 tensor", e.name);
                }
            } else {
                // lib.rs:163-181
                bool dtype_ok = e.dtype == "BF16" || (quantized && e.dtype == "U16");
                if (!dtype_ok || elements > SIZE_MAX / 2 || elements * 2 != at.bytes)
                    return fmt_error("expected BF16 tensor", e.name);
                if (tensors.count(e.name)) return fmt_error("duplicate tensor");
                IndexTensor t;
                t.name = e.name;
                t.dtype = JL_BF16;
                t.shape = e.shape;
                t.data = at;
                tensors.emplace(e.name, std::move(t));
            }
        }
    }
    // lib.rs:184-197: pair packed nibbles with their scales
    for (auto& kv : packed) {
        auto sc = scales.find(kv.first);
        if (sc == scales.end()) return fmt_error("missing MXFP4 scales");
        const auto& shape = kv.second.shape;
        if (shape.size() != 2 || shape[1] % 16 != 0 || sc->second.shape.size() != 2 ||
            sc->second.shape[0] != shape[0] || sc->second.shape[1] != shape[1] / 16)
            return fmt_error("invalid MXFP4 tensor shape", kv.first);
        size_t rows = shape[0], cols = shape[1] * 2;
        // Tensor::quantized -> Mxfp4::validate (engine/src/mxfp4.rs:11-25)
        if (rows == 0 || cols == 0 || cols % 32)
            return fmt_error("MXFP4 requires nonempty rows with a width divisible by 32");
        if (kv.second.at.bytes != rows * cols / 2 || sc->second.bytes.size() != rows * cols / 32)
            return fmt_error("MXFP4 data length does not match shape");
        if (std::find(sc->second.bytes.begin(), sc->second.bytes.end(), 255) != sc->second.bytes.end())
            return fmt_error("MXFP4 checkpoint contains a NaN scale");
        if (tensors.count(kv.first)) return fmt_error("duplicate tensor");
        IndexTensor t;
        t.name = kv.first;
        t.dtype = JL_MXFP4;
        t.shape = {rows, cols};
        t.data = kv.second.at;
        t.scales = std::move(sc->second.bytes);
        tensors.emplace(kv.first, std::move(t));
        scales.erase(sc);
    }
    if (!scales.empty()) return fmt_error("MXFP4 scales have no matching packed weights");
    return JL_OK;
}

jl_status read_range(const FileRange& r, void* dst, size_t offset, size_t bytes) {
    if (offset > r.bytes || bytes > r.bytes - offset) {
        set_error("read past the end of a tensor in %s", r.path.c_str());
        return JL_ERR_INVALID_ARG;
    }
    FILE* f = fopen(r.path.c_str(), "rb");
    if (!f) {
        set_error("cannot open %s", r.path.c_str());
        return JL_ERR_IO;
    }
    std::unique_ptr<FILE, int (*)(FILE*)> guard(f, fclose);
    if (fseeko(f, (off_t)(r.offset + offset), SEEK_SET) != 0 ||
        (bytes && fread(dst, 1, bytes, f) != bytes)) {
        set_error("short read in %s", r.path.c_str());
        return JL_ERR_IO;
    }
    return JL_OK;
}

jl_status load_weights(const std::string& dir, jl_weights* out) {
    // engine/src/lib.rs:85-202: the whole checkpoint in host memory.
    WeightIndex idx;
    JL_TRY(scan_weights(dir, &idx));
    for (auto& kv : idx.tensors) {
        IndexTensor& it = kv.second;
        HostTensor t;
        t.name = it.name;
        t.dtype = it.dtype;
        t.shape = it.shape;
        std::vector<uint8_t> bytes(it.data.bytes);
        JL_TRY(read_range(it.data, bytes.data(), 0, bytes.size()));
        if (it.dtype == JL_MXFP4) {
            t.packed = std::move(bytes);
            t.scales = std::move(it.scales);
        } else {
            t.bf16.resize(bytes.size() / 2);
            for (size_t i = 0; i < t.bf16.size(); ++i)
                t.bf16[i] = (uint16_t)(bytes[2 * i] | (bytes[2 * i + 1] << 8));
        }
        out->tensors.emplace(kv.first, std::move(t));
    }
    return JL_OK;
}

}  // namespace jl
