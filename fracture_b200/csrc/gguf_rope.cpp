// RoPE frequencies from a GGUF model file, llama3 scaling included.
//
// The reference reads only `{arch}.rope.freq_base` (crates/fracture-gguf/src/parser.rs:482,
// default 500000) and builds its table with precompute_rope_freqs(head_dim, theta)
// (backends/fracture-cuda/src/lib.rs:133-155, called at bins/fracture-server-cuda/src/main.rs:104),
// so Llama 3.1 models run with unscaled frequencies. This file reads what a GGUF file can say
// about the scaling and turns it into the frequency table the RoPE kernels take:
//
//   * a `rope_freqs.weight` F32 tensor of head_dim/2 per-pair divisors (what llama.cpp's converter
//     writes for rope_type "llama3"): freq_i = base_i / divisor_i;
//   * else `{arch}.rope.scaling.type` = "llama3" with `{arch}.rope.scaling.factor`,
//     `{arch}.rope.scaling.original_context_length` and, when present,
//     `{arch}.rope.scaling.low_freq_factor` / `.high_freq_factor` (defaults 1 and 4, the Llama 3.1
//     values): the published llama3 rule (fb_rope_freqs_llama3);
//   * else type "linear" with a factor: freq_i = base_i / factor;
//   * else the reference's table, base_i = 1 / theta^(2i/d) rounded as it rounds it.
//
// The reader walks the GGUF v2/v3 layout: the header, the metadata key/value pairs (every value
// type, arrays included, is parsed or skipped by its size), the tensor infos, and the aligned data
// section (`general.alignment`, default 32) from which the one F32 tensor is read. It reads the
// file with stdio and allocates only host memory.

#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <string>
#include <vector>

#include "fracture_b200.h"

namespace {

enum GgufType : uint32_t {
    T_U8 = 0, T_I8 = 1, T_U16 = 2, T_I16 = 3, T_U32 = 4, T_I32 = 5, T_F32 = 6, T_BOOL = 7,
    T_STRING = 8, T_ARRAY = 9, T_U64 = 10, T_I64 = 11, T_F64 = 12
};

struct Reader {
    FILE* f = nullptr;
    bool ok = true;
    ~Reader() {
        if (f) fclose(f);
    }
    bool read(void* p, size_t n) {
        if (ok && fread(p, 1, n, f) != n) ok = false;
        return ok;
    }
    template <typename T> T get() {
        T v{};
        read(&v, sizeof v);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (1u << 20)) {
            ok = false;
            return {};
        }
        std::string s(n, '\0');
        read(&s[0], n);
        return s;
    }
    bool skip(uint64_t n) {
        if (ok && fseek(f, (long)n, SEEK_CUR) != 0) ok = false;
        return ok;
    }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case T_U8: case T_I8: case T_BOOL: return 1;
        case T_U16: case T_I16: return 2;
        case T_U32: case T_I32: case T_F32: return 4;
        case T_U64: case T_I64: case T_F64: return 8;
        default: return 0;
    }
}

// A metadata value kept when it is a number or a string; arrays are skipped.
struct Value {
    uint32_t type = 0xffffffffu;
    double num = 0.0;
    std::string s;
    bool is_num() const { return scalar_size(type) != 0 && type != T_BOOL; }
};

bool read_value(Reader& r, uint32_t type, Value* out) {
    out->type = type;
    switch (type) {
        case T_U8: out->num = r.get<uint8_t>(); break;
        case T_I8: out->num = r.get<int8_t>(); break;
        case T_U16: out->num = r.get<uint16_t>(); break;
        case T_I16: out->num = r.get<int16_t>(); break;
        case T_U32: out->num = r.get<uint32_t>(); break;
        case T_I32: out->num = r.get<int32_t>(); break;
        case T_F32: out->num = r.get<float>(); break;
        case T_BOOL: out->num = r.get<uint8_t>(); break;
        case T_U64: out->num = (double)r.get<uint64_t>(); break;
        case T_I64: out->num = (double)r.get<int64_t>(); break;
        case T_F64: out->num = r.get<double>(); break;
        case T_STRING: out->s = r.str(); break;
        case T_ARRAY: {
            const uint32_t et = r.get<uint32_t>();
            const uint64_t n = r.get<uint64_t>();
            if (!r.ok) return false;
            if (et == T_STRING) {
                for (uint64_t i = 0; i < n && r.ok; ++i) r.str();
            } else if (et == T_ARRAY || scalar_size(et) == 0) {
                return r.ok = false;  // nested arrays do not occur in GGUF files
            } else {
                r.skip(n * scalar_size(et));
            }
            break;
        }
        default: return r.ok = false;
    }
    return r.ok;
}

struct Model {
    std::vector<std::pair<std::string, Value>> kv;
    bool has_factors = false;
    std::vector<float> factors;  // rope_freqs.weight
    const Value* find(const std::string& key) const {
        for (auto& p : kv)
            if (p.first == key) return &p.second;
        return nullptr;
    }
};

thread_local std::string g_gguf_error;

int fail(const std::string& msg) {
    g_gguf_error = msg;
    return 1;
}

int load(const char* path, Model* m) {
    Reader r;
    r.f = fopen(path, "rb");
    if (!r.f) return fail(std::string("cannot open ") + path);
    char magic[4];
    if (!r.read(magic, 4) || memcmp(magic, "GGUF", 4) != 0) return fail("not a GGUF file (bad magic)");
    const uint32_t version = r.get<uint32_t>();
    if (!r.ok || version < 2 || version > 3) return fail("unsupported GGUF version " + std::to_string(version));
    const uint64_t n_tensors = r.get<uint64_t>();
    const uint64_t n_kv = r.get<uint64_t>();
    if (!r.ok || n_kv > (1u << 20) || n_tensors > (1u << 24)) return fail("corrupt GGUF header");
    for (uint64_t i = 0; i < n_kv; ++i) {
        std::string key = r.str();
        const uint32_t type = r.get<uint32_t>();
        Value v;
        if (!r.ok || !read_value(r, type, &v)) return fail("corrupt GGUF metadata at key " + key);
        m->kv.emplace_back(std::move(key), std::move(v));
    }
    // tensor infos: the rope_freqs tensor, if any
    uint64_t rf_offset = 0, rf_elems = 0;
    uint32_t rf_type = 0;
    bool rf = false;
    for (uint64_t i = 0; i < n_tensors; ++i) {
        const std::string name = r.str();
        const uint32_t nd = r.get<uint32_t>();
        if (!r.ok || nd > 8) return fail("corrupt GGUF tensor info");
        uint64_t elems = 1;
        for (uint32_t d = 0; d < nd; ++d) elems *= r.get<uint64_t>();
        const uint32_t type = r.get<uint32_t>();
        const uint64_t off = r.get<uint64_t>();
        if (!r.ok) return fail("corrupt GGUF tensor info");
        if (name == "rope_freqs.weight") {
            rf = true;
            rf_offset = off;
            rf_elems = elems;
            rf_type = type;
        }
    }
    if (rf) {
        if (rf_type != 0 /* GGML F32 */ || rf_elems == 0 || rf_elems > 4096)
            return fail("rope_freqs.weight must be an F32 vector of head_dim/2 divisors");
        uint64_t align = 32;
        if (const Value* a = m->find("general.alignment"))
            if (a->is_num() && a->num >= 1) align = (uint64_t)a->num;
        const long here = ftell(r.f);
        if (here < 0) return fail("cannot seek in GGUF file");
        const uint64_t data = ((uint64_t)here + align - 1) / align * align;
        if (fseek(r.f, (long)(data + rf_offset), SEEK_SET) != 0) return fail("cannot seek to rope_freqs.weight");
        m->factors.resize(rf_elems);
        if (!r.read(m->factors.data(), rf_elems * sizeof(float))) return fail("truncated rope_freqs.weight");
        m->has_factors = true;
    }
    return 0;
}

double num_or(const Model& m, const std::string& key, double dflt) {
    const Value* v = m.find(key);
    return v && v->is_num() ? v->num : dflt;
}

}  // namespace

extern "C" const char* fb_gguf_last_error(void) { return g_gguf_error.c_str(); }

namespace {

void params_of(const Model& m, fb_rope_params* out) {
    memset(out, 0, sizeof *out);
    const Value* arch = m.find("general.architecture");
    const std::string a = arch && arch->type == T_STRING ? arch->s : "llama";
    out->theta = num_or(m, a + ".rope.freq_base", 500000.0);
    out->head_dim = (int32_t)num_or(m, a + ".rope.dimension_count", 0.0);
    out->factor = num_or(m, a + ".rope.scaling.factor", 1.0);
    out->original_context = num_or(m, a + ".rope.scaling.original_context_length", 8192.0);
    out->low_freq_factor = num_or(m, a + ".rope.scaling.low_freq_factor", 1.0);
    out->high_freq_factor = num_or(m, a + ".rope.scaling.high_freq_factor", 4.0);
    out->num_freq_factors = m.has_factors ? (int32_t)m.factors.size() : 0;
    const Value* t = m.find(a + ".rope.scaling.type");
    const std::string type = t && t->type == T_STRING ? t->s : "";
    if (m.has_factors) out->scaling = FB_ROPE_SCALING_FACTORS;
    else if (type == "llama3") out->scaling = FB_ROPE_SCALING_LLAMA3;
    else if (type == "linear" && out->factor > 0.0 && out->factor != 1.0) out->scaling = FB_ROPE_SCALING_LINEAR;
    else out->scaling = FB_ROPE_SCALING_NONE;
}

}  // namespace

extern "C" int fb_gguf_rope_params(const char* path, fb_rope_params* out) {
    if (!path || !out) return fail("null argument");
    Model m;
    if (load(path, &m)) return 1;
    params_of(m, out);
    return 0;
}

extern "C" int fb_rope_freqs_from_gguf(const char* path, int head_dim, float* out) {
    if (!path || !out || head_dim <= 0 || (head_dim & 1)) return fail("invalid arguments");
    Model m;
    if (load(path, &m)) return 1;
    fb_rope_params p;
    params_of(m, &p);
    const int half = head_dim / 2;
    switch (p.scaling) {
        case FB_ROPE_SCALING_FACTORS:
            if ((int)m.factors.size() != half) return fail("rope_freqs.weight has " + std::to_string(m.factors.size()) +
                                                            " entries, head_dim/2 is " + std::to_string(half));
            if (fb_rope_freqs(head_dim, p.theta, out)) return fail("invalid rope.freq_base");
            for (int i = 0; i < half; ++i) {
                if (!(m.factors[i] > 0.0f)) return fail("rope_freqs.weight holds a non-positive divisor");
                out[i] = out[i] / m.factors[i];
            }
            return 0;
        case FB_ROPE_SCALING_LLAMA3:
            if (fb_rope_freqs_llama3(head_dim, p.theta, p.factor, p.low_freq_factor, p.high_freq_factor,
                                     p.original_context, out))
                return fail("invalid llama3 rope scaling parameters");
            return 0;
        case FB_ROPE_SCALING_LINEAR:
            if (fb_rope_freqs(head_dim, p.theta, out)) return fail("invalid rope.freq_base");
            for (int i = 0; i < half; ++i) out[i] = (float)((double)out[i] / p.factor);
            return 0;
        default:
            if (fb_rope_freqs(head_dim, p.theta, out)) return fail("invalid rope.freq_base");
            return 0;
    }
}
