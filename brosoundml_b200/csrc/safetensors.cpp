// safetensors reading (the file format the reference loads its converted Kokoro
// checkpoint from, src/kokoro_modules.cpp:99-125): an 8-byte little-endian
// header length, a JSON header {name: {dtype, shape, data_offsets}, __metadata__:
// {...}}, then the raw little-endian data. Host-side IO: tensors are read into
// host memory as fp32 (F32 / F16 / BF16 / F64 sources).
#include "safetensors.h"

#include <cmath>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace bsml {

namespace {

// A minimal JSON reader for the header: objects, arrays, strings, numbers,
// true / false / null. Only what the header needs is kept.
struct Json {
    const std::string& s;
    size_t i = 0;
    std::string where;

    [[noreturn]] void bad(const std::string& why) { fail(where.c_str(), "bad header: " + why); }
    void ws() {
        while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
    }
    void expect(char c) {
        ws();
        if (i >= s.size() || s[i] != c) bad(std::string("expected '") + c + "'");
        ++i;
    }
    bool peek(char c) {
        ws();
        return i < s.size() && s[i] == c;
    }
    std::string str() {
        expect('"');
        std::string out;
        while (i < s.size() && s[i] != '"') {
            char c = s[i++];
            if (c == '\\') {
                if (i >= s.size()) bad("truncated escape");
                const char e = s[i++];
                switch (e) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {
                        if (i + 4 > s.size()) bad("truncated \\u escape");
                        const unsigned cp = (unsigned)std::stoul(s.substr(i, 4), nullptr, 16);
                        i += 4;
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
                    default: out += e;
                }
            } else {
                out += c;
            }
        }
        if (i >= s.size()) bad("unterminated string");
        ++i;
        return out;
    }
    int64_t integer() {
        ws();
        size_t j = i;
        if (j < s.size() && s[j] == '-') ++j;
        while (j < s.size() && s[j] >= '0' && s[j] <= '9') ++j;
        if (j == i) bad("expected an integer");
        const int64_t v = std::stoll(s.substr(i, j - i));
        i = j;
        return v;
    }
    void skip() {   // any value
        ws();
        if (i >= s.size()) bad("truncated");
        const char c = s[i];
        if (c == '"') {
            str();
        } else if (c == '{') {
            ++i;
            if (peek('}')) { ++i; return; }
            for (;;) {
                str();
                expect(':');
                skip();
                if (peek(',')) { ++i; continue; }
                expect('}');
                return;
            }
        } else if (c == '[') {
            ++i;
            if (peek(']')) { ++i; return; }
            for (;;) {
                skip();
                if (peek(',')) { ++i; continue; }
                expect(']');
                return;
            }
        } else {
            while (i < s.size() && s[i] != ',' && s[i] != '}' && s[i] != ']') ++i;
        }
    }
};

int dtype_code(const std::string& d) {
    if (d == "F32") return ST_F32;
    if (d == "F16") return ST_F16;
    if (d == "BF16") return ST_BF16;
    if (d == "F64") return ST_F64;
    return ST_OTHER;
}

int dtype_size(int code) {
    switch (code) {
        case ST_F32: return 4;
        case ST_F16: return 2;
        case ST_BF16: return 2;
        case ST_F64: return 8;
        default: return 0;
    }
}

float half_to_float(uint16_t h) {
    const int s = (h >> 15) & 1, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    float v;
    if (e == 0) v = std::ldexp((float)m, -24);
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = std::ldexp((float)(m | 0x400), e - 25);
    return s ? -v : v;
}

}  // namespace

SafeTensors::SafeTensors(const std::string& path) : path_(path) {
    const char* where = "safetensors";
    f_ = std::fopen(path.c_str(), "rb");
    if (!f_) fail(where, "cannot open " + path);
    uint8_t hb[8];
    if (std::fread(hb, 1, 8, f_) != 8) fail(where, "truncated file " + path);
    uint64_t n = 0;
    for (int k = 7; k >= 0; --k) n = (n << 8) | hb[k];
    std::fseek(f_, 0, SEEK_END);
    const int64_t size = std::ftell(f_);
    if (n == 0 || (int64_t)n > size - 8) fail(where, "header length out of range in " + path);
    std::string h(n, '\0');
    std::fseek(f_, 8, SEEK_SET);
    if (std::fread(&h[0], 1, n, f_) != n) fail(where, "truncated header in " + path);
    data0_ = 8 + (int64_t)n;
    const int64_t data_size = size - data0_;
    Json js{h};
    js.where = where;
    js.expect('{');
    if (js.peek('}')) return;
    for (;;) {
        const std::string key = js.str();
        js.expect(':');
        if (key == "__metadata__") {
            js.expect('{');
            if (!js.peek('}')) {
                for (;;) {
                    const std::string k = js.str();
                    js.expect(':');
                    if (js.peek('"')) meta_[k] = js.str();
                    else js.skip();
                    if (js.peek(',')) { ++js.i; continue; }
                    break;
                }
            }
            js.expect('}');
        } else {
            Entry e;
            e.name = key;
            bool have_off = false;
            js.expect('{');
            for (;;) {
                const std::string f = js.str();
                js.expect(':');
                if (f == "dtype") {
                    e.dtype = dtype_code(js.str());
                } else if (f == "shape") {
                    js.expect('[');
                    if (!js.peek(']')) {
                        for (;;) {
                            e.shape.push_back(js.integer());
                            if (js.peek(',')) { ++js.i; continue; }
                            break;
                        }
                    }
                    js.expect(']');
                } else if (f == "data_offsets") {
                    js.expect('[');
                    e.begin = js.integer();
                    js.expect(',');
                    e.end = js.integer();
                    js.expect(']');
                    have_off = true;
                } else {
                    js.skip();
                }
                if (js.peek(',')) { ++js.i; continue; }
                break;
            }
            js.expect('}');
            if (!have_off) fail(where, "tensor '" + key + "' has no data_offsets");
            e.numel = 1;
            for (int64_t d : e.shape) e.numel *= d;
            const int es = dtype_size(e.dtype);
            if (e.begin < 0 || e.end < e.begin || e.end > data_size)
                fail(where, "tensor '" + key + "' data out of range");
            if (es && e.end - e.begin != e.numel * es)
                fail(where, "tensor '" + key + "' byte size does not match its shape");
            index_[key] = (int)entries_.size();
            entries_.push_back(std::move(e));
        }
        if (js.peek(',')) { ++js.i; continue; }
        js.expect('}');
        break;
    }
}

SafeTensors::~SafeTensors() {
    if (f_) std::fclose(f_);
}

const SafeTensors::Entry* SafeTensors::find(const std::string& name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &entries_[it->second];
}

void SafeTensors::read_f32(const Entry& e, float* dst) const {
    const int es = dtype_size(e.dtype);
    if (!es) fail("safetensors", "tensor '" + e.name + "' has a dtype other than F32/F16/BF16/F64");
    std::vector<uint8_t> raw((size_t)(e.end - e.begin));
    std::fseek(f_, (long)(data0_ + e.begin), SEEK_SET);
    if (!raw.empty() && std::fread(raw.data(), 1, raw.size(), f_) != raw.size())
        fail("safetensors", "truncated data of '" + e.name + "'");
    for (int64_t i = 0; i < e.numel; ++i) {
        const uint8_t* p = raw.data() + i * es;
        switch (e.dtype) {
            case ST_F32: std::memcpy(&dst[i], p, 4); break;
            case ST_F64: { double v; std::memcpy(&v, p, 8); dst[i] = (float)v; break; }
            case ST_F16: { uint16_t h; std::memcpy(&h, p, 2); dst[i] = half_to_float(h); break; }
            case ST_BF16: {
                uint16_t h;
                std::memcpy(&h, p, 2);
                const uint32_t u = (uint32_t)h << 16;
                std::memcpy(&dst[i], &u, 4);
                break;
            }
            default: break;
        }
    }
}

// Parameters by table: key = prefix + name. A weight stored under PyTorch's
// weight-norm parameterisation (name_g = ...weight_g, ...weight_v) is fused as
// weight = g * v / ||v||, the norm over every axis but the first
// (torch.nn.utils.weight_norm dim 0), as the reference's converter does
// (scripts/convert-kokoro.py:71-110).
void SafeTensors::load_params(const bsml_param_entry* table, int n_entries, const std::string& prefix, float* params,
                              int64_t n_params) const {
    const char* where = "bsml_params_from_safetensors";
    for (int t = 0; t < n_entries; ++t) {
        const bsml_param_entry& pe = table[t];
        if (pe.offset < 0 || pe.offset + pe.numel > n_params) fail(where, "table entry outside the parameter vector");
        const std::string key = prefix + pe.name;
        float* dst = params + pe.offset;
        if (const Entry* e = find(key)) {
            if (e->numel != pe.numel)
                fail(where, "tensor '" + key + "' has " + std::to_string(e->numel) + " elements; expected " +
                                std::to_string(pe.numel));
            read_f32(*e, dst);
            continue;
        }
        const std::string nm(pe.name);
        const size_t dot = nm.rfind(".weight");
        const Entry* g = nullptr;
        const Entry* v = nullptr;
        if (dot != std::string::npos && dot + 7 == nm.size()) {
            g = find(prefix + nm + "_g");
            v = find(prefix + nm + "_v");
        }
        if (!g || !v) fail(where, "missing safetensors key '" + key + "'");
        if (v->numel != pe.numel) fail(where, "tensor '" + key + "_v' has the wrong element count");
        const int64_t rows = pe.shape[0];
        if (rows <= 0 || g->numel != rows || pe.numel % rows != 0)
            fail(where, "tensor '" + key + "_g' does not match the weight's first axis");
        std::vector<float> gv(rows);
        read_f32(*g, gv.data());
        read_f32(*v, dst);
        const int64_t per = pe.numel / rows;
        for (int64_t r = 0; r < rows; ++r) {
            double ss = 0.0;
            for (int64_t j = 0; j < per; ++j) ss += (double)dst[r * per + j] * dst[r * per + j];
            const double scale = gv[r] / std::max(std::sqrt(ss), 1e-12);
            for (int64_t j = 0; j < per; ++j) dst[r * per + j] = (float)(dst[r * per + j] * scale);
        }
    }
}

}  // namespace bsml
