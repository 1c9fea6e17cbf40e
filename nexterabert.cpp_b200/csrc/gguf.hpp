// GGUF reader of libnexterabert.so (host side).
//
// Parses the published GGUF layout (v2 / v3): header, typed key/value pairs,
// tensor records, aligned data section.  Replaces the ggml gguf reader the
// reference loads with (src/nexterabert.cpp:1555-1557, :1682-1693).
#pragma once

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace nxg {

enum vtype : uint32_t { U8 = 0, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 };

struct Value {
    uint32_t type = 0;
    uint32_t arr_type = 0;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0.0;
    std::string s;
    std::vector<std::string> arr_s;
    uint64_t arr_n = 0;
};

struct TensorInfo {
    std::string name;
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    int type = 0;
    uint64_t offset = 0;
    size_t nbytes = 0;
};

// (block size, bytes per block) of a ggml type id; 0 when unknown
inline int64_t blck_size(int t) {
    switch (t) {
        case 0: case 1: case 24: case 25: case 26: case 27: case 28: case 30: return 1;
        case 2: case 3: case 6: case 7: case 8: case 9: return 32;
        case 10: case 11: case 12: case 13: case 14: case 15: return 256;
        default: return 0;
    }
}
inline size_t type_size(int t) {
    switch (t) {
        case 0: return 4; case 1: return 2; case 2: return 18; case 3: return 20; case 6: return 22;
        case 7: return 24; case 8: return 34; case 9: return 36; case 10: return 84; case 11: return 110;
        case 12: return 144; case 13: return 176; case 14: return 210; case 15: return 292;
        case 24: return 1; case 25: return 2; case 26: return 4; case 27: return 8; case 28: return 8; case 30: return 2;
        default: return 0;
    }
}
inline size_t row_size(int t, int64_t ne0) {
    const int64_t bs = blck_size(t);
    return bs > 0 ? (size_t) (ne0 / bs) * type_size(t) : 0;
}
inline bool is_quantized(int t) { return (t >= 2 && t <= 9 && t != 4 && t != 5) || (t >= 10 && t <= 15); }

class File {
public:
    std::unordered_map<std::string, Value> kv;
    std::vector<TensorInfo> tensors;
    uint64_t data_offset = 0;
    std::string error;

    bool open(const char * path) {
        FILE * f = fopen(path, "rb");
        if (!f) { error = "cannot open file"; return false; }
        fp_ = f;
        bool ok = parse();
        fclose(f);
        fp_ = nullptr;
        return ok;
    }

    const Value * get(const char * key) const {
        auto it = kv.find(key);
        return it == kv.end() ? nullptr : &it->second;
    }
    uint32_t u32(const char * key, uint32_t def) const {
        const Value * v = get(key);
        return v ? (uint32_t) v->u : def;
    }
    float f32(const char * key, float def) const {
        const Value * v = get(key);
        return v ? (float) v->f : def;
    }
    std::string str(const char * key, const char * def) const {
        const Value * v = get(key);
        return v && v->type == STR ? v->s : std::string(def);
    }

private:
    FILE * fp_ = nullptr;
    bool ok_ = true;

    void rd(void * p, size_t n) {
        if (ok_ && fread(p, 1, n, fp_) != n) ok_ = false;
    }
    uint64_t rd64() { uint64_t v = 0; rd(&v, 8); return v; }
    uint32_t rd32() { uint32_t v = 0; rd(&v, 4); return v; }
    std::string rdstr() {
        const uint64_t n = rd64();
        if (!ok_ || n > (1ull << 31)) { ok_ = false; return {}; }
        std::string s(n, '\0');
        rd(&s[0], n);
        return s;
    }
    static size_t scalar_bytes(uint32_t t) {
        switch (t) {
            case U8: case I8: case BOOL: return 1;
            case U16: case I16: return 2;
            case U32: case I32: case F32: return 4;
            case U64: case I64: case F64: return 8;
            default: return 0;
        }
    }
    void rdscalar(uint32_t t, Value & v) {
        unsigned char b[8] = {0};
        const size_t n = scalar_bytes(t);
        if (!n) { ok_ = false; return; }
        rd(b, n);
        switch (t) {
            case U8: case BOOL: v.u = b[0]; v.i = b[0]; break;
            case I8: v.i = (int8_t) b[0]; v.u = (uint64_t) v.i; break;
            case U16: { uint16_t x; memcpy(&x, b, 2); v.u = x; v.i = x; break; }
            case I16: { int16_t x; memcpy(&x, b, 2); v.i = x; v.u = (uint64_t) x; break; }
            case U32: { uint32_t x; memcpy(&x, b, 4); v.u = x; v.i = x; break; }
            case I32: { int32_t x; memcpy(&x, b, 4); v.i = x; v.u = (uint64_t) x; break; }
            case F32: { float x; memcpy(&x, b, 4); v.f = x; break; }
            case U64: { uint64_t x; memcpy(&x, b, 8); v.u = x; v.i = (int64_t) x; break; }
            case I64: { int64_t x; memcpy(&x, b, 8); v.i = x; v.u = (uint64_t) x; break; }
            case F64: { double x; memcpy(&x, b, 8); v.f = x; break; }
        }
    }

    bool parse() {
        char magic[4];
        rd(magic, 4);
        if (!ok_ || memcmp(magic, "GGUF", 4) != 0) { error = "not a GGUF file"; return false; }
        const uint32_t version = rd32();
        const uint64_t n_tensors = rd64(), n_kv = rd64();
        if (!ok_ || version < 2 || n_kv > 100000 || n_tensors > 1000000) { error = "bad GGUF header"; return false; }
        uint32_t alignment = 32;
        for (uint64_t i = 0; ok_ && i < n_kv; ++i) {
            const std::string key = rdstr();
            Value v;
            v.type = rd32();
            if (v.type == STR) {
                v.s = rdstr();
            } else if (v.type == ARR) {
                v.arr_type = rd32();
                v.arr_n = rd64();
                if (v.arr_n > (1ull << 28)) { ok_ = false; break; }
                if (v.arr_type == STR) {
                    for (uint64_t j = 0; ok_ && j < v.arr_n; ++j) v.arr_s.push_back(rdstr());
                } else {
                    const size_t es = scalar_bytes(v.arr_type);
                    if (!es) { ok_ = false; break; }
                    std::vector<unsigned char> skip(es * v.arr_n);
                    rd(skip.data(), skip.size());
                }
            } else {
                rdscalar(v.type, v);
            }
            if (key == "general.alignment" && v.type == U32) alignment = (uint32_t) v.u;
            kv[key] = std::move(v);
        }
        for (uint64_t i = 0; ok_ && i < n_tensors; ++i) {
            TensorInfo t;
            t.name = rdstr();
            t.n_dims = (int) rd32();
            if (t.n_dims < 1 || t.n_dims > 4) { ok_ = false; break; }
            for (int d = 0; d < t.n_dims; ++d) t.ne[d] = (int64_t) rd64();
            t.type = (int) rd32();
            t.offset = rd64();
            const size_t rs = row_size(t.type, t.ne[0]);
            t.nbytes = rs * (size_t) (t.ne[1] * t.ne[2] * t.ne[3]);
            tensors.push_back(std::move(t));
        }
        if (!ok_) { error = "truncated or malformed GGUF"; return false; }
        const uint64_t pos = (uint64_t) ftello(fp_);
        const uint64_t a = alignment ? alignment : 32;
        data_offset = (pos + a - 1) / a * a;
        return true;
    }
};

} // namespace nxg
