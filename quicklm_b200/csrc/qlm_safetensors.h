// qlm_safetensors.h — host-side reader of safetensors files and small JSON
// documents (internal): a depth- and size-limited JSON parser and a mapped
// file whose tensor entries are checked against the file's bounds. Used by the
// pre-quantized store (qlm_store.cu) and the model loader (qlm_model.cu).
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/qlm_b200.h"

namespace qlm_st {

constexpr uint64_t kMaxHeader = 100u << 20;  // safetensors' own header limit
constexpr int kMaxDepth = 16;

// ---- a small JSON reader for the safetensors header ----------------------
struct JValue {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    double num = 0;
    std::string str;
    std::vector<JValue> arr;
    std::map<std::string, JValue> obj;
};

struct JParser {
    const char* p;
    const char* end;
    std::string err;

    void ws() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool fail(const char* what) {
        if (err.empty()) err = what;
        return false;
    }
    bool str(std::string& out) {
        if (p >= end || *p != '"') return fail("expected a string");
        ++p;
        while (p < end && *p != '"') {
            char c = *p++;
            if (c == '\\') {
                if (p >= end) return fail("truncated escape");
                const char e = *p++;
                switch (e) {
                    case '"': case '\\': case '/': out.push_back(e); break;
                    case 'b': out.push_back('\b'); break;
                    case 'f': out.push_back('\f'); break;
                    case 'n': out.push_back('\n'); break;
                    case 'r': out.push_back('\r'); break;
                    case 't': out.push_back('\t'); break;
                    case 'u': {
                        if (end - p < 4) return fail("truncated \\u escape");
                        unsigned v = 0;
                        for (int i = 0; i < 4; ++i) {
                            const char h = *p++;
                            v <<= 4;
                            if (h >= '0' && h <= '9') v |= (unsigned)(h - '0');
                            else if (h >= 'a' && h <= 'f') v |= (unsigned)(h - 'a' + 10);
                            else if (h >= 'A' && h <= 'F') v |= (unsigned)(h - 'A' + 10);
                            else return fail("bad \\u escape");
                        }
                        // Names are ASCII in practice; other code points are kept as UTF-8.
                        if (v < 0x80) {
                            out.push_back((char)v);
                        } else if (v < 0x800) {
                            out.push_back((char)(0xC0 | (v >> 6)));
                            out.push_back((char)(0x80 | (v & 0x3F)));
                        } else {
                            out.push_back((char)(0xE0 | (v >> 12)));
                            out.push_back((char)(0x80 | ((v >> 6) & 0x3F)));
                            out.push_back((char)(0x80 | (v & 0x3F)));
                        }
                        break;
                    }
                    default: return fail("bad escape");
                }
            } else {
                out.push_back(c);
            }
        }
        if (p >= end) return fail("unterminated string");
        ++p;
        return true;
    }
    bool value(JValue& v, int depth) {
        if (depth > kMaxDepth) return fail("header nested too deeply");
        ws();
        if (p >= end) return fail("truncated header");
        const char c = *p;
        if (c == '{') {
            v.kind = JValue::Obj;
            ++p;
            ws();
            if (p < end && *p == '}') { ++p; return true; }
            for (;;) {
                ws();
                std::string key;
                if (!str(key)) return false;
                ws();
                if (p >= end || *p != ':') return fail("expected ':'");
                ++p;
                JValue item;
                if (!value(item, depth + 1)) return false;
                v.obj[key] = std::move(item);
                ws();
                if (p < end && *p == ',') { ++p; continue; }
                if (p < end && *p == '}') { ++p; return true; }
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.kind = JValue::Arr;
            ++p;
            ws();
            if (p < end && *p == ']') { ++p; return true; }
            for (;;) {
                JValue item;
                if (!value(item, depth + 1)) return false;
                v.arr.push_back(std::move(item));
                ws();
                if (p < end && *p == ',') { ++p; continue; }
                if (p < end && *p == ']') { ++p; return true; }
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = JValue::Str;
            return str(v.str);
        }
        if (c == '-' || (c >= '0' && c <= '9')) {
            // Shapes and offsets are non-negative integers: read the digits exactly;
            // anything else reads as -1, which every such use rejects. The
            // literal is kept in `str` for readers of other numbers.
            const char* start = p;
            const bool neg = c == '-';
            if (neg) ++p;
            if (p >= end || *p < '0' || *p > '9') return fail("bad number");
            double x = 0;
            while (p < end && *p >= '0' && *p <= '9') x = x * 10 + (*p++ - '0');
            bool integral = !neg;
            if (p < end && (*p == '.' || *p == 'e' || *p == 'E')) {
                integral = false;
                ++p;
                while (p < end && ((*p >= '0' && *p <= '9') || *p == '+' || *p == '-' || *p == 'e' || *p == 'E')) ++p;
            }
            v.kind = JValue::Num;
            v.num = integral ? x : -1.0;
            v.str.assign(start, p);  // the literal, for readers of non-integers
            return true;
        }
        auto word = [&](const char* w, JValue::Kind k) {
            const size_t n = std::strlen(w);
            if ((size_t)(end - p) < n || std::strncmp(p, w, n) != 0) return fail("bad literal");
            p += n;
            v.kind = k;
            return true;
        };
        if (c == 't') return word("true", JValue::Bool);
        if (c == 'f') return word("false", JValue::Bool);
        if (c == 'n') return word("null", JValue::Null);
        return fail("unexpected character");
    }
};

// ---- the mapped file --------------------------------------------------------
struct Mapped {
    int fd = -1;
    void* base = MAP_FAILED;
    size_t size = 0;
    ~Mapped() {
        if (base != MAP_FAILED) munmap(base, size);
        if (fd >= 0) close(fd);
    }
};

struct TensorRef {
    std::string dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;  // absolute byte offsets in the file
};

struct Store {
    Mapped m;
    uint64_t data0 = 0;  // first byte after the header
    std::map<std::string, TensorRef> tensors;
    std::map<std::string, std::string> meta;
};

inline int open_store(const char* path, Store& st, std::string& err) {
    auto bad = [&](const char* fmt, auto... args) {
        char buf[512];
        std::snprintf(buf, sizeof buf, fmt, args...);
        err = buf;
        return QLM_ERR_INVALID_ARG;
    };
    if (!path) return bad("%s", "path is NULL");
    st.m.fd = open(path, O_RDONLY);
    if (st.m.fd < 0) return bad("cannot open %s: %s", path, std::strerror(errno));
    struct stat sb;
    if (fstat(st.m.fd, &sb) != 0) return bad("cannot stat %s", path);
    st.m.size = (size_t)sb.st_size;
    if (st.m.size < 8) return bad("%s: file too small for a safetensors header", path);
    st.m.base = mmap(nullptr, st.m.size, PROT_READ, MAP_PRIVATE, st.m.fd, 0);
    if (st.m.base == MAP_FAILED) return bad("cannot map %s", path);
    const uint8_t* b = static_cast<const uint8_t*>(st.m.base);
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | b[i];
    if (hlen > kMaxHeader || hlen > st.m.size - 8)
        return bad("%s: header length %llu out of bounds", path, (unsigned long long)hlen);
    st.data0 = 8 + hlen;
    JParser jp{reinterpret_cast<const char*>(b + 8), reinterpret_cast<const char*>(b + 8 + hlen), {}};
    JValue root;
    if (!jp.value(root, 0)) return bad("%s: bad header (%s)", path, jp.err.c_str());
    if (root.kind != JValue::Obj) return bad("%s: header is not an object", path);
    for (auto& kv : root.obj) {
        if (kv.first == "__metadata__") {
            if (kv.second.kind != JValue::Obj) return bad("%s: bad __metadata__", path);
            for (auto& mv : kv.second.obj)
                if (mv.second.kind == JValue::Str) st.meta[mv.first] = mv.second.str;
            continue;
        }
        const JValue& t = kv.second;
        auto dt = t.obj.find("dtype");
        auto sh = t.obj.find("shape");
        auto off = t.obj.find("data_offsets");
        if (t.kind != JValue::Obj || dt == t.obj.end() || sh == t.obj.end() || off == t.obj.end() ||
            dt->second.kind != JValue::Str || sh->second.kind != JValue::Arr || off->second.kind != JValue::Arr ||
            off->second.arr.size() != 2)
            return bad("%s: malformed entry '%s'", path, kv.first.c_str());
        TensorRef r;
        r.dtype = dt->second.str;
        for (const JValue& d : sh->second.arr) {
            if (d.kind != JValue::Num || d.num < 0 || d.num > 9.0e15)
                return bad("%s: bad shape of '%s'", path, kv.first.c_str());
            r.shape.push_back((int64_t)d.num);
        }
        const JValue& o0 = off->second.arr[0];
        const JValue& o1 = off->second.arr[1];
        if (o0.kind != JValue::Num || o1.kind != JValue::Num || o0.num < 0 || o1.num < o0.num || o1.num > 9.0e15)
            return bad("%s: bad data_offsets of '%s'", path, kv.first.c_str());
        r.begin = st.data0 + (uint64_t)o0.num;
        r.end = st.data0 + (uint64_t)o1.num;
        if (r.end > st.m.size)
            return bad("%s: '%s' goes out of the file's bounds", path, kv.first.c_str());
        st.tensors[kv.first] = std::move(r);
    }
    return QLM_OK;
}

}  // namespace qlm_st
