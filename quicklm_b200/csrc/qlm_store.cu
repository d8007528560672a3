// qlm_store.cu — pre-quantized weights on disk (host code).
//
// QuickLM's loader accepts only F32 and BF16 safetensors (src/io/
// safetensors.cpp:524-527) and quantizes every matmul weight at load
// (get_tensor_keep_int8 :517-585, get_tensor_keep_int4 :587-656). This file
// stores the quantized result instead, as a standard safetensors file:
//
//   <name>          codes in the reference Tensor's layout: dtype "I8", shape
//                   [rows, K] (int8), or dtype "U8", shape [rows, (K+1)/2]
//                   (int4: value + 8, low nibble = even column)
//   <name>.qscale   dtype "F32", shape [rows, ceil(K/32)]: the block scales
//   __metadata__    "qlm.<name>": "int8 k=<K>" or "int4 k=<K>"
//
// so a load maps the file and moves the bytes to the device (qlm_weight_import_*:
// a staged copy and a repack kernel), skipping quantization. The header is
// parsed with the bounds checks the reference loader applies (offsets inside
// the file, sizes equal to shape x element size).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "qlm_b200.h"
#include "qlm_handle.h"
#include "qlm_safetensors.h"

namespace qlm_internal {
void set_last_error(const std::string& msg);
}

namespace {

int set_err(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    qlm_internal::set_last_error(buf);
    return code;
}

using namespace qlm_st;

int open_store(const char* path, Store& st) {
    std::string err;
    const int rc = qlm_st::open_store(path, st, err);
    if (rc) return set_err(rc, "%s", err.c_str());
    return QLM_OK;
}

// The codes and scales of weight `name`, checked against each other.
struct WeightRef {
    const TensorRef* codes;
    const TensorRef* scales;
    int bits;
    int64_t rows, k;
};

int find_weight(const Store& st, const char* path, const char* name, WeightRef& w) {
    if (!name) return set_err(QLM_ERR_INVALID_ARG, "name is NULL");
    auto mi = st.meta.find(std::string("qlm.") + name);
    auto ci = st.tensors.find(name);
    auto si = st.tensors.find(std::string(name) + ".qscale");
    if (mi == st.meta.end() || ci == st.tensors.end() || si == st.tensors.end())
        return set_err(QLM_ERR_INVALID_ARG, "%s: no quantized weight '%s'", path, name);
    char kind[8] = {0};
    long long k = -1;
    if (std::sscanf(mi->second.c_str(), "%7s k=%lld", kind, &k) != 2 || k <= 0 || k > 0x7fffffff)
        return set_err(QLM_ERR_INVALID_ARG, "%s: bad metadata for '%s'", path, name);
    w.bits = std::strcmp(kind, "int8") == 0 ? 8 : std::strcmp(kind, "int4") == 0 ? 4 : 0;
    if (!w.bits) return set_err(QLM_ERR_INVALID_ARG, "%s: unknown code kind '%s' for '%s'", path, kind, name);
    const TensorRef& c = ci->second;
    const TensorRef& s = si->second;
    const int64_t code_row = w.bits == 8 ? k : (k + 1) / 2;
    const int64_t nb = (k + QLM_BLOCK - 1) / QLM_BLOCK;
    if (c.dtype != (w.bits == 8 ? "I8" : "U8") || c.shape.size() != 2 || c.shape[1] != code_row)
        return set_err(QLM_ERR_INVALID_ARG, "%s: '%s' is not %s [rows, %lld]", path, name, w.bits == 8 ? "I8" : "U8",
                       (long long)code_row);
    if (c.shape[0] <= 0 || c.shape[0] > 0x7fffffff)
        return set_err(QLM_ERR_INVALID_ARG, "%s: '%s' has %lld rows", path, name, (long long)c.shape[0]);
    if (s.dtype != "F32" || s.shape.size() != 2 || s.shape[0] != c.shape[0] || s.shape[1] != nb)
        return set_err(QLM_ERR_INVALID_ARG, "%s: '%s.qscale' is not F32 [%lld, %lld]", path, name,
                       (long long)c.shape[0], (long long)nb);
    if (c.end - c.begin != (uint64_t)(c.shape[0] * code_row) || s.end - s.begin != (uint64_t)(s.shape[0] * nb * 4))
        return set_err(QLM_ERR_INVALID_ARG, "%s: byte ranges of '%s' do not match their shapes", path, name);
    w.codes = &c;
    w.scales = &s;
    w.rows = c.shape[0];
    w.k = k;
    return QLM_OK;
}

void json_string(std::string& out, const std::string& s) {
    out.push_back('"');
    for (unsigned char c : s) {
        if (c == '"' || c == '\\') {
            out.push_back('\\');
            out.push_back((char)c);
        } else if (c < 0x20) {
            char buf[8];
            std::snprintf(buf, sizeof buf, "\\u%04x", c);
            out += buf;
        } else {
            out.push_back((char)c);
        }
    }
    out.push_back('"');
}

}  // namespace

extern "C" {

int qlm_store_info(const char* path, const char* name, int* bits, int64_t* rows, int64_t* k) {
    Store st;
    int rc = open_store(path, st);
    if (rc) return rc;
    WeightRef w;
    if ((rc = find_weight(st, path, name, w))) return rc;
    if (bits) *bits = w.bits;
    if (rows) *rows = w.rows;
    if (k) *k = w.k;
    return QLM_OK;
}

int qlm_store_load(const char* path, const char* name, int row_begin, int row_end, int device, void* stream,
                   qlm_w8** out) {
    if (!out) return set_err(QLM_ERR_INVALID_ARG, "out is NULL");
    *out = nullptr;
    Store st;
    int rc = open_store(path, st);
    if (rc) return rc;
    WeightRef w;
    if ((rc = find_weight(st, path, name, w))) return rc;
    if (row_end < 0) row_end = (int)w.rows;
    const uint8_t* base = static_cast<const uint8_t*>(st.m.base);
    const float* scales = reinterpret_cast<const float*>(base + w.scales->begin);
    if (reinterpret_cast<uintptr_t>(scales) % alignof(float) != 0)
        return set_err(QLM_ERR_INVALID_ARG, "%s: '%s.qscale' is not 4-byte aligned in the file", path, name);
    if (w.bits == 8)
        return qlm_weight_import_int8(reinterpret_cast<const int8_t*>(base + w.codes->begin), scales, (int)w.rows,
                                      (int)w.k, row_begin, row_end, device, stream, out);
    return qlm_weight_import_int4(base + w.codes->begin, scales, (int)w.rows, (int)w.k, row_begin, row_end, device,
                                  stream, out);
}

int qlm_store_save(const char* path, int n, const char* const* names, const qlm_w8* const* weights) {
    if (!path || n <= 0 || !names || !weights) return set_err(QLM_ERR_INVALID_ARG, "bad arguments");
    struct Item {
        std::string name;
        std::vector<uint8_t> codes;
        std::vector<float> scales;
        int bits, rows, k;
    };
    std::vector<Item> items((size_t)n);
    for (int i = 0; i < n; ++i) {
        const qlm_w8* w = weights[i];
        if (!w || !names[i] || !names[i][0]) return set_err(QLM_ERR_INVALID_ARG, "weight %d: NULL handle or name", i);
        Item& it = items[(size_t)i];
        it.name = names[i];
        it.bits = w->bits;
        it.rows = w->rows;
        it.k = w->k;
        const size_t code_row = w->bits == 8 ? (size_t)w->k : (size_t)(w->k + 1) / 2;
        const size_t nb = (size_t)(w->k + QLM_BLOCK - 1) / QLM_BLOCK;
        try {
            it.codes.resize((size_t)w->rows * code_row);
            it.scales.resize((size_t)w->rows * nb);
        } catch (...) {
            return set_err(QLM_ERR_OUT_OF_MEMORY, "host staging allocation failed");
        }
        const int rc = w->bits == 8
                           ? qlm_weight_export_int8(w, reinterpret_cast<int8_t*>(it.codes.data()), it.scales.data())
                           : qlm_weight_export_int4(w, it.codes.data(), it.scales.data());
        if (rc) return rc;
        for (int j = 0; j < i; ++j)
            if (items[(size_t)j].name == it.name) return set_err(QLM_ERR_INVALID_ARG, "duplicate name '%s'", names[i]);
    }
    // Byte buffer without holes (as safetensors requires): every weight's
    // scales first (4-byte multiples, so they stay 4-aligned after the
    // 8-aligned header), then every weight's codes.
    std::string h = "{\"__metadata__\":{\"qlm.format\":\"1\"";
    for (const Item& it : items) {
        h += ",";
        json_string(h, "qlm." + it.name);
        h += ":";
        json_string(h, std::string(it.bits == 8 ? "int8" : "int4") + " k=" + std::to_string(it.k));
    }
    h += "}";
    uint64_t off = 0;
    for (const Item& it : items) {
        const uint64_t sb = it.scales.size() * 4;
        h += ",";
        json_string(h, it.name + ".qscale");
        h += ":{\"dtype\":\"F32\",\"shape\":[" + std::to_string(it.rows) + "," +
             std::to_string(it.scales.size() / (size_t)it.rows) + "],\"data_offsets\":[" + std::to_string(off) + "," +
             std::to_string(off + sb) + "]}";
        off += sb;
    }
    for (const Item& it : items) {
        const uint64_t cb = it.codes.size();
        h += ",";
        json_string(h, it.name);
        h += ":{\"dtype\":\"" + std::string(it.bits == 8 ? "I8" : "U8") + "\",\"shape\":[" + std::to_string(it.rows) +
             "," + std::to_string(cb / (uint64_t)it.rows) + "],\"data_offsets\":[" + std::to_string(off) + "," +
             std::to_string(off + cb) + "]}";
        off += cb;
    }
    h += "}";
    while ((8 + h.size()) % 8) h.push_back(' ');  // data starts 8-aligned
    FILE* f = std::fopen(path, "wb");
    if (!f) return set_err(QLM_ERR_INVALID_ARG, "cannot create %s: %s", path, std::strerror(errno));
    uint8_t len[8];
    for (int i = 0; i < 8; ++i) len[i] = (uint8_t)((uint64_t)h.size() >> (8 * i));
    bool ok = std::fwrite(len, 1, 8, f) == 8 && std::fwrite(h.data(), 1, h.size(), f) == h.size();
    for (size_t i = 0; ok && i < items.size(); ++i)
        ok = std::fwrite(items[i].scales.data(), 4, items[i].scales.size(), f) == items[i].scales.size();
    for (size_t i = 0; ok && i < items.size(); ++i)
        ok = std::fwrite(items[i].codes.data(), 1, items[i].codes.size(), f) == items[i].codes.size();
    if (std::fclose(f) != 0) ok = false;
    if (!ok) return set_err(QLM_ERR_INVALID_ARG, "write to %s failed", path);
    return QLM_OK;
}

}  // extern "C"
