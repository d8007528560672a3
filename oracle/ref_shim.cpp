// TEST INFRASTRUCTURE ONLY — the parity checker, never the product path.
//
// extern "C" entry points over QuickLM's OWN int8 path, compiled from the
// reference sources (src/ops/math_ops.cpp, src/io/safetensors.cpp) by
// oracle/Makefile into oracle/_ref/libqlm_refcpu.so. Only tests/, the smoke
// check and bench.py's CPU-baseline / reference arm load this library.
//
// What each entry point drives in the reference:
//   qlmref_quantize     -> SafetensorsLoader::open + get_tensor_keep_int8
//                          (io/safetensors.cpp:121-189, 517-585), which runs
//                          st_quantize_row_f32 / st_quantize_row_bf16
//                          (io/safetensors.cpp:348-391 / 296-345)
//   qlmref_matmul_int8  -> math::matmul with an int8 B operand
//                          (ops/math_ops.cpp:820-900 -> int8_gemv_range 558-579
//                          -> dot8/dot4/dot_avx2_int8 414-553)
//   qlmref_init_threads -> math::init_thread_pool (ops/math_ops.cpp:161-171)
//   qlmref_rms_norm / qlmref_add_rms_norm / qlmref_silu_mul / qlmref_rope_neox
//                       -> math::rms_norm, add_rms_norm, silu_mul, apply_rope_neox
//                          (ops/math_ops.cpp:1055-1074, 1133-1174, 1122-1131, 1237-1291)
//   qlmref_greedy_sample -> DecoderModel::sample(logits, 0, 0), the greedy branch
//                          (model/model.cpp:259-272)
//   qlmref_quantize_int4 -> SafetensorsLoader::get_tensor_keep_int4, which runs
//                          st_quantize_row_f32_int4 / st_quantize_row_bf16_int4
//                          (io/safetensors.cpp:393-515)
//   qlmref_matmul_int4  -> math::matmul with an int4 B operand
//                          (ops/math_ops.cpp:852-855 -> int4_gemv_range 771-794
//                          -> dot8/dot4/dot_avx2_int4 581-769)
//
// The reference quantizer only reads safetensors files, so qlmref_quantize
// writes the matrix to a private temporary file first.

#include "math_ops.hpp"
#include "model.hpp"
#include "safetensors.hpp"

#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <unistd.h>
#include <vector>

namespace {

thread_local std::string g_err;

int fail(const std::string& msg) {
    g_err = msg;
    return 1;
}

bool write_safetensors(const std::string& path, const void* data, int dtype, int n, int k) {
    const size_t elem = dtype == 1 ? 2 : 4;
    const size_t nbytes = (size_t)n * (size_t)k * elem;
    std::string hdr = std::string("{\"w\":{\"dtype\":\"") + (dtype == 1 ? "BF16" : "F32") +
                      "\",\"shape\":[" + std::to_string(n) + "," + std::to_string(k) +
                      "],\"data_offsets\":[0," + std::to_string(nbytes) + "]}}";
    while (hdr.size() % 8) hdr.push_back(' ');
    FILE* f = std::fopen(path.c_str(), "wb");
    if (!f) return false;
    uint64_t hlen = hdr.size();
    bool ok = std::fwrite(&hlen, 8, 1, f) == 1 && std::fwrite(hdr.data(), 1, hdr.size(), f) == hdr.size() &&
              (nbytes == 0 || std::fwrite(data, 1, nbytes, f) == nbytes);
    ok = (std::fclose(f) == 0) && ok;
    return ok;
}

}  // namespace

extern "C" {

const char* qlmref_last_error(void) { return g_err.c_str(); }

// The reference's greedy sampling over n logits (a view, not a copy).
int qlmref_greedy_sample(const float* logits, int n, int* out) {
    if (!logits || n <= 0 || !out) return fail("bad arguments");
    Tensor t;
    t.shape = {1, n};
    t.data = const_cast<float*>(logits);
    DecoderModel model;
    *out = model.sample(t, 0.0f, 0);
    return 0;
}

int qlmref_init_threads(int n) {
    try {
        math::init_thread_pool(n > 0 ? (size_t)n : 1);
        return 0;
    } catch (const std::exception& e) {
        return fail(e.what());
    }
}

// W: [n, k] row-major, dtype 0 = F32 (float*), 1 = BF16 (uint16_t*).
// q_out: [n, k] int8; s_out: [n, ceil(k/32)] fp32 (the reference layout).
int qlmref_quantize(const void* w, int dtype, int n, int k, int8_t* q_out, float* s_out) {
    if (!w || n <= 0 || k <= 0 || !q_out || !s_out || (dtype != 0 && dtype != 1)) return fail("bad args");
    const char* tmp = std::getenv("TMPDIR");
    std::string pat = std::string(tmp && *tmp ? tmp : "/tmp") + "/qlmref_XXXXXX";
    std::vector<char> buf(pat.begin(), pat.end());
    buf.push_back('\0');
    int fd = mkstemp(buf.data());
    if (fd < 0) return fail("mkstemp failed");
    close(fd);
    std::string path(buf.data());
    int rc = 0;
    try {
        if (!write_safetensors(path, w, dtype, n, k)) {
            rc = fail("could not write temporary safetensors file");
        } else {
            SafetensorsLoader loader;
            if (!loader.open(path)) {
                rc = fail("SafetensorsLoader::open failed");
            } else {
                Tensor t = loader.get_tensor_keep_int8("w");
                const int nb = (k + Tensor::INT8_BLOCK_SIZE - 1) / Tensor::INT8_BLOCK_SIZE;
                std::memcpy(q_out, t.int8_data, (size_t)n * k);
                std::memcpy(s_out, t.int8_scales->data(), (size_t)n * nb * sizeof(float));
            }
        }
    } catch (const std::exception& e) {
        rc = fail(e.what());
    }
    std::remove(path.c_str());
    return rc;
}

// The int4 counterpart of qlmref_quantize: packed_out [n, (k+1)/2] bytes (two
// values per byte, low nibble = even column, value + 8), s_out [n, ceil(k/32)].
int qlmref_quantize_int4(const void* w, int dtype, int n, int k, uint8_t* packed_out, float* s_out) {
    if (!w || n <= 0 || k <= 0 || !packed_out || !s_out || (dtype != 0 && dtype != 1)) return fail("bad args");
    const char* tmp = std::getenv("TMPDIR");
    std::string pat = std::string(tmp && *tmp ? tmp : "/tmp") + "/qlmref_XXXXXX";
    std::vector<char> buf(pat.begin(), pat.end());
    buf.push_back('\0');
    int fd = mkstemp(buf.data());
    if (fd < 0) return fail("mkstemp failed");
    close(fd);
    std::string path(buf.data());
    int rc = 0;
    try {
        if (!write_safetensors(path, w, dtype, n, k)) {
            rc = fail("could not write temporary safetensors file");
        } else {
            SafetensorsLoader loader;
            if (!loader.open(path)) {
                rc = fail("SafetensorsLoader::open failed");
            } else {
                Tensor t = loader.get_tensor_keep_int4("w");
                const int nb = (k + Tensor::INT4_BLOCK_SIZE - 1) / Tensor::INT4_BLOCK_SIZE;
                std::memcpy(packed_out, t.int4_data, (size_t)n * ((k + 1) / 2));
                std::memcpy(s_out, t.int4_scales->data(), (size_t)n * nb * sizeof(float));
            }
        }
    } catch (const std::exception& e) {
        rc = fail(e.what());
    }
    std::remove(path.c_str());
    return rc;
}

// y = x . W^T through math::matmul with W in the reference's int4 layout.
int qlmref_matmul_int4(const float* x, int m, int k, const uint8_t* packed, const float* s, int n, float* c,
                       int ldc) {
    if (!x || !packed || !s || !c || m <= 0 || k <= 0 || n <= 0 || ldc < n) return fail("bad args");
    try {
        const int nb = (k + Tensor::INT4_BLOCK_SIZE - 1) / Tensor::INT4_BLOCK_SIZE;
        Tensor A(std::vector<int>{m, k}, const_cast<float*>(x));
        Tensor B;
        B.shape = {n, k};
        B.compute_strides();
        B.int4_data = packed;
        B.int4_scales = std::make_shared<std::vector<float>>(s, s + (size_t)n * nb);
        Tensor C(std::vector<int>{m, n}, c);
        C.strides[0] = ldc;
        math::matmul(A, B, C, true);
        return 0;
    } catch (const std::exception& e) {
        return fail(e.what());
    }
}

// y[m, :] = x[m, :] . W^T through math::matmul, W given in the reference's
// int8 layout. Runs `reps` times (>= 1) and writes the best wall time (ms)
// to *best_ms when non-null. C has row stride ldc (>= n).
int qlmref_matmul_int8(const float* x, int m, int k, const int8_t* q, const float* s, int n, float* c,
                       int ldc, int reps, double* best_ms) {
    if (!x || !q || !s || !c || m <= 0 || k <= 0 || n <= 0 || ldc < n) return fail("bad args");
    try {
        const int nb = (k + Tensor::INT8_BLOCK_SIZE - 1) / Tensor::INT8_BLOCK_SIZE;
        Tensor A(std::vector<int>{m, k}, const_cast<float*>(x));
        Tensor B;
        B.shape = {n, k};
        B.compute_strides();
        B.int8_data = q;
        B.int8_scales = std::make_shared<std::vector<float>>(s, s + (size_t)n * nb);
        Tensor C(std::vector<int>{m, n}, c);
        C.strides[0] = ldc;
        double best = 1e300;
        for (int r = 0; r < (reps > 0 ? reps : 1); ++r) {
            auto t0 = std::chrono::steady_clock::now();
            math::matmul(A, B, C, true);
            auto t1 = std::chrono::steady_clock::now();
            double ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
            if (ms < best) best = ms;
        }
        if (best_ms) *best_ms = best;
        return 0;
    } catch (const std::exception& e) {
        return fail(e.what());
    }
}

// Per-layer ops on host buffers, through the reference's own functions.
int qlmref_rms_norm(const float* x, const float* w, float* y, int rows, int size, float eps) {
    if (!x || !w || !y || rows <= 0 || size <= 0) return fail("bad args");
    Tensor in(std::vector<int>{rows, size}, const_cast<float*>(x));
    Tensor wt(std::vector<int>{size}, const_cast<float*>(w));
    Tensor out(std::vector<int>{rows, size}, y);
    math::rms_norm(in, wt, out, eps);
    return 0;
}

int qlmref_add_rms_norm(float* res, const float* delta, const float* w, float* out, int rows, int size, float eps) {
    if (!res || !delta || !w || !out || rows <= 0 || size <= 0) return fail("bad args");
    Tensor r(std::vector<int>{rows, size}, res);
    Tensor d(std::vector<int>{rows, size}, const_cast<float*>(delta));
    Tensor wt(std::vector<int>{size}, const_cast<float*>(w));
    Tensor o(std::vector<int>{rows, size}, out);
    math::add_rms_norm(r, d, wt, o, eps);
    return 0;
}

int qlmref_silu_mul(float* a, const float* b, int n) {
    if (!a || !b || n <= 0) return fail("bad args");
    Tensor A(std::vector<int>{n}, a);
    Tensor B(std::vector<int>{n}, const_cast<float*>(b));
    math::silu_mul(A, B);
    return 0;
}

int qlmref_silu(float* x, int n) {
    if (!x || n <= 0) return fail("bad args");
    Tensor X(std::vector<int>{n}, x);
    math::silu(X, X);
    return 0;
}

int qlmref_conv1d_update_tapmajor(const float* input, float* state, int oldest_tap, const float* weight_t,
                                  float* output, int conv_dim, int kernel_size) {
    if (!input || !state || !weight_t || !output) return fail("bad args");
    math::causal_conv1d_update_tapmajor(input, state, oldest_tap, weight_t, output, conv_dim, kernel_size);
    return 0;
}

// The gated-delta-net q/k normalisation as the model writes it
// (model/attention.cpp:466-469), through the reference's sumsq / vec_div_inplace.
int qlmref_l2norm_heads(float* x, int heads, int head_dim, float eps) {
    if (!x || heads <= 0 || head_dim <= 0) return fail("bad args");
    for (int h = 0; h < heads; ++h) {
        float* xh = x + (size_t)h * head_dim;
        const float n = std::sqrt(math::sumsq(xh, head_dim) + eps);
        math::vec_div_inplace(xh, n, head_dim);
    }
    return 0;
}

// One token: t [num_heads, head_dim] at position pos.
int qlmref_rope_neox(float* t, int num_heads, int head_dim, int pos, float theta, int rotary_dim) {
    if (!t || num_heads <= 0 || head_dim <= 0) return fail("bad args");
    Tensor T(std::vector<int>{num_heads, head_dim}, t);
    math::apply_rope_neox(T, pos, theta, head_dim, rotary_dim);
    return 0;
}

// Streams `g` distinct int8 weights (all [n, k]) through math::matmul once
// each, in order, `rounds` times; returns total wall time in ms. This is the
// CPU-side analogue of a decode step that reads a stack of weight matrices.
int qlmref_matmul_int8_stack(const float* x, int m, int k, const int8_t* const* qs, const float* const* ss,
                             int g, int n, float* c, int rounds, double* total_ms) {
    if (!x || !qs || !ss || !c || m <= 0 || k <= 0 || n <= 0 || g <= 0) return fail("bad args");
    try {
        const int nb = (k + Tensor::INT8_BLOCK_SIZE - 1) / Tensor::INT8_BLOCK_SIZE;
        Tensor A(std::vector<int>{m, k}, const_cast<float*>(x));
        std::vector<Tensor> Bs(g);
        for (int i = 0; i < g; ++i) {
            Bs[i].shape = {n, k};
            Bs[i].compute_strides();
            Bs[i].int8_data = qs[i];
            Bs[i].int8_scales = std::make_shared<std::vector<float>>(ss[i], ss[i] + (size_t)n * nb);
        }
        Tensor C(std::vector<int>{m, n}, c);
        auto t0 = std::chrono::steady_clock::now();
        for (int r = 0; r < (rounds > 0 ? rounds : 1); ++r)
            for (int i = 0; i < g; ++i) math::matmul(A, Bs[i], C, true);
        auto t1 = std::chrono::steady_clock::now();
        if (total_ms) *total_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
        return 0;
    } catch (const std::exception& e) {
        return fail(e.what());
    }
}

}  // extern "C"
