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

#include "attention.hpp"
#include "math_ops.hpp"
#include "model.hpp"
#include "safetensors.hpp"

#include <algorithm>
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

// ---- gated-delta-net decode step (model/attention.cpp:414-591) ----------------
//
// qlmref_gdn_module_steps drives the reference module itself
// (Qwen3_5GatedDeltaNet::init + forward, seq_len 1) over `steps` tokens.
// qlmref_gdn_restated_steps is this oracle's restatement of the same step,
// built on the reference's standalone functions where the model calls them
// (matmul, causal_conv1d_update_tapmajor, sumsq, vec_div_inplace,
// norm_apply_gain) and restating the inline parts: the SiLU, the gates
// (attention.cpp:472-482) and the delta-rule recurrence (qlmref_gdn_recurrence,
// attention.cpp:498-560). Equal outputs over several steps pin the restated
// recurrence, which the device kernel is then tested against.

// The recurrence for all heads: state [heads][d][d] row-major, q/k/v [heads][d],
// dec/beta [heads]; out [heads][d]. The model's 8-wide body uses FMAs, its scalar
// tail (j >= d - d % 8) separate products and sums.
int qlmref_gdn_recurrence(float* state, const float* q, const float* k, const float* v, const float* dec,
                          const float* beta, int heads, int d, float* out) {
    if (!state || !q || !k || !v || !dec || !beta || !out || heads <= 0 || d <= 0) return fail("bad args");
    const int d8 = d - d % 8;
    const float q_scale = 1.0f / std::sqrt(static_cast<float>(d));
    std::vector<float> kv(d), delta(d);
    for (int h = 0; h < heads; ++h) {
        float* S = state + (size_t)h * d * d;
        const float* qh = q + (size_t)h * d;
        const float* kh = k + (size_t)h * d;
        const float* vh = v + (size_t)h * d;
        float* oh = out + (size_t)h * d;
        std::fill(kv.begin(), kv.end(), 0.0f);
        for (int i = 0; i < d; ++i) {
            float* row = S + (size_t)i * d;
            for (int j = 0; j < d; ++j) {
                const float r = row[j] * dec[h];
                row[j] = r;
                kv[j] = j < d8 ? std::fma(kh[i], r, kv[j]) : kv[j] + kh[i] * r;
            }
        }
        for (int j = 0; j < d; ++j) delta[j] = vh[j] - kv[j];
        for (int i = 0; i < d; ++i) {
            const float s = beta[h] * kh[i];
            float* row = S + (size_t)i * d;
            for (int j = 0; j < d; ++j) row[j] = j < d8 ? std::fma(s, delta[j], row[j]) : row[j] + s * delta[j];
        }
        for (int j = 0; j < d; ++j) oh[j] = 0.0f;
        for (int i = 0; i < d; ++i) {
            const float* row = S + (size_t)i * d;
            for (int j = 0; j < d; ++j) oh[j] = j < d8 ? std::fma(qh[i], row[j], oh[j]) : oh[j] + qh[i] * row[j];
        }
        for (int j = 0; j < d; ++j) oh[j] *= q_scale;
    }
    return 0;
}

// The per-head decay and write gates (model/attention.cpp:472-482).
int qlmref_gdn_gates(const float* a_raw, const float* b_raw, const float* A_log, const float* dt_bias, float* dec,
                     float* beta, int heads) {
    if (!a_raw || !b_raw || !A_log || !dt_bias || !dec || !beta || heads <= 0) return fail("bad args");
    for (int h = 0; h < heads; ++h) {
        const float dt_in = a_raw[h] + dt_bias[h];
        const float sp = (dt_in > 20.0f) ? dt_in : std::log1p(std::exp(dt_in));
        const float alpha = -std::exp(A_log[h]) * sp;
        dec[h] = std::exp(alpha);
        beta[h] = 1.0f / (1.0f + std::exp(-b_raw[h]));
    }
    return 0;
}

// The head-wise output norm with a plain gain (model/attention.cpp:573-577).
int qlmref_rms_norm_gain(const float* x, const float* w, float* y, int rows, int size, float eps) {
    if (!x || !w || !y || rows <= 0 || size <= 0) return fail("bad args");
    for (int r = 0; r < rows; ++r) {
        const float sc = 1.0f / std::sqrt((math::sumsq(x + (size_t)r * size, size) / size) + eps);
        math::norm_apply_gain(x + (size_t)r * size, w, y + (size_t)r * size, sc, size);
    }
    return 0;
}

namespace {
struct GdnWeights {
    int hin, heads, d, ks, hout;
    const float *w_qkv, *w_z, *w_b, *w_a, *conv_w, *norm_w, *A_log, *dt_bias, *w_out;
};
Tensor owned(const std::vector<int>& shape, const float* src, size_t n) {
    Tensor t(shape);
    std::memcpy(t.data, src, n * sizeof(float));
    return t;
}
}  // namespace

int qlmref_gdn_module_steps(int hin, int heads, int d, int ks, int hout, const float* w_qkv, const float* w_z,
                            const float* w_b, const float* w_a, const float* conv_w, const float* norm_w,
                            const float* A_log, const float* dt_bias, const float* w_out, int steps,
                            const float* inputs, float* outputs) {
    if (steps <= 0 || !inputs || !outputs) return fail("bad args");
    try {
        const int H = heads * d;
        Qwen3_5GatedDeltaNet m;
        m.init(owned({3 * H, hin}, w_qkv, (size_t)3 * H * hin), owned({H, hin}, w_z, (size_t)H * hin),
               owned({heads, hin}, w_b, (size_t)heads * hin), owned({heads, hin}, w_a, (size_t)heads * hin),
               owned({3 * H, 1, ks}, conv_w, (size_t)3 * H * ks), owned({d}, norm_w, (size_t)d),
               owned({heads}, A_log, (size_t)heads), owned({heads}, dt_bias, (size_t)heads),
               owned({hout, H}, w_out, (size_t)hout * H), heads, d, steps);
        m.reset_states();
        for (int s = 0; s < steps; ++s) {
            Tensor in(std::vector<int>{hin}, const_cast<float*>(inputs + (size_t)s * hin));
            Tensor out(std::vector<int>{hout}, outputs + (size_t)s * hout);
            Context ctx;
            ctx.pos = s;
            ctx.seq_len = 1;
            m.forward(in, out, ctx);
        }
        return 0;
    } catch (const std::exception& e) {
        return fail(e.what());
    }
}

int qlmref_gdn_restated_steps(int hin, int heads, int d, int ks, int hout, const float* w_qkv, const float* w_z,
                              const float* w_b, const float* w_a, const float* conv_w, const float* norm_w,
                              const float* A_log, const float* dt_bias, const float* w_out, int steps,
                              const float* inputs, float* outputs) {
    if (steps <= 0 || !inputs || !outputs) return fail("bad args");
    try {
        const int H = heads * d, C = 3 * H, ntaps = ks - 1;
        Tensor Wqkv = owned({C, hin}, w_qkv, (size_t)C * hin), Wz = owned({H, hin}, w_z, (size_t)H * hin);
        Tensor Wb = owned({heads, hin}, w_b, (size_t)heads * hin), Wa = owned({heads, hin}, w_a, (size_t)heads * hin);
        Tensor Wout = owned({hout, H}, w_out, (size_t)hout * H);
        std::vector<float> wt((size_t)ks * C), conv_state((size_t)ntaps * C, 0.0f), S((size_t)heads * d * d, 0.0f);
        for (int c = 0; c < C; ++c)
            for (int t = 0; t < ks; ++t) wt[(size_t)t * C + c] = conv_w[(size_t)c * ks + t];
        std::vector<float> qkv(C), z(H), b(heads), a(heads), conv(C), y(H), dec(heads), beta(heads);
        int ring = 0;
        for (int s = 0; s < steps; ++s) {
            Tensor in(std::vector<int>{hin}, const_cast<float*>(inputs + (size_t)s * hin));
            Tensor tq(std::vector<int>{C}, qkv.data()), tz(std::vector<int>{H}, z.data());
            Tensor tb(std::vector<int>{heads}, b.data()), ta(std::vector<int>{heads}, a.data());
            math::matmul(in, Wqkv, tq, true);
            math::matmul(in, Wz, tz, true);
            math::matmul(in, Wb, tb, true);
            math::matmul(in, Wa, ta, true);
            math::causal_conv1d_update_tapmajor(qkv.data(), conv_state.data(), ring, wt.data(), conv.data(), C, ks);
            ring = (ring + 1) % ntaps;
            for (int i = 0; i < C; ++i) conv[i] = conv[i] / (1.0f + std::exp(-conv[i]));
            float* qp = conv.data();
            float* kp = conv.data() + H;
            const float* vp = conv.data() + 2 * H;
            for (int h = 0; h < heads; ++h) {
                const float qn = std::sqrt(math::sumsq(qp + (size_t)h * d, d) + 1e-6f);
                const float kn = std::sqrt(math::sumsq(kp + (size_t)h * d, d) + 1e-6f);
                math::vec_div_inplace(qp + (size_t)h * d, qn, d);
                math::vec_div_inplace(kp + (size_t)h * d, kn, d);
            }
            qlmref_gdn_gates(a.data(), b.data(), A_log, dt_bias, dec.data(), beta.data(), heads);
            qlmref_gdn_recurrence(S.data(), qp, kp, vp, dec.data(), beta.data(), heads, d, y.data());
            qlmref_rms_norm_gain(y.data(), norm_w, y.data(), heads, d, 1e-6f);
            for (int i = 0; i < H; ++i) y[i] *= z[i] / (1.0f + std::exp(-z[i]));
            Tensor ty(std::vector<int>{1, H}, y.data());
            Tensor to(std::vector<int>{hout}, outputs + (size_t)s * hout);
            math::matmul(ty, Wout, to, true);
        }
        return 0;
    } catch (const std::exception& e) {
        return fail(e.what());
    }
}

// ---- GQA attention decode step (model/attention.cpp:138-235) ---------------
//
// qlmref_attn_module_steps drives Qwen3_5Attention::init + forward (seq_len 1,
// F32 weights, no biases, gated q_proj) over `steps` tokens;
// qlmref_attn_restated_steps restates the step on the reference's standalone
// functions (matmul, sumsq, norm_apply_zc, apply_rope_neox) with the restated
// per-head attention (qlmref_gqa_attend, attention.cpp:17-81) and output gate.

namespace {
// dot_f32 (attention.cpp:17-37): two 8-lane FMA accumulators over 16-wide
// steps, an 8-wide remainder into the first, the lane tree, the scalar tail.
float dot_ref(const float* a, const float* b, int n) {
    float a0[8] = {0, 0, 0, 0, 0, 0, 0, 0}, a1[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 16 <= n; i += 16)
        for (int l = 0; l < 8; ++l) {
            a0[l] = std::fma(a[i + l], b[i + l], a0[l]);
            a1[l] = std::fma(a[i + 8 + l], b[i + 8 + l], a1[l]);
        }
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) a0[l] = std::fma(a[i + l], b[i + l], a0[l]);
    float s[8], lo[4];
    for (int l = 0; l < 8; ++l) s[l] = a0[l] + a1[l];
    for (int l = 0; l < 4; ++l) lo[l] = s[l] + s[l + 4];
    float r = (lo[0] + lo[1]) + (lo[2] + lo[3]);
    for (; i < n; ++i) r += a[i] * b[i];
    return r;
}
}  // namespace

// All heads of one token: q [heads][q_stride] (query in the first d), caches
// [T][kv_heads][d] with positions 0..pos valid, out [heads][d].
int qlmref_gqa_attend(const float* q, int q_stride, const float* k_cache, const float* v_cache, float* out, int pos,
                      int heads, int kv_heads, int d) {
    if (!q || !k_cache || !v_cache || !out || heads <= 0 || kv_heads <= 0 || d <= 0 || pos < 0) return fail("bad args");
    const int kv_size = kv_heads * d, group = heads / kv_heads, d8 = d - d % 8;
    const float scale = 1.0f / std::sqrt(static_cast<float>(d));
    std::vector<float> sc(pos + 1);
    for (int h = 0; h < heads; ++h) {
        const float* qh = q + (size_t)h * q_stride;
        const int off = (h / group) * d;
        for (int p = 0; p <= pos; ++p) sc[p] = dot_ref(qh, k_cache + (size_t)p * kv_size + off, d) * scale;
        float m = sc[0];
        for (int p = 1; p <= pos; ++p)
            if (sc[p] > m) m = sc[p];
        float sum = 0.0f;
        for (int p = 0; p <= pos; ++p) {
            sc[p] = std::exp(sc[p] - m);
            sum += sc[p];
        }
        for (int p = 0; p <= pos; ++p) sc[p] /= sum;
        float* oh = out + (size_t)h * d;
        for (int i = 0; i < d; ++i) oh[i] = 0.0f;
        for (int p = 0; p <= pos; ++p) {
            const float* vp = v_cache + (size_t)p * kv_size + off;
            for (int i = 0; i < d; ++i) oh[i] = i < d8 ? std::fma(sc[p], vp[i], oh[i]) : oh[i] + sc[p] * vp[i];
        }
    }
    return 0;
}

int qlmref_attn_module_steps(int hin, int heads, int kv_heads, int d, int rot, float theta, int hout,
                             const float* w_q, const float* w_k, const float* w_v, const float* w_o,
                             const float* q_norm, const float* k_norm, int steps, const float* inputs,
                             float* outputs) {
    if (steps <= 0 || !inputs || !outputs) return fail("bad args");
    try {
        Qwen3_5Attention m;
        m.init(owned({heads * 2 * d, hin}, w_q, (size_t)heads * 2 * d * hin),
               owned({kv_heads * d, hin}, w_k, (size_t)kv_heads * d * hin),
               owned({kv_heads * d, hin}, w_v, (size_t)kv_heads * d * hin),
               owned({hout, heads * d}, w_o, (size_t)hout * heads * d), Tensor(), Tensor(), Tensor(),
               owned({d}, q_norm, (size_t)d), owned({d}, k_norm, (size_t)d), heads, kv_heads, d, rot, theta, steps);
        m.reset_states();
        for (int s = 0; s < steps; ++s) {
            Tensor in(std::vector<int>{hin}, const_cast<float*>(inputs + (size_t)s * hin));
            Tensor out(std::vector<int>{hout}, outputs + (size_t)s * hout);
            Context ctx;
            ctx.pos = s;
            ctx.seq_len = 1;
            m.forward(in, out, ctx);
        }
        return 0;
    } catch (const std::exception& e) {
        return fail(e.what());
    }
}

int qlmref_attn_restated_steps(int hin, int heads, int kv_heads, int d, int rot, float theta, int hout,
                               const float* w_q, const float* w_k, const float* w_v, const float* w_o,
                               const float* q_norm, const float* k_norm, int steps, const float* inputs,
                               float* outputs) {
    if (steps <= 0 || !inputs || !outputs) return fail("bad args");
    try {
        const int qd = 2 * d, kv_size = kv_heads * d;
        Tensor Wq = owned({heads * qd, hin}, w_q, (size_t)heads * qd * hin);
        Tensor Wk = owned({kv_size, hin}, w_k, (size_t)kv_size * hin);
        Tensor Wv = owned({kv_size, hin}, w_v, (size_t)kv_size * hin);
        Tensor Wo = owned({hout, heads * d}, w_o, (size_t)hout * heads * d);
        std::vector<float> kc((size_t)steps * kv_size), vc((size_t)steps * kv_size);
        std::vector<float> qv((size_t)heads * qd), kv(kv_size), vv(kv_size), att((size_t)heads * d);
        for (int s = 0; s < steps; ++s) {
            Tensor in(std::vector<int>{hin}, const_cast<float*>(inputs + (size_t)s * hin));
            Tensor tq(std::vector<int>{heads, qd}, qv.data()), tk(std::vector<int>{kv_heads, d}, kv.data());
            Tensor tv(std::vector<int>{kv_heads, d}, vv.data());
            math::matmul(in, Wq, tq, true);
            math::matmul(in, Wk, tk, true);
            math::matmul(in, Wv, tv, true);
            for (int h = 0; h < heads; ++h) {
                float* qh = qv.data() + (size_t)h * qd;
                const float sc = 1.0f / std::sqrt((math::sumsq(qh, d) / d) + 1e-6f);
                math::norm_apply_zc(qh, q_norm, qh, sc, d);
            }
            for (int h = 0; h < kv_heads; ++h) {
                float* kh = kv.data() + (size_t)h * d;
                const float sc = 1.0f / std::sqrt((math::sumsq(kh, d) / d) + 1e-6f);
                math::norm_apply_zc(kh, k_norm, kh, sc, d);
            }
            math::apply_rope_neox(tk, s, theta, d, rot);
            for (int h = 0; h < heads; ++h) {
                Tensor qview(std::vector<int>{1, d}, qv.data() + (size_t)h * qd);
                math::apply_rope_neox(qview, s, theta, d, rot);
            }
            std::memcpy(kc.data() + (size_t)s * kv_size, kv.data(), kv_size * sizeof(float));
            std::memcpy(vc.data() + (size_t)s * kv_size, vv.data(), kv_size * sizeof(float));
            qlmref_gqa_attend(qv.data(), qd, kc.data(), vc.data(), att.data(), s, heads, kv_heads, d);
            for (int h = 0; h < heads; ++h)
                for (int i = 0; i < d; ++i) {
                    const float g = qv[(size_t)h * qd + d + i];
                    att[(size_t)h * d + i] *= 1.0f / (1.0f + std::exp(-g));
                }
            Tensor ta(std::vector<int>{1, heads * d}, att.data());
            Tensor to(std::vector<int>{hout}, outputs + (size_t)s * hout);
            math::matmul(ta, Wo, to, true);
        }
        return 0;
    } catch (const std::exception& e) {
        return fail(e.what());
    }
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
