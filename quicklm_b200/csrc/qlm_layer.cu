// qlm_layer.cu — per-layer elementwise/normalisation ops on device-resident
// activations, so a decoder layer's activations can stay in HBM between its
// projections. Restatements of QuickLM src/ops/math_ops.cpp:
//
//   rms_norm      (:1055-1074, sumsq :990-1019, norm_apply_zc :1021-1032)
//   add_rms_norm  (:1133-1174)
//   silu_mul      (:1122-1131), silu (:1076-1084)
//   apply_rope_neox (:1237-1291)
//   causal_conv1d_update_tapmajor (:1321-1366)
//   the GQA attention of one decode token (src/model/attention.cpp:17-81,
//     gqa_attend_head: dot_f32 scores, max, exp, sum, normalise, axpy over V)
//   the gated-delta-net decode step (src/model/attention.cpp): the per-head
//     L2 normalisation (:462-470), the decay/write gates (:472-482), the
//     delta-rule recurrence (:498-560) and the head-wise output norm (:573-577)
//
// rms_norm, add_rms_norm and the RoPE rotation are bit-identical to the
// reference (strict build, no contraction): the sums of squares follow its
// exact accumulation order and reduction tree, the scale is the IEEE
// 1 / sqrt(ss / n + eps), and the RoPE cos/sin tables are computed on the host
// with the same libm calls the reference makes (qlm_rope_neox_tables). SiLU
// needs exp: the device evaluates it in double precision and rounds once, so
// it agrees with the host's expf except where that is not correctly rounded;
// a 1-ulp difference there can move 1 + e, the quotient and the product by one
// rounding each, so silu_mul is specified to 2 ulp of the reference (equal on
// more than 99% of inputs, NaN/Inf alike).
#include <cmath>
#include <cstdint>
#include <string>

#include "qlm_b200.h"
#include "qlm_device.cuh"

namespace qlm {
namespace {

constexpr int kThreads = 256;
constexpr int kStageFloats = 12000;  // rows up to this size are staged in shared memory (< 48 KB with the static part)

// ---- sums of squares, in the reference's order ------------------------------

// sumsq (math_ops.cpp:990-1019): accumulators a0..a3 of 8 lanes; a_g lane l
// takes x[32 i + 8 g + l] by FMA, i ascending; then the 8-wide remainder
// into a0; then per lane (a0 + a1) + (a2 + a3), the 8 -> 4 -> 1 tree
// (lo_i = s_i + s_{i+4}; two hadds), then the scalar tail r += x * x. Warp 0.
__device__ float sumsq_ref(const float* __restrict__ x, int n) {
    const int t = threadIdx.x & 31;
    const int g = t >> 3, l = t & 7;
    const int limit = n - (n % 32);
    float a = 0.0f;
#pragma unroll 4
    for (int i = 0; i < limit; i += 32) a = __fmaf_rn(x[i + 8 * g + l], x[i + 8 * g + l], a);
    int i = limit;
    for (; i + 8 <= n; i += 8)
        if (g == 0) a = __fmaf_rn(x[i + l], x[i + l], a);
    // per lane: (a0 + a1) + (a2 + a3)
    const float a1 = __shfl_sync(0xffffffffu, a, 8 + l);
    const float a2 = __shfl_sync(0xffffffffu, a, 16 + l);
    const float a3 = __shfl_sync(0xffffffffu, a, 24 + l);
    const float s = __fadd_rn(__fadd_rn(a, a1), __fadd_rn(a2, a3));  // valid in lanes 0..7
    const float s_hi = __shfl_sync(0xffffffffu, s, (l & 3) + 4);
    const float lo = __fadd_rn(s, s_hi);  // lanes 0..3: lo_l = s_l + s_{l+4}
    const float lo0 = __shfl_sync(0xffffffffu, lo, 0), lo1 = __shfl_sync(0xffffffffu, lo, 1);
    const float lo2 = __shfl_sync(0xffffffffu, lo, 2), lo3 = __shfl_sync(0xffffffffu, lo, 3);
    float r = __fadd_rn(__fadd_rn(lo0, lo1), __fadd_rn(lo2, lo3));
    for (; i < n; ++i) r = __fadd_rn(r, __fmul_rn(x[i], x[i]));
    return r;
}

// add_rms_norm's sum (math_ops.cpp:1148-1166): one 8-lane accumulator, lane l
// takes v[8 i + l] by FMA; the 8 -> 4 -> 1 tree; then ss += v * v over the tail.
__device__ float sumsq_one_acc(const float* __restrict__ v, int n) {
    const int l = threadIdx.x & 7;
    const int full = n - (n % 8);
    float a = 0.0f;
#pragma unroll 8
    for (int i = 0; i < full; i += 8) a = __fmaf_rn(v[i + l], v[i + l], a);
    const float a_hi = __shfl_sync(0xffffffffu, a, (l & 3) + 4);
    const float lo = __fadd_rn(a, a_hi);
    const float lo0 = __shfl_sync(0xffffffffu, lo, 0), lo1 = __shfl_sync(0xffffffffu, lo, 1);
    const float lo2 = __shfl_sync(0xffffffffu, lo, 2), lo3 = __shfl_sync(0xffffffffu, lo, 3);
    float r = __fadd_rn(__fadd_rn(lo0, lo1), __fadd_rn(lo2, lo3));
    for (int i = full; i < n; ++i) r = __fadd_rn(r, __fmul_rn(v[i], v[i]));
    return r;
}

__device__ __forceinline__ float rms_scale(float ss, int n, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
}

// norm_apply_zc: out = (in * s) * (1 + w); norm_apply_gain (ZC = false):
// out = (in * s) * w; vector body and scalar tail alike. in and out may be the
// same row (each element is read and written by one thread).
template <bool ZC = true>
__device__ __forceinline__ void apply_zc(const float* in, const float* __restrict__ w, float* out, float s, int n) {
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        out[i] = __fmul_rn(__fmul_rn(in[i], s), ZC ? __fadd_rn(1.0f, w[i]) : w[i]);
}

// One CTA per row. Rows up to kStageFloats are first staged in shared memory
// with coalesced loads, so the ordered accumulation chains read on-chip data.
// ZC: zero-centred gain (1 + w) as math::rms_norm; else the plain gain w.
// ld: row stride of x and y in floats (>= size; the rows' first `size` values
// are normalized, the rest untouched).
// Programmatic launch: the decode step launches this kernel and the others it
// runs (qlm_model.cu) as secondaries of the kernel before them. Each waits for
// its predecessor first (pdl_wait), reads data other kernels wrote through L2,
// and then lets its own successor start — usually a GEMV whose weight copies
// then overlap it (the GEMV reads its activations only after its own wait).
// Triggering after the wait keeps the stream at most one kernel ahead: a
// trigger before it let later GEMVs launch while an earlier one still ran
// (620 vs 662-673 tok/s on configuration 3). Launched plainly (the C ABI), the
// wait and the trigger do nothing.
template <bool ZC>
__global__ void __launch_bounds__(kThreads) rms_norm_kernel(const float* x, const float* __restrict__ w, float* y,
                                                            int size, float eps, int64_t ld) {
    extern __shared__ float stage[];
    __shared__ float s_scale;
    pdl_wait();
    pdl_launch_dependents();
    const float* xr = x + (int64_t)blockIdx.x * ld;
    if (size <= kStageFloats) {
        for (int i = threadIdx.x; i < size; i += blockDim.x) stage[i] = __ldcg(xr + i);
        __syncthreads();
        xr = stage;
    }
    if (threadIdx.x < 32) {
        const float ss = sumsq_ref(xr, size);
        if (threadIdx.x == 0) s_scale = rms_scale(ss, size, eps);
    }
    __syncthreads();
    apply_zc<ZC>(xr, w, y + (int64_t)blockIdx.x * ld, s_scale, size);
}

// The decoder layer's unfused residual step (src/model/modules.hpp:228-231,
// 239-240 with the next layer's norm1): x += delta (stored, one rounding per
// element, math::elementwise_add), then y = math::rms_norm(x) in rms_norm's
// own accumulation order — the same bits as the two separate kernels, in one
// launch. One CTA per row; lets a following GEMV start (see rms_norm_kernel).
__global__ void __launch_bounds__(kThreads) add_then_rms_norm_kernel(float* x, const float* __restrict__ delta,
                                                                     const float* __restrict__ w, float* y, int size,
                                                                     float eps) {
    extern __shared__ float stage[];
    __shared__ float s_scale;
    pdl_wait();
    pdl_launch_dependents();
    float* xr = x + (int64_t)blockIdx.x * size;
    const float* dr = delta + (int64_t)blockIdx.x * size;
    const bool staged = size <= kStageFloats;
    for (int i = threadIdx.x; i < size; i += blockDim.x) {
        const float v = __fadd_rn(__ldcg(xr + i), __ldcg(dr + i));
        xr[i] = v;
        if (staged) stage[i] = v;
    }
    __syncthreads();  // the row's sums are visible to warp 0
    const float* v = staged ? stage : xr;
    if (threadIdx.x < 32) {
        const float ss = sumsq_ref(v, size);
        if (threadIdx.x == 0) s_scale = rms_scale(ss, size, eps);
    }
    __syncthreads();
    apply_zc<true>(v, w, y + (int64_t)blockIdx.x * size, s_scale, size);
}

// The gated attention's QK-norm (attention.cpp:166-178) in one launch: CTA r
// < nq normalizes query head r (row stride q_ld, the query half of each
// [query | gate] row) with wq, the others key head r - nq (row stride k_ld)
// with wk; rms_norm_kernel<true>'s arithmetic, in place.
__global__ void __launch_bounds__(kThreads) qk_norm_kernel(float* q, int q_ld, const float* __restrict__ wq,
                                                           float* k, int k_ld, const float* __restrict__ wk, int nq,
                                                           int size, float eps) {
    extern __shared__ float stage[];
    __shared__ float s_scale;
    pdl_wait();
    pdl_launch_dependents();
    const bool isq = (int)blockIdx.x < nq;
    float* xr = isq ? q + (int64_t)blockIdx.x * q_ld : k + (int64_t)(blockIdx.x - nq) * k_ld;
    const float* w = isq ? wq : wk;
    const float* src = xr;
    if (size <= kStageFloats) {
        for (int i = threadIdx.x; i < size; i += blockDim.x) stage[i] = __ldcg(xr + i);
        __syncthreads();
        src = stage;
    }
    if (threadIdx.x < 32) {
        const float ss = sumsq_ref(src, size);
        if (threadIdx.x == 0) s_scale = rms_scale(ss, size, eps);
    }
    __syncthreads();
    apply_zc<true>(src, w, xr, s_scale, size);
}

// Gated-delta-net steps 8-9 (attention.cpp:573-584) in one launch, one CTA per
// head row: o = (x * s) * w with s from rms_norm's accumulation order (the
// arithmetic of rms_norm_kernel<false>), then z = silu(z) * o (that of
// silu_mul_kernel); o itself is not stored. Precedes out_proj's GEMV.
__global__ void __launch_bounds__(kThreads) head_norm_gate_kernel(const float* x, const float* __restrict__ w,
                                                                  float* __restrict__ z, int size, float eps) {
    extern __shared__ float stage[];
    __shared__ float s_scale;
    pdl_wait();
    pdl_launch_dependents();
    const float* xr = x + (int64_t)blockIdx.x * size;
    if (size <= kStageFloats) {
        for (int i = threadIdx.x; i < size; i += blockDim.x) stage[i] = __ldcg(xr + i);
        __syncthreads();
        xr = stage;
    }
    if (threadIdx.x < 32) {
        const float ss = sumsq_ref(xr, size);
        if (threadIdx.x == 0) s_scale = rms_scale(ss, size, eps);
    }
    __syncthreads();
    float* zr = z + (int64_t)blockIdx.x * size;
    for (int i = threadIdx.x; i < size; i += blockDim.x) {
        const float o = __fmul_rn(__fmul_rn(xr[i], s_scale), w[i]);
        const float zx = __ldcg(zr + i);
        const float e = (float)exp(-(double)zx);
        zr[i] = __fmul_rn(__fdiv_rn(zx, __fadd_rn(1.0f, e)), o);
    }
}

// One CTA per row: residual += delta (stored), then out = rms_norm(residual).
__global__ void __launch_bounds__(kThreads) add_rms_norm_kernel(float* res, const float* __restrict__ delta,
                                                                const float* __restrict__ w, float* out, int size,
                                                                float eps) {
    extern __shared__ float stage[];
    __shared__ float s_scale;
    float* rr = res + (int64_t)blockIdx.x * size;
    const float* dr = delta + (int64_t)blockIdx.x * size;
    const bool staged = size <= kStageFloats;
    for (int i = threadIdx.x; i < size; i += blockDim.x) {
        const float v = __fadd_rn(rr[i], dr[i]);
        rr[i] = v;
        if (staged) stage[i] = v;
    }
    __syncthreads();  // the row's sums are visible to warp 0
    const float* v = staged ? stage : rr;
    if (threadIdx.x < 32) {
        const float ss = sumsq_one_acc(v, size);
        if (threadIdx.x == 0) s_scale = rms_scale(ss, size, eps);
    }
    __syncthreads();
    apply_zc(v, w, out + (int64_t)blockIdx.x * size, s_scale, size);
}

// a = (x / (1 + exp(-x))) * b with exp evaluated in double and rounded once.
__global__ void __launch_bounds__(kThreads) silu_mul_kernel(float* __restrict__ a, const float* __restrict__ b,
                                                            int64_t n) {
    pdl_wait();
    pdl_launch_dependents();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float x = __ldcg(a + i);
        const float e = (float)exp(-(double)x);
        a[i] = __fmul_rn(__fdiv_rn(x, __fadd_rn(1.0f, e)), __ldcg(b + i));
    }
}

// x = x / (1 + exp(-x)), exp as in silu_mul_kernel.
__global__ void __launch_bounds__(kThreads) silu_kernel(float* __restrict__ x, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        x[i] = __fdiv_rn(v, __fadd_rn(1.0f, (float)exp(-(double)v)));
    }
}

// Depthwise causal conv step on a tap-major ring (state [ntaps][conv_dim],
// row (oldest + j) % ntaps is the j-th oldest tap; weight_t [ntaps + 1][conv_dim]):
// out[c] = (((0 + s_0 w_0) + s_1 w_1) + ...) + in w_last, products and sums
// rounded separately; the oldest row then takes the input. One thread per channel.
// d_oldest: when set, the ring position is read from device memory (a
// captured decode step replays at every position). SILU: the output then goes
// through silu_kernel's arithmetic (the gated-delta-net's next step,
// attention.cpp:452-457) in the same launch.
template <bool SILU>
__global__ void __launch_bounds__(kThreads) conv1d_tapmajor_kernel(const float* __restrict__ in, float* state,
                                                                   int oldest, const int* __restrict__ d_oldest,
                                                                   const float* __restrict__ wt,
                                                                   float* __restrict__ out, int conv_dim, int ntaps) {
    pdl_wait();
    pdl_launch_dependents();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= conv_dim) return;
    if (d_oldest) oldest = __ldcg(d_oldest);
    float sum = 0.0f;
    for (int j = 0; j < ntaps; ++j) {
        const int row = (oldest + j) % ntaps;
        sum = __fadd_rn(sum, __fmul_rn(__ldcg(state + (int64_t)row * conv_dim + c), wt[(int64_t)j * conv_dim + c]));
    }
    const float x = __ldcg(in + c);
    float y = __fadd_rn(sum, __fmul_rn(x, wt[(int64_t)ntaps * conv_dim + c]));
    if (SILU) y = __fdiv_rn(y, __fadd_rn(1.0f, (float)exp(-(double)y)));
    out[c] = y;
    state[(int64_t)oldest * conv_dim + c] = x;
}

// x_h /= sqrt(sumsq(x_h) + eps) for each head row (one warp per head).
__global__ void __launch_bounds__(kThreads) l2norm_heads_kernel(float* x, int heads, int head_dim, float eps) {
    const int h = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (h >= heads) return;  // whole warps
    float* xh = x + (int64_t)h * head_dim;
    const float ss = sumsq_ref(xh, head_dim);
    const float n = __fsqrt_rn(__fadd_rn(ss, eps));
    __syncwarp();
    for (int i = threadIdx.x & 31; i < head_dim; i += 32) xh[i] = __fdiv_rn(xh[i], n);
}

// The gated-delta-net gates of one head (attention.cpp:472-482): softplus,
// decay = exp(-exp(A_log) * softplus), beta = sigmoid(b); each libm call
// evaluated in double and rounded once, as a correctly rounded float function
// would. Shared by gdn_gates_kernel and the recurrence that folds it in.
__device__ __forceinline__ void gdn_gate(float a_raw, float b_raw, float A_log, float dt_bias, float& dec,
                                         float& beta) {
    const float dt_in = __fadd_rn(a_raw, dt_bias);
    const float sp = dt_in > 20.0f ? dt_in : (float)log1p((double)(float)exp((double)dt_in));
    const float alpha = __fmul_rn(-(float)exp((double)A_log), sp);
    dec = (float)exp((double)alpha);
    beta = __fdiv_rn(1.0f, __fadd_rn(1.0f, (float)exp(-(double)b_raw)));
}

// The delta-rule recurrence; CTA (head h, block of 32 state columns), one
// thread per column j: S = dec * S; kv = k . S; S += (beta k) outer (v - kv);
// out = (q . S) / sqrt(d). The reference's 8-wide body (j < d - d % 8) uses
// FMAs, its scalar tail separate products and sums; each column's operations
// run in the reference's order, and the update of a column and its output sum
// touch only that column, so fusing the update and output passes changes no
// rounding. The CTA's [d][32] slice of the state is loaded into shared memory
// with independent coalesced loads (128 bytes per row), updated there, and
// written back. GATES: the head's decay and beta are computed here from the
// raw gate inputs (gdn_gate, parameters repeating every `per` heads) instead
// of being read from dec / beta — the gates step folded into this launch.
// NORM: q and k are L2-normalized here, in their shared-memory copies, with
// l2norm_heads_kernel's arithmetic (sumsq in the reference's order,
// sqrt(ss + eps), one division per element) — that step folded in as well.
template <bool GATES, bool NORM = false>
__global__ void __launch_bounds__(32) gdn_recurrence_kernel(float* __restrict__ state, const float* __restrict__ q,
                                                            const float* __restrict__ k, const float* __restrict__ v,
                                                            const float* __restrict__ dec,
                                                            const float* __restrict__ beta, float* __restrict__ out,
                                                            int d, const float* __restrict__ a_raw,
                                                            const float* __restrict__ b_raw,
                                                            const float* __restrict__ A_log,
                                                            const float* __restrict__ dt_bias, int per,
                                                            float norm_eps) {
    extern __shared__ float sh[];  // q_h [d], k_h [d], slice [d][32]
    pdl_wait();
    pdl_launch_dependents();
    const int h = blockIdx.x, lane = threadIdx.x, j = blockIdx.y * 32 + lane;
    float* qs = sh;
    float* ks = sh + d;
    float* tile = sh + 2 * d;
    for (int i = lane; i < d; i += 32) {
        qs[i] = __ldcg(q + (int64_t)h * d + i);
        ks[i] = __ldcg(k + (int64_t)h * d + i);
    }
    if (NORM) {
        __syncwarp();
        const float nq = __fsqrt_rn(__fadd_rn(sumsq_ref(qs, d), norm_eps));
        const float nk = __fsqrt_rn(__fadd_rn(sumsq_ref(ks, d), norm_eps));
        __syncwarp();
        for (int i = lane; i < d; i += 32) {
            qs[i] = __fdiv_rn(qs[i], nq);
            ks[i] = __fdiv_rn(ks[i], nk);
        }
    }
    float* S = state + (int64_t)h * d * d + j;
    const bool live = j < d;
#pragma unroll 8
    for (int i = 0; i < d; ++i) tile[i * 32 + lane] = live ? __ldcg(S + (int64_t)i * d) : 0.0f;
    __syncwarp();
    if (live) {
        const bool body = j < d - d % 8;
        float dh, bh;
        if (GATES) {
            gdn_gate(__ldcg(a_raw + h), __ldcg(b_raw + h), A_log[h % per], dt_bias[h % per], dh, bh);
        } else {
            dh = dec[h];
            bh = beta[h];
        }
        float kv = 0.0f;
#pragma unroll 8
        for (int i = 0; i < d; ++i) {
            const float r = __fmul_rn(tile[i * 32 + lane], dh);
            tile[i * 32 + lane] = r;
            kv = body ? __fmaf_rn(ks[i], r, kv) : __fadd_rn(kv, __fmul_rn(ks[i], r));
        }
        const float delta = __fsub_rn(__ldcg(v + (int64_t)h * d + j), kv);
        float o = 0.0f;
#pragma unroll 8
        for (int i = 0; i < d; ++i) {
            const float s = __fmul_rn(bh, ks[i]);
            float r = tile[i * 32 + lane];
            r = body ? __fmaf_rn(s, delta, r) : __fadd_rn(r, __fmul_rn(s, delta));
            tile[i * 32 + lane] = r;
            o = body ? __fmaf_rn(qs[i], r, o) : __fadd_rn(o, __fmul_rn(qs[i], r));
        }
        out[(int64_t)h * d + j] = __fmul_rn(o, __fdiv_rn(1.0f, __fsqrt_rn((float)d)));
#pragma unroll 8
        for (int i = 0; i < d; ++i) S[(int64_t)i * d] = tile[i * 32 + lane];
    }
}

// GQA attention for one decode token, one CTA per query head h (kv head
// h / (heads / kv_heads)). Scores follow dot_f32 (attention.cpp:17-37) exactly:
// a 16-thread group per position, lane a accumulating elements 16c + a (the
// two 8-lane accumulators), an 8-wide remainder into the first, the lane tree,
// the scalar tail, times 1/sqrt(d). The max is order-free (the sign of a zero
// maximum cannot change s - max's exp), except that a NaN first score makes it
// NaN as in the sequential scan. exp is evaluated in double and rounded once;
// the sum runs in position order on one thread; each output element then
// accumulates its positions in order (FMA in the 8-wide body, mul+add in the
// tail), as axpy_f32 does. Shared memory: q [d], scores [pos + 1], 34 floats.
__global__ void __launch_bounds__(256) gqa_attend_kernel(const float* __restrict__ q, int q_stride,
                                                         const float* __restrict__ kc, const float* __restrict__ vc,
                                                         float* __restrict__ out, int pos, int heads, int kv_heads,
                                                         int d) {
    extern __shared__ float sh[];
    float* qs = sh;
    float* sc = sh + d;
    float* red = sc + pos + 1;  // 32 partial maxima, the max, the sum
    const int h = blockIdx.x, tid = threadIdx.x;
    const int kv_size = kv_heads * d, off = (h / (heads / kv_heads)) * d;
    for (int i = tid; i < d; i += blockDim.x) qs[i] = q[(int64_t)h * q_stride + i];
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)d));
    const int groups = blockDim.x / 16, g = tid >> 4, a = tid & 15;
    const int n16 = d / 16, i8 = 16 * n16;
    for (int p0 = 0; p0 <= pos; p0 += groups) {  // warp-uniform trip count
        const int p = min(p0 + g, pos);
        const float* kp = kc + (int64_t)p * kv_size + off;
        float acc = 0.0f;
        for (int c0 = 0; c0 < n16; c0 += 8) {  // this position's K loads first, then the ordered chain
            float kk[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (c0 + u < n16) kk[u] = kp[16 * (c0 + u) + a];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (c0 + u < n16) acc = __fmaf_rn(qs[16 * (c0 + u) + a], kk[u], acc);
        }
        int tail = i8;
        if (i8 + 8 <= d) {
            if (a < 8) acc = __fmaf_rn(qs[i8 + a], kp[i8 + a], acc);
            tail = i8 + 8;
        }
        const float s = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 8, 16));   // lanes 0..7: a0 + a1
        const float lo = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, 4, 16));      // lanes 0..3
        const float l1 = __shfl_down_sync(0xffffffffu, lo, 1, 16);
        const float l2 = __shfl_down_sync(0xffffffffu, lo, 2, 16);
        const float l3 = __shfl_down_sync(0xffffffffu, lo, 3, 16);
        if (a == 0 && p0 + g <= pos) {
            float r = __fadd_rn(__fadd_rn(lo, l1), __fadd_rn(l2, l3));
            for (int i = tail; i < d; ++i) r = __fadd_rn(r, __fmul_rn(qs[i], kp[i]));
            sc[p] = __fmul_rn(r, scale);
        }
    }
    __syncthreads();
    // max over the non-NaN scores
    float m = -INFINITY;
    for (int p = tid; p <= pos; p += blockDim.x)
        if (sc[p] > m) m = sc[p];
    for (int o = 16; o; o >>= 1) {
        const float t = __shfl_xor_sync(0xffffffffu, m, o);
        m = t > m ? t : m;
    }
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    if (tid == 0) {
        float mm = red[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) mm = red[w] > mm ? red[w] : mm;
        red[32] = isnan(sc[0]) ? sc[0] : mm;
    }
    __syncthreads();
    m = red[32];
    for (int p = tid; p <= pos; p += blockDim.x) sc[p] = (float)exp((double)__fsub_rn(sc[p], m));
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
#pragma unroll 8
        for (int p = 0; p <= pos; ++p) sum = __fadd_rn(sum, sc[p]);
        red[33] = sum;
    }
    __syncthreads();
    const float sum = red[33];
    for (int p = tid; p <= pos; p += blockDim.x) sc[p] = __fdiv_rn(sc[p], sum);
    __syncthreads();
    const int d8 = d - d % 8;
    constexpr int kVBatch = 32;  // V rows loaded ahead of the ordered accumulation
    for (int i = tid; i < d; i += blockDim.x) {
        float o = 0.0f;
        const float* vp = vc + off + i;
        const bool body = i < d8;
        for (int p0 = 0; p0 <= pos; p0 += kVBatch) {
            const int n = min(kVBatch, pos + 1 - p0);
            float vv[kVBatch];
#pragma unroll
            for (int u = 0; u < kVBatch; ++u)
                if (u < n) vv[u] = vp[(int64_t)(p0 + u) * kv_size];
#pragma unroll
            for (int u = 0; u < kVBatch; ++u)
                if (u < n) {
                    const float w = sc[p0 + u];
                    o = body ? __fmaf_rn(w, vv[u], o) : __fadd_rn(o, __fmul_rn(w, vv[u]));
                }
        }
        out[(int64_t)h * d + i] = o;
    }
}

// Position-parallel form of gqa_attend_kernel for long contexts, in three
// launches with the same arithmetic. Scores: CTA (head, block of 64 positions),
// 16-thread groups as above, into scratch [heads][pos + 1].
// d_pos: when set, the position is read from device memory and the grid
// covers the longest context (CTAs past the position return at once).
__global__ void __launch_bounds__(256) gqa_scores_kernel(const float* __restrict__ q, int q_stride,
                                                         const float* __restrict__ kc, float* __restrict__ scores,
                                                         int pos, const int* __restrict__ d_pos, int heads,
                                                         int kv_heads, int d) {
    extern __shared__ float qs[];
    pdl_wait();
    pdl_launch_dependents();
    if (d_pos) pos = __ldcg(d_pos);
    if ((int)blockIdx.y * 64 > pos) return;
    const int h = blockIdx.x, tid = threadIdx.x;
    const int kv_size = kv_heads * d, off = (h / (heads / kv_heads)) * d;
    for (int i = tid; i < d; i += blockDim.x) qs[i] = __ldcg(q + (int64_t)h * q_stride + i);
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)d));
    const int g = tid >> 4, a = tid & 15;
    const int n16 = d / 16, i8 = 16 * n16;
    const int pbeg = blockIdx.y * 64;
    for (int it = 0; it < 4; ++it) {  // warp-uniform
        const int pw = pbeg + it * 16 + g;
        const int p = min(pw, pos);
        const float* kp = kc + (int64_t)p * kv_size + off;
        float acc = 0.0f;
        for (int c0 = 0; c0 < n16; c0 += 8) {
            float kk[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (c0 + u < n16) kk[u] = __ldcg(kp + (16 * (c0 + u) + a));
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (c0 + u < n16) acc = __fmaf_rn(qs[16 * (c0 + u) + a], kk[u], acc);
        }
        int tail = i8;
        if (i8 + 8 <= d) {
            if (a < 8) acc = __fmaf_rn(qs[i8 + a], __ldcg(kp + (i8 + a)), acc);
            tail = i8 + 8;
        }
        const float s = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 8, 16));
        const float lo = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, 4, 16));
        const float l1 = __shfl_down_sync(0xffffffffu, lo, 1, 16);
        const float l2 = __shfl_down_sync(0xffffffffu, lo, 2, 16);
        const float l3 = __shfl_down_sync(0xffffffffu, lo, 3, 16);
        if (a == 0 && pw <= pos) {
            float r = __fadd_rn(__fadd_rn(lo, l1), __fadd_rn(l2, l3));
            for (int i = tail; i < d; ++i) r = __fadd_rn(r, __fmul_rn(qs[i], __ldcg(kp + (i))));
            scores[(int64_t)h * (pos + 1) + p] = __fmul_rn(r, scale);
        }
    }
}

// Softmax of one head's scores in place, one CTA per head: max with the NaN
// rule, exp in double, the sum in position order, the division.
__global__ void __launch_bounds__(256) gqa_softmax_kernel(float* __restrict__ scores, int pos,
                                                          const int* __restrict__ d_pos) {
    __shared__ float red[34];
    pdl_wait();
    pdl_launch_dependents();
    if (d_pos) pos = __ldcg(d_pos);
    float* sc = scores + (int64_t)blockIdx.x * (pos + 1);
    const int tid = threadIdx.x;
    float m = -INFINITY;
    for (int p = tid; p <= pos; p += blockDim.x)
        if (__ldcg(sc + p) > m) m = __ldcg(sc + p);
    for (int o = 16; o; o >>= 1) {
        const float t = __shfl_xor_sync(0xffffffffu, m, o);
        m = t > m ? t : m;
    }
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    if (tid == 0) {
        float mm = red[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) mm = red[w] > mm ? red[w] : mm;
        const float s0 = __ldcg(sc);
        red[32] = isnan(s0) ? s0 : mm;
    }
    __syncthreads();
    m = red[32];
    for (int p = tid; p <= pos; p += blockDim.x) sc[p] = (float)exp((double)__fsub_rn(__ldcg(sc + p), m));
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
#pragma unroll 8
        for (int p = 0; p <= pos; ++p) sum = __fadd_rn(sum, __ldcg(sc + p));
        red[33] = sum;
    }
    __syncthreads();
    const float sum = red[33];
    for (int p = tid; p <= pos; p += blockDim.x) sc[p] = __fdiv_rn(__ldcg(sc + p), sum);
}

// V: CTA (head, block of 32 output elements), one warp; the head's weights are
// staged in shared memory, then each lane accumulates its output element over
// the positions in order.
// gate: when set, each output is multiplied by the gated attention's sigmoid
// output gate (attention.cpp:216-226) of its element, gate[h * gate_ld + i]
// (exp in double, rounded once), so the gate needs no launch of its own.
__global__ void __launch_bounds__(32) gqa_v_kernel(const float* __restrict__ probs, const float* __restrict__ vc,
                                                   float* __restrict__ out, int pos, const int* __restrict__ d_pos,
                                                   int heads, int kv_heads, int d, const float* __restrict__ gate,
                                                   int gate_ld) {
    extern __shared__ float pr[];  // [pos + 1]
    pdl_wait();
    pdl_launch_dependents();  // usually precedes o_proj's GEMV (see rms_norm_kernel)
    if (d_pos) pos = __ldcg(d_pos);
    const int h = blockIdx.x, lane = threadIdx.x;
    const int kv_size = kv_heads * d, off = (h / (heads / kv_heads)) * d;
    const float* src = probs + (int64_t)h * (pos + 1);
    for (int p = lane; p <= pos; p += 32) pr[p] = __ldcg(src + p);
    __syncwarp();
    const int i = blockIdx.y * 32 + lane;
    if (i >= d) return;
    const bool body = i < d - d % 8;
    const float* vp = vc + off + i;
    constexpr int kVBatch = 32;
    float o = 0.0f;
    for (int p0 = 0; p0 <= pos; p0 += kVBatch) {
        const int n = min(kVBatch, pos + 1 - p0);
        float vv[kVBatch];
#pragma unroll
        for (int u = 0; u < kVBatch; ++u)
            if (u < n) vv[u] = __ldcg(vp + (int64_t)(p0 + u) * kv_size);
#pragma unroll
        for (int u = 0; u < kVBatch; ++u)
            if (u < n) {
                const float w = pr[p0 + u];
                o = body ? __fmaf_rn(w, vv[u], o) : __fadd_rn(o, __fmul_rn(w, vv[u]));
            }
    }
    if (gate) {
        const float e = (float)exp(-(double)__ldcg(gate + (int64_t)h * gate_ld + i));
        o = __fmul_rn(o, __fdiv_rn(1.0f, __fadd_rn(1.0f, e)));
    }
    out[(int64_t)h * d + i] = o;
}

// Per-head gates; each libm call is evaluated in double and rounded once, as
// a correctly rounded float function would.
__global__ void gdn_gates_kernel(const float* __restrict__ a_raw, const float* __restrict__ b_raw,
                                 const float* __restrict__ A_log, const float* __restrict__ dt_bias,
                                 float* __restrict__ dec, float* __restrict__ beta, int heads, int per) {
    // heads of several sequences in a row: the per-head parameters repeat every `per` heads
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h >= heads) return;
    const int hp = h % per;
    gdn_gate(a_raw[h], b_raw[h], A_log[hp], dt_bias[hp], dec[h], beta[h]);
}

// t [tokens][heads][head_dim]; cos/sin [tokens][rotary_dim / 2].
__global__ void __launch_bounds__(kThreads) rope_neox_kernel(float* __restrict__ t, const float* __restrict__ ct,
                                                             const float* __restrict__ st, int heads, int head_dim,
                                                             int half) {
    const int tok = blockIdx.y;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)heads * half) return;
    const int h = (int)(idx / half), i = (int)(idx % half);
    float* hd = t + ((int64_t)tok * heads + h) * head_dim;
    const float c = ct[(int64_t)tok * half + i], s = st[(int64_t)tok * half + i];
    const float x1 = hd[i], x2 = hd[i + half];
    hd[i] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    hd[i + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
}

// Steps 3-4 of the gated attention's decode (attention.cpp:183-187 RoPE,
// 190-200 cache append) in one launch, at the position *d_pos: thread i <
// nq * half rotates query pair i in place (rope_neox_kernel's arithmetic, head
// stride q_ld); the next nk * head_dim threads each write one element of the
// rotated keys straight into the key cache row (the rotated value of its
// pair, or the element itself past rotary_dim), the last nk * head_dim copy
// the values into the value cache. The keys themselves are not rewritten.
__global__ void __launch_bounds__(kThreads) rope_append_kernel(float* __restrict__ q, int q_ld, int nq,
                                                               const float* __restrict__ k,
                                                               const float* __restrict__ v, int nk, int head_dim,
                                                               int half, const float* __restrict__ cos_all,
                                                               const float* __restrict__ sin_all,
                                                               const int* __restrict__ d_pos, float* __restrict__ kc,
                                                               float* __restrict__ vc) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int pos = __ldcg(d_pos);
    const float* ct = cos_all + (int64_t)pos * half;
    const float* st = sin_all + (int64_t)pos * half;
    const int64_t nqp = (int64_t)nq * half, nke = (int64_t)nk * head_dim;
    if (i < nqp) {
        const int h = (int)(i / half), e = (int)(i % half);
        float* hd = q + (int64_t)h * q_ld;
        const float c = ct[e], sn = st[e];
        const float x1 = __ldcg(hd + e), x2 = __ldcg(hd + e + half);
        hd[e] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
        hd[e + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
    } else if (i < nqp + nke) {
        const int64_t j = i - nqp;
        const int h = (int)(j / head_dim), e = (int)(j % head_dim);
        const float* hd = k + (int64_t)h * head_dim;
        float r;
        if (e < half) {
            r = __fsub_rn(__fmul_rn(__ldcg(hd + e), ct[e]), __fmul_rn(__ldcg(hd + e + half), st[e]));
        } else if (e < 2 * half) {
            r = __fadd_rn(__fmul_rn(__ldcg(hd + e), ct[e - half]), __fmul_rn(__ldcg(hd + e - half), st[e - half]));
        } else {
            r = __ldcg(hd + e);
        }
        kc[(int64_t)pos * nke + j] = r;
    } else if (i < nqp + 2 * nke) {
        const int64_t j = i - nqp - nke;
        vc[(int64_t)pos * nke + j] = __ldcg(v + j);
    }
}


}  // namespace
}  // namespace qlm

namespace qlm_internal {
void set_last_error(const std::string& msg);
}

namespace {

int layer_fail(int code, const char* msg) {
    qlm_internal::set_last_error(msg);
    return code;
}

int launched(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return QLM_OK;
    qlm_internal::set_last_error(std::string(what) + ": " + cudaGetErrorString(e));
    return QLM_ERR_CUDA;
}

}  // namespace

namespace qlm {

// math::rms_norm on `rows` rows of `size` floats spaced `ld` apart (in place
// when x == y): the per-head QK-norm of a query laid out [query | gate].
// The internal launchers below launch as programmatic-dependent secondaries
// when pdl is set; the norm kernels only when their rows are staged in shared
// memory (their unstaged form reads the row again through L1).
cudaError_t launch_add_then_rms_norm(float* x, const float* delta, const float* w, float* y, int rows, int size,
                                     float eps, cudaStream_t stream, bool pdl) {
    const bool staged = size <= kStageFloats;
    return launch_pdl(pdl && staged, add_then_rms_norm_kernel, dim3(rows), dim3(kThreads),
                      staged ? (size_t)size * sizeof(float) : 0, stream, x, delta, w, y, size, eps);
}

cudaError_t launch_rms_norm(const float* x, const float* w, float* y, int rows, int size, float eps,
                            cudaStream_t stream, bool pdl) {
    const bool staged = size <= kStageFloats;
    return launch_pdl(pdl && staged, rms_norm_kernel<true>, dim3(rows), dim3(kThreads),
                      staged ? (size_t)size * sizeof(float) : 0, stream, x, w, y, size, eps, (int64_t)size);
}

cudaError_t launch_silu_mul(float* a, const float* b, int64_t n, cudaStream_t stream, bool pdl) {
    int64_t blocks = (n + kThreads - 1) / kThreads;
    if (blocks > 148 * 64) blocks = 148 * 64;
    return launch_pdl(pdl, silu_mul_kernel, dim3((unsigned)blocks), dim3(kThreads), 0, stream, a, b, n);
}

// Position-from-device forms for a decode step that is captured once and
// replayed at every position (same kernels and arithmetic as the C ABI's).
cudaError_t launch_conv1d_silu_dev(const float* input, float* state, const int* d_oldest, const float* weight_t,
                                   float* output, int conv_dim, int kernel_size, cudaStream_t stream, bool pdl) {
    return launch_pdl(pdl, conv1d_tapmajor_kernel<true>, dim3((conv_dim + kThreads - 1) / kThreads), dim3(kThreads), 0,
                      stream, input, state, 0, d_oldest, weight_t, output, conv_dim, kernel_size - 1);
}

cudaError_t launch_rope_append(float* q, int q_ld, int nq, const float* k, const float* v, int nk, int head_dim,
                               int rotary_dim, const float* cos_all, const float* sin_all, const int* d_pos,
                               float* k_cache, float* v_cache, cudaStream_t stream, bool pdl) {
    const int half = rotary_dim / 2;
    const int64_t n = (int64_t)nq * half + 2 * (int64_t)nk * head_dim;
    return launch_pdl(pdl, rope_append_kernel, dim3((unsigned)((n + kThreads - 1) / kThreads)), dim3(kThreads), 0,
                      stream, q, q_ld, nq, k, v, nk, head_dim, half, cos_all, sin_all, d_pos, k_cache, v_cache);
}

cudaError_t launch_qk_norm(float* q, int q_ld, const float* wq, int nq, float* k, int k_ld, const float* wk, int nk,
                           int size, float eps, cudaStream_t stream, bool pdl) {
    const bool staged = size <= kStageFloats;
    return launch_pdl(pdl && staged, qk_norm_kernel, dim3(nq + nk), dim3(kThreads),
                      staged ? (size_t)size * sizeof(float) : 0, stream, q, q_ld, wq, k, k_ld, wk, nq, size, eps);
}

cudaError_t launch_head_norm_gate(const float* x, const float* w, float* z, int rows, int size, float eps,
                                  cudaStream_t stream, bool pdl) {
    const bool staged = size <= kStageFloats;
    return launch_pdl(pdl && staged, head_norm_gate_kernel, dim3(rows), dim3(kThreads),
                      staged ? (size_t)size * sizeof(float) : 0, stream, x, w, z, size, eps);
}

cudaError_t launch_gdn_recurrence_fused(float* state, const float* q, const float* k, const float* v,
                                        const float* a_raw, const float* b_raw, const float* A_log,
                                        const float* dt_bias, int per, float norm_eps, float* out, int heads,
                                        int head_dim, cudaStream_t stream, bool pdl) {
    if (heads <= 0 || head_dim <= 0 || head_dim > 1024 || per <= 0) return cudaErrorInvalidValue;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        if ((e = cudaFuncSetAttribute(gdn_recurrence_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (2 + 32) * 1024 * (int)sizeof(float))) != cudaSuccess)
            return e;
        attr_set[dev] = true;
    }
    const dim3 grid((unsigned)heads, (unsigned)((head_dim + 31) / 32));
    const size_t smem = (size_t)(2 + 32) * head_dim * sizeof(float);
    return launch_pdl(pdl, gdn_recurrence_kernel<true, true>, grid, dim3(32), smem, stream, state, q, k, v,
                      (const float*)nullptr, (const float*)nullptr, out, head_dim, a_raw, b_raw, A_log, dt_bias, per,
                      norm_eps);
}

size_t gqa_dev_smem_bytes(int max_pos) { return (size_t)(max_pos + 1) * sizeof(float); }

cudaError_t launch_gqa_attend_dev(const float* q, int q_stride, const float* k_cache, const float* v_cache,
                                  float* out, const int* d_pos, int max_pos, int heads, int kv_heads, int head_dim,
                                  float* scratch, const float* gate, int gate_ld, cudaStream_t stream, bool pdl) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        if ((e = cudaFuncSetAttribute(gqa_v_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) !=
            cudaSuccess)
            return e;
        attr_set[dev] = true;
    }
    const dim3 g1((unsigned)heads, (unsigned)((max_pos + 64) / 64));
    if ((e = launch_pdl(pdl, gqa_scores_kernel, g1, dim3(256), (size_t)head_dim * sizeof(float), stream, q, q_stride,
                        k_cache, scratch, 0, d_pos, heads, kv_heads, head_dim)) != cudaSuccess)
        return e;
    if ((e = launch_pdl(pdl, gqa_softmax_kernel, dim3(heads), dim3(256), 0, stream, scratch, 0, d_pos)) != cudaSuccess)
        return e;
    const dim3 g2((unsigned)heads, (unsigned)((head_dim + 31) / 32));
    return launch_pdl(pdl, gqa_v_kernel, g2, dim3(32), gqa_dev_smem_bytes(max_pos), stream, (const float*)scratch,
                      v_cache, out, 0, d_pos, heads, kv_heads, head_dim, gate, gate_ld);
}
}  // namespace qlm

extern "C" {

int qlm_rms_norm(const float* x, const float* w, float* y, int rows, int size, float eps, void* stream) {
    if (!x || !w || !y) return layer_fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (rows <= 0 || size <= 0) return layer_fail(QLM_ERR_INVALID_ARG, "rows and size must be positive");
    const size_t smem = size <= qlm::kStageFloats ? (size_t)size * sizeof(float) : 0;
    qlm::rms_norm_kernel<true><<<rows, qlm::kThreads, smem, static_cast<cudaStream_t>(stream)>>>(x, w, y, size, eps, size);
    return launched("rms_norm launch");
}

int qlm_rms_norm_gain(const float* x, const float* w, float* y, int rows, int size, float eps, void* stream) {
    if (!x || !w || !y) return layer_fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (rows <= 0 || size <= 0) return layer_fail(QLM_ERR_INVALID_ARG, "rows and size must be positive");
    const size_t smem = size <= qlm::kStageFloats ? (size_t)size * sizeof(float) : 0;
    qlm::rms_norm_kernel<false><<<rows, qlm::kThreads, smem, static_cast<cudaStream_t>(stream)>>>(x, w, y, size, eps, size);
    return launched("rms_norm_gain launch");
}

int qlm_gdn_recurrence(float* state, const float* q, const float* k, const float* v, const float* decay,
                       const float* beta, float* out, int heads, int head_dim, void* stream) {
    if (!state || !q || !k || !v || !decay || !beta || !out) return layer_fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (heads <= 0 || head_dim <= 0 || head_dim > 1024)
        return layer_fail(QLM_ERR_INVALID_ARG, "heads must be positive and head_dim in [1, 1024]");
    const dim3 grid((unsigned)heads, (unsigned)((head_dim + 31) / 32));
    const size_t smem = (size_t)(2 + 32) * head_dim * sizeof(float);  // <= 136 KB at head_dim 1024
    static bool attr_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return layer_fail(QLM_ERR_CUDA, "cudaGetDevice");
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(qlm::gdn_recurrence_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (2 + 32) * 1024 * (int)sizeof(float)) != cudaSuccess)
            return launched("gdn_recurrence attribute");
        attr_set[dev] = true;
    }
    qlm::gdn_recurrence_kernel<false><<<grid, 32, smem, static_cast<cudaStream_t>(stream)>>>(
        state, q, k, v, decay, beta, out, head_dim, nullptr, nullptr, nullptr, nullptr, 1, 0.0f);
    return launched("gdn_recurrence launch");
}

int qlm_gqa_attend(const float* q, int q_stride, const float* k_cache, const float* v_cache, float* out, int pos,
                   int heads, int kv_heads, int head_dim, float* scratch, void* stream) {
    if (!q || !k_cache || !v_cache || !out) return layer_fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || head_dim <= 0 || pos < 0 || q_stride < head_dim)
        return layer_fail(QLM_ERR_INVALID_ARG, "bad attention shape");
    constexpr size_t kMaxSmem = 200 * 1024;
    const size_t smem = ((size_t)head_dim + (size_t)pos + 1 + 34) * sizeof(float);
    if (smem > kMaxSmem) return layer_fail(QLM_ERR_UNSUPPORTED, "context too long for the attention kernels");
    static bool attr_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return layer_fail(QLM_ERR_CUDA, "cudaGetDevice");
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(qlm::gqa_attend_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kMaxSmem) != cudaSuccess ||
            cudaFuncSetAttribute(qlm::gqa_v_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kMaxSmem) != cudaSuccess)
            return launched("gqa_attend attribute");
        attr_set[dev] = true;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!scratch) {
        qlm::gqa_attend_kernel<<<heads, 256, smem, s>>>(q, q_stride, k_cache, v_cache, out, pos, heads, kv_heads,
                                                        head_dim);
        return launched("gqa_attend launch");
    }
    const dim3 g1((unsigned)heads, (unsigned)((pos + 64) / 64));
    qlm::gqa_scores_kernel<<<g1, 256, (size_t)head_dim * sizeof(float), s>>>(q, q_stride, k_cache, scratch, pos,
                                                                            nullptr, heads, kv_heads, head_dim);
    int rc = launched("gqa_scores launch");
    if (rc) return rc;
    qlm::gqa_softmax_kernel<<<heads, 256, 0, s>>>(scratch, pos, nullptr);
    if ((rc = launched("gqa_softmax launch"))) return rc;
    const dim3 g2((unsigned)heads, (unsigned)((head_dim + 31) / 32));
    qlm::gqa_v_kernel<<<g2, 32, (size_t)(pos + 1) * sizeof(float), s>>>(scratch, v_cache, out, pos, nullptr, heads,
                                                                        kv_heads, head_dim, nullptr, 0);
    return launched("gqa_v launch");
}

int qlm_gdn_gates(const float* a_raw, const float* b_raw, const float* A_log, const float* dt_bias, float* decay,
                  float* beta, int heads, void* stream) {
    if (!a_raw || !b_raw || !A_log || !dt_bias || !decay || !beta) return layer_fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (heads <= 0) return layer_fail(QLM_ERR_INVALID_ARG, "heads must be positive");
    qlm::gdn_gates_kernel<<<(heads + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        a_raw, b_raw, A_log, dt_bias, decay, beta, heads, heads);
    return launched("gdn_gates launch");
}

int qlm_add_then_rms_norm(float* residual, const float* delta, const float* w, float* out, int rows, int size,
                          float eps, void* stream) {
    if (!residual || !delta || !w || !out) return layer_fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (rows <= 0 || size <= 0) return layer_fail(QLM_ERR_INVALID_ARG, "rows and size must be positive");
    const cudaError_t e =
        qlm::launch_add_then_rms_norm(residual, delta, w, out, rows, size, eps, static_cast<cudaStream_t>(stream), false);
    if (e != cudaSuccess) return layer_fail(QLM_ERR_CUDA, cudaGetErrorString(e));
    return launched("add_then_rms_norm launch");
}

int qlm_add_rms_norm(float* residual, const float* delta, const float* w, float* out, int rows, int size, float eps,
                     void* stream) {
    if (!residual || !delta || !w || !out) return layer_fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (rows <= 0 || size <= 0) return layer_fail(QLM_ERR_INVALID_ARG, "rows and size must be positive");
    const size_t smem = size <= qlm::kStageFloats ? (size_t)size * sizeof(float) : 0;
    qlm::add_rms_norm_kernel<<<rows, qlm::kThreads, smem, static_cast<cudaStream_t>(stream)>>>(residual, delta, w,
                                                                                             out, size, eps);
    return launched("add_rms_norm launch");
}

int qlm_silu_mul(float* a, const float* b, int64_t n, void* stream) {
    if (!a || !b) return layer_fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (n <= 0) return layer_fail(QLM_ERR_INVALID_ARG, "n must be positive");
    int64_t blocks = (n + qlm::kThreads - 1) / qlm::kThreads;
    if (blocks > 148 * 64) blocks = 148 * 64;
    qlm::silu_mul_kernel<<<(unsigned)blocks, qlm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a, b, n);
    return launched("silu_mul launch");
}

int qlm_rope_neox(float* t, int num_tokens, int num_heads, int head_dim, int rotary_dim, const float* cos_tab,
                  const float* sin_tab, void* stream) {
    if (!t || !cos_tab || !sin_tab) return layer_fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (num_tokens <= 0 || num_heads <= 0 || head_dim <= 0 || rotary_dim < 2 || rotary_dim > head_dim ||
        rotary_dim % 2 || num_tokens > 65535)
        return layer_fail(QLM_ERR_INVALID_ARG, "bad RoPE shape");
    const int half = rotary_dim / 2;
    const int64_t per_tok = (int64_t)num_heads * half;
    const dim3 grid((unsigned)((per_tok + qlm::kThreads - 1) / qlm::kThreads), (unsigned)num_tokens);
    qlm::rope_neox_kernel<<<grid, qlm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(t, cos_tab, sin_tab,
                                                                                       num_heads, head_dim, half);
    return launched("rope_neox launch");
}

int qlm_silu(float* x, int64_t n, void* stream) {
    if (!x) return layer_fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (n <= 0) return layer_fail(QLM_ERR_INVALID_ARG, "n must be positive");
    int64_t blocks = (n + qlm::kThreads - 1) / qlm::kThreads;
    if (blocks > 148 * 64) blocks = 148 * 64;
    qlm::silu_kernel<<<(unsigned)blocks, qlm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(x, n);
    return launched("silu launch");
}

int qlm_conv1d_update_tapmajor(const float* input, float* state, int oldest_tap, const float* weight_t,
                               float* output, int conv_dim, int kernel_size, void* stream) {
    if (!input || !state || !weight_t || !output) return layer_fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (conv_dim <= 0 || kernel_size < 2 || oldest_tap < 0 || oldest_tap >= kernel_size - 1)
        return layer_fail(QLM_ERR_INVALID_ARG, "bad conv1d shape or ring position");
    qlm::conv1d_tapmajor_kernel<false><<<(conv_dim + qlm::kThreads - 1) / qlm::kThreads, qlm::kThreads, 0,
                                  static_cast<cudaStream_t>(stream)>>>(input, state, oldest_tap, nullptr, weight_t,
                                                                       output, conv_dim, kernel_size - 1);
    return launched("conv1d launch");
}

int qlm_l2norm_heads(float* x, int heads, int head_dim, float eps, void* stream) {
    if (!x) return layer_fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (heads <= 0 || head_dim <= 0) return layer_fail(QLM_ERR_INVALID_ARG, "heads and head_dim must be positive");
    const int per_cta = qlm::kThreads / 32;
    qlm::l2norm_heads_kernel<<<(heads + per_cta - 1) / per_cta, qlm::kThreads, 0,
                               static_cast<cudaStream_t>(stream)>>>(x, heads, head_dim, eps);
    return launched("l2norm launch");
}

int qlm_rope_neox_tables(int pos0, int num_tokens, float rope_theta, int rotary_dim, float* cos_out, float* sin_out) {
    if (!cos_out || !sin_out) return layer_fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (num_tokens <= 0 || rotary_dim < 2 || rotary_dim % 2 || pos0 < 0)
        return layer_fail(QLM_ERR_INVALID_ARG, "bad RoPE table shape");
    const int half = rotary_dim / 2;
    for (int tok = 0; tok < num_tokens; ++tok) {
        const int pos = pos0 + tok;
        for (int i = 0; i < half; ++i) {
            // The reference's float expressions (math_ops.cpp:1260-1270), same libm calls.
            const float inv_freq = 1.0f / std::pow(rope_theta, (2.0f * i) / rotary_dim);
            const float angle = pos * inv_freq;
            cos_out[(size_t)tok * half + i] = std::cos(angle);
            sin_out[(size_t)tok * half + i] = std::sin(angle);
        }
    }
    return QLM_OK;
}

}  // extern "C"
