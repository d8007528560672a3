// qlm_gemv.cu — bit-exact int8 decode GEMV / small-M matmul for sm_100a.
//
// Replaces the int8 branch of math::matmul (QuickLM src/ops/math_ops.cpp:
// 820-900 -> int8_gemv_range 558-579 -> dot8/dot4/dot_avx2_int8 414-553).
// Every output element is computed with the reference's exact sequence of
// IEEE-754 binary32 operations (no contraction, no reassociation):
//   lane l in [0,8), block b ascending:
//     p_j = x[32b+8j+l] * q[32b+8j+l]                    j = 0..3
//     bs  = (p_0 + p_1) + (p_2 + p_3)
//     t_l = fma(bs, s[b], t_l)                             t_l starts at +0
//   y = ((t_0+t_4) + (t_1+t_5)) + ((t_2+t_6) + (t_3+t_7))
//   ragged tail (k % 32): acc = sum x[k]*q[k] in order from 0; y += acc*s[last]
// so the result is bit-identical to the CPU engine for every M, shape and
// input (including NaN/Inf propagation).
//
// Mapping: one thread per (output row, lane l), 8 consecutive threads per row,
// 4 rows per warp. The chain t_l is the thread's register; the final 8->1 tree
// is three xor-shuffles inside the row's 8 threads. Each thread streams its
// 16-byte slice of every 128-element chunk (packed layout in qlm_device.cuh)
// with a register prefetch ring of kDepth chunks, so a warp keeps
// 4 rows x 128 B x kDepth bytes of weights in flight. The activations for all
// MM rows are staged once per CTA in shared memory in a lane-permuted order
// (one conflict-free float4 per lane per block). Scales are applied
// in-register by the chain's FMA.
//
// Grid: about one CTA per SM, each owning a contiguous, balanced range of
// 4-row units (one unit per warp per pass), so the whole matrix streams in a
// single wave without tail imbalance.
#include "qlm_device.cuh"
#include "qlm_kernels.h"

namespace qlm {
namespace {

constexpr int kDepth = 4;  // chunks prefetched per thread

struct GemvParams {
    const float* x;
    int64_t ldx;
    const uint8_t* q;
    const float* s;
    float* y;
    int64_t ldy;
    int rows, k, k_pad, nb_pad;
    int units;  // ceil(rows / 4)
};

template <int MM>
__device__ __forceinline__ void chunk_update(const float* __restrict__ xs, int k_pad, int c, int lane, uint4 qv,
                                             float4 sv, float (&t)[MM], int nblocks) {
    float qf[4][4];
    s8x4_to_f32(qv.x, qf[0]);
    s8x4_to_f32(qv.y, qf[1]);
    s8x4_to_f32(qv.z, qf[2]);
    s8x4_to_f32(qv.w, qf[3]);
    const float sc[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
    for (int bb = 0; bb < 4; ++bb) {
        if (bb < nblocks) {
#pragma unroll
            for (int m = 0; m < MM; ++m) {
                const float4 xv =
                    *reinterpret_cast<const float4*>(xs + (size_t)m * k_pad + c * kChunk + bb * 32 + lane * 4);
                const float p0 = __fmul_rn(xv.x, qf[bb][0]);
                const float p1 = __fmul_rn(xv.y, qf[bb][1]);
                const float p2 = __fmul_rn(xv.z, qf[bb][2]);
                const float p3 = __fmul_rn(xv.w, qf[bb][3]);
                const float bs = __fadd_rn(__fadd_rn(p0, p1), __fadd_rn(p2, p3));
                t[m] = __fmaf_rn(bs, sc[bb], t[m]);
            }
        }
    }
}

template <int MM>
__global__ void __launch_bounds__(512) gemv_exact_kernel(const GemvParams p) {
    extern __shared__ __align__(16) float xs[];  // [MM][k_pad], lane-permuted

    pdl_launch_dependents();

    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    const int lane = threadIdx.x & 7;   // reference lane l
    const int rsub = (threadIdx.x >> 3) & 3;  // row within the warp's 4-row unit

    // Balanced contiguous unit range for this CTA.
    const int u_begin = (int)(((int64_t)blockIdx.x * p.units) / gridDim.x);
    const int u_end = (int)(((int64_t)(blockIdx.x + 1) * p.units) / gridDim.x);

    const int nbf = p.k / kBlock;   // full blocks
    const int cfull = nbf / 4;      // chunks made of 4 full blocks
    const int rem_blocks = nbf - cfull * 4;
    const int nchunks = cfull + (rem_blocks ? 1 : 0);

    // Wait for the producer of x (previous kernel in the stream) before
    // touching activations; weights are constant and need no wait.
    pdl_wait();

    // Stage x for all MM rows: xs[m][xperm(k)] = x[m][k], 0 beyond k.
    for (int i = threadIdx.x; i < MM * p.k_pad; i += blockDim.x) {
        const int m = i / p.k_pad, kk = i - m * p.k_pad;
        const float v = (kk < p.k) ? p.x[(int64_t)m * p.ldx + kk] : 0.0f;
        xs[m * p.k_pad + xperm_offset(kk)] = v;
    }
    __syncthreads();

    for (int u = u_begin + warp; u < u_end; u += nwarps) {
        const int row_raw = u * 4 + rsub;
        const bool valid = row_raw < p.rows;
        const int row = valid ? row_raw : p.rows - 1;  // keep shuffles uniform
        const uint8_t* qrow = p.q + (int64_t)row * p.k_pad + lane * 16;
        const float* srow = p.s + (int64_t)row * p.nb_pad;

        float t[MM];
#pragma unroll
        for (int m = 0; m < MM; ++m) t[m] = 0.0f;

        uint4 qb[kDepth];
        float4 sb[kDepth];
#pragma unroll
        for (int i = 0; i < kDepth; ++i) {
            if (i < nchunks) {
                qb[i] = ldg_stream_u4(qrow + (int64_t)i * kChunk);
                sb[i] = ldg_f4(srow + i * 4);
            }
        }
        for (int c0 = 0; c0 < nchunks; c0 += kDepth) {
#pragma unroll
            for (int i = 0; i < kDepth; ++i) {
                const int c = c0 + i;
                if (c < nchunks) {
                    const uint4 qv = qb[i];
                    const float4 sv = sb[i];
                    if (c + kDepth < nchunks) {
                        qb[i] = ldg_stream_u4(qrow + (int64_t)(c + kDepth) * kChunk);
                        sb[i] = ldg_f4(srow + (c + kDepth) * 4);
                    }
                    chunk_update<MM>(xs, p.k_pad, c, lane, qv, sv, t, c < cfull ? 4 : rem_blocks);
                }
            }
        }

        // 8 -> 1 tree across the row's lanes: u_i = t_i + t_{i+4};
        // (u_0 + u_1) + (u_2 + u_3). IEEE addition is commutative bitwise.
#pragma unroll
        for (int m = 0; m < MM; ++m) {
            float v = t[m];
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
            t[m] = v;
        }

        if (lane == 0 && valid) {
            if (p.k > nbf * kBlock) {
                // Ragged tail: sequential scalar sum times the last block's scale.
                const uint8_t* qr = p.q + (int64_t)row * p.k_pad;
                const float st = srow[nbf];
#pragma unroll
                for (int m = 0; m < MM; ++m) {
                    float acc = 0.0f;
                    for (int kk = nbf * kBlock; kk < p.k; ++kk) {
                        const float qv = (float)(int8_t)qr[packed_offset(kk)];
                        acc = __fadd_rn(acc, __fmul_rn(xs[m * p.k_pad + xperm_offset(kk)], qv));
                    }
                    t[m] = __fadd_rn(t[m], __fmul_rn(acc, st));
                }
            }
#pragma unroll
            for (int m = 0; m < MM; ++m) p.y[(int64_t)m * p.ldy + row] = t[m];
        }
    }
}

template <int MM>
cudaError_t launch_mm(const GemvParams& p, int sm_count, cudaStream_t stream, bool pdl) {
    const size_t smem = (size_t)MM * p.k_pad * sizeof(float);
    static bool attr_set[64] = {};  // the attribute is per function and device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(gemv_exact_kernel<MM>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    // Warps per CTA: enough that every unit of a one-CTA-per-SM grid is one
    // warp-pass, capped at 16 warps; small problems use fewer CTAs.
    const int ctas = p.units < sm_count ? p.units : sm_count;
    int warps = (p.units + ctas - 1) / ctas;
    if (warps > 16) warps = 16;
    if (warps < 1) warps = 1;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3((unsigned)(warps * 32));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_exact_kernel<MM>, p);
}

}  // namespace

size_t gemv_smem_bytes(int mm, int k) { return (size_t)mm * packed_k(k) * sizeof(float); }

cudaError_t launch_gemv_exact(const float* x, int64_t ldx, int mm, const uint8_t* q, const float* s, int rows,
                              int k, float* y, int64_t ldy, int sm_count, cudaStream_t stream, bool pdl) {
    GemvParams p;
    p.x = x;
    p.ldx = ldx;
    p.q = q;
    p.s = s;
    p.y = y;
    p.ldy = ldy;
    p.rows = rows;
    p.k = k;
    p.k_pad = packed_k(k);
    p.nb_pad = p.k_pad / kBlock;
    p.units = (rows + 3) / 4;
    switch (mm) {
        case 1: return launch_mm<1>(p, sm_count, stream, pdl);
        case 2: return launch_mm<2>(p, sm_count, stream, pdl);
        case 3: return launch_mm<3>(p, sm_count, stream, pdl);
        case 4: return launch_mm<4>(p, sm_count, stream, pdl);
        case 5: return launch_mm<5>(p, sm_count, stream, pdl);
        case 6: return launch_mm<6>(p, sm_count, stream, pdl);
        case 7: return launch_mm<7>(p, sm_count, stream, pdl);
        case 8: return launch_mm<8>(p, sm_count, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace qlm
