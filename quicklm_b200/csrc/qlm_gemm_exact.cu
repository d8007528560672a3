// qlm_gemm_exact.cu — bit-exact int8/int4 product for 9..64 activation rows
// (batched decode, exact prefill chunks), streaming each weight once per launch.
//
// Same arithmetic as the decode GEMV (QuickLM src/ops/math_ops.cpp:414-553,
// one output element = one row n of W and one activation row m): lane l of
// the reference kernel, blocks b ascending,
//   bs(b) = (x[32b+l]q + x[32b+8+l]q) + (x[32b+16+l]q + x[32b+24+l]q)
//   t_l   = fma(bs(b), s[n][b], t_l)
//   y     = ((t_0+t_4) + (t_1+t_5)) + ((t_2+t_6) + (t_3+t_7))   (+ ragged tail)
// so y[m][n] is bit-identical to the reference for every m.
//
// Mapping: a thread runs the chains t_l of 4 weight rows x 8 activation rows
// for one lane l, across all of K: 32 accumulators. The f32x2 ops pair two
// activation rows (m, m+1) of the same weight row, so a weight value q enters
// as the pair (q, q) — converted once per 128-element chunk and reused for the
// 8 activation rows — and the activations arrive as pairs straight from shared
// memory: the chunk's activations are staged interleaved by row pair,
// (x[m][k], x[m+1][k], x[m][k+8], x[m+1][k+8]) per 128-bit word, so every
// 128-bit load gives two ready pairs and the 8 lanes of a quarter warp read
// 128 consecutive bytes. That layout is written once per call by a small
// pre-pass (xpair_kernel) into scratch, so each CTA fills a stage with plain
// 16-byte copies. M is staged in buckets of 16, 32 or 64 rows (MS = 2, 4, 8
// sets of 8); a CTA's 64 groups of 8 lanes cover the MS sets of 256 / MS x 4
// weight rows per pass. The grid is one CTA per SM, each owning a balanced
// contiguous range of weight rows that it works in passes, so no SM idles
// while another runs a last wave. Codes, scales and activations of an item
// (pass, chunk) arrive by cp.async in a 3-stage ring that runs across passes,
// so item i+2 is in flight while item i computes.
#include "qlm_device.cuh"
#include "qlm_kernels.h"

#include <algorithm>

namespace qlm {
namespace {

constexpr int kMtStages = 3;
constexpr int kMtMaxM = 64;     // activation rows per launch
constexpr int kMtThreads = 512; // 64 groups of the 8 reference lanes

struct MtParams {
    const float* x;
    int64_t ldx;
    int M;
    const uint8_t* q;  // packed codes [rows][row_bytes]
    const float* s;    // [rows][nb_pad]
    float* y;
    int64_t ldy;
    int rows, k, nb_pad, nck, row_bytes;
    int m_alloc;       // activation rows staged: 16, 32 or 64
    int row_q, row_r;  // rows per CTA: CTA b owns [b*q + min(b, r), +q + (b < r))
    const float* xp;   // the activations in the pair-interleaved chunk layout
    float zero_neg;    // -0.0f: the product addend (see qlm_gemv.cu)
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint4 lds_u4(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}

// Rows of W per pass: each group of 8 threads (the reference lanes) runs 4
// weight rows x 8 activation rows, and the 64 groups of a CTA cover all
// MS x 8 staged activation rows: 32 rows per pass at MS = 8 (M <= 64), 64 at
// MS = 4 (M <= 32), 128 at MS = 2 (M <= 16).
template <int MS>
__host__ __device__ constexpr int pass_rows() { return 4 * (kMtThreads / 8) / MS; }

// Stage layout (bytes): activations [MS*4 pairs][4 blocks][2 halves][8 lanes]
// float4 (MS * 4 KB), then codes [pass rows][128 or 64], then scales
// [pass rows][4]. The scratch holds the same activation layout per chunk.
template <int MS, bool Q4>
struct MtStage {
    static constexpr int kX = MS * 8 * kChunk * 4;
    static constexpr int kRows = pass_rows<MS>();
    static constexpr int kCodes = kRows * (Q4 ? 64 : 128);
    static constexpr int kScales = kRows * 16;
    static constexpr int kBytes = kX + kCodes + kScales;
};

// xp[c][mp][b][h][l] = float4(x[2mp][k], x[2mp+1][k], x[2mp][k+8], x[2mp+1][k+8])
// with k = c*128 + 32b + 16h + l: the activation pairs of lane l, block b,
// steps 2h and 2h+1. Rows past M and columns past K are zero.
__global__ void xpair_kernel(const float* __restrict__ x, int64_t ldx, int M, int k, int m_alloc, int nck,
                             float4* __restrict__ xp) {
    const int64_t n = (int64_t)nck * (m_alloc / 2) * 64;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int l = (int)(i & 7), h = (int)((i >> 3) & 1), b = (int)((i >> 4) & 3);
        const int64_t r = i >> 6;
        const int mp = (int)(r % (m_alloc / 2));
        const int c = (int)(r / (m_alloc / 2));
        const int kk = c * kChunk + 32 * b + 16 * h + l;
        const int m0 = 2 * mp, m1 = m0 + 1;
        auto at = [&](int m, int kx) { return m < M && kx < k ? __ldg(x + (int64_t)m * ldx + kx) : 0.0f; };
        xp[i] = make_float4(at(m0, kk), at(m1, kk), at(m0, kk + 8), at(m1, kk + 8));
    }
}

template <int MS, bool Q4>
__global__ void __launch_bounds__(kMtThreads, 1) gemm_exact_kernel(const __grid_constant__ MtParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int CB = Q4 ? 64 : 128;
    constexpr int PR = pass_rows<MS>();
    using St = MtStage<MS, Q4>;
    const int tid = threadIdx.x, l = tid & 7, oct = tid >> 3;
    const int ms = oct % MS, rq = oct / MS;  // activation set, row quad of the pass
    const int mbase = ms * 8;                // this thread's 8 activation rows
    const uint32_t sbase = __cvta_generic_to_shared(smem);
    // Balanced contiguous row range of this CTA, worked in passes of PR rows;
    // groups whose 4 rows lie past the range skip the arithmetic, so a short
    // last pass costs little more than its activation copies.
    const int b = (int)blockIdx.x;
    const int r_begin = b * p.row_q + min(b, p.row_r);
    const int r_end = r_begin + p.row_q + (b < p.row_r ? 1 : 0);
    const int npass = (r_end - r_begin + PR - 1) / PR;

    const int nbf = p.k / kBlock;  // full blocks
    const int cfull = nbf / 4;
    const int rem_blocks = nbf - cfull * 4;
    // Chunks holding full blocks; one (empty) item per pass when K < 32, so
    // the pass still ends in the ragged tail and the stores.
    const int nchunks = max(1, cfull + (rem_blocks ? 1 : 0));
    const int items = npass * nchunks;  // (pass, chunk), chunk fastest

    // Fill stage st with item it: the chunk's activations (contiguous in the
    // scratch), the pass rows' code bytes and scales. Zero past the range.
    auto issue = [&](int it, int st) {
        const int pass = it / nchunks, c = it - pass * nchunks;
        const int row0 = r_begin + pass * PR;
        const uint32_t dst = sbase + st * St::kBytes;
        const uint8_t* xs = reinterpret_cast<const uint8_t*>(p.xp) + (int64_t)c * St::kX;
        for (int o = tid * 16; o < St::kX; o += kMtThreads * 16) cp_async16(dst + o, xs + o, true);
        constexpr int nq = PR * (CB / 16);  // 16-byte pieces of codes
        for (int i = tid; i < nq + PR; i += kMtThreads) {
            if (i < nq) {
                const int r = i / (CB / 16), piece = i % (CB / 16);
                const bool ok = row0 + r < r_end;
                cp_async16(dst + St::kX + r * CB + piece * 16,
                           ok ? p.q + (int64_t)(row0 + r) * p.row_bytes + (int64_t)c * CB + piece * 16 : p.q, ok);
            } else {
                const int r = i - nq;
                const bool ok = row0 + r < r_end;
                cp_async16(dst + St::kX + St::kCodes + r * 16, ok ? p.s + (int64_t)(row0 + r) * p.nb_pad + c * 4 : p.s,
                           ok);
            }
        }
    };

    for (int i = 0; i < kMtStages - 1; ++i) {
        if (i < items) issue(i, i);
        cp_async_commit();
    }
    const unsigned long long nz = f2pack(p.zero_neg, p.zero_neg);
    const unsigned long long bias = Q4 ? 0x4B0000084B000008ull : 0x4B0000804B000080ull;
    unsigned long long t[4][4];  // [weight row][activation pair]: (t for m, t for m+1)
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int i = 0; i < 4; ++i) t[r][i] = 0ull;  // (+0, +0)

    int c = 0, pass = 0;
    for (int it = 0; it < items; ++it) {
        const int nxt = it + kMtStages - 1;
        if (nxt < items) issue(nxt, nxt % kMtStages);
        cp_async_commit();
        cp_async_wait<kMtStages - 1>();
        __syncthreads();
        const uint32_t sb = sbase + (it % kMtStages) * St::kBytes;
        const int nblk = c < cfull ? 4 : rem_blocks;
        const int row0 = r_begin + pass * PR;
        const bool active = row0 + 4 * rq < r_end && mbase < p.M;
        if (active) {
            for (int bb = 0; bb < nblk; ++bb) {
                unsigned long long xq[4][4];  // [pair][step]
#pragma unroll
                for (int pi = 0; pi < 4; ++pi) {
                    const int mp = (mbase >> 1) + pi;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint4 v = lds_u4(sb + ((((mp * 4 + bb) * 2 + h) * 8 + l) * 16));
                        xq[pi][2 * h] = u2pack(v.x, v.y);
                        xq[pi][2 * h + 1] = u2pack(v.z, v.w);
                    }
                }
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int rr = rq * 4 + r;
                    uint32_t w;
                    if (Q4) {
                        w = lds_u32(sb + St::kX + rr * 64 + l * 8 + (bb >> 1) * 4);
                        w = (bb & 1) ? (w >> 4) & 0x0F0F0F0Fu : w & 0x0F0F0F0Fu;
                    } else {
                        w = lds_u32(sb + St::kX + rr * 128 + l * 16 + bb * 4) ^ 0x80808080u;
                    }
                    const uint32_t sv = lds_u32(sb + St::kX + St::kCodes + rr * 16 + bb * 4);
                    const unsigned long long ss = u2pack(sv, sv);
                    unsigned long long qq[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t f = __byte_perm(w, 0x4B000000u, 0x7540u | (uint32_t)j);
                        qq[j] = f2sub(u2pack(f, f), bias);  // (q, q), exact
                    }
#pragma unroll
                    for (int pi = 0; pi < 4; ++pi) {
                        const unsigned long long p0 = f2fma(xq[pi][0], qq[0], nz);
                        const unsigned long long p1 = f2fma(xq[pi][1], qq[1], nz);
                        const unsigned long long p2 = f2fma(xq[pi][2], qq[2], nz);
                        const unsigned long long p3 = f2fma(xq[pi][3], qq[3], nz);
                        t[r][pi] = f2fma(f2add(f2add(p0, p1), f2add(p2, p3)), ss, t[r][pi]);
                    }
                }
            }
        }
        __syncthreads();  // the stage is read: item it + kMtStages may refill it
        if (++c < nchunks) continue;
        // Pass done: 8 -> 1 tree over the lanes of each group (every lane of
        // the warp takes part in the shuffles), then the ragged tail and the
        // stores of the group's valid rows.
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int pi = 0; pi < 4; ++pi) {
                float a, b2;
                f2unpack(t[r][pi], a, b2);
                a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));
                b2 = __fadd_rn(b2, __shfl_xor_sync(0xffffffffu, b2, 4));
                a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));
                b2 = __fadd_rn(b2, __shfl_xor_sync(0xffffffffu, b2, 1));
                a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 2));
                b2 = __fadd_rn(b2, __shfl_xor_sync(0xffffffffu, b2, 2));
                t[r][pi] = f2pack(a, b2);
            }
        if (l == 0 && active) {
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int row = row0 + rq * 4 + r;
                if (row >= r_end) break;
                const uint8_t* qr = p.q + (int64_t)row * p.row_bytes;
#pragma unroll
                for (int pi = 0; pi < 4; ++pi) {
                    float v[2];
                    f2unpack(t[r][pi], v[0], v[1]);
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int m = mbase + 2 * pi + e;
                        if (m >= p.M) continue;
                        float y = v[e];
                        if (p.k > nbf * kBlock) {
                            // ragged tail: sequential scalar sum times the last block's scale
                            float acc = 0.0f;
                            for (int kk = nbf * kBlock; kk < p.k; ++kk) {
                                const float qf =
                                    Q4 ? (float)((int)((qr[packed_offset_q4(kk)] >> packed_shift_q4(kk)) & 0xF) - 8)
                                       : (float)(int8_t)qr[packed_offset(kk)];
                                acc = __fadd_rn(acc, __fmul_rn(__ldg(p.x + (int64_t)m * p.ldx + kk), qf));
                            }
                            y = __fadd_rn(y, __fmul_rn(acc, p.s[(int64_t)row * p.nb_pad + nbf]));
                        }
                        p.y[(int64_t)m * p.ldy + row] = y;
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int i = 0; i < 4; ++i) t[r][i] = 0ull;
        c = 0;
        ++pass;
    }
    cp_async_wait<0>();
}

}  // namespace

bool gemm_exact_supported(int M, int k) { return M >= 2 && M <= kMtMaxM && k >= 1; }

size_t gemm_exact_scratch_bytes(int M, int k) {
    const int m_alloc = M <= 16 ? 16 : M <= 32 ? 32 : kMtMaxM;
    return (size_t)(packed_k(k) / kChunk) * m_alloc * kChunk * 4;
}

namespace {
template <int MS, bool Q4>
cudaError_t launch_ms(const MtParams& p, int ctas, cudaStream_t stream) {
    static bool attr[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const size_t smem = (size_t)kMtStages * MtStage<MS, Q4>::kBytes;
    if (!attr[dev]) {
        if ((e = cudaFuncSetAttribute(gemm_exact_kernel<MS, Q4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem)) != cudaSuccess)
            return e;
        attr[dev] = true;
    }
    gemm_exact_kernel<MS, Q4><<<ctas, kMtThreads, smem, stream>>>(p);
    return cudaGetLastError();
}
}  // namespace

cudaError_t launch_gemm_exact(const float* x, int64_t ldx, int M, const uint8_t* q, const float* s, int rows, int k,
                              bool q4, float* y, int64_t ldy, void* scratch, int sm_count, cudaStream_t stream) {
    if (!gemm_exact_supported(M, k) || rows < 1 || sm_count < 1) return cudaErrorInvalidValue;
    MtParams p{};
    p.x = x;
    p.ldx = ldx;
    p.M = M;
    p.q = q;
    p.s = s;
    p.y = y;
    p.ldy = ldy;
    p.rows = rows;
    p.k = k;
    const int k_pad = packed_k(k);
    p.nb_pad = k_pad / kBlock;
    p.nck = k_pad / kChunk;
    p.row_bytes = q4 ? k_pad / 2 : k_pad;
    p.m_alloc = M <= 16 ? 16 : M <= 32 ? 32 : kMtMaxM;
    p.xp = static_cast<const float*>(scratch);
    p.zero_neg = -0.0f;
    // One CTA per SM (fewer for matrices of fewer than 4 rows per SM).
    const int ctas = std::min(sm_count, (rows + 3) / 4);
    p.row_q = rows / ctas;
    p.row_r = rows % ctas;
    const int64_t n4 = (int64_t)p.nck * (p.m_alloc / 2) * 64;
    xpair_kernel<<<(int)((n4 + 255) / 256), 256, 0, stream>>>(x, ldx, M, k, p.m_alloc, p.nck,
                                                              static_cast<float4*>(scratch));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    switch (p.m_alloc) {
        case 16: return q4 ? launch_ms<2, true>(p, ctas, stream) : launch_ms<2, false>(p, ctas, stream);
        case 32: return q4 ? launch_ms<4, true>(p, ctas, stream) : launch_ms<4, false>(p, ctas, stream);
        default: return q4 ? launch_ms<8, true>(p, ctas, stream) : launch_ms<8, false>(p, ctas, stream);
    }
}

}  // namespace qlm
