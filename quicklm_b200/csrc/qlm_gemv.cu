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
// 4 rows ("a unit") per warp. The chain t_l is the thread's register; the
// 8->1 tree is three xor-shuffles inside the row's 8 threads. The exact
// int8 -> fp32 conversion runs on paired fp32 subtracts; every product, sum
// and FMA of the reference's sequence is a scalar round-to-nearest op.
//
// Memory: each warp streams its units' packed rows (and their scales) into
// private shared-memory slots with 1-D cp.async.bulk copies completing on an
// mbarrier. A warp issues its first slots BEFORE the programmatic-dependent-
// launch wait, so a kernel in a stream or CUDA graph starts pulling weights
// from HBM while its predecessor is still computing; with one CTA per SM and
// a balanced contiguous unit range per CTA, a decode-sized matrix is in
// flight in full within the first microsecond. The activations for all MM
// rows are staged once per CTA in a lane-permuted shared layout (one
// conflict-free float4 per lane per step). Waits are bounded: on give-up the
// kernel records a status code and stops.
#include "qlm_device.cuh"
#include "qlm_kernels.h"
#include "qlm_sm100.cuh"

namespace qlm {
namespace {

constexpr long long kWaitBudget = 4000000000LL;  // ~2 s of SM clock
constexpr int kMaxSegChunks = 16;                // chunks per slot (2048 K elements)
constexpr int kSlotBytesPerChunk = 4 * (kChunk + 16);  // 4 rows x (128 int8 + 4 fp32 scales)
constexpr int kStatusTimeout = 0x201;
constexpr int kStatusGatherTimeout = 0x202;

struct GemvParams {
    const float* x;
    int64_t ldx;
    const uint8_t* q;
    const float* s;
    float* y;
    int64_t ldy;
    int* status;
    int rows, k, k_pad, nb_pad;
    int units;       // ceil(rows / 4)
    int sc, nseg;    // chunks per segment, segments per row
    int d;           // slots per warp
    int xs_bytes;    // activation staging bytes (128-aligned)
    int ucta_q, ucta_r;  // units per CTA: CTA b owns [b*q + min(b, r), +q + (b < r))
    // Row-sharded all-gather (M = 1): every output row is also stored into each
    // rank's exchange buffer over NVLink, at column col0 + row.
    GatherArgs ga;
};

// Balanced contiguous unit range of this CTA without any integer division.
__device__ __forceinline__ void cta_units(const GemvParams& p, int& u_begin, int& u_end) {
    const int b = (int)blockIdx.x;
    u_begin = b * p.ucta_q + min(b, p.ucta_r);
    u_end = u_begin + p.ucta_q + (b < p.ucta_r ? 1 : 0);
}

// x element k lives at (k/128)*128 + j*32 + l*4 + bb (block bb = (k/32)%4,
// step j = (k/8)%4, lane l = k%8): lane l reads the four blocks' x for step j
// as one float4 at chunk*128 + j*32 + l*4.
__device__ __forceinline__ int xperm(int k) {
    return (k & ~(kChunk - 1)) + ((k >> 3) & 3) * 32 + (k & 7) * 4 + ((k >> 5) & 3);
}

// One 128-element chunk for this lane: 4 blocks x 4 steps, scales sv[0..3].
// Every product, sum and FMA of the reference's sequence is a scalar
// round-to-nearest op (the scalar .rn forms are never contracted by ptxas;
// paired f32x2 mul/add were seen to be contracted into a paired FMA).
template <int MM>
__device__ __forceinline__ void chunk_update(const float* __restrict__ xs_chunk, int k_pad, int lane, uint4 qv,
                                             float4 sv, float (&t)[MM], int nblocks) {
    const uint32_t w[4] = {qv.x ^ 0x80808080u, qv.y ^ 0x80808080u, qv.z ^ 0x80808080u, qv.w ^ 0x80808080u};
    const float sc[4] = {sv.x, sv.y, sv.z, sv.w};
    float qf[4][4];  // [block][step], exact: (2^23 + q + 128) - (2^23 + 128)
#pragma unroll
    for (int bb = 0; bb < 4; ++bb)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            qf[bb][j] = __fsub_rn(__uint_as_float(__byte_perm(w[bb], 0x4B000000u, 0x7540u | (uint32_t)j)),
                                  8388736.0f);
#pragma unroll
    for (int m = 0; m < MM; ++m) {
        const float* xm = xs_chunk + (size_t)m * k_pad + lane * 4;
        float4 xv[4];  // step j: blocks 0..3
#pragma unroll
        for (int j = 0; j < 4; ++j) xv[j] = *reinterpret_cast<const float4*>(xm + j * 32);
        float tt = t[m];
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
            if (bb < nblocks) {
                const float x0 = bb == 0 ? xv[0].x : bb == 1 ? xv[0].y : bb == 2 ? xv[0].z : xv[0].w;
                const float x1 = bb == 0 ? xv[1].x : bb == 1 ? xv[1].y : bb == 2 ? xv[1].z : xv[1].w;
                const float x2 = bb == 0 ? xv[2].x : bb == 1 ? xv[2].y : bb == 2 ? xv[2].z : xv[2].w;
                const float x3 = bb == 0 ? xv[3].x : bb == 1 ? xv[3].y : bb == 2 ? xv[3].z : xv[3].w;
                const float p0 = __fmul_rn(x0, qf[bb][0]);
                const float p1 = __fmul_rn(x1, qf[bb][1]);
                const float p2 = __fmul_rn(x2, qf[bb][2]);
                const float p3 = __fmul_rn(x3, qf[bb][3]);
                tt = __fmaf_rn(__fadd_rn(__fadd_rn(p0, p1), __fadd_rn(p2, p3)), sc[bb], tt);
            }
        }
        t[m] = tt;
    }
}

template <int MM>
__global__ void __launch_bounds__(512, 1) gemv_stream_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    using namespace sm100;
    const int warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5, lane32 = threadIdx.x & 31;
    const int lane = threadIdx.x & 7;         // reference lane l
    const int rsub = (threadIdx.x >> 3) & 3;  // row within the warp's unit

    const int slot_bytes = p.sc * kSlotBytesPerChunk;
    float* xs = reinterpret_cast<float*>(smem);
    uint8_t* my_slots = smem + p.xs_bytes + (size_t)warp * p.d * slot_bytes;
    const uint32_t bars = smem_u32(smem + p.xs_bytes + (size_t)nwarps * p.d * slot_bytes) + warp * p.d * 8;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(
        smem + p.xs_bytes + (size_t)nwarps * p.d * slot_bytes + (size_t)nwarps * p.d * 8);

    // Balanced contiguous unit range for this CTA; warp w takes units w, w+nwarps, ...
    int u_begin, u_end;
    cta_units(p, u_begin, u_end);
    const int my_units = warp < (u_end - u_begin) ? (u_end - u_begin - warp + nwarps - 1) / nwarps : 0;
    const int items = my_units * p.nseg;
    const int nck = p.k_pad / kChunk;

    auto issue = [&](int item, int slot) {
        // lane 0 only: unit's 4 rows, chunks [g*sc, g*sc + n) of segment g
        const int u = u_begin + warp + (item / p.nseg) * nwarps;
        const int g = item % p.nseg;
        const int c0 = g * p.sc;
        const int n = min(p.sc, nck - c0);
        const uint32_t bar = bars + slot * 8;
        const uint32_t dst = smem_u32(my_slots + (size_t)slot * slot_bytes);
        int valid = min(4, p.rows - 4 * u);
        mbar_arrive_expect_tx(bar, (uint32_t)(valid * n * (kChunk + 16)));
        for (int r = 0; r < valid; ++r) {
            const int row = 4 * u + r;
            bulk_copy_g2s(dst + r * p.sc * kChunk, p.q + (int64_t)row * p.k_pad + (int64_t)c0 * kChunk,
                          (uint32_t)(n * kChunk), bar);
            bulk_copy_g2s(dst + 4 * p.sc * kChunk + r * p.sc * 16, p.s + (int64_t)row * p.nb_pad + c0 * 4,
                          (uint32_t)(n * 16), bar);
        }
    };

    if (lane32 == 0) {
        for (int i = 0; i < p.d; ++i) mbar_init(bars + i * 8, 1);
        if (warp == 0) *abort_flag = 0;
        mbar_fence_init();
        for (int i = 0; i < p.d && i < items; ++i) issue(i, i);
    }
    pdl_launch_dependents();
    // Activations are produced by the previous kernel in the stream.
    pdl_wait();
    // All of a thread's loads are issued before its first store, so staging
    // costs one L2 round trip per 8 elements per thread, not one per element.
#pragma unroll 1
    for (int m = 0; m < MM; ++m) {
        const float* xr = p.x + (int64_t)m * p.ldx;
        float* xd = xs + m * p.k_pad;
        for (int base = 0; base < p.k_pad; base += 8 * (int)blockDim.x) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int kk = base + (int)threadIdx.x + i * (int)blockDim.x;
                v[i] = kk < p.k ? __ldg(xr + kk) : 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int kk = base + (int)threadIdx.x + i * (int)blockDim.x;
                if (kk < p.k_pad) xd[xperm(kk)] = v[i];
            }
        }
    }
    __syncthreads();

    const int nbf = p.k / kBlock;  // full blocks
    const int cfull = nbf / 4;     // chunks of 4 full blocks
    const int rem_blocks = nbf - cfull * 4;
    const int nchunks = cfull + (rem_blocks ? 1 : 0);

    float t[MM];
#pragma unroll
    for (int m = 0; m < MM; ++m) t[m] = 0.0f;

    int stop = items;  // first item not consumed (== items on the normal path)
    for (int i = 0; i < items; ++i) {
        const int slot = i % p.d;
        const int u = u_begin + warp + (i / p.nseg) * nwarps;
        const int g = i % p.nseg;
        if (!mbar_wait(bars + slot * 8, (uint32_t)((i / p.d) & 1), abort_flag, kWaitBudget)) {
            *abort_flag = 1;
            if (lane32 == 0 && p.status) atomicCAS(p.status, 0, kStatusTimeout);
            stop = i;
            break;
        }
        const uint8_t* sq = my_slots + (size_t)slot * slot_bytes + rsub * p.sc * kChunk + lane * 16;
        const uint8_t* ss = my_slots + (size_t)slot * slot_bytes + 4 * p.sc * kChunk + rsub * p.sc * 16;
        const int c0 = g * p.sc;
        const int c1 = min(c0 + p.sc, nchunks);
        const int cf = min(c1, cfull);  // chunks made of four full blocks
        int c = c0;
#pragma unroll 2
        for (; c < cf; ++c) {
            const uint4 qv = *reinterpret_cast<const uint4*>(sq + (c - c0) * kChunk);
            const float4 sv = *reinterpret_cast<const float4*>(ss + (c - c0) * 16);
            chunk_update<MM>(xs + c * kChunk, p.k_pad, lane, qv, sv, t, 4);
        }
        if (c < c1) {  // the chunk holding the last (1..3) full blocks
            const uint4 qv = *reinterpret_cast<const uint4*>(sq + (c - c0) * kChunk);
            const float4 sv = *reinterpret_cast<const float4*>(ss + (c - c0) * 16);
            chunk_update<MM>(xs + c * kChunk, p.k_pad, lane, qv, sv, t, rem_blocks);
        }
        __syncwarp();
        if (lane32 == 0 && i + p.d < items) {
            fence_proxy_async_smem();
            issue(i + p.d, slot);
        }
        if (g == p.nseg - 1) {
            const int row_raw = 4 * u + rsub;
            const bool valid = row_raw < p.rows;
            const int row = valid ? row_raw : p.rows - 1;
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
                    const float st = p.s[(int64_t)row * p.nb_pad + nbf];
#pragma unroll
                    for (int m = 0; m < MM; ++m) {
                        float acc = 0.0f;
                        for (int kk = nbf * kBlock; kk < p.k; ++kk) {
                            const float qf = (float)(int8_t)qr[packed_offset(kk)];
                            acc = __fadd_rn(acc, __fmul_rn(xs[m * p.k_pad + xperm(kk)], qf));
                        }
                        t[m] = __fadd_rn(t[m], __fmul_rn(acc, st));
                    }
                }
#pragma unroll
                for (int m = 0; m < MM; ++m) p.y[(int64_t)m * p.ldy + row] = t[m];
            }
#pragma unroll
            for (int m = 0; m < MM; ++m) t[m] = 0.0f;
        }
    }
    // Drain after a give-up: items [stop, stop + d) were issued but not
    // consumed; their copies must land before this warp's slots are released.
    if (lane32 == 0)
        for (int j = stop; j < stop + p.d && j < items; ++j)
            mbar_wait(bars + (j % p.d) * 8, (uint32_t)((j / p.d) & 1), nullptr, kWaitBudget);
}

// ---------------------------------------------------------------------------
// M = 1 (decode) kernel. Same arithmetic, organised for more warps per SM:
// a warp owns a 2-row unit; phase 1 (all 32 threads, uniform): every thread
// turns its 16-byte slices into the four block sums bs = (p0+p1)+(p2+p3) of
// the reference and writes them over the int8 bytes it just consumed (same 16
// bytes); phase 2: one thread per (row, lane) runs the FMA chain
// t = fma(bs, s, t) over every block in order from shared memory. The block
// sums have no ordering constraint, so phase 1 splits each row's chunks
// between two thread halves; the chain stays sequential per (row, lane).
// Activations are staged block-major: x of (chunk c, block bb, lane l, step j)
// at c*128 + bb*32 + l*4 + j, one float4 per lane per block.
__device__ __forceinline__ int xperm_bm(int k) {
    return (k & ~(kChunk - 1)) + ((k >> 5) & 3) * 32 + (k & 7) * 4 + ((k >> 3) & 3);
}

constexpr int kM1SlotBytesPerChunk = 2 * (kChunk + 16);  // 2 rows x (128 int8 + 4 fp32 scales)

// Block sums of one 16-byte lane slice: bs[bb] = (p0 + p1) + (p2 + p3) with
// p_j = x_j * q_j. The int8 -> fp32 bias subtracts and the products run as
// paired fp32 ops; the two products of a pair are then added horizontally
// with scalar .rn adds, a shape ptxas cannot contract into a paired FMA (it
// did contract paired products feeding a paired add).
__device__ __forceinline__ float4 block_sums(const float* __restrict__ xc, uint4 qv, int nblocks) {
    const uint32_t w[4] = {qv.x ^ 0x80808080u, qv.y ^ 0x80808080u, qv.z ^ 0x80808080u, qv.w ^ 0x80808080u};
    const unsigned long long bias = 0x4B0000804B000080ull;  // (2^23 + 128) x 2
    float bs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int bb = 0; bb < 4; ++bb) {
        if (bb < nblocks) {
            const float4 xv = *reinterpret_cast<const float4*>(xc + bb * 32);
            const uint32_t f0 = __byte_perm(w[bb], 0x4B000000u, 0x7540u);
            const uint32_t f1 = __byte_perm(w[bb], 0x4B000000u, 0x7541u);
            const uint32_t f2 = __byte_perm(w[bb], 0x4B000000u, 0x7542u);
            const uint32_t f3 = __byte_perm(w[bb], 0x4B000000u, 0x7543u);
            const unsigned long long q01 = f2sub(((unsigned long long)f1 << 32) | f0, bias);
            const unsigned long long q23 = f2sub(((unsigned long long)f3 << 32) | f2, bias);
            float p0, p1, p2, p3;
            f2unpack(f2mul(f2pack(xv.x, xv.y), q01), p0, p1);
            f2unpack(f2mul(f2pack(xv.z, xv.w), q23), p2, p3);
            bs[bb] = __fadd_rn(__fadd_rn(p0, p1), __fadd_rn(p2, p3));
        }
    }
    return make_float4(bs[0], bs[1], bs[2], bs[3]);
}

// dst[i] = src[i] for i in [c0, c1) by all threads of the CTA: 16-byte moves
// for the aligned middle (four loads in flight per thread), scalar edges.
__device__ __forceinline__ void cta_copy(float* __restrict__ dst, const float* __restrict__ src, int c0, int c1) {
    const int a0 = min(c1, (c0 + 3) & ~3), a1 = max(a0, c1 & ~3);
    for (int i = c0 + (int)threadIdx.x; i < a0; i += blockDim.x) dst[i] = src[i];
    for (int i = a1 + (int)threadIdx.x; i < c1; i += blockDim.x) dst[i] = src[i];
    const float4* s4 = reinterpret_cast<const float4*>(src + a0);
    float4* d4 = reinterpret_cast<float4*>(dst + a0);
    const int n4 = (a1 - a0) / 4, step = (int)blockDim.x;
    for (int base = 0; base < n4; base += 4 * step) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = base + u * step + (int)threadIdx.x;
            if (i < n4) v[u] = s4[i];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = base + u * step + (int)threadIdx.x;
            if (i < n4) d4[i] = v[u];
        }
    }
}

template <bool GATHER>
__global__ void __launch_bounds__(704, 2) gemv_m1_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    using namespace sm100;
    const int warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5, lane32 = threadIdx.x & 31;
    const int lane = threadIdx.x & 7;           // reference lane l
    const int rsub = (threadIdx.x >> 3) & 1;    // row within the warp's 2-row unit
    const int half = (threadIdx.x >> 4) & 1;    // phase-1 chunk parity

    const int slot_bytes = p.sc * kM1SlotBytesPerChunk;
    float* xs = reinterpret_cast<float*>(smem);
    uint8_t* my_slots = smem + p.xs_bytes + (size_t)warp * p.d * slot_bytes;
    const uint32_t bars = smem_u32(smem + p.xs_bytes + (size_t)nwarps * p.d * slot_bytes) + warp * p.d * 8;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(
        smem + p.xs_bytes + (size_t)nwarps * p.d * slot_bytes + (size_t)nwarps * p.d * 8);

    int u_begin, u_end;
    cta_units(p, u_begin, u_end);
    // Work items of this warp: (unit u_begin + warp + j*nwarps, segment g),
    // g fastest. Counted without division.
    int my_units = 0;
    for (int u = u_begin + warp; u < u_end; u += nwarps) ++my_units;
    const int items = my_units * p.nseg;
    const int nck = p.k_pad >> 7;

    auto issue = [&](int uu, int g, int slot) {  // lane 0 only: unit index uu of this warp, segment g
        const int u = u_begin + warp + uu * nwarps;
        const int c0 = g * p.sc;
        const int n = min(p.sc, nck - c0);
        const uint32_t bar = bars + slot * 8;
        const uint32_t dst = smem_u32(my_slots + (size_t)slot * slot_bytes);
        const int valid = min(2, p.rows - 2 * u);
        mbar_arrive_expect_tx(bar, (uint32_t)(valid * n * (kChunk + 16)));
        for (int r = 0; r < valid; ++r) {
            const int row = 2 * u + r;
            bulk_copy_g2s(dst + r * p.sc * kChunk, p.q + (int64_t)row * p.k_pad + (int64_t)c0 * kChunk,
                          (uint32_t)(n * kChunk), bar);
            bulk_copy_g2s(dst + 2 * p.sc * kChunk + r * p.sc * 16, p.s + (int64_t)row * p.nb_pad + c0 * 4,
                          (uint32_t)(n * 16), bar);
        }
    };

    if (lane32 == 0) {
        for (int i = 0; i < p.d; ++i) mbar_init(bars + i * 8, 1);
        if (warp == 0) *abort_flag = 0;
        mbar_fence_init();
        int uu = 0, g = 0;
        for (int i = 0; i < p.d && i < items; ++i) {
            issue(uu, g, i);
            if (++g == p.nseg) { g = 0; ++uu; }
        }
    }
    pdl_launch_dependents();
    pdl_wait();  // activations are produced by the previous kernel in the stream
    {
        const float* xr = p.x;
        for (int base = 0; base < p.k_pad; base += 8 * (int)blockDim.x) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int kk = base + (int)threadIdx.x + i * (int)blockDim.x;
                v[i] = kk < p.k ? __ldg(xr + kk) : 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int kk = base + (int)threadIdx.x + i * (int)blockDim.x;
                if (kk < p.k_pad) xs[xperm_bm(kk)] = v[i];
            }
        }
    }
    __syncthreads();

    const int nbf = p.k / kBlock;
    const int cfull = nbf / 4;
    const int rem_blocks = nbf - cfull * 4;
    const int nchunks = cfull + (rem_blocks ? 1 : 0);

    float t = 0.0f;
    int stop = items;
    // item i = (unit index uu, segment g); slot = i mod d with phase parity;
    // (uu2, g2) tracks item i + d, the next one issued into this slot.
    int uu = 0, g = 0, slot = 0;
    uint32_t parity = 0;
    int uu2 = 0, g2 = 0;
    for (int j = 0; j < p.d; ++j)
        if (++g2 == p.nseg) { g2 = 0; ++uu2; }
    for (int i = 0; i < items; ++i) {
        const int u = u_begin + warp + uu * nwarps;
        if (!mbar_wait(bars + slot * 8, parity, abort_flag, kWaitBudget)) {
            *abort_flag = 1;
            if (lane32 == 0 && p.status) atomicCAS(p.status, 0, kStatusTimeout);
            stop = i;
            break;
        }
        uint8_t* sq = my_slots + slot * slot_bytes + rsub * p.sc * kChunk + lane * 16;
        const uint8_t* ss = my_slots + slot * slot_bytes + 2 * p.sc * kChunk + rsub * p.sc * 16;
        const int c0 = g * p.sc;
        const int c1 = min(c0 + p.sc, nchunks);
        const int cf = min(c1, cfull);  // chunks of four full blocks in this segment
        // phase 1: block sums for chunks c0 + half, c0 + half + 2, ... written in place
#pragma unroll 2
        for (int c = c0 + half; c < cf; c += 2) {
            const uint4 qv = *reinterpret_cast<const uint4*>(sq + (c - c0) * kChunk);
            const float4 bs = block_sums(xs + c * kChunk + lane * 4, qv, 4);
            *reinterpret_cast<float4*>(sq + (c - c0) * kChunk) = bs;
        }
        if (cf < c1 && ((cf - c0) & 1) == half) {  // the chunk with the last 1..3 full blocks
            const uint4 qv = *reinterpret_cast<const uint4*>(sq + (cf - c0) * kChunk);
            const float4 bs = block_sums(xs + cf * kChunk + lane * 4, qv, rem_blocks);
            *reinterpret_cast<float4*>(sq + (cf - c0) * kChunk) = bs;
        }
        __syncwarp();
        // phase 2: the chain over every block of the segment, in order
        if (half == 0) {
#pragma unroll 4
            for (int c = c0; c < cf; ++c) {
                const float4 bs = *reinterpret_cast<const float4*>(sq + (c - c0) * kChunk);
                const float4 sv = *reinterpret_cast<const float4*>(ss + (c - c0) * 16);
                t = __fmaf_rn(bs.x, sv.x, t);
                t = __fmaf_rn(bs.y, sv.y, t);
                t = __fmaf_rn(bs.z, sv.z, t);
                t = __fmaf_rn(bs.w, sv.w, t);
            }
            if (cf < c1) {
                const float4 bs = *reinterpret_cast<const float4*>(sq + (cf - c0) * kChunk);
                const float4 sv = *reinterpret_cast<const float4*>(ss + (cf - c0) * 16);
                t = __fmaf_rn(bs.x, sv.x, t);
                if (rem_blocks > 1) t = __fmaf_rn(bs.y, sv.y, t);
                if (rem_blocks > 2) t = __fmaf_rn(bs.z, sv.z, t);
            }
        }
        __syncwarp();
        if (lane32 == 0 && i + p.d < items) {
            fence_proxy_async_smem();
            issue(uu2, g2, slot);
        }
        if (++g2 == p.nseg) { g2 = 0; ++uu2; }
        const bool unit_done = g == p.nseg - 1;
        if (++g == p.nseg) { g = 0; ++uu; }
        if (++slot == p.d) { slot = 0; parity ^= 1u; }
        if (unit_done) {
            const int row_raw = 2 * u + rsub;
            const bool valid = row_raw < p.rows;
            const int row = valid ? row_raw : p.rows - 1;
            float v = t;
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
            if (half == 0 && lane == 0 && valid) {
                if (p.k > nbf * kBlock) {
                    const uint8_t* qr = p.q + (int64_t)row * p.k_pad;
                    const float st = p.s[(int64_t)row * p.nb_pad + nbf];
                    float acc = 0.0f;
                    for (int kk = nbf * kBlock; kk < p.k; ++kk) {
                        const float qf = (float)(int8_t)qr[packed_offset(kk)];
                        acc = __fadd_rn(acc, __fmul_rn(xs[xperm_bm(kk)], qf));
                    }
                    v = __fadd_rn(v, __fmul_rn(acc, st));
                }
                if (GATHER) {
                    // this rank's own exchange buffer; the last CTA pushes the shard to the peers
                    p.ga.peer_out[p.ga.rank][((*p.ga.epoch + 1) & 1) * p.ga.out_stride + p.ga.col0 + row] = v;
                } else {
                    p.y[row] = v;
                }
            }
            t = 0.0f;
        }
    }
    if (lane32 == 0)
        for (int j = stop; j < stop + p.d && j < items; ++j)
            mbar_wait(bars + (j % p.d) * 8, (uint32_t)((j / p.d) & 1), nullptr, kWaitBudget);  // give-up path only
    if (GATHER) {
        // Completion: each CTA's rows are in this rank's own buffer; it counts
        // itself done with a GPU-scope release. The last CTA acquires them,
        // pushes the whole shard to every peer with 16-byte stores, releases
        // them at system scope once, publishes this call's epoch e to every
        // rank, waits (bounded) until every rank has published e, copies the
        // gathered row into y and records e.
        __shared__ int is_last, bad;
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            is_last = atomicAdd(p.ga.counter, 1) == (int)gridDim.x - 1;
            bad = 0;
        }
        __syncthreads();
        if (is_last) {
            __threadfence();
            const int e = *p.ga.epoch + 1;
            const long long half = (e & 1) * p.ga.out_stride;
            const float* mine = p.ga.peer_out[p.ga.rank] + half;
#pragma unroll 1
            for (int r = 0; r < p.ga.nranks; ++r)
                if (r != p.ga.rank) cta_copy(p.ga.peer_out[r] + half, mine, p.ga.col0, p.ga.col0 + p.rows);
            __syncthreads();
            if (threadIdx.x == 0) {
                fence_acq_rel_sys();
#pragma unroll 1
                for (int r = 0; r < p.ga.nranks; ++r) st_release_sys(p.ga.peer_flags[r] + p.ga.rank, e);
            }
            if ((int)threadIdx.x < p.ga.nranks) {
                const int* flag = p.ga.peer_flags[p.ga.rank] + threadIdx.x;  // this rank's own flag array
                const long long t0 = clock64();
                while (ld_acquire_sys(flag) - e < 0) {
                    if (clock64() - t0 > kWaitBudget) {
                        bad = 1;
                        if (p.status) atomicCAS(p.status, 0, kStatusGatherTimeout);
                        break;
                    }
                    __nanosleep(32);
                }
            }
            __syncthreads();
            if (!bad) {
                if ((reinterpret_cast<uintptr_t>(p.y) & 15) == 0) {
                    cta_copy(p.y, mine, 0, p.ga.n_total);
                } else {
                    for (int i = threadIdx.x; i < p.ga.n_total; i += blockDim.x) p.y[i] = mine[i];
                }
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                *p.ga.counter = 0;
                *const_cast<int*>(p.ga.epoch) = e;
            }
        }
    }
}

struct Plan {
    int mm, sc, nseg, d, nwarps, ctas, xs_bytes, smem;
};

bool make_plan(int mm, int rows, int k, int sm_count, Plan* pl) {
    const int k_pad = packed_k(k);
    const int nck = k_pad / kChunk;
    const int rpu = mm == 1 ? 2 : 4;  // rows per warp unit
    const int max_warps = mm == 1 ? 22 : 16;
    pl->mm = mm;
    pl->sc = nck < kMaxSegChunks ? nck : kMaxSegChunks;
    pl->nseg = (nck + pl->sc - 1) / pl->sc;
    const int slot_bytes = pl->sc * (mm == 1 ? kM1SlotBytesPerChunk : kSlotBytesPerChunk);
    pl->xs_bytes = round_up(mm * k_pad * 4, 128);
    const int units = (rows + rpu - 1) / rpu;
    pl->ctas = units < sm_count ? units : sm_count;
    const int upc = (units + pl->ctas - 1) / pl->ctas;
    // Short kernels: everything in flight at once within ~113 KB, leaving room
    // for the next kernel's CTA on the same SM. Long ones: up to 200 KB.
    const int small_budget = 113 * 1024, big_budget = 200 * 1024;
    int max_slots = (small_budget - pl->xs_bytes - 1024) / slot_bytes;
    const int upw_all = upc;  // with one warp per unit
    if (max_slots >= 1 && upc <= max_warps && upw_all * pl->nseg <= max_slots) {
        pl->nwarps = upc;
        pl->d = pl->nseg;
    } else {
        max_slots = (big_budget - pl->xs_bytes - 1024) / slot_bytes;
        if (max_slots < 1) return false;
        pl->nwarps = upc < max_warps ? upc : max_warps;
        if (pl->nwarps > max_slots) pl->nwarps = max_slots;
        pl->d = max_slots / pl->nwarps;
        if (pl->d > 4) pl->d = 4;
        const int items_per_warp = ((upc + pl->nwarps - 1) / pl->nwarps) * pl->nseg;
        if (pl->d > items_per_warp) pl->d = items_per_warp;
    }
    pl->smem = pl->xs_bytes + pl->nwarps * pl->d * (slot_bytes + 8) + 16;
    return true;
}

template <int MM>
cudaError_t launch_mm(const GemvParams& p0, const Plan& pl, cudaStream_t stream, bool pdl) {
    static bool attr_set[2][64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    auto kern = MM == 1 ? (p0.ga.nranks > 0 ? gemv_m1_kernel<true> : gemv_m1_kernel<false>) : gemv_stream_kernel<MM>;
    const int gi = p0.ga.nranks > 0 ? 1 : 0;
    if (!attr_set[gi][dev]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 224 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[gi][dev] = true;
    }
    GemvParams p = p0;
    p.units = (p.rows + (MM == 1 ? 1 : 3)) / (MM == 1 ? 2 : 4);
    p.ucta_q = p.units / pl.ctas;
    p.ucta_r = p.units % pl.ctas;
    p.sc = pl.sc;
    p.nseg = pl.nseg;
    p.d = pl.d;
    p.xs_bytes = pl.xs_bytes;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)pl.ctas);
    cfg.blockDim = dim3((unsigned)(pl.nwarps * 32));
    cfg.dynamicSmemBytes = (size_t)pl.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p);
}


}  // namespace

bool gemv_supported(int mm, int rows, int k, int sm_count) {
    Plan pl;
    return make_plan(mm, rows, k, sm_count, &pl);
}

cudaError_t launch_gemv_exact(const float* x, int64_t ldx, int mm, const uint8_t* q, const float* s, int rows,
                              int k, float* y, int64_t ldy, int* status, int sm_count, cudaStream_t stream, bool pdl,
                              const GatherArgs* gather) {
    Plan pl;
    if (!make_plan(mm, rows, k, sm_count, &pl)) return cudaErrorInvalidValue;
    if (gather && mm != 1) return cudaErrorInvalidValue;
    GemvParams p{};
    if (gather) p.ga = *gather;
    p.x = x;
    p.ldx = ldx;
    p.q = q;
    p.s = s;
    p.y = y;
    p.ldy = ldy;
    p.status = status;
    p.rows = rows;
    p.k = k;
    p.k_pad = packed_k(k);
    p.nb_pad = p.k_pad / kBlock;
    p.units = (rows + 3) / 4;
    switch (mm) {
        case 1: return launch_mm<1>(p, pl, stream, pdl);
        case 2: return launch_mm<2>(p, pl, stream, pdl);
        case 3: return launch_mm<3>(p, pl, stream, pdl);
        case 4: return launch_mm<4>(p, pl, stream, pdl);
        case 5: return launch_mm<5>(p, pl, stream, pdl);
        case 6: return launch_mm<6>(p, pl, stream, pdl);
        case 7: return launch_mm<7>(p, pl, stream, pdl);
        case 8: return launch_mm<8>(p, pl, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace qlm
