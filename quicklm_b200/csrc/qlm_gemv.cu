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
// 4 rows ("a unit") per warp; every thread runs its own chain t_l over all
// blocks in order, and the 8->1 tree is three xor-shuffles inside the row's 8
// threads. Within a thread two neighbouring blocks are independent until their
// FMA, so the int8 -> fp32 conversion, the products and the three sums of
// blocks b and b+1 run as paired fp32 ops (one f32x2 instruction for both
// blocks); only the FMA chain is scalar.
//
// The products are fma.rn.f32x2(x, q, z) with z = -0.0 read from the kernel
// parameters: fma(x, q, -0) rounds x*q once and keeps its sign, so it is
// bit-identical to mul.rn(x, q) for every input, but ptxas cannot see that z
// is a zero. With mul.rn.f32x2 products, ptxas (CUDA 12.9, sm_100a) contracts
// the paired add.rn.f32x2 that consumes them into fma(x0, q0, p1) despite the
// .rn qualifiers, with or without --fmad=false and through an opaque mov
// (identified bit-for-bit against a CPU emulation of that contraction); a
// compile-time -0.0 addend is folded and contracted the same way.
//
// Memory: each warp streams its units' packed rows (and their scales) into
// private shared-memory slots, one slot per (unit, segment of the row), so the
// chain starts on a row's first segment while the rest is still in flight.
// Kernels that refill slots (more items than slots) fill each slot with two
// TMA loads (codes, scales) issued by one lane: the packed codes are described
// as a 2-D tensor of 8-byte elements [rows][row bytes / 8] and the scales as
// [rows][k_pad / 32], so one box of 4R rows x one segment lands in the
// [row][chunk][bytes] order the arithmetic reads. Per-row 1-D bulk copies
// issued by 16 lanes cost about as many instructions as the arithmetic there
// (the copy takes uniform operands, so a lane-divergent issue is serialised
// lane by lane): the lm_head 151936 x 2560 runs in 79 us with TMA, 102 us with
// bulk copies. Kernels whose slots are all issued at the start (a decode-sized
// matrix) keep the per-row bulk copies, which start sooner than a first TMA
// load (config 1: 5.6 us vs 5.8 us per launch in a graph). A warp issues its
// first slots BEFORE the programmatic-dependent-launch wait, so a kernel in a
// stream or CUDA graph starts pulling weights from HBM while its predecessor
// is still computing; with one CTA per SM and a balanced contiguous unit range
// per CTA, a decode-sized matrix is in flight in full within the first
// microsecond. The activations for all MM rows are staged once per CTA in a
// lane-permuted shared layout (one conflict-free float4 per lane per step).
// Waits are bounded: on give-up the kernel records a status code and stops.
#include <cstdlib>

#include "qlm_device.cuh"
#include "qlm_kernels.h"
#include "qlm_sm100.cuh"

namespace qlm {
namespace {

constexpr long long kWaitBudget = 4000000000LL;  // ~2 s of SM clock
constexpr int kMaxSegChunks = 8;                 // chunks per slot (1024 K elements)
// One row x one chunk in a slot: the weights (128 int8 or 64 bytes of int4)
// plus its 4 fp32 scales.
template <bool Q4>
__host__ __device__ constexpr int row_chunk_bytes() { return (Q4 ? 64 : 128) + 16; }
// Bytes of one slot (4R rows x sc chunks), padded so that every slot and its
// scale part start on a 128-byte boundary (TMA destinations).
template <bool Q4>
__host__ __device__ constexpr int slot_stride(int sc, int unit_rows) {
    return (unit_rows * sc * row_chunk_bytes<Q4>() + 127) / 128 * 128;
}
// Chunks per segment: about four segments per row, so a row's chain starts on
// its first quarter while the rest is in flight. The GEMV descriptors are
// built with the same value.
int seg_chunks(int nck) {
    int sc = (nck + 3) / 4;
    sc = sc < 2 ? 2 : sc > kMaxSegChunks ? kMaxSegChunks : sc;
    return sc < nck ? sc : nck;
}
constexpr int kStatusTimeout = 0x201;
constexpr int kStatusGatherTimeout = 0x202;

// One weight of a launch. A launch serves up to kMaxGroup weights that share
// the activations (q/k/v, gate/up): their units are concatenated, weight g
// owning units [ubase, ubase + ceil(rows / (4 R))).
struct GemvGroup {
    const CUtensorMap* mq;  // codes, box of 4R rows x sc chunks (device copy of GemvMaps::q[R - 1])
    const CUtensorMap* ms;  // scales, same box
    const uint8_t* q;
    const float* s;
    float* y;
    int64_t ldy;
    int rows;
    int ubase;
};

struct GemvParams {
    const float* x;
    int64_t ldx;
    float zero_neg;  // -0.0f: the product addend (see the file header)
    GemvGroup grp[kMaxGroup];
    int ngroup;
    int* status;
    int k, k_pad, nb_pad;
    int units;       // total units over the weights
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

// Weight of global unit u (the last one whose first unit is <= u).
__device__ __forceinline__ int unit_group(const GemvParams& p, int u) {
    int g = 0;
    for (int i = 1; i < p.ngroup; ++i)
        if (u >= p.grp[i].ubase) g = i;
    return g;
}

// x element k lives at (k/128)*128 + j*32 + l*4 + bb (block bb = (k/32)%4,
// step j = (k/8)%4, lane l = k%8): lane l reads the four blocks' x for step j
// as one float4 at chunk*128 + j*32 + l*4.
__device__ __forceinline__ int xperm(int k) {
    return (k & ~(kChunk - 1)) + ((k >> 3) & 3) * 32 + (k & 7) * 4 + ((k >> 5) & 3);
}

// One 128-element chunk of this lane for the thread's R rows. Row i's 16-byte
// slice (at sq + i * qstride) holds blocks 0..3 (one word each) x steps 0..3
// (one byte each); its four scales are at ss + i * sstride. The activations
// are loaded once per chunk and reused for all R rows. Blocks are processed in
// pairs (0,1) and (2,3): each f32x2 op below is the reference's scalar op for
// both blocks of a pair, so every rounding matches, and the FMAs run in block
// order. nz = (-0, -0) from the kernel parameters. With FULL = false only
// the first nblocks blocks enter the chain (the last chunk of a row with
// K % 128 != 0).
template <int MM, int R, bool FULL, bool Q4>
__device__ __forceinline__ void chunk_update(const float* __restrict__ xs_chunk, int k_pad, int lane,
                                             const uint8_t* sq, int qstride, const uint8_t* ss, int sstride,
                                             unsigned long long nz, float (&t)[MM][R], int nblocks) {
    // w4[i][bb]: byte j = the (biased) value of block bb, step j, this lane.
    uint32_t w4[R][4];
    float4 sv[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
        if (Q4) {
            const uint2 a = *reinterpret_cast<const uint2*>(sq + i * qstride);
            w4[i][0] = a.x & 0x0F0F0F0Fu;
            w4[i][1] = (a.x >> 4) & 0x0F0F0F0Fu;
            w4[i][2] = a.y & 0x0F0F0F0Fu;
            w4[i][3] = (a.y >> 4) & 0x0F0F0F0Fu;
        } else {
            const uint4 a = *reinterpret_cast<const uint4*>(sq + i * qstride);
            w4[i][0] = a.x ^ 0x80808080u;
            w4[i][1] = a.y ^ 0x80808080u;
            w4[i][2] = a.z ^ 0x80808080u;
            w4[i][3] = a.w ^ 0x80808080u;
        }
        sv[i] = *reinterpret_cast<const float4*>(ss + i * sstride);
    }
    // (2^23 + bias) x 2: the byte sits in the mantissa of 2^23; int8 bytes
    // are biased by 128 above, int4 nibbles carry QuickLM's +8.
    const unsigned long long bias = Q4 ? 0x4B0000084B000008ull : 0x4B0000804B000080ull;
#pragma unroll
    for (int m = 0; m < MM; ++m) {
        const float* xm = xs_chunk + (size_t)m * k_pad + lane * 4;
        float4 xv[4];  // step j: blocks 0..3
#pragma unroll
        for (int j = 0; j < 4; ++j) xv[j] = *reinterpret_cast<const float4*>(xm + j * 32);
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const uint32_t* w = w4[i];
            float tt = t[m][i];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                unsigned long long qp[4];  // step j: (q of block 2h, q of block 2h+1), exact
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    qp[j] = f2sub(u2pack(__byte_perm(w[2 * h], 0x4B000000u, 0x7540u | (uint32_t)j),
                                         __byte_perm(w[2 * h + 1], 0x4B000000u, 0x7540u | (uint32_t)j)),
                                  bias);
                const unsigned long long p0 =
                    f2fma(h ? f2pack(xv[0].z, xv[0].w) : f2pack(xv[0].x, xv[0].y), qp[0], nz);
                const unsigned long long p1 =
                    f2fma(h ? f2pack(xv[1].z, xv[1].w) : f2pack(xv[1].x, xv[1].y), qp[1], nz);
                const unsigned long long p2 =
                    f2fma(h ? f2pack(xv[2].z, xv[2].w) : f2pack(xv[2].x, xv[2].y), qp[2], nz);
                const unsigned long long p3 =
                    f2fma(h ? f2pack(xv[3].z, xv[3].w) : f2pack(xv[3].x, xv[3].y), qp[3], nz);
                float b0, b1;  // block sums of blocks 2h and 2h+1
                f2unpack(f2add(f2add(p0, p1), f2add(p2, p3)), b0, b1);
                if (FULL || 2 * h < nblocks) tt = __fmaf_rn(b0, h ? sv[i].z : sv[i].x, tt);
                if (FULL || 2 * h + 1 < nblocks) tt = __fmaf_rn(b1, h ? sv[i].w : sv[i].y, tt);
            }
            t[m][i] = tt;
        }
    }
}

// R rows per thread (4R per warp unit): the activations a thread loads from
// shared memory serve R rows, which halves the shared-memory traffic and the
// load instructions per weight byte at R = 2 (every 128-bit shared load is
// served per quarter-warp, so rows of one warp cannot share a load). M = 1:
// up to 12 warps and 80 registers, so two CTAs fit on an SM and the next
// kernel's CTA can start its weight copies while this one finishes.
// TMA: fill slots by TMA (GemvGroup::mq/ms) instead of per-row bulk copies.
template <int MM, int R, bool GATHER, bool Q4, bool TMA>
__global__ void __launch_bounds__(MM == 1 || R == 2 ? 384 : 512, MM == 1 ? 2 : 1)
    gemv_kernel(const __grid_constant__ GemvParams p) {
    constexpr int CB = Q4 ? 64 : 128;  // weight bytes per row per 128-element chunk
    constexpr int kRowChunkBytes = row_chunk_bytes<Q4>();
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // TMA destinations need 128-byte alignment: align the base explicitly (the
    // plan requests 128 spare bytes).
    uint8_t* smem = smem_raw + ((128u - (sm100::smem_u32(smem_raw) & 127u)) & 127u);
    using namespace sm100;
    const int warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5, lane32 = threadIdx.x & 31;
    const int lane = threadIdx.x & 7;                // reference lane l
    const int rsub = ((threadIdx.x >> 3) & 3) * R;   // first of the thread's R rows within the unit
    constexpr int kUnitRows = 4 * R;

    const int slot_bytes = slot_stride<Q4>(p.sc, kUnitRows);
    float* xs = reinterpret_cast<float*>(smem);
    uint8_t* my_slots = smem + p.xs_bytes + (size_t)warp * p.d * slot_bytes;
    const uint32_t bars = smem_u32(smem + p.xs_bytes + (size_t)nwarps * p.d * slot_bytes) + warp * p.d * 8;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(
        smem + p.xs_bytes + (size_t)nwarps * p.d * slot_bytes + (size_t)nwarps * p.d * 8);

    // Balanced contiguous unit range for this CTA; warp w takes units w,
    // w + nwarps, ...; its work items are (unit, segment g), g fastest.
    int u_begin, u_end;
    cta_units(p, u_begin, u_end);
    int my_units = 0;
    for (int u = u_begin + warp; u < u_end; u += nwarps) ++my_units;
    const int items = my_units * p.nseg;

    // Fill `slot` with the unit's codes and scales for segment g; called by
    // the whole warp. TMA: one lane, two boxes; rows past the weight's end and
    // chunks past k_pad arrive as zeros (never stored), and the transaction
    // count is the full box either way. Bulk: lane r < 4R copies row r's
    // codes, lane 16 + r its scales, valid rows and chunks only.
    auto issue = [&](int uu, int g, int slot) {
        const int u = u_begin + warp + uu * nwarps;
        const GemvGroup& W = p.grp[unit_group(p, u)];
        const int lu = u - W.ubase;  // unit within its weight
        const uint32_t bar = bars + slot * 8;
        const uint32_t dst = smem_u32(my_slots + (size_t)slot * slot_bytes);
        if (TMA) {
            if (lane32 == 0) {
                mbar_arrive_expect_tx(bar, (uint32_t)(kUnitRows * p.sc * kRowChunkBytes));
                tma_load_2d(dst, W.mq, g * p.sc * (CB / 8), kUnitRows * lu, bar);
                tma_load_2d(dst + kUnitRows * p.sc * CB, W.ms, g * p.sc * 4, kUnitRows * lu, bar);
            }
            return;
        }
        const int c0 = g * p.sc;
        const int n = min(p.sc, (p.k_pad >> 7) - c0);
        const int valid = min(kUnitRows, W.rows - kUnitRows * lu);
        if (lane32 == 0) mbar_arrive_expect_tx(bar, (uint32_t)(valid * n * kRowChunkBytes));
        const int r = lane32 & 15, row = kUnitRows * lu + r;
        if (lane32 < 16 && r < valid)
            bulk_copy_g2s(dst + r * p.sc * CB, W.q + (int64_t)row * (p.k_pad / kChunk) * CB + (int64_t)c0 * CB,
                          (uint32_t)(n * CB), bar);
        else if (lane32 >= 16 && r < valid)
            bulk_copy_g2s(dst + kUnitRows * p.sc * CB + r * p.sc * 16, W.s + (int64_t)row * p.nb_pad + c0 * 4,
                          (uint32_t)(n * 16), bar);
    };

    if (lane32 == 0) {
        for (int i = 0; i < p.d; ++i) mbar_init(bars + i * 8, 1);
        if (warp == 0) *abort_flag = 0;
        mbar_fence_init();
    }
    __syncwarp();
    {
        int uu = 0, g = 0;
        for (int i = 0; i < p.d && i < items; ++i) {
            issue(uu, g, i);
            if (++g == p.nseg) { g = 0; ++uu; }
        }
    }
    pdl_launch_dependents();
    // Activations are produced by the previous kernel in the stream. All of a
    // thread's loads are issued before its first store, so staging costs one
    // L2 round trip per 8 elements per thread, not one per element. They are
    // L2 loads (ld.global.cg), never the non-coherent read-only path: under
    // programmatic launch this kernel starts while its producer still writes
    // x, so x is not read-only for this kernel's lifetime and an L1/texture
    // line of an earlier read of the buffer could be served stale.
    pdl_wait();
    // Gather: a communicator whose bounded wait gave up is failed, and such a
    // call does nothing (the host reports QLM_ERR_TIMEOUT until the
    // communicator is freed and recreated). The status word is read after the
    // dependency wait, so it includes the previous call's collect kernel; one
    // thread reads it and the CTA decides together after the staging barrier.
    // Then this call's epoch (the previous call's collect kernel, which
    // advanced it, has completed) and the exchange half it selects.
    __shared__ int comm_failed;
    int g_epoch = 0;
    long long g_half = 0;
    if (GATHER) {
        if (threadIdx.x == 0) comm_failed = ld_relaxed_sys_i32(p.status);
        g_epoch = *reinterpret_cast<volatile const int*>(p.ga.epochs + blockIdx.x) + 1;
        g_half = (long long)(g_epoch & 1) * p.ga.out_stride;
    }
#pragma unroll 1
    for (int m = 0; m < MM; ++m) {
        const float* xr = p.x + (int64_t)m * p.ldx;
        float* xd = xs + m * p.k_pad;
        for (int base = 0; base < p.k_pad; base += 8 * (int)blockDim.x) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int kk = base + (int)threadIdx.x + i * (int)blockDim.x;
                v[i] = kk < p.k ? __ldcg(xr + kk) : 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int kk = base + (int)threadIdx.x + i * (int)blockDim.x;
                if (kk < p.k_pad) xd[xperm(kk)] = v[i];
            }
        }
    }
    __syncthreads();
    if (GATHER && comm_failed) {
        // Let this warp's copies land before leaving (bounded).
        if (lane32 == 0)
            for (int j = 0; j < p.d && j < items; ++j)
                mbar_wait(bars + j * 8, 0u, nullptr, kWaitBudget);
        return;
    }

    const int nbf = p.k / kBlock;  // full blocks
    const int cfull = nbf / 4;     // chunks of 4 full blocks
    const int rem_blocks = nbf - cfull * 4;
    const int nchunks = cfull + (rem_blocks ? 1 : 0);

    const unsigned long long nz = f2pack(p.zero_neg, p.zero_neg);
    float t[MM][R];
#pragma unroll
    for (int m = 0; m < MM; ++m)
#pragma unroll
        for (int i = 0; i < R; ++i) t[m][i] = 0.0f;

    int stop = items;  // first item not consumed (== items on the normal path)
    // item i = (unit index uu, segment g) in slot i mod d with phase parity;
    // (uu2, g2) tracks item i + d, the next one issued into the same slot.
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
        const uint8_t* sq = my_slots + (size_t)slot * slot_bytes + rsub * p.sc * CB + lane * (CB / 8);
        const uint8_t* ss = my_slots + (size_t)slot * slot_bytes + kUnitRows * p.sc * CB + rsub * p.sc * 16;
        const int qstride = p.sc * CB, sstride = p.sc * 16;
        const int c0 = g * p.sc;
        const int c1 = min(c0 + p.sc, nchunks);
        const int cf = min(c1, cfull);  // chunks made of four full blocks
        const float* xc = xs + c0 * kChunk;
#pragma unroll 1
        for (int c = 0; c < cf - c0; ++c) {
            chunk_update<MM, R, true, Q4>(xc + c * kChunk, p.k_pad, lane, sq + c * CB, qstride, ss + c * 16, sstride,
                                      nz, t, 4);
        }
        if (cf < c1) {  // the chunk holding the last (1..3) full blocks
            chunk_update<MM, R, false, Q4>(xs + cf * kChunk, p.k_pad, lane, sq + (cf - c0) * CB, qstride,
                                       ss + (cf - c0) * 16, sstride, nz, t, rem_blocks);
        }
        __syncwarp();
        if (i + p.d < items) {
            fence_proxy_async_smem();
            __syncwarp();
            issue(uu2, g2, slot);
        }
        if (++g2 == p.nseg) { g2 = 0; ++uu2; }
        const bool unit_done = g == p.nseg - 1;
        if (++g == p.nseg) { g = 0; ++uu; }
        if (++slot == p.d) { slot = 0; parity ^= 1u; }
        if (unit_done) {
#pragma unroll
            for (int m = 0; m < MM; ++m)
#pragma unroll
                for (int i = 0; i < R; ++i) {
                    float v = t[m][i];
                    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
                    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
                    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
                    t[m][i] = v;
                }
            if (lane == 0) {
                const GemvGroup& W = p.grp[unit_group(p, u)];
                const int lu = u - W.ubase;
#pragma unroll
                for (int i = 0; i < R; ++i) {
                    const int row = kUnitRows * lu + rsub + i;
                    if (row >= W.rows) break;
                    if (p.k > nbf * kBlock) {
                        // Ragged tail: sequential scalar sum times the last block's scale.
                        const uint8_t* qr = W.q + (int64_t)row * (p.k_pad / kChunk) * CB;
                        const float st = W.s[(int64_t)row * p.nb_pad + nbf];
#pragma unroll
                        for (int m = 0; m < MM; ++m) {
                            float acc = 0.0f;
                            for (int kk = nbf * kBlock; kk < p.k; ++kk) {
                                const float qf =
                                    Q4 ? (float)((int)((qr[packed_offset_q4(kk)] >> packed_shift_q4(kk)) & 0xF) - 8)
                                       : (float)(int8_t)qr[packed_offset(kk)];
                                acc = __fadd_rn(acc, __fmul_rn(xs[m * p.k_pad + xperm(kk)], qf));
                            }
                            t[m][i] = __fadd_rn(t[m][i], __fmul_rn(acc, st));
                        }
                    }
                    if (GATHER) {
                        // one word per rank: this call's epoch with the value
                        const unsigned long long word =
                            ((unsigned long long)(uint32_t)g_epoch << 32) | __float_as_uint(t[0][i]);
#pragma unroll 1
                        for (int r = 0; r < p.ga.nranks; ++r)
                            st_relaxed_sys_u64(p.ga.peer_slots[r] + g_half + p.ga.col0 + row, word);
                    } else {
#pragma unroll
                        for (int m = 0; m < MM; ++m) W.y[(int64_t)m * W.ldy + row] = t[m][i];
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < MM; ++m)
#pragma unroll
                for (int i = 0; i < R; ++i) t[m][i] = 0.0f;
        }
    }
    // Drain after a give-up: items [stop, stop + d) were issued but not
    // consumed; their copies must land before this warp's slots are released.
    if (lane32 == 0)
        for (int j = stop; j < stop + p.d && j < items; ++j)
            mbar_wait(bars + (j % p.d) * 8, (uint32_t)((j / p.d) & 1), nullptr, kWaitBudget);
}

struct Plan {
    int mm, r, sc, nseg, d, nwarps, ctas, xs_bytes, smem, tma;
};

// Rows per thread (measured on B200, M = 1): R = 2 pays from ~48 rows per SM
// (lm_head 151936 x 2560: 98.5 us vs 115 us at R = 1; 9728 x 2560: 10.3 vs
// 12.1 us); below that R = 1 keeps enough warps per SM and two CTAs per SM
// (config 1, 6144 x 2048: 5.5 us vs 8.2 us at R = 2). R = 4 was slower than
// R = 2 everywhere. M > 1 keeps R = 1.
// M > 1: two rows per thread halve the activations' shared-memory traffic,
// which bounds the one-row form (per activation row and 128-element chunk a
// warp issues ~22 instructions against four 128-bit activation loads, 16
// shared-memory wavefronts). QLM_GEMV_R2=0 keeps one row per thread (for
// comparisons).
int pick_rows_per_thread(int mm, int rows, int sm_count) {
    static const bool r2_multi = [] {
        const char* e = std::getenv("QLM_GEMV_R2");
        return !(e && e[0] == '0');
    }();
    if (mm > 1 && !r2_multi) return 1;
    return rows / sm_count >= 48 ? 2 : 1;
}

// rows: the rows the launch covers (for several weights, the sum of their
// rows each rounded up to whole units of the forced R).
bool make_plan(int mm, int rows, int k, int sm_count, Plan* pl, int force_r = 0, bool q4 = false) {
    const int k_pad = packed_k(k);
    const int nck = k_pad / kChunk;
    const int max_warps = mm == 1 ? 12 : (force_r == 2 || pick_rows_per_thread(mm, rows, sm_count) == 2 ? 12 : 16);
    pl->mm = mm;
    pl->r = force_r ? force_r : pick_rows_per_thread(mm, rows, sm_count);
    const int unit_rows = 4 * pl->r;
    pl->sc = seg_chunks(nck);
    pl->nseg = (nck + pl->sc - 1) / pl->sc;
    const int slot_bytes = q4 ? slot_stride<true>(pl->sc, unit_rows) : slot_stride<false>(pl->sc, unit_rows);
    pl->xs_bytes = round_up(mm * k_pad * 4, 128);
    const int units = (rows + unit_rows - 1) / unit_rows;
    pl->ctas = units < sm_count ? units : sm_count;
    const int upc = (units + pl->ctas - 1) / pl->ctas;
    // Short kernels: everything in flight at once within ~110 KB, leaving room
    // for the next kernel's CTA on the same SM. Long ones: up to 200 KB.
    const int small_budget = 110 * 1024, big_budget = 200 * 1024;
    int max_slots = (small_budget - pl->xs_bytes - 1024) / slot_bytes;
    pl->tma = 0;
    if (max_slots >= 1 && upc <= max_warps && upc * pl->nseg <= max_slots) {
        pl->nwarps = upc;
        pl->d = pl->nseg;
    } else {
        pl->tma = 1;
        max_slots = (big_budget - pl->xs_bytes - 1024) / slot_bytes;
        if (max_slots < 1) return false;
        pl->nwarps = upc < max_warps ? upc : max_warps;
        if (pl->nwarps > max_slots) pl->nwarps = max_slots;
        pl->d = max_slots / pl->nwarps;
        if (pl->d > 4) pl->d = 4;
        const int items_per_warp = ((upc + pl->nwarps - 1) / pl->nwarps) * pl->nseg;
        if (pl->d > items_per_warp) pl->d = items_per_warp;
    }
    pl->smem = 128 + pl->xs_bytes + pl->nwarps * pl->d * (slot_bytes + 8) + 16;
    return true;
}

template <int MM, int R, bool Q4>
cudaError_t launch_mm(const GemvParams& p0, const Plan& pl, cudaStream_t stream, bool pdl) {
    static bool attr_set[4][64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const bool gather = p0.ga.nranks > 0;
    auto kern = MM == 1 && gather ? (pl.tma ? gemv_kernel<1, R, true, Q4, true> : gemv_kernel<1, R, true, Q4, false>)
                                  : (pl.tma ? gemv_kernel<MM, R, false, Q4, true> : gemv_kernel<MM, R, false, Q4, false>);
    const int gi = (gather ? 2 : 0) + (pl.tma ? 1 : 0);
    if (!attr_set[gi][dev]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 224 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[gi][dev] = true;
    }
    GemvParams p = p0;
    int ub = 0;
    for (int g = 0; g < p.ngroup; ++g) {
        p.grp[g].ubase = ub;
        ub += (p.grp[g].rows + 4 * R - 1) / (4 * R);
    }
    p.units = ub;
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

bool gemv_supported(int mm, int rows, int k, int sm_count, bool q4) {
    Plan pl;
    return make_plan(mm, rows, k, sm_count, &pl, 0, q4);
}

namespace {

// QLM_GEMV_DECODE=0 selects the single-role kernel for every M = 1 launch,
// =2 the producer/consumer form wherever its plan fits (for comparisons); by
// default the producer/consumer form takes the small matrices (below).
int decode_form_mode() {
    static const int mode = [] {
        const char* e = std::getenv("QLM_GEMV_DECODE");
        return e && e[0] == '0' ? 0 : e && e[0] == '2' ? 2 : 1;
    }();
    return mode;
}

template <bool Q4>
cudaError_t launch_mm_any(int mm, const GemvParams& p, const Plan& pl, cudaStream_t stream, bool pdl) {
    switch (mm) {
        case 1: return pl.r == 2 ? launch_mm<1, 2, Q4>(p, pl, stream, pdl) : launch_mm<1, 1, Q4>(p, pl, stream, pdl);
        case 2: return pl.r == 2 ? launch_mm<2, 2, Q4>(p, pl, stream, pdl) : launch_mm<2, 1, Q4>(p, pl, stream, pdl);
        case 3: return pl.r == 2 ? launch_mm<3, 2, Q4>(p, pl, stream, pdl) : launch_mm<3, 1, Q4>(p, pl, stream, pdl);
        case 4: return pl.r == 2 ? launch_mm<4, 2, Q4>(p, pl, stream, pdl) : launch_mm<4, 1, Q4>(p, pl, stream, pdl);
        case 5: return pl.r == 2 ? launch_mm<5, 2, Q4>(p, pl, stream, pdl) : launch_mm<5, 1, Q4>(p, pl, stream, pdl);
        case 6: return pl.r == 2 ? launch_mm<6, 2, Q4>(p, pl, stream, pdl) : launch_mm<6, 1, Q4>(p, pl, stream, pdl);
        case 7: return pl.r == 2 ? launch_mm<7, 2, Q4>(p, pl, stream, pdl) : launch_mm<7, 1, Q4>(p, pl, stream, pdl);
        case 8: return pl.r == 2 ? launch_mm<8, 2, Q4>(p, pl, stream, pdl) : launch_mm<8, 1, Q4>(p, pl, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_gemv_grouped(const float* x, int64_t ldx, int mm, const GemvWeight* ws, int nw, int k,
                                int* status, int sm_count, cudaStream_t stream, bool pdl, const GatherArgs* gather,
                                bool q4) {
    if (nw < 1 || nw > kMaxGroup || (gather && (mm != 1 || nw != 1))) return cudaErrorInvalidValue;
    int rows_total = 0;
    for (int g = 0; g < nw; ++g) {
        if (ws[g].rows < 1 || !ws[g].maps) return cudaErrorInvalidValue;
        rows_total += ws[g].rows;
    }
    // M = 1: the producer/consumer form serves matrices of fewer than 32 rows
    // per SM, where one thread per (row, lane) would leave most of the SM idle;
    // measured on B200 (CUDA graph, rotating weights): [512,2560] 3.2 vs 8.0 us,
    // [2560,9728] 12.0 vs 16.1 us, [1024,3584] 3.6 vs 7.0 us, while from ~40 rows
    // per SM the single-role kernel is faster (config 1 [6144,2048] 5.6 vs
    // 6.9 us, lm_head [151936,2560] 76 vs 107 us).
    const int dmode = decode_form_mode();
    if (mm == 1 && !gather && dmode != 0 && (dmode == 2 || rows_total < 32 * sm_count) &&
        gemv_decode_supported(rows_total, nw, k, sm_count, q4))
        return launch_gemv_decode(x, ws, nw, k, status, sm_count, stream, pdl, q4);
    const int r = pick_rows_per_thread(mm, rows_total, sm_count);
    int rows_eff = 0;  // whole units per weight
    for (int g = 0; g < nw; ++g) rows_eff += round_up(ws[g].rows, 4 * r);
    Plan pl;
    if (!make_plan(mm, rows_eff, k, sm_count, &pl, r, q4)) return cudaErrorInvalidValue;
    GemvParams p{};
    if (gather) p.ga = *gather;
    p.x = x;
    p.ldx = ldx;
    p.zero_neg = -0.0f;
    for (int g = 0; g < nw; ++g) {
        if (ws[g].maps->sc != pl.sc || !ws[g].maps->dev) return cudaErrorInvalidValue;  // built for another k
        p.grp[g].mq = ws[g].maps->dev + (r - 1);
        p.grp[g].ms = ws[g].maps->dev + 2 + (r - 1);
        p.grp[g].q = ws[g].q;
        p.grp[g].s = ws[g].s;
        p.grp[g].y = ws[g].y;
        p.grp[g].ldy = ws[g].ldy;
        p.grp[g].rows = ws[g].rows;
    }
    p.ngroup = nw;
    p.status = status;
    p.k = k;
    p.k_pad = packed_k(k);
    p.nb_pad = p.k_pad / kBlock;
    return q4 ? launch_mm_any<true>(mm, p, pl, stream, pdl) : launch_mm_any<false>(mm, p, pl, stream, pdl);
}

cudaError_t launch_gemv_exact(const float* x, int64_t ldx, int mm, const uint8_t* q, const float* s,
                              const GemvMaps& maps, int rows, int k, float* y, int64_t ldy, int* status, int sm_count,
                              cudaStream_t stream, bool pdl, const GatherArgs* gather, bool q4) {
    const GemvWeight w{q, s, &maps, rows, y, ldy};
    return launch_gemv_grouped(x, ldx, mm, &w, 1, k, status, sm_count, stream, pdl, gather, q4);
}

cudaError_t gemv_make_maps(const uint8_t* q, const float* s, int rows, int k, bool q4, GemvMaps* out) {
    auto enc = tensor_map_encoder();
    if (!enc) return cudaErrorNotSupported;
    const int nck = packed_k(k) / kChunk;
    const int cb = q4 ? 64 : 128;
    out->sc = seg_chunks(nck);
    // Codes as 8-byte elements: a segment of sc chunks is sc * cb / 8 <= 128
    // elements, one box row. Scales: 4 per chunk.
    for (int r = 1; r <= 2; ++r) {
        const cuuint32_t ur = 4 * r;
        const cuuint32_t estr[2] = {1, 1};
        {
            const cuuint64_t dims[2] = {(cuuint64_t)nck * cb / 8, (cuuint64_t)rows};
            const cuuint64_t strides[1] = {(cuuint64_t)nck * cb};
            const cuuint32_t box[2] = {(cuuint32_t)(out->sc * cb / 8), ur};
            if (enc(&out->q[r - 1], CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(q), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                return cudaErrorInvalidValue;
        }
        {
            const cuuint64_t dims[2] = {(cuuint64_t)nck * 4, (cuuint64_t)rows};
            const cuuint64_t strides[1] = {(cuuint64_t)nck * 16};
            const cuuint32_t box[2] = {(cuuint32_t)(out->sc * 4), ur};
            if (enc(&out->s[r - 1], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(s), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                return cudaErrorInvalidValue;
        }
    }
    static_assert(offsetof(GemvMaps, s) == 2 * sizeof(CUtensorMap), "q and s descriptors must be contiguous");
    cudaError_t e = cudaMalloc(&out->dev, 4 * sizeof(CUtensorMap));
    if (e != cudaSuccess) return e;
    e = cudaMemcpy(out->dev, out->q, 4 * sizeof(CUtensorMap), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(out->dev);
        out->dev = nullptr;
    }
    return e;
}

namespace {

constexpr int kCollectThreads = 256;

// Second half of the fused all-gather: the GEMV of a call stores its rows'
// words into every rank's exchange buffer and ends; this kernel, next in the
// stream, waits (bounded) until every word of the gathered row in this rank's
// buffer carries the call's epoch, copies the values into y and advances the
// epoch words, so no GEMV ends in a cross-GPU barrier. The trigger comes
// first: the next kernel (typically the next GEMV, which waits for this one's
// completion before it reads anything) can then take an SM beside this call's
// GEMV and issue its weight copies during that GEMV's compute and this
// kernel's wait, as consecutive GEMVs do on one GPU.
__global__ void __launch_bounds__(kCollectThreads) gather_collect_kernel(const __grid_constant__ GatherArgs ga,
                                                                         float* __restrict__ y, int* status) {
    using namespace sm100;
    constexpr int kBatch = 4;  // words of a thread in flight at once
    pdl_launch_dependents();
    pdl_wait();  // this call's GEMV has completed (its own stores are issued)
    const int failed = ld_relaxed_sys_i32(status);
    const int e = *reinterpret_cast<volatile const int*>(ga.epochs + blockIdx.x) + 1;
    if (failed) return;  // the GEMV returned at entry; nothing was stored
    const unsigned long long* mine = ga.peer_slots[ga.rank] + (long long)(e & 1) * ga.out_stride;
    const long long t0 = globaltimer_ns();
    const int stride = (int)(gridDim.x * blockDim.x);
    for (int base = (int)(blockIdx.x * blockDim.x + threadIdx.x); base < ga.n_total; base += kBatch * stride) {
        unsigned long long v[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int i = base + u * stride;
            v[u] = i < ga.n_total ? ld_relaxed_sys_u64(mine + i) : 0ull;
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int i = base + u * stride;
            if (i >= ga.n_total) break;
            while ((int)(v[u] >> 32) != e) {
                if (globaltimer_ns() - t0 > ga.wait_ns) {
                    atomicCAS(status, 0, kStatusGatherTimeout);
                    break;
                }
                __nanosleep(32);
                v[u] = ld_relaxed_sys_u64(mine + i);
            }
            if ((int)(v[u] >> 32) == e) y[i] = __uint_as_float((uint32_t)v[u]);
        }
    }
    __syncthreads();  // every thread's wait has ended (or recorded a give-up)
    // CTA b advances words b, b + grid, ... (see GatherArgs). After a give-up
    // the communicator is failed and its epoch words are not used again.
    if (threadIdx.x == 0 && ld_relaxed_sys_i32(status) == 0)
        for (int sl = (int)blockIdx.x; sl < ga.nepochs; sl += (int)gridDim.x)
            reinterpret_cast<volatile int*>(ga.epochs)[sl] = e;
}

}  // namespace

cudaError_t launch_gather_collect(const GatherArgs& ga, float* y, int* status, int sm_count, cudaStream_t stream,
                                  bool pdl) {
    if (ga.nranks <= 0 || ga.n_total <= 0 || !status || !ga.epochs) return cudaErrorInvalidValue;
    int ctas = (ga.n_total + kCollectThreads - 1) / kCollectThreads;
    if (ctas > sm_count) ctas = sm_count;
    if (ctas > ga.nepochs) ctas = ga.nepochs;
    if (ctas < 1) ctas = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3((unsigned)kCollectThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gather_collect_kernel, ga, y, status);
}

}  // namespace qlm
