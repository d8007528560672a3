// qlm_gemv_decode.cu — bit-exact int8/int4 decode GEMV (M = 1) for sm_100a,
// in producer/consumer form.
//
// Same arithmetic as qlm_gemv.cu (QuickLM src/ops/math_ops.cpp:414-553): for
// output row n, reference lane l in [0, 8) and 32-block b,
//   p_j   = x[32b+8j+l] * q[32b+8j+l]                j = 0..3
//   bs(b) = (p_0 + p_1) + (p_2 + p_3)
//   t_l   = fma(bs(b), s[b], t_l)   for b ascending, t_l from +0
//   y     = ((t_0+t_4) + (t_1+t_5)) + ((t_2+t_6) + (t_3+t_7))
// (+ the ragged scalar tail), so every output is bit-identical to the CPU
// engine's. What differs is how the work is spread over the SM.
//
// The block sums bs(b) carry almost all of the work (conversion, products,
// three adds per 4 elements) and are independent of one another; only the FMA
// chain over b is ordered. So the kernel splits them:
//   * producer warps: thread = (128-element chunk c, lane l). Its 16
//     activations x[c*128 + 32bb + 8j + l] sit in registers for the whole
//     kernel, so weights are the only operand it reads: one 128-bit shared
//     load per row gives its 16 codes (the packed layout puts a lane's bytes of
//     a chunk side by side), from which it forms the four block sums of the
//     chunk and stores them back to shared memory. A warp covers 4 chunks (8
//     with two chunks per thread) of a row; S warps cover the row.
//   * chain warps: thread = (row of a 4-row group, lane l): runs the ordered
//     FMA chain over the staged block sums of all chunks (one 128-bit shared
//     load of sums and one of scales per chunk), then the fixed 8 -> 1 tree.
// Producers and chain warps hand 4-row groups over through a ring of shared
// memory slots per "pipe" (S producer warps + C chain warps), completing on
// mbarriers (landed: the group's codes and scales arrived; full: the S
// producer warps stored its block sums).
//
// Memory: a group's codes (4 consecutive rows) and scales are contiguous in
// HBM, so each arrives in its slot with two bulk copies issued by one lane of
// the chain warp: the ring of D slots per pipe is filled before the
// programmatic-dependent-launch wait, and a chain warp refills a slot as soon
// as it has read it. Groups beyond the ring are requested into L2 ahead of
// time (cp.async.bulk.prefetch.L2). So in a stream or CUDA graph the weights
// of this GEMV stream from HBM while the previous kernel computes. Waits are
// bounded: on give-up the kernel records a status code, raises a CTA-wide
// abort flag and stops.
#include "qlm_device.cuh"
#include "qlm_kernels.h"
#include "qlm_sm100.cuh"

namespace qlm {
namespace {

constexpr long long kDecWaitBudget = 4000000000LL;  // ~2 s of SM clock
constexpr int kDecStatusTimeout = 0x203;
constexpr int kDecMaxWarps = 16;
// Slot bytes per 128-element chunk of a 4-row group: codes overwritten in
// place by the block sums (int8), or codes + sums (int4); then the scales.
constexpr int kDecSlotPerChunkI8 = 4 * 128 + 4 * 16;
constexpr int kDecSlotPerChunkI4 = 4 * 64 + 4 * 128 + 4 * 16;

struct DecWeight {
    const uint8_t* q;  // packed codes [rows][row_bytes]
    const float* s;    // scales [rows][nb_pad]
    float* y;
    int rows;
    int gbase;         // first 4-row group of this weight in the launch
};

struct DecParams {
    const float* x;
    float zero_neg;    // -0.0f: the product addend (see qlm_gemv.cu)
    DecWeight w[kMaxGroup];
    int nw;
    int* status;
    int k, nb_pad, nck;
    int row_bytes;     // packed code bytes per row
    int cta_q, cta_r;  // groups per CTA: CTA b owns [b*q + min(b, r), +q + (b < r))
    int S, P, C, D;    // producer warps per pipe, pipes, chain warps per pipe, slots per pipe
    int slot_bytes;
    int ahead;         // L2 prefetch distance, in groups of the pipe
};

__device__ __forceinline__ int dec_weight_of(const DecParams& p, int g) {
    int w = 0;
    for (int i = 1; i < p.nw; ++i)
        if (g >= p.w[i].gbase) w = i;
    return w;
}

__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ void sts_u64x2(uint32_t addr, unsigned long long a, unsigned long long b) {
    asm volatile("st.shared.v2.u64 [%0], {%1, %2};" ::"r"(addr), "l"(a), "l"(b) : "memory");
}

// The four block sums of one chunk for this lane: a = the lane's codes of the
// chunk (int8: 16 bytes, byte 4bb + j = block bb, step j; int4: 8 bytes,
// bytes 0..3 blocks 0/1 in the low/high nibble, bytes 4..7 blocks 2/3), xp[h][j]
// = (x of block 2h, x of block 2h+1) at step j. Returns (bs0, bs1) and
// (bs2, bs3). Each paired op is the reference's scalar op for both blocks.
template <bool Q4>
__device__ __forceinline__ void chunk_block_sums(const uint4& a, const unsigned long long (&xp)[2][4],
                                                 unsigned long long nz, unsigned long long& b01,
                                                 unsigned long long& b23) {
    uint32_t w4[4];
    if (Q4) {
        w4[0] = a.x & 0x0F0F0F0Fu;
        w4[1] = (a.x >> 4) & 0x0F0F0F0Fu;
        w4[2] = a.y & 0x0F0F0F0Fu;
        w4[3] = (a.y >> 4) & 0x0F0F0F0Fu;
    } else {
        w4[0] = a.x ^ 0x80808080u;
        w4[1] = a.y ^ 0x80808080u;
        w4[2] = a.z ^ 0x80808080u;
        w4[3] = a.w ^ 0x80808080u;
    }
    // (2^23 + bias) x 2: the byte sits in the mantissa of 2^23; int8 bytes are
    // biased by 128 above, int4 nibbles carry QuickLM's +8.
    const unsigned long long bias = Q4 ? 0x4B0000084B000008ull : 0x4B0000804B000080ull;
    unsigned long long out[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        unsigned long long pr[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const unsigned long long qp =
                f2sub(u2pack(__byte_perm(w4[2 * h], 0x4B000000u, 0x7540u | (uint32_t)j),
                             __byte_perm(w4[2 * h + 1], 0x4B000000u, 0x7540u | (uint32_t)j)),
                      bias);
            pr[j] = f2fma(xp[h][j], qp, nz);
        }
        out[h] = f2add(f2add(pr[0], pr[1]), f2add(pr[2], pr[3]));
    }
    b01 = out[0];
    b23 = out[1];
}

// CPT: chunks per producer thread (1, or 2 for long rows; registers hold
// CPT x 16 activations). A slot holds one 4-row group: the rows' packed codes
// as they lie in HBM (4 x row_bytes), overwritten in place by the block sums
// for int8 (a lane's 16 code bytes of a chunk become its float4 of sums at the
// same address; int4 codes are half as wide, so their sums go to a separate
// area), then the rows' scales (4 x nck float4). Shared memory: P*D slots,
// then the landed and full mbarriers and the last group issued into each
// slot (P*D each), the abort flag, and 512 bytes per producer warp that lanes
// past a row's end compute into (so the loop has no divergent branch).
template <bool Q4, int CPT>
__global__ void __launch_bounds__(CPT == 1 ? 512 : 384, 2) gemv_dec_kernel(const __grid_constant__ DecParams p) {
    using namespace sm100;
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int CB = Q4 ? 64 : 128;  // code bytes per row per chunk
    const int warp = threadIdx.x >> 5, lane32 = threadIdx.x & 31;
    const int nprod = p.S * p.P;
    const int b = (int)blockIdx.x;
    const int g_begin = b * p.cta_q + min(b, p.cta_r);
    const int g_count = p.cta_q + (b < p.cta_r ? 1 : 0);
    const int nslots = p.P * p.D;
    uint8_t* slots = smem;
    const uint32_t landed0 = smem_u32(smem + (size_t)nslots * p.slot_bytes);
    const uint32_t full0 = landed0 + nslots * 8;
    int* issued = reinterpret_cast<int*>(smem + (size_t)nslots * p.slot_bytes + nslots * 16);
    volatile int* abort_flag = issued + nslots;
    // Per producer warp, 512 bytes that lanes past a row's end compute into.
    uint8_t* dummy_base = smem + (((size_t)nslots * p.slot_bytes + nslots * 20 + 4 + 15) & ~(size_t)15);
    const int codes_bytes = 4 * p.row_bytes;                // codes of a group
    const int bs_off = Q4 ? codes_bytes : 0;                // block sums
    const int sc_off = Q4 ? codes_bytes + 512 * p.nck : codes_bytes;  // scales

    if (threadIdx.x == 0) {
        for (int i = 0; i < nslots; ++i) {
            mbar_init(landed0 + i * 8, 1);
            mbar_init(full0 + i * 8, 32 * p.S);
            issued[i] = -1;
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();

    if (warp < nprod) {
        // ---------------- producer: block sums of chunks cj[] of each row ----
        const int sw = warp % p.S, pp = warp / p.S;
        const int l = lane32 & 7, cl = lane32 >> 3;
        const int n = g_count > pp ? (g_count - pp + p.P - 1) / p.P : 0;  // groups of this pipe
        int cj[CPT];
        bool vj[CPT];
        uint32_t loff[CPT], soff[CPT];  // this lane's code / block-sum bytes of row 0 within a slot
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
            cj[j] = sw * 4 * CPT + cl + 4 * j;
            vj[j] = cj[j] < p.nck;
            loff[j] = (uint32_t)(cj[j] * CB + l * (CB / 8));
            soff[j] = (uint32_t)(bs_off + (cj[j] * 8 + l) * 16);
        }
        const uint32_t rs_ld = (uint32_t)(p.nck * CB), rs_st = (uint32_t)(p.nck * 128);  // per row of a group
        const uint32_t dummy = smem_u32(dummy_base) + (uint32_t)(warp * 512 + lane32 * 16);
        pdl_launch_dependents();
        pdl_wait();
        // L2 loads of x, not the read-only path: this kernel may start while
        // its producer still writes x (see the staging in qlm_gemv.cu).
        unsigned long long xp[CPT][2][4];
#pragma unroll
        for (int j = 0; j < CPT; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const int k0 = cj[j] * kChunk + (2 * h) * kBlock + jj * 8 + l, k1 = k0 + kBlock;
                    const float x0 = vj[j] && k0 < p.k ? __ldcg(p.x + k0) : 0.0f;
                    const float x1 = vj[j] && k1 < p.k ? __ldcg(p.x + k1) : 0.0f;
                    xp[j][h][jj] = f2pack(x0, x1);
                }
        const unsigned long long nz = f2pack(p.zero_neg, p.zero_neg);
        // Group i sits in slot i % D of the pipe, phase (i / D) & 1; tracked
        // incrementally.
        int si = 0;
        uint32_t par = 0;
        for (int i = 0; i < n; ++i) {
            const int slot = pp * p.D + si;
            if (++si == p.D) si = 0;
            const uint32_t this_par = par;
            if (si == 0) par ^= 1u;
            const bool ok = mbar_wait(landed0 + slot * 8, this_par, abort_flag, kDecWaitBudget);
            if (!__all_sync(0xffffffffu, ok)) {
                *abort_flag = 1;
                if (lane32 == 0 && p.status) atomicCAS(p.status, 0, kDecStatusTimeout);
                break;
            }
            const uint32_t sb = smem_u32(slots + (size_t)slot * p.slot_bytes);
            // Branch-free: a lane whose chunk is past the row's end computes on
            // its private dummy line instead (its result is never read). The
            // rows' codes are loaded ahead of their arithmetic (all four rows
            // with one chunk per thread, two ahead with two), so the loads of
            // later rows are in flight while earlier rows compute.
            constexpr int PRE = CPT == 1 ? 4 : 2;
            uint4 cw[4][CPT];
            auto load_row = [&](int r) {
#pragma unroll
                for (int j = 0; j < CPT; ++j) {
                    const uint32_t la = vj[j] ? sb + r * rs_ld + loff[j] : dummy;
                    if (Q4) {
                        asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(cw[r][j].x), "=r"(cw[r][j].y) : "r"(la));
                        cw[r][j].z = cw[r][j].w = 0u;
                    } else {
                        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                                     : "=r"(cw[r][j].x), "=r"(cw[r][j].y), "=r"(cw[r][j].z), "=r"(cw[r][j].w)
                                     : "r"(la));
                    }
                }
            };
#pragma unroll
            for (int r = 0; r < PRE; ++r) load_row(r);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                if (r + PRE < 4) load_row(r + PRE);
#pragma unroll
                for (int j = 0; j < CPT; ++j) {
                    const uint32_t sa = vj[j] ? sb + r * (Q4 ? rs_st : rs_ld) + (Q4 ? soff[j] : loff[j]) : dummy;
                    unsigned long long b01, b23;
                    chunk_block_sums<Q4>(cw[r][j], xp[j], nz, b01, b23);
                    sts_u64x2(sa, b01, b23);
                }
            }
            // This slot's next writer is the copy engine (after the chain warp
            // has read it): order the generic-proxy accesses first.
            fence_proxy_async_smem();
            __syncwarp();
            mbar_arrive(full0 + slot * 8);
        }
        return;
    }

    // ---------------- chain warps: ordered FMA chain + 8 -> 1 tree ------------
    const int cwi = warp - nprod;
    const int pp = cwi / p.C, cc = cwi % p.C;
    const int n = g_count > pp ? (g_count - pp + p.P - 1) / p.P : 0;
    const int ri = lane32 >> 3, l = lane32 & 7;
    // Group i of this pipe: its weight, first row and row count.
    auto group_rows = [&](int i, const DecWeight*& W, int& row0, int& nr) {
        const int g = g_begin + pp + i * p.P;
        W = &p.w[dec_weight_of(p, g)];
        row0 = (g - W->gbase) * 4;
        nr = min(4, W->rows - row0);
    };
    // Codes and scales of group i into pipe slot `slot` (lane 0 only).
    auto issue = [&](int i, int slot) {
        const DecWeight* W;
        int row0, nr;
        group_rows(i, W, row0, nr);
        uint8_t* sb = slots + (size_t)slot * p.slot_bytes;
        const uint32_t cbytes = (uint32_t)(nr * p.row_bytes), sbytes = (uint32_t)(nr * p.nb_pad * 4);
        const uint32_t bar = landed0 + slot * 8;
        issued[slot] = i;
        mbar_arrive_expect_tx(bar, cbytes + sbytes);
        bulk_copy_g2s(smem_u32(sb), W->q + (int64_t)row0 * p.row_bytes, cbytes, bar);
        bulk_copy_g2s(smem_u32(sb + sc_off), W->s + (int64_t)row0 * p.nb_pad, sbytes, bar);
    };
    auto prefetch = [&](int i) {
        const DecWeight* W;
        int row0, nr;
        group_rows(i, W, row0, nr);
        prefetch_l2_bulk(W->q + (int64_t)row0 * p.row_bytes, (uint32_t)(nr * p.row_bytes));
        prefetch_l2_bulk(W->s + (int64_t)row0 * p.nb_pad, (uint32_t)(nr * p.nb_pad * 4));
    };
    // Before the dependency wait: fill the ring (group i by chain warp i % C)
    // and ask L2 for the groups after it.
    if (lane32 == 0) {
        for (int i = cc; i < n && i < p.D; i += p.C) issue(i, pp * p.D + i);
        for (int i = p.D + cc; i < n && i < p.D + p.ahead; i += p.C) prefetch(i);
    }
    pdl_launch_dependents();
    pdl_wait();
    const int nbf = p.k / kBlock;  // full blocks
    const int cfull = nbf / 4;     // chunks of four full blocks
    const int rem_blocks = nbf - cfull * 4;
    // This warp's groups i = cc, cc + C, ... sit in slots i % D (D is a
    // multiple of C), phase (i / D) & 1; tracked incrementally.
    int si = cc;
    uint32_t par = 0;
    for (int i = cc; i < n; i += p.C) {
        const int slot = pp * p.D + si;
        const uint32_t this_par = par;
        si += p.C;
        if (si >= p.D) {
            si -= p.D;
            par ^= 1u;
        }
        const bool ok = mbar_wait(full0 + slot * 8, this_par, abort_flag, kDecWaitBudget);
        if (!__all_sync(0xffffffffu, ok)) {
            *abort_flag = 1;
            if (lane32 == 0 && p.status) atomicCAS(p.status, 0, kDecStatusTimeout);
            break;
        }
        const uint32_t sb = smem_u32(slots + (size_t)slot * p.slot_bytes);
        const uint32_t bsp = sb + bs_off + (ri * p.nck * 8 + l) * 16;  // + c * 128 per chunk
        const uint32_t scp = sb + sc_off + ri * p.nck * 16;             // + c * 16 per chunk
        float t = 0.0f;
#pragma unroll 4
        for (int c = 0; c < cfull; ++c) {
            const float4 v = lds_f4(bsp + c * 128), s = lds_f4(scp + c * 16);
            t = __fmaf_rn(v.x, s.x, t);
            t = __fmaf_rn(v.y, s.y, t);
            t = __fmaf_rn(v.z, s.z, t);
            t = __fmaf_rn(v.w, s.w, t);
        }
        if (rem_blocks) {
            const float4 v = lds_f4(bsp + cfull * 128), s = lds_f4(scp + cfull * 16);
            t = __fmaf_rn(v.x, s.x, t);
            if (rem_blocks > 1) t = __fmaf_rn(v.y, s.y, t);
            if (rem_blocks > 2) t = __fmaf_rn(v.z, s.z, t);
        }
        // The slot is read: refill it with group i + D (after ordering this
        // warp's reads before the copy engine's writes).
        fence_proxy_async_smem();
        __syncwarp();
        if (lane32 == 0) {
            if (i + p.D < n) issue(i + p.D, slot);
            if (i + p.D + p.ahead < n) prefetch(i + p.D + p.ahead);
        }
        t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 4));
        t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 1));
        t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
        if (l == 0) {
            const DecWeight* W;
            int row0, nr;
            group_rows(i, W, row0, nr);
            if (ri < nr) {
                const int row = row0 + ri;
                if (p.k > nbf * kBlock) {
                    // Ragged tail: sequential scalar sum times the last block's scale.
                    const uint8_t* qr = W->q + (int64_t)row * p.row_bytes;
                    float acc = 0.0f;
                    for (int kk = nbf * kBlock; kk < p.k; ++kk) {
                        const float qf = Q4 ? (float)((int)((qr[packed_offset_q4(kk)] >> packed_shift_q4(kk)) & 0xF) - 8)
                                            : (float)(int8_t)qr[packed_offset(kk)];
                        acc = __fadd_rn(acc, __fmul_rn(__ldcg(p.x + kk), qf));
                    }
                    t = __fadd_rn(t, __fmul_rn(acc, W->s[(int64_t)row * p.nb_pad + nbf]));
                }
                W->y[row] = t;
            }
        }
    }
    // After a give-up, the copies this warp issued into the CTA's shared
    // memory must land before the CTA leaves (they normally have: every issued
    // group is consumed). One outstanding copy per slot at most. Bounded.
    if (*abort_flag && lane32 == 0) {
        for (int s = pp * p.D; s < (pp + 1) * p.D; ++s) {
            const int j = issued[s];
            if (j >= 0)
                mbar_wait(landed0 + s * 8, (uint32_t)((j / p.D) & 1), nullptr, kDecWaitBudget);
        }
    }
}

}  // namespace

namespace {

struct DecPlan {
    int cpt, S, P, C, D, ctas, slot_bytes, smem, threads, ahead;
};

// Launch shape for `groups` 4-row groups of length k. One chunk per producer
// thread while a pipe (S producer warps + its chain warp) is at most 5 warps,
// else two; chain warps per pipe so that the ordered chain (4 cycles per
// block) keeps up with its producers; as many pipes as fit 16 warps (12 with
// two chunks per thread); ring slots within ~110 KB of shared memory, so the
// next GEMV's CTA fits on the SM beside this one.
bool dec_plan(int groups, int k, bool q4, int sm_count, DecPlan* pl) {
    const int nck = packed_k(k) / kChunk;
    int cpt = 1, S = (nck + 3) / 4;
    if (S + 1 > 5) {
        cpt = 2;
        S = (nck + 7) / 8;
    }
    const int max_warps = cpt == 1 ? kDecMaxWarps : 12;
    const int C = nck * 16 > 500 * cpt ? 2 : 1;
    if (S + C > max_warps || groups < 1) return false;
    pl->cpt = cpt;
    pl->S = S;
    pl->C = C;
    // One CTA per SM, so the next GEMV's CTA fits beside it and starts its
    // copies early; long matrices (>= 24 groups per SM) run two per SM
    // instead, for twice the warps and slots in flight.
    const int max_ctas = groups >= 24 * sm_count ? 2 * sm_count : sm_count;
    pl->ctas = groups < max_ctas ? groups : max_ctas;
    const int gpc = (groups + pl->ctas - 1) / pl->ctas;
    int P = max_warps / (S + C);
    if (P > 4) P = 4;
    if (P > gpc) P = gpc;
    pl->P = P;
    pl->slot_bytes = (q4 ? kDecSlotPerChunkI4 : kDecSlotPerChunkI8) * nck;
    int D = (110 * 1024) / (P * pl->slot_bytes);
    if (D < 2 && 2 * P * pl->slot_bytes <= 200 * 1024) D = 2;  // long rows: two slots, one CTA per SM
    if (D > 4) D = 4;
    const int per_pipe = (gpc + P - 1) / P;
    if (D > per_pipe) D = per_pipe;
    if (D < 1) return false;
    // Each slot must be consumed by one chain warp, in group order: chain warp
    // c takes groups i = c (mod C) and slot i % D, so D must be a multiple of
    // C. (A slot shared by two chain warps would have one of them wait on a
    // barrier phase whose predecessor has not completed, which the parity wait
    // cannot tell from a completed one.)
    if (pl->C > D) pl->C = D;
    D -= D % pl->C;
    pl->D = D;
    pl->smem = P * D * (pl->slot_bytes + 24) + 16 + P * S * 512 + 16;
    if (pl->smem > 220 * 1024) return false;
    pl->threads = P * (S + pl->C) * 32;
    pl->ahead = D + 3;
    return true;
}

template <bool Q4, int CPT>
cudaError_t dec_launch(const DecParams& p, const DecPlan& pl, cudaStream_t stream, bool pdl) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    auto kern = gemv_dec_kernel<Q4, CPT>;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)pl.ctas);
    cfg.blockDim = dim3((unsigned)pl.threads);
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

bool gemv_decode_supported(int rows_total, int nw, int k, int sm_count, bool q4) {
    DecPlan pl;
    return dec_plan((rows_total + 3 * nw + 3) / 4, k, q4, sm_count, &pl);
}

cudaError_t launch_gemv_decode(const float* x, const GemvWeight* ws, int nw, int k, int* status, int sm_count,
                               cudaStream_t stream, bool pdl, bool q4) {
    if (nw < 1 || nw > kMaxGroup) return cudaErrorInvalidValue;
    DecParams p{};
    int groups = 0;
    for (int g = 0; g < nw; ++g) {
        if (ws[g].rows < 1) return cudaErrorInvalidValue;
        p.w[g].q = ws[g].q;
        p.w[g].s = ws[g].s;
        p.w[g].y = ws[g].y;
        p.w[g].rows = ws[g].rows;
        p.w[g].gbase = groups;
        groups += (ws[g].rows + 3) / 4;
    }
    DecPlan pl;
    if (!dec_plan(groups, k, q4, sm_count, &pl)) return cudaErrorInvalidValue;
    if (pl.D % pl.C != 0) return cudaErrorInvalidValue;  // a slot must belong to one chain warp
    p.x = x;
    p.zero_neg = -0.0f;
    p.nw = nw;
    p.status = status;
    p.k = k;
    const int k_pad = packed_k(k);
    p.nb_pad = k_pad / kBlock;
    p.nck = k_pad / kChunk;
    p.row_bytes = q4 ? k_pad / 2 : k_pad;
    p.cta_q = groups / pl.ctas;
    p.cta_r = groups % pl.ctas;
    p.S = pl.S;
    p.P = pl.P;
    p.C = pl.C;
    p.D = pl.D;
    p.slot_bytes = pl.slot_bytes;
    p.ahead = pl.ahead;
    if (pl.cpt == 1) return q4 ? dec_launch<true, 1>(p, pl, stream, pdl) : dec_launch<false, 1>(p, pl, stream, pdl);
    return q4 ? dec_launch<true, 2>(p, pl, stream, pdl) : dec_launch<false, 2>(p, pl, stream, pdl);
}

}  // namespace qlm
