// qlm_gemm_tc.cu — tcgen05 tensor-core prefill GEMM for the int8 path (sm_100a).
//
// Computes y[m, n] = sum_k x[m, k] * q[n, k] * s[n, k/32] for prefill-sized
// batches (QuickLM runs the same per-row GEMV for every row:
// src/ops/math_ops.cpp:845-894). The reference does not quantize activations
// and applies an arbitrary fp32 scale per (row, 32-block), so neither
// kind::i8 nor block-scaled MMA applies; this kernel dequantizes the weight
// tile on chip and runs a kind::f16 MMA with fp32 accumulation.
//
// Numerics: x is pre-scaled per row by an exact power of two 2^ea so its
// largest magnitude sits in [2^13, 2^14), then rounded to fp16; each weight
// block's scale is pre-scaled per row by 2^ew, rounded to fp16, and
// multiplied (in fp16) with the exactly-converted int8 value. The epilogue
// undoes 2^-(ea+ew) exactly. Result: within relative L2 ~4e-4 of the
// reference (the bar for a reduced-precision prefill MMA is 2e-3).
//
// K order. A K-step is 64 elements (two 32-blocks). The MMA only needs A and
// B to agree on the order of K inside a step, so both use the order in which
// the packed int8 layout hands the bytes to a converter thread: a 32-bit word
// of a row's lane slice l holds elements 8j + l (j = 0..3) of one block, and
// bytes (0, 2) and (1, 3) of that word become one fp16 pair each with a
// single mask-and-xor (plus a shift for the second pair). Step position
// pos = 32*bl + 4*l + 2*p + h holds element 32*bl + 8*(p + 2h) + l of the
// step; the activation converter writes x16 in that order.
//
// Data flow per CTA (one 128-row weight tile x BN tokens, all of K; BN is a
// run-time multiple of 16 picked so the grid fills the SMs):
//   warp 2 lane 0  TMA producer for the weights: int8 chunks (128 rows x
//                  128 B, one packed 128-element chunk per row, 128-byte
//                  swizzle) and their fp32 scales, 8 chunks per stage.
//   warp 0 lane 0  TMA producer for the activations: 64-wide fp16 tiles of BN
//                  tokens (128-byte swizzle, the MMA's K-major B operand).
//   warps 4..      NG converter groups of 4 warps, one thread per weight row;
//                  group g takes the chunks c = g mod NG. int8 -> fp16 with
//                  1.5 integer + 2 fp16x2 ops per pair, written with
//                  tcgen05.st straight into tensor memory as the MMA's A
//                  operand (no shared-memory round trip for the fp16 tile).
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma (K = 16) per 64-wide step;
//                  commits release the tensor-memory A stage and the
//                  activation stage.
//   warps 4..      epilogue: tcgen05.ld of the fp32 accumulator (TMEM lane =
//                  weight row, column = token), exact 2^-(ea+ew), stores of y
//                  coalesced along the weight rows.
// Every wait is bounded; on give-up the CTA records a status code, drains
// its in-flight copies and MMAs, frees its tensor memory and returns. No TMA
// load in this file uses multicast.
#include "qlm_device.cuh"
#include "qlm_kernels.h"
#include "qlm_sm100.cuh"

#include <cuda_fp16.h>
#include <cudaTypedefs.h>

namespace qlm {
namespace {

using namespace sm100;

constexpr int BM = 128;      // weight rows per tile (MMA M)
constexpr int BK = 64;       // fp16 K elements per MMA step (one 128-B swizzle row)
constexpr int NG = 4;        // converter groups
constexpr int NTHREADS = 128 * (1 + NG);
constexpr int BN_MAX = 192;  // tokens per tile (MMA N), multiple of 16
constexpr int SW = 4;        // int8 weight stages (one 128-element chunk each)
constexpr int SS = 2;        // scale stages
constexpr int S_CHUNKS = 4;  // chunks per scale stage (16 fp32 scales per row, unswizzled)
constexpr int SX = 3;        // activation slots (one 128-wide chunk = two 64-wide boxes each)
constexpr int NSLOT = 4;     // tensor-memory A slots (one chunk = 64 columns each)
constexpr int TMEM_COLS = 512;
constexpr int A_COL0 = 256;  // accumulator in columns [0, BN), A slots above
constexpr int W_STAGE_BYTES = BM * 128;           // [row 128][128 B], 128-byte swizzle
constexpr int S_STAGE_BYTES = BM * S_CHUNKS * 16;  // [row 128][S_CHUNKS x 4 scales]
constexpr int OFF_W = 0;
constexpr int OFF_S = OFF_W + SW * W_STAGE_BYTES;
constexpr int OFF_X = OFF_S + SS * S_STAGE_BYTES;
constexpr int NBAR = 2 * SW + 2 * SS + SX + 2 * NSLOT + 1;
constexpr long long WAIT_BUDGET = 4000000000LL;  // ~2 s of SM clock per wait

__host__ __device__ constexpr int x_slot_bytes(int bn) { return 2 * bn * 128; }
__host__ __device__ constexpr int off_bar(int bn) { return OFF_X + SX * x_slot_bytes(bn); }
__host__ __device__ constexpr int off_misc(int bn) { return off_bar(bn) + NBAR * 8; }
__host__ __device__ constexpr int off_ea(int bn) { return off_misc(bn) + 16; }
__host__ __device__ constexpr int smem_bytes(int bn) { return off_ea(bn) + 4 * BN_MAX + 1024; }  // + base alignment
static_assert(smem_bytes(BN_MAX) <= 232448, "shared memory budget");
static_assert(BN_MAX % (16 * NG) == 0, "epilogue column blocks");
static_assert(SW <= S_CHUNKS, "the first weight chunks issued at set-up all use scale stage 0");
static_assert(BM * 4 <= SX * 2 * 128, "epilogue staging (BM x bn fp32) fits below the barriers for every bn");
constexpr long long DRAIN_BUDGET = 1LL << 25;  // ~17 ms: bound for copies still in flight after an abort

enum : int { ST_OK = 0, ST_TIMEOUT_PRODUCER = 0x101, ST_TIMEOUT_MMA = 0x102, ST_TIMEOUT_CONVERT = 0x103 };

struct TcParams {
    float* y;
    int64_t ldy;
    const int* ew;  // [rows] per-row weight exponents
    const int* ea;  // [M] per-row activation exponents
    int rows, M, bn, nchunks;
    int y_vec4;  // y and ldy allow 16-byte stores
    int* status;
};

// Exact v * 2^e for |e| <= 378 (three normal power-of-two factors).
__device__ __forceinline__ float mul_pow2(float v, int e) {
    const int e1 = e / 3, e2 = (e - e1) / 2, e3 = e - e1 - e2;
    v = __fmul_rn(v, __int_as_float((e1 + 127) << 23));
    v = __fmul_rn(v, __int_as_float((e2 + 127) << 23));
    return __fmul_rn(v, __int_as_float((e3 + 127) << 23));
}

// v * 2^e with one multiply when 2^e is a normal float, else mul_pow2.
__device__ __forceinline__ float scale_pow2(float v, int e) {
    if ((unsigned)(e + 126) <= 253u) return __fmul_rn(v, __int_as_float((e + 127) << 23));
    return mul_pow2(v, e);
}

// E such that v = f * 2^E with f in [0.5, 1), for finite v > 0.
__device__ __forceinline__ int frexp_exponent(float v) {
    uint32_t b = __float_as_uint(v);
    int be = (int)((b >> 23) & 0xFF);
    if (be == 0) {  // subnormal: scale up by 2^64 exactly
        b = __float_as_uint(__fmul_rn(v, 18446744073709551616.0f));
        return (int)((b >> 23) & 0xFF) - 64 - 126;
    }
    return be - 126;
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<const uint32_t*>(&h); }

// Synchronise the converter warps only (named barrier 1).
__device__ __forceinline__ void converters_sync() { asm volatile("bar.sync 1, %0;" ::"r"(128 * NG) : "memory"); }

// Named barrier 2: warp 0 arrives once the mbarriers are initialised (it
// starts its weight copies right away); warp 1 arrives after allocating
// tensor memory; every other warp waits for both.
__device__ __forceinline__ void setup_arrive() { asm volatile("bar.arrive 2, %0;" ::"r"(NTHREADS) : "memory"); }
__device__ __forceinline__ void setup_sync() { asm volatile("bar.sync 2, %0;" ::"r"(NTHREADS) : "memory"); }

__global__ void __launch_bounds__(NTHREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
               const __grid_constant__ CUtensorMap tm_x, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int bn = p.bn;
    const uint32_t x_box_bytes = (uint32_t)bn * 128u;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + off_bar(bn);
    const uint32_t WFULL = bar0, WEMPTY = WFULL + 8 * SW;
    const uint32_t SFULL = WEMPTY + 8 * SW, SEMPTY = SFULL + 8 * SS;
    const uint32_t XEMPTY = SEMPTY + 8 * SS;
    const uint32_t AFULL = XEMPTY + 8 * SX, AEMPTY = AFULL + 8 * NSLOT;
    const uint32_t ACCFULL = AEMPTY + 8 * NSLOT;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + off_misc(bn));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + off_misc(bn) + 4);
    int* ea_s = reinterpret_cast<int*>(smem + off_ea(bn));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BM, m0 = blockIdx.y * bn;
    const int nchunks = p.nchunks;

    if (warp == 0) {
        // ------------------ TMA producer: weights + scales ------------------
        int w_issued = 0, s_issued = 0;
        if (lane == 0) {
            for (int i = 0; i < SW; ++i) {
                mbar_init(WFULL + 8 * i, 1);
                mbar_init(WEMPTY + 8 * i, 4);  // the 4 warps of the group that owns the chunk
            }
            for (int i = 0; i < SS; ++i) {
                mbar_init(SFULL + 8 * i, 1);
                mbar_init(SEMPTY + 8 * i, 4 * NG);
            }
            mbar_fence_init();
            // The first scale stage and weight chunks go out before anything
            // else is set up (the stages are empty: no wait needed).
            mbar_arrive_expect_tx(SFULL, S_STAGE_BYTES);
            tma_load_2d(sbase + OFF_S, &tm_s, 0, n0, SFULL);
            for (int c = 0; c < SW && c < nchunks; ++c) {
                mbar_arrive_expect_tx(WFULL + 8 * c, W_STAGE_BYTES);
                tma_load_2d(sbase + OFF_W + c * W_STAGE_BYTES, &tm_w, c * 128, n0, WFULL + 8 * c);
            }
            for (int i = 0; i < SX; ++i) mbar_init(XEMPTY + 8 * i, 1);
            for (int i = 0; i < NSLOT; ++i) {
                // the owning converter group's 4 warps + the activation producer (with the bytes)
                mbar_init(AFULL + 8 * i, 5);
                mbar_init(AEMPTY + 8 * i, 1);
            }
            mbar_init(ACCFULL, 1);
            *abort_flag = 0;
            mbar_fence_init();
        }
        __syncwarp();
        setup_arrive();
        // Weights are not written by the preceding kernel, so these copies
        // start before the programmatic-dependent-launch wait.
        bool ok = true;
        s_issued = 1;
        w_issued = min(SW, nchunks);
        for (int c = w_issued; c < nchunks && ok; ++c) {
            if (c % S_CHUNKS == 0) {
                const int g = c / S_CHUNKS, ss = g % SS;
                if (!mbar_wait_warp(SEMPTY + 8 * ss, ((g / SS) & 1) ^ 1, abort_flag, WAIT_BUDGET)) {
                    ok = false;
                    break;
                }
                if (elect_one()) {
                    mbar_arrive_expect_tx(SFULL + 8 * ss, S_STAGE_BYTES);
                    tma_load_2d(sbase + OFF_S + ss * S_STAGE_BYTES, &tm_s, 4 * c, n0, SFULL + 8 * ss);
                }
                ++s_issued;
            }
            const int ws = c % SW;
            if (!mbar_wait_warp(WEMPTY + 8 * ws, ((c / SW) & 1) ^ 1, abort_flag, WAIT_BUDGET)) {
                ok = false;
                break;
            }
            if (elect_one()) {
                mbar_arrive_expect_tx(WFULL + 8 * ws, W_STAGE_BYTES);
                tma_load_2d(sbase + OFF_W + ws * W_STAGE_BYTES, &tm_w, c * 128, n0, WFULL + 8 * ws);
            }
            ++w_issued;
        }
        pdl_launch_dependents();
        if (!ok && lane == 0) {
            *abort_flag = 1;
            atomicCAS(p.status, 0, ST_TIMEOUT_PRODUCER);
        }
        // Drain: the last load issued into every stage must have landed
        // before this CTA's shared memory can be released.
        for (int i = (w_issued > SW ? w_issued - SW : 0); i < w_issued; ++i)
            mbar_wait(WFULL + 8 * (i % SW), (i / SW) & 1, nullptr, WAIT_BUDGET);
        for (int i = (s_issued > SS ? s_issued - SS : 0); i < s_issued; ++i)
            mbar_wait(SFULL + 8 * (i % SS), (i / SS) & 1, nullptr, WAIT_BUDGET);
    } else if (warp == 1) {
        // --------------------------- MMA issuer -------------------------
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
        tc_fence_before();
        setup_sync();
        tc_fence_after();
        const uint32_t tmem = *tmem_slot;
        // One chunk (128 of K: the A slot and both activation boxes, one
        // barrier) per step: 8 MMAs of K = 16.
        const uint32_t idesc = idesc_f16_f32(BM, bn);
        bool ok = true;
        for (int c = 0; c < nchunks && ok; ++c) {
            const int slot = c % NSLOT, xs = c % SX;
            if (!mbar_wait_warp(AFULL + 8 * slot, (c / NSLOT) & 1, abort_flag, WAIT_BUDGET)) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (elect_one()) {
                const uint32_t a_tmem = tmem + A_COL0 + slot * 64;
                const uint64_t b_desc = smem_desc_sw128(sbase + OFF_X + xs * x_slot_bytes(bn));
                const uint64_t b_step = (uint64_t)(x_box_bytes >> 4);  // second 64-wide box
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        mma_f16_ts(tmem, a_tmem + h * 32 + kk * 8, b_desc + h * b_step + (uint64_t)(kk * 2), idesc,
                                   (c | h | kk) != 0);
                tc_commit(XEMPTY + 8 * xs);
                tc_commit(AEMPTY + 8 * slot);
            }
            __syncwarp();
        }
        pdl_launch_dependents();
        if (!ok && lane == 0) {
            *abort_flag = 1;
            atomicCAS(p.status, 0, ST_TIMEOUT_MMA);
        }
        if (elect_one()) tc_commit(ACCFULL);  // fires once every MMA issued above has completed
        __syncwarp();
    } else if (warp == 2) {
        // ------------------- TMA producer: activations -------------------
        // Both 64-wide boxes of chunk c complete on the chunk's A-slot barrier.
        setup_sync();
        if (elect_one()) tma_prefetch_desc(&tm_x);
        pdl_wait();  // x16 is written by the preceding conversion kernel
        bool ok = true;
        int x_issued = 0;
        for (int c = 0; c < nchunks; ++c) {
            const int xs = c % SX, slot = c % NSLOT;
            if (!mbar_wait_warp(XEMPTY + 8 * xs, ((c / SX) & 1) ^ 1, abort_flag, WAIT_BUDGET)) {
                ok = false;
                break;
            }
            if (elect_one()) {
                const uint32_t dst = sbase + OFF_X + xs * x_slot_bytes(bn);
                mbar_arrive_expect_tx(AFULL + 8 * slot, 2 * x_box_bytes);
                tma_load_2d(dst, &tm_x, c * 128, m0, AFULL + 8 * slot);
                tma_load_2d(dst + x_box_bytes, &tm_x, c * 128 + BK, m0, AFULL + 8 * slot);
            }
            __syncwarp();
            ++x_issued;
        }
        pdl_launch_dependents();
        if (!ok && lane == 0) {
            *abort_flag = 1;
            atomicCAS(p.status, 0, ST_TIMEOUT_PRODUCER);
        }
        // On the normal path the MMA warp has waited for every copy issued
        // here. After an abort, the last SX copies may still be in flight and
        // their A-slot phases may never complete (the converters stopped):
        // wait a bounded time for them to land before shared memory is freed.
        if (*abort_flag)
            for (int c = (x_issued > SX ? x_issued - SX : 0); c < x_issued; ++c)
                mbar_wait(AFULL + 8 * (c % NSLOT), (c / NSLOT) & 1, nullptr, DRAIN_BUDGET);
    } else if (warp >= 4) {
        // ------------------- converters, then the epilogue -------------------
        setup_sync();
        tc_fence_after();
        const uint32_t tmem = *tmem_slot;
        const int grp = (warp - 4) >> 2;  // converter group
        const int qw = warp & 3;          // tensor-memory lane quarter of this warp
        const int r = 32 * qw + lane;
        const int row = n0 + r;
        const int ewr = row < p.rows ? p.ew[row] : 0;
        const uint32_t lane_addr = (uint32_t)(32 * qw) << 16;
        const int sw = r & 7;  // this row's 128-byte swizzle phase
        const __half2 bias2 = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
        bool ok = true;
        for (int c = grp; c < nchunks && ok; c += NG) {
            const int g = c / S_CHUNKS, ss = g % SS, cc = c % S_CHUNKS;
            const int ws = c % SW, slot = c % NSLOT;
            if (!mbar_wait_warp(SFULL + 8 * ss, (g / SS) & 1, abort_flag, WAIT_BUDGET) ||
                !mbar_wait_warp(WFULL + 8 * ws, (c / SW) & 1, abort_flag, WAIT_BUDGET)) {
                ok = false;
                break;
            }
            const uint8_t* wst = smem + OFF_W + ws * W_STAGE_BYTES + r * 128;
            uint4 v[8];
#pragma unroll
            for (int l = 0; l < 8; ++l) v[l] = *reinterpret_cast<const uint4*>(wst + ((l ^ sw) << 4));
            const float4 s4 =
                *reinterpret_cast<const float4*>(smem + OFF_S + ss * S_STAGE_BYTES + r * (S_CHUNKS * 16) + cc * 16);
            // These generic-proxy reads must be performed before the stage is
            // handed back to the TMA (async proxy) that refills it.
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(WEMPTY + 8 * ws);
                // this group's last chunk of the scale stage
                if (c + NG >= S_CHUNKS * (g + 1) || c + NG >= nchunks) mbar_arrive(SEMPTY + 8 * ss);
            }
            const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
            __half2 s16[4];
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) s16[bb] = __float2half2_rn(scale_pow2(sv[bb], ewr));

            // Both steps of the chunk go to the chunk's A slot (64 columns):
            // convert, wait for the slot, store; one wait for the stores, then
            // the slot is published.
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t out[32];
#pragma unroll
                for (int bl = 0; bl < 2; ++bl) {
                    const int bb = 2 * h + bl;
#pragma unroll
                    for (int l = 0; l < 8; ++l) {
                        // bytes (0,2) and (1,3) of the word: elements 8j + l of block bb, j = (0,2) / (1,3);
                        // fp16 bit pattern 0x64XX = 1024 + XX with XX = q + 128
                        const uint32_t w = word_of(v[l], bb);
                        const uint32_t u02 = (w & 0x00FF00FFu) ^ 0x64806480u;
                        const uint32_t u13 = ((w >> 8) & 0x00FF00FFu) ^ 0x64806480u;
                        const __half2 q02 = __hsub2(*reinterpret_cast<const __half2*>(&u02), bias2);
                        const __half2 q13 = __hsub2(*reinterpret_cast<const __half2*>(&u13), bias2);
                        out[16 * bl + 2 * l] = h2_bits(__hmul2(q02, s16[bb]));
                        out[16 * bl + 2 * l + 1] = h2_bits(__hmul2(q13, s16[bb]));
                    }
                }
                // warp-collective wait: the tcgen05.st below is .sync.aligned and
                // must be executed by the whole, converged warp
                if (h == 0 && !mbar_wait_warp(AEMPTY + 8 * slot, ((c / NSLOT) & 1) ^ 1, abort_flag, WAIT_BUDGET)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                tmem_st_32x32b_x32(tmem + lane_addr + A_COL0 + slot * 64 + h * 32, out);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(AFULL + 8 * slot);
        }
        pdl_launch_dependents();
        if (!ok) {
            *abort_flag = 1;
            atomicCAS(p.status, 0, ST_TIMEOUT_CONVERT);
        }
        // y and ea belong to the stream's earlier work.
        pdl_wait();
        const int ct = (warp - 4) * 32 + lane;
        for (int i = ct; i < bn; i += 128 * NG) ea_s[i] = m0 + i < p.M ? p.ea[m0 + i] : 0;
        converters_sync();
        // The accumulator (or, after an abort, the drained MMA pipe). Every
        // copy into the stage buffers has been consumed by now (the MMAs read
        // all activation stages, the converters all weight/scale stages), so
        // the tile is restaged in [token][128 rows] order over them and
        // written out one token row (512 contiguous bytes) per warp store.
        mbar_wait_warp(ACCFULL, 0, nullptr, WAIT_BUDGET);  // converged before tcgen05.ld (.sync.aligned)
        tc_fence_after();
        float* stage = reinterpret_cast<float*>(smem);
        const int cols = min(bn, p.M - m0);
        if (!*abort_flag) {
            // All of this warp's column blocks (16 wide, every NG-th) are
            // loaded before a single wait, so the TMEM load latency is paid
            // once. Columns past the tile are allocated and simply not stored.
            constexpr int NCB = BN_MAX / (16 * NG);
            uint32_t acc[NCB][16];
#pragma unroll
            for (int j = 0; j < NCB; ++j) tmem_ld_32x32b_x16(tmem + lane_addr + 16 * (grp + NG * j), acc[j]);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < NCB; ++j) {
                const int col0 = 16 * (grp + NG * j);
                if (col0 < cols) {
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        stage[(col0 + i) * BM + r] = scale_pow2(__uint_as_float(acc[j][i]), -(ewr + ea_s[col0 + i]));
                }
            }
        }
        converters_sync();
        if (!*abort_flag) {
            const int nrow = min(BM, p.rows - n0);
            if (p.y_vec4 && nrow == BM) {
                for (int i = ct; i < cols * (BM / 4); i += 128 * NG) {
                    const int t = i / (BM / 4), seg = i % (BM / 4);
                    const float4 v = *reinterpret_cast<const float4*>(stage + t * BM + 4 * seg);
                    *reinterpret_cast<float4*>(p.y + (int64_t)(m0 + t) * p.ldy + n0 + 4 * seg) = v;
                }
            } else {
                for (int i = ct; i < cols * BM; i += 128 * NG) {
                    const int t = i / BM, rr = i % BM;
                    if (rr < nrow) p.y[(int64_t)(m0 + t) * p.ldy + n0 + rr] = stage[t * BM + rr];
                }
            }
        }
    } else {
        setup_sync();
        pdl_launch_dependents();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(*tmem_slot, TMEM_COLS);
    }
}

// Activations fp32 [M][ldx] -> fp16 [M][k_pad] in the MMA's K order, scaled
// by 2^ea[m] so the row's largest finite magnitude lands in [2^13, 2^14);
// zeros past k. One CTA per row; each thread writes 8 consecutive positions
// (16 bytes), reading their sources back from L1.
// early: every row's CTA is resident from the start (few rows), so the GEMM
// may launch at once: its set-up and first weight chunks then overlap this
// kernel (it waits for x16 and ea before reading them). Otherwise the trigger
// comes last, since an early GEMM CTA would hold an SM this grid still needs.
__global__ void __launch_bounds__(256) act_to_f16_kernel(const float* __restrict__ x, int64_t ldx, int K, int k_pad,
                                                         __half* __restrict__ x16, int* __restrict__ ea, int early) {
    __shared__ float red[8];
    if (early) pdl_launch_dependents();
    pdl_wait();  // x comes from the previous kernel; x16/ea may still be read by the previous GEMM
    // x is read through L2 (ld.global.cg): under programmatic launch its producer may
    // still be running when this kernel starts, so the read-only path is not safe.
    const int m = blockIdx.x;
    const float* xr = x + (int64_t)m * ldx;
    float mx = 0.0f;
    // eight independent loads in flight per thread per pass over the row
    for (int base = 0; base < K; base += 8 * (int)blockDim.x) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int k = base + i * (int)blockDim.x + (int)threadIdx.x;
            v[i] = k < K ? fabsf(__ldcg(xr + k)) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (v[i] > mx && v[i] <= 3.4028234663852886e38f) mx = v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, red[i]);
    const int e = mx > 0.0f ? 14 - frexp_exponent(mx) : 0;
    uint4* dst = reinterpret_cast<uint4*>(x16 + (int64_t)m * k_pad);
    for (int pos0 = 8 * (int)threadIdx.x; pos0 < k_pad; pos0 += 8 * (int)blockDim.x) {
        // positions pos0..pos0+7: lanes l0, l0+1; (p, h) in {0,1}^2 each
        const int base = pos0 & ~63, pl = pos0 & 63;
        const int bl = pl >> 5, l0 = (pl >> 2) & 7;
        uint32_t hw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int l = l0 + (i >> 1), pp = i & 1;  // output pair i = positions 2i, 2i+1: h = 0, 1
            const int k0 = base + 32 * bl + 8 * pp + l, k1 = k0 + 16;
            const float a = k0 < K ? __ldcg(xr + k0) : 0.0f;
            const float b = k1 < K ? __ldcg(xr + k1) : 0.0f;
            const __half2 v = __halves2half2(__float2half_rn(scale_pow2(a, e)), __float2half_rn(scale_pow2(b, e)));
            hw[i] = h2_bits(v);
        }
        dst[pos0 >> 3] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    }
    if (threadIdx.x == 0) ea[m] = e;
    if (!early) pdl_launch_dependents();
}

// Per weight row: ew so that 127 * max(finite block scale) * 2^ew is in
// [2^13, 2^14). One warp per row.
__global__ void weight_exp_kernel(const float* __restrict__ s, int rows, int nb, int nb_pad, int* __restrict__ ew) {
    const int wpr = (int)(blockDim.x >> 5);
    const int row = blockIdx.x * wpr + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int lane = threadIdx.x & 31;
    float mx = 0.0f;
    for (int b = lane; b < nb; b += 32) {
        const float v = s[(int64_t)row * nb_pad + b];
        if (v > mx && v <= 3.4028234663852886e38f) mx = v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) {
        const float v = __fmul_rn(mx, 127.0f);
        ew[row] = (v > 0.0f && v <= 3.4028234663852886e38f) ? 14 - frexp_exponent(v) : 0;
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

int sm_count_of_current_device() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() { return encode_fn(); }

cudaError_t tc_make_weight_maps(const uint8_t* q, const float* s, int rows, int k_pad, TcMaps* out) {
    auto enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)k_pad, (cuuint64_t)rows};
        const cuuint64_t strides[1] = {(cuuint64_t)k_pad};
        const cuuint32_t box[2] = {128, (cuuint32_t)BM};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&out->w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(q), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    }
    {
        const int nb_pad = k_pad / kBlock;
        const cuuint64_t dims[2] = {(cuuint64_t)nb_pad, (cuuint64_t)rows};
        const cuuint64_t strides[1] = {(cuuint64_t)nb_pad * 4};
        const cuuint32_t box[2] = {4 * S_CHUNKS, (cuuint32_t)BM};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&out->s, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(s), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    }
    return cudaSuccess;
}

cudaError_t launch_weight_exponents(const float* s, int rows, int k, int* ew, cudaStream_t stream) {
    const int nb = (k + kBlock - 1) / kBlock, nb_pad = packed_k(k) / kBlock;
    weight_exp_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(s, rows, nb, nb_pad, ew);
    return cudaGetLastError();
}

// Token-tile width: a CTA spends about max(2 * BN, kConvCycles) cycles per
// 64-wide K step (the MMA at 2 BN cycles, or converting 128 rows x 64
// weights), one CTA per SM. Pick the multiple of 16 with the least
// (waves x step time), then the least padding, then the widest tile.
int tc_pick_bn(int M, int rows, int sm_count) {
    constexpr long kConvCycles = 320;
    const long tiles_n = (rows + BM - 1) / BM;
    int best = 16;
    long best_cost = -1, best_pad = 0;
    for (int bn = 16; bn <= BN_MAX; bn += 16) {
        const long tiles_m = (M + bn - 1) / bn;
        const long waves = (tiles_n * tiles_m + sm_count - 1) / sm_count;
        const long cost = waves * (2L * bn > kConvCycles ? 2L * bn : kConvCycles);
        const long pad = tiles_m * bn;
        if (best_cost < 0 || cost < best_cost || (cost == best_cost && (pad < best_pad || (pad == best_pad && bn > best)))) {
            best = bn;
            best_cost = cost;
            best_pad = pad;
        }
    }
    return best;
}

cudaError_t launch_gemm_tc(const TcMaps& maps, const int* ew, int rows, int k, const float* x, int64_t ldx, int M,
                           void* x16_scratch, int* ea_scratch, float* y, int64_t ldy, int* status,
                           cudaStream_t stream, bool pdl) {
    auto enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    const int k_pad = packed_k(k);
    const int bn = tc_pick_bn(M, rows, sm_count_of_current_device());
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)M);
        cfg.blockDim = dim3(256);
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 1 : 0;
        // at most 4 of its 256-thread CTAs per SM: all resident at once
        const int early = pdl && M <= 4 * sm_count_of_current_device() ? 1 : 0;
        cudaError_t e = cudaLaunchKernelEx(&cfg, act_to_f16_kernel, x, ldx, k, k_pad,
                                           static_cast<__half*>(x16_scratch), ea_scratch, early);
        if (e != cudaSuccess) return e;
    }
    CUtensorMap tm_x;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)k_pad, (cuuint64_t)M};
        const cuuint64_t strides[1] = {(cuuint64_t)k_pad * 2};
        const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)bn};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&tm_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x16_scratch, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    }
    TcParams p;
    p.y = y;
    p.ldy = ldy;
    p.ew = ew;
    p.ea = ea_scratch;
    p.rows = rows;
    p.M = M;
    p.bn = bn;
    p.nchunks = k_pad / 128;
    p.y_vec4 = ((reinterpret_cast<uintptr_t>(y) & 15) == 0 && (ldy & 3) == 0) ? 1 : 0;
    p.status = status;

    static bool attr_set[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(BN_MAX));
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((rows + BM - 1) / BM), (unsigned)((M + bn - 1) / bn));
    cfg.blockDim = dim3(NTHREADS);
    // Always the full budget: one CTA per SM, so the 512-column TMEM
    // allocation never waits for another CTA of this kernel.
    cfg.dynamicSmemBytes = smem_bytes(BN_MAX);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemm_tc_kernel, maps.w, maps.s, tm_x, p);
}

}  // namespace qlm
