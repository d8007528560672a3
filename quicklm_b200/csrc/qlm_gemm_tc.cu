// qlm_gemm_tc.cu — tcgen05 tensor-core prefill GEMM for the int8 path (sm_100a).
//
// Computes y[m, n] = sum_k x[m, k] * q[n, k] * s[n, k/32] for M >= 64 style
// prefill batches (QuickLM runs the same per-row GEMV for every row:
// src/ops/math_ops.cpp:845-894). The reference does not quantize activations
// and applies an arbitrary fp32 scale per (row, 32-block), so neither
// kind::i8 nor block-scaled MMA applies; this kernel dequantizes the weight
// tile on chip and runs a kind::f16 MMA with fp32 accumulation.
//
// Numerics: x is pre-scaled per row by an exact power of two 2^ea so its
// largest magnitude sits in [2^13, 2^14), then rounded to fp16; each weight
// block's scale is pre-scaled per row by 2^ew, rounded to fp16, and
// multiplied (in fp16) with the exactly-converted int8 value. The epilogue
// undoes 2^-(ea+ew) exactly. Result: within relative L2 ~1e-3 of the
// reference (the bar for a reduced-precision prefill MMA is 2e-3).
//
// Data flow per CTA (one 128-row weight tile x BN tokens, all of K):
//   warp 0 lane 0  TMA producer: int8 weight chunks (128 rows x 128 B, one
//                  packed chunk per row, 128-byte swizzle so a thread per
//                  row reads its 16-byte lane slices without bank
//                  conflicts), their scales 8 chunks at a time (also
//                  swizzled), and 64-wide fp16 activation tiles (128-byte
//                  swizzle, the MMA's K-major B operand).
//   warps 4-7      converters, one thread per weight row: int8 -> fp16 with
//                  two integer ops and two fp16x2 ops per pair, written with
//                  tcgen05.st straight into tensor memory as the MMA's A
//                  operand (no shared-memory round trip for the fp16 tile).
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma (K=16) per 64-wide step,
//                  commits release the TMEM A stage and the activation stage.
//   warps 4-7      epilogue: tcgen05.ld of the fp32 accumulator (TMEM lane =
//                  weight row, column = token), exact 2^-(ea+ew), coalesced
//                  stores of y.
// Every wait is bounded; on give-up the CTA records a status code, drains
// its in-flight copies and MMAs, frees its tensor memory and returns.
#include "qlm_device.cuh"
#include "qlm_kernels.h"
#include "qlm_sm100.cuh"

#include <cuda_fp16.h>
#include <cudaTypedefs.h>

namespace qlm {
namespace {

using namespace sm100;

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BK = 64;   // fp16 K elements per activation stage (one 128-B swizzle row)
constexpr int SW = 3;    // int8 weight stages (one 128-element chunk each)
constexpr int SS = 2;    // scale stages (8 chunks each)
constexpr int S_CHUNKS = 8;
constexpr int SX = 4;    // activation stages
constexpr int SA = 4;    // tensor-memory A stages (one BK step = 32 columns each)
constexpr int W_STAGE_BYTES = BM * 128;  // [row 128][128 B], 128-byte swizzle
constexpr int S_STAGE_BYTES = BM * 128;  // [row 128][8 chunks x 4 scales], 128-byte swizzle
constexpr long long WAIT_BUDGET = 4000000000LL;  // ~2 s of SM clock per wait

enum : int { ST_OK = 0, ST_TIMEOUT_PRODUCER = 0x101, ST_TIMEOUT_MMA = 0x102, ST_TIMEOUT_CONVERT = 0x103 };

struct TcParams {
    float* y;
    int64_t ldy;
    const int* ew;  // [rows] per-row weight exponents
    const int* ea;  // [M] per-row activation exponents
    int rows, M, nchunks, nksteps;
    int* status;
};

template <int BN>
struct TcCfg {
    static constexpr int X_STAGE_BYTES = BN * 128;
    static constexpr int TMEM_COLS = BN <= 128 ? 256 : 512;
    static constexpr int A_COL0 = BN <= 128 ? 128 : 256;
    static constexpr int OFF_X = 0;
    static constexpr int OFF_W = OFF_X + SX * X_STAGE_BYTES;
    static constexpr int OFF_S = OFF_W + SW * W_STAGE_BYTES;
    static constexpr int OFF_BAR = OFF_S + SS * S_STAGE_BYTES;
    static constexpr int NBAR = 2 * SW + 2 * SX + 2 * SA + 2 * SS + 1;
    static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
    static constexpr int SMEM = OFF_MISC + 16 + 1024;  // + slack to align the base to 1024 B
};

// Exact v * 2^e for |e| <= 378 (three normal power-of-two factors).
__device__ __forceinline__ float mul_pow2(float v, int e) {
    const int e1 = e / 3, e2 = (e - e1) / 2, e3 = e - e1 - e2;
    v = __fmul_rn(v, __int_as_float((e1 + 127) << 23));
    v = __fmul_rn(v, __int_as_float((e2 + 127) << 23));
    return __fmul_rn(v, __int_as_float((e3 + 127) << 23));
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

template <int BN>
__global__ void __launch_bounds__(256, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
               const __grid_constant__ CUtensorMap tm_x, const TcParams p) {
    using C = TcCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + C::OFF_BAR;
    const uint32_t WFULL = bar0, WEMPTY = bar0 + 8 * SW;
    const uint32_t XFULL = bar0 + 8 * (2 * SW), XEMPTY = XFULL + 8 * SX;
    const uint32_t AFULL = bar0 + 8 * (2 * SW + 2 * SX), AEMPTY = AFULL + 8 * SA;
    const uint32_t ACCFULL = bar0 + 8 * (2 * SW + 2 * SX + 2 * SA);
    const uint32_t SFULL = ACCFULL + 8, SEMPTY = SFULL + 8 * SS;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BM, m0 = blockIdx.y * BN;

    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        for (int i = 0; i < SW; ++i) {
            mbar_init(WFULL + 8 * i, 1);
            mbar_init(WEMPTY + 8 * i, 4);
        }
        for (int i = 0; i < SX; ++i) {
            mbar_init(XFULL + 8 * i, 1);
            mbar_init(XEMPTY + 8 * i, 1);
        }
        for (int i = 0; i < SA; ++i) {
            mbar_init(AFULL + 8 * i, 4);
            mbar_init(AEMPTY + 8 * i, 1);
        }
        mbar_init(ACCFULL, 1);
        for (int i = 0; i < SS; ++i) {
            mbar_init(SFULL + 8 * i, 1);
            mbar_init(SEMPTY + 8 * i, 4);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------- TMA producer -------------------------
            tma_prefetch_desc(&tm_w);
            tma_prefetch_desc(&tm_s);
            tma_prefetch_desc(&tm_x);
            bool ok = true;
            int w_issued = 0, x_issued = 0, s_issued = 0;
            for (int c = 0; c < p.nchunks && ok; ++c) {
                if (c % S_CHUNKS == 0) {
                    const int g = c / S_CHUNKS, ss = g % SS;
                    if (!mbar_wait(SEMPTY + 8 * ss, ((g / SS) & 1) ^ 1, abort_flag, WAIT_BUDGET)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(SFULL + 8 * ss, S_STAGE_BYTES);
                    tma_load_2d(sbase + C::OFF_S + ss * S_STAGE_BYTES, &tm_s, 4 * c, n0, SFULL + 8 * ss);
                    ++s_issued;
                }
                const int ws = c % SW;
                if (!mbar_wait(WEMPTY + 8 * ws, ((c / SW) & 1) ^ 1, abort_flag, WAIT_BUDGET)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(WFULL + 8 * ws, W_STAGE_BYTES);
                tma_load_2d(sbase + C::OFF_W + ws * W_STAGE_BYTES, &tm_w, c * 128, n0, WFULL + 8 * ws);
                ++w_issued;
                if (c == 0) pdl_wait();  // activations are produced by the previous kernel
                for (int h = 0; h < 2; ++h) {
                    const int ks = 2 * c + h;
                    if (ks >= p.nksteps) break;
                    const int xs = ks % SX;
                    if (!mbar_wait(XEMPTY + 8 * xs, ((ks / SX) & 1) ^ 1, abort_flag, WAIT_BUDGET)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(XFULL + 8 * xs, C::X_STAGE_BYTES);
                    tma_load_2d(sbase + C::OFF_X + xs * C::X_STAGE_BYTES, &tm_x, ks * BK, m0, XFULL + 8 * xs);
                    ++x_issued;
                }
            }
            if (!ok) {
                *abort_flag = 1;
                atomicCAS(p.status, 0, ST_TIMEOUT_PRODUCER);
            }
            // Drain: the last load issued into every stage must have landed
            // before this CTA's shared memory can be released.
            for (int i = (w_issued > SW ? w_issued - SW : 0); i < w_issued; ++i)
                mbar_wait(WFULL + 8 * (i % SW), (i / SW) & 1, nullptr, WAIT_BUDGET);
            for (int i = (x_issued > SX ? x_issued - SX : 0); i < x_issued; ++i)
                mbar_wait(XFULL + 8 * (i % SX), (i / SX) & 1, nullptr, WAIT_BUDGET);
            for (int i = (s_issued > SS ? s_issued - SS : 0); i < s_issued; ++i)
                mbar_wait(SFULL + 8 * (i % SS), (i / SS) & 1, nullptr, WAIT_BUDGET);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // --------------------------- MMA issuer -------------------------
            pdl_wait();
            constexpr uint32_t idesc = idesc_f16_f32(BM, BN);
            bool ok = true;
            for (int ks = 0; ks < p.nksteps; ++ks) {
                const int as = ks % SA, xs = ks % SX;
                if (!mbar_wait(AFULL + 8 * as, (ks / SA) & 1, abort_flag, WAIT_BUDGET) ||
                    !mbar_wait(XFULL + 8 * xs, (ks / SX) & 1, abort_flag, WAIT_BUDGET)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a_tmem = tmem + C::A_COL0 + as * 32;
                const uint64_t b_desc = smem_desc_sw128(sbase + C::OFF_X + xs * C::X_STAGE_BYTES);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
                    mma_f16_ts(tmem, a_tmem + kk * 8, b_desc + (uint64_t)(kk * 2), idesc, (ks | kk) != 0);
                tc_commit(AEMPTY + 8 * as);
                tc_commit(XEMPTY + 8 * xs);
            }
            if (!ok) {
                *abort_flag = 1;
                atomicCAS(p.status, 0, ST_TIMEOUT_MMA);
            }
            tc_commit(ACCFULL);  // fires once every MMA issued above has completed
        }
    } else if (warp >= 4) {
        // ------------------- converters, then the epilogue -------------------
        pdl_wait();
        const int qw = warp & 3;
        const int r = 32 * qw + lane;
        const int row = n0 + r;
        const int ewr = row < p.rows ? p.ew[row] : 0;
        const uint32_t lane_addr = (uint32_t)(32 * qw) << 16;
        bool ok = true;
        const int sw = r & 7;  // this row's 128-byte swizzle phase
        for (int c = 0; c < p.nchunks && ok; ++c) {
            const int g = c / S_CHUNKS, ss = g % SS, cc = c % S_CHUNKS;
            if (cc == 0 && !mbar_wait(SFULL + 8 * ss, (g / SS) & 1, abort_flag, WAIT_BUDGET)) {
                ok = false;
                break;
            }
            const int ws = c % SW;
            if (!mbar_wait(WFULL + 8 * ws, (c / SW) & 1, abort_flag, WAIT_BUDGET)) {
                ok = false;
                break;
            }
            const uint8_t* wst = smem + C::OFF_W + ws * W_STAGE_BYTES + r * 128;
            uint4 v[8];
#pragma unroll
            for (int l = 0; l < 8; ++l) v[l] = *reinterpret_cast<const uint4*>(wst + ((l ^ sw) << 4));
            const float4 s4 = *reinterpret_cast<const float4*>(smem + C::OFF_S + ss * S_STAGE_BYTES + r * 128 +
                                                               ((cc ^ sw) << 4));
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(WEMPTY + 8 * ws);
                if (cc == S_CHUNKS - 1 || c == p.nchunks - 1) mbar_arrive(SEMPTY + 8 * ss);
            }
            const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
            __half2 s16[4];
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) s16[bb] = __float2half2_rn(mul_pow2(sv[bb], ewr));

#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int ks = 2 * c + h;
                if (ks >= p.nksteps) break;
                const int as = ks % SA;
                if (!mbar_wait(AEMPTY + 8 * as, ((ks / SA) & 1) ^ 1, abort_flag, WAIT_BUDGET)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t out[32];
#pragma unroll
                for (int bbl = 0; bbl < 2; ++bbl) {
                    const int bb = 2 * h + bbl;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        // bytes j of lanes (2lp, 2lp+1), block bb -> K elements (k, k+1)
                        const uint32_t sel = (uint32_t)j | ((uint32_t)j << 4) | ((uint32_t)(4 + j) << 8) |
                                             ((uint32_t)(4 + j) << 12);
#pragma unroll
                        for (int lp = 0; lp < 4; ++lp) {
                            const uint32_t t = __byte_perm(word_of(v[2 * lp], bb), word_of(v[2 * lp + 1], bb), sel);
                            // fp16 bit patterns 0x64XX = 1024 + XX with XX = q + 128
                            const uint32_t u = (t & 0x00FF00FFu) ^ 0x64806480u;
                            __half2 hq = __hsub2(*reinterpret_cast<const __half2*>(&u),
                                                 __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));
                            const __half2 wv = __hmul2(hq, s16[bb]);
                            out[16 * bbl + 4 * j + lp] = *reinterpret_cast<const uint32_t*>(&wv);
                        }
                    }
                }
                tmem_st_32x32b_x32(tmem + lane_addr + C::A_COL0 + as * 32, out);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(AFULL + 8 * as);
            }
        }
        if (!ok) {
            *abort_flag = 1;
            atomicCAS(p.status, 0, ST_TIMEOUT_CONVERT);
        }
        // The accumulator (or, after an abort, the drained MMA pipe).
        mbar_wait(ACCFULL, 0, nullptr, WAIT_BUDGET);
        tc_fence_after();
        if (!*abort_flag) {
            for (int col0 = 0; col0 < BN; col0 += 16) {
                if (m0 + col0 >= p.M) break;  // warp-uniform
                uint32_t acc[16];
                tmem_ld_32x32b_x16(tmem + lane_addr + col0, acc);
                tmem_ld_wait();
                if (row < p.rows) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int tok = m0 + col0 + i;
                        if (tok < p.M)
                            p.y[(int64_t)tok * p.ldy + row] = mul_pow2(__uint_as_float(acc[i]), -(ewr + p.ea[tok]));
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// Activations fp32 [M][ldx] -> fp16 [M][k_pad] scaled by 2^ea[m] so the row's
// largest finite magnitude lands in [2^13, 2^14); zeros past k.
__global__ void __launch_bounds__(256) act_to_f16_kernel(const float* __restrict__ x, int64_t ldx, int K, int k_pad,
                                                         __half* __restrict__ x16, int* __restrict__ ea) {
    __shared__ float red[8];
    pdl_launch_dependents();
    pdl_wait();  // x comes from the previous kernel; x16/ea may still be read by the previous GEMM
    const int m = blockIdx.x;
    const float* xr = x + (int64_t)m * ldx;
    float mx = 0.0f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float a = fabsf(xr[k]);
        if (a > mx && a <= 3.4028234663852886e38f) mx = a;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, red[i]);
    const int e = mx > 0.0f ? 14 - frexp_exponent(mx) : 0;
    __half* dst = x16 + (int64_t)m * k_pad;
    for (int k = threadIdx.x; k < k_pad; k += blockDim.x)
        dst[k] = k < K ? __float2half_rn(mul_pow2(xr[k], e)) : __ushort_as_half(0);
    if (threadIdx.x == 0) ea[m] = e;
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

template <int BN>
cudaError_t launch_bn(const TcMaps& maps, const CUtensorMap& tm_x, const TcParams& p, cudaStream_t stream,
                      bool pdl) {
    using C = TcCfg<BN>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(gemm_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((p.rows + BM - 1) / BM), (unsigned)((p.M + BN - 1) / BN));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN>, maps.w, maps.s, tm_x, p);
}

}  // namespace

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
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
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

int tc_pick_bn(int M) { return M <= 64 ? 64 : (M <= 128 ? 128 : 256); }

cudaError_t launch_gemm_tc(const TcMaps& maps, const int* ew, int rows, int k, const float* x, int64_t ldx, int M,
                           void* x16_scratch, int* ea_scratch, float* y, int64_t ldy, int* status,
                           cudaStream_t stream, bool pdl) {
    auto enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    const int k_pad = packed_k(k);
    const int bn = tc_pick_bn(M);
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
        cudaError_t e = cudaLaunchKernelEx(&cfg, act_to_f16_kernel, x, ldx, k, k_pad,
                                           static_cast<__half*>(x16_scratch), ea_scratch);
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
    p.nchunks = k_pad / 128;
    p.nksteps = k_pad / BK;
    p.status = status;
    switch (bn) {
        case 64: return launch_bn<64>(maps, tm_x, p, stream, pdl);
        case 128: return launch_bn<128>(maps, tm_x, p, stream, pdl);
        default: return launch_bn<256>(maps, tm_x, p, stream, pdl);
    }
}

}  // namespace qlm
