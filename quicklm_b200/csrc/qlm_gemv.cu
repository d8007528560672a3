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
};

// x element k lives at (k/128)*128 + j*32 + l*4 + bb (block bb = (k/32)%4,
// step j = (k/8)%4, lane l = k%8): lane l reads the four blocks' x for step j
// as one float4 at chunk*128 + j*32 + l*4.
__device__ __forceinline__ int xperm(int k) {
    return (k & ~(kChunk - 1)) + ((k >> 3) & 3) * 32 + (k & 7) * 4 + ((k >> 5) & 3);
}

// One 128-element chunk for this lane: 4 blocks x 4 steps, scales sv[0..3].
// int8 -> fp32 uses paired subtracts (no multiply feeds them). Products and
// their sums stay scalar mul.rn / add.rn: ptxas (CUDA 12.9, sm_100a) was seen
// to contract a paired mul.rn.f32x2 into the add.rn.f32x2 consuming it, which
// changes the reference's rounding; the scalar .rn forms are never contracted.
template <int MM>
__device__ __forceinline__ void chunk_update(const float* __restrict__ xs_chunk, int k_pad, int lane, uint4 qv,
                                             float4 sv, float (&t)[MM], int nblocks) {
    const uint32_t u0 = qv.x ^ 0x80808080u, u1 = qv.y ^ 0x80808080u;
    const uint32_t u2 = qv.z ^ 0x80808080u, u3 = qv.w ^ 0x80808080u;
    const unsigned long long bias = 0x4B0000804B000080ull;  // (2^23 + 128) x 2
    float qf[4][4];  // [block][step]
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t sel = 0x7540u | (uint32_t)j;
        const uint32_t f0 = __byte_perm(u0, 0x4B000000u, sel), f1 = __byte_perm(u1, 0x4B000000u, sel);
        const uint32_t f2 = __byte_perm(u2, 0x4B000000u, sel), f3 = __byte_perm(u3, 0x4B000000u, sel);
        f2unpack(f2sub(((unsigned long long)f1 << 32) | f0, bias), qf[0][j], qf[1][j]);
        f2unpack(f2sub(((unsigned long long)f3 << 32) | f2, bias), qf[2][j], qf[3][j]);
    }
    const float sc[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
    for (int m = 0; m < MM; ++m) {
        const float* xm = xs_chunk + (size_t)m * k_pad + lane * 4;
        float xv[4][4];  // [step][block]
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 v = *reinterpret_cast<const float4*>(xm + j * 32);
            xv[j][0] = v.x;
            xv[j][1] = v.y;
            xv[j][2] = v.z;
            xv[j][3] = v.w;
        }
        float tt = t[m];
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
            if (bb < nblocks) {
                const float p0 = __fmul_rn(xv[0][bb], qf[bb][0]);
                const float p1 = __fmul_rn(xv[1][bb], qf[bb][1]);
                const float p2 = __fmul_rn(xv[2][bb], qf[bb][2]);
                const float p3 = __fmul_rn(xv[3][bb], qf[bb][3]);
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
    const int u_begin = (int)(((int64_t)blockIdx.x * p.units) / gridDim.x);
    const int u_end = (int)(((int64_t)(blockIdx.x + 1) * p.units) / gridDim.x);
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
    for (int i = threadIdx.x; i < MM * p.k_pad; i += blockDim.x) {
        const int m = i / p.k_pad, kk = i - m * p.k_pad;
        xs[m * p.k_pad + xperm(kk)] = (kk < p.k) ? p.x[(int64_t)m * p.ldx + kk] : 0.0f;
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
        for (int c = c0; c < c1; ++c) {
            const uint4 qv = *reinterpret_cast<const uint4*>(sq + (c - c0) * kChunk);
            const float4 sv = *reinterpret_cast<const float4*>(ss + (c - c0) * 16);
            chunk_update<MM>(xs + c * kChunk, p.k_pad, lane, qv, sv, t, c < cfull ? 4 : rem_blocks);
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

struct Plan {
    int mm, sc, nseg, d, nwarps, ctas, xs_bytes, smem;
};

bool make_plan(int mm, int rows, int k, int sm_count, Plan* pl) {
    const int k_pad = packed_k(k);
    const int nck = k_pad / kChunk;
    pl->mm = mm;
    pl->sc = nck < kMaxSegChunks ? nck : kMaxSegChunks;
    pl->nseg = (nck + pl->sc - 1) / pl->sc;
    const int slot_bytes = pl->sc * kSlotBytesPerChunk;
    pl->xs_bytes = round_up(mm * k_pad * 4, 128);
    const int units = (rows + 3) / 4;
    pl->ctas = units < sm_count ? units : sm_count;
    const int upc = (units + pl->ctas - 1) / pl->ctas;
    // Short kernels: everything in flight at once within ~113 KB, leaving room
    // for the next kernel's CTA on the same SM. Long ones: up to 200 KB.
    const int small_budget = 113 * 1024, big_budget = 200 * 1024;
    int max_slots = (small_budget - pl->xs_bytes - 1024) / slot_bytes;
    const int upw_all = upc;  // with one warp per unit
    if (max_slots >= 1 && upc <= 16 && upw_all * pl->nseg <= max_slots) {
        pl->nwarps = upc;
        pl->d = pl->nseg;
    } else {
        max_slots = (big_budget - pl->xs_bytes - 1024) / slot_bytes;
        if (max_slots < 1) return false;
        pl->nwarps = upc < 16 ? upc : 16;
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
    static bool attr_set[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(gemv_stream_kernel<MM>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    GemvParams p = p0;
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
    return cudaLaunchKernelEx(&cfg, gemv_stream_kernel<MM>, p);
}

}  // namespace

bool gemv_supported(int mm, int rows, int k, int sm_count) {
    Plan pl;
    return make_plan(mm, rows, k, sm_count, &pl);
}

cudaError_t launch_gemv_exact(const float* x, int64_t ldx, int mm, const uint8_t* q, const float* s, int rows,
                              int k, float* y, int64_t ldy, int* status, int sm_count, cudaStream_t stream, bool pdl) {
    Plan pl;
    if (!make_plan(mm, rows, k, sm_count, &pl)) return cudaErrorInvalidValue;
    GemvParams p{};
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
