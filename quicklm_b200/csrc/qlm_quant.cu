// qlm_quant.cu — load-time int8 quantize-and-pack on the device.
//
// Replaces st_quantize_row_f32 / st_quantize_row_bf16 (QuickLM
// src/io/safetensors.cpp:348-391 / 296-345) as driven by
// get_tensor_keep_int8 (src/io/safetensors.cpp:517-585). Per 32-element block:
//   max_abs = max |v| (8 strided lanes, then the fixed 8->1 tree, then a
//             scalar pass over the < 8 elements left in a ragged block)
//   scale   = max_abs > 0 ? max_abs / 127 : 1          (IEEE division)
//   inv     = 1 / scale                                (IEEE division)
//   q       = clamp(round(v * inv), -127, 127)
// with round-half-even for elements covered by an 8-wide step and
// round-half-away (lround) for the scalar remainder, exactly as the reference.
// NaN/Inf follow the x86 semantics the reference inherits (MAXPS returns its
// second operand when unordered; cvtps2dq returns 0x80000000; (int)lround of
// NaN/Inf is 0), so the bytes and scales are identical for every input.
//
// The int4 variant (Q4 = true) replaces st_quantize_row_f32_int4 /
// st_quantize_row_bf16_int4 (src/io/safetensors.cpp:393-515, driven by
// get_tensor_keep_int4): the same block loop with scale = max_abs / 8 and
// values clamped to [-8, 7], stored as value + 8 in the P128/4 nibble layout
// (qlm_device.cuh); padding nibbles are 8 (value 0).
//
// Work mapping: one warp per (row, 32 consecutive blocks). The warp stages the
// 1024 source values through shared memory with coalesced loads, each lane
// quantizes one block, and the packed bytes go back out through shared memory
// as one contiguous 1 KB store (the P128 layout keeps 8 chunks contiguous).
//
// repack_kernel moves codes that are already quantized, in the reference
// Tensor's own layouts (int8 [rows][k]; int4 [rows][(k+1)/2] bytes, low nibble
// = even column), into the packed layouts, with the scales copied into the
// padded [rows][k_pad/32] array: the load path of pre-quantized weights.
#include "qlm_device.cuh"
#include "qlm_kernels.h"

namespace qlm {
namespace {

constexpr int kWarpsPerCta = 8;

__device__ __forceinline__ float maxps(float a, float b) { return (a > b) ? a : b; }
__device__ __forceinline__ float stdmax(float a, float b) { return (a < b) ? b : a; }

__device__ __forceinline__ int32_t cvt_rne_indefinite(float v) {
    const float r = rintf(v);  // cvt.rni: round to nearest, ties to even
    if (!(fabsf(r) < 2147483648.0f)) return INT32_MIN;
    return (int32_t)r;
}

// (int)std::lround(v): ties away from zero; NaN/Inf/|v| >= 2^63 give
// (int)LONG_MIN == 0; otherwise the low 32 bits of the long.
__device__ __forceinline__ int32_t cvt_lround_int(float v) {
    if (!(fabsf(v) < 9.2233720368547758e18f)) return 0;
    float t = truncf(v);
    if (fabsf(__fsub_rn(v, t)) >= 0.5f) t = __fadd_rn(t, copysignf(1.0f, v));
    const long long l = (long long)t;
    return (int32_t)(uint32_t)(unsigned long long)l;
}

__device__ __forceinline__ uint32_t clamp127_byte(int32_t q) {
    q = q < -127 ? -127 : (q > 127 ? 127 : q);
    return (uint32_t)(q & 0xFF);
}

__device__ __forceinline__ float load_src(const void* src, int dtype, int64_t idx) {
    if (dtype == 1) {
        const uint16_t h = static_cast<const uint16_t*>(src)[idx];
        return __uint_as_float((uint32_t)h << 16);
    }
    return static_cast<const float*>(src)[idx];
}

template <bool Q4>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
quantize_pack_kernel(const void* __restrict__ src, int dtype, int64_t src_stride, int rows, int k,
                     int k_pad, uint8_t* __restrict__ q, float* __restrict__ scales) {
    __shared__ float vals[kWarpsPerCta][32][33];
    __shared__ __align__(16) uint8_t packed[kWarpsPerCta][1024];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb_pad = k_pad / kBlock;
    const int nseg = (nb_pad + 31) / 32;
    const int64_t gw = (int64_t)blockIdx.x * kWarpsPerCta + warp;
    if (gw >= (int64_t)rows * nseg) return;  // whole warp exits together
    const int row = (int)(gw / nseg), seg = (int)(gw % nseg);
    const int64_t base = (int64_t)row * src_stride;
    const int e0 = seg * 1024;

    // Coalesced staging: element e0 + 32*i + lane -> vals[i][lane].
#pragma unroll 4
    for (int i = 0; i < 32; ++i) {
        const int e = e0 + 32 * i + lane;
        vals[warp][i][lane] = (e < k) ? load_src(src, dtype, base + e) : 0.0f;
    }
    __syncwarp();

    const int blk = seg * 32 + lane;  // this lane's block
    const int k0 = blk * kBlock;
    uint32_t words[8];  // word l holds bytes j=0..3 of lane l for this block
    float scale = 0.0f;
    if (blk < nb_pad && k0 < k) {
        const int k1 = min(k0 + kBlock, k);
        const float* v = vals[warp][lane];  // v[i] = element k0 + i
        const int len = k1 - k0;
        float lanemax[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        int i = 0;
        for (; i + 8 <= len; i += 8)
#pragma unroll
            for (int t = 0; t < 8; ++t) lanemax[t] = maxps(lanemax[t], fabsf(v[i + t]));
        float m0 = maxps(lanemax[0], lanemax[4]), m1 = maxps(lanemax[1], lanemax[5]);
        const float m2 = maxps(lanemax[2], lanemax[6]), m3 = maxps(lanemax[3], lanemax[7]);
        m0 = maxps(m0, m2);
        m1 = maxps(m1, m3);
        float max_abs = maxps(m0, m1);
        for (; i < len; ++i) max_abs = stdmax(max_abs, fabsf(v[i]));
        scale = (max_abs > 0.0f) ? __fdiv_rn(max_abs, Q4 ? 8.0f : 127.0f) : 1.0f;
        const float inv = __fdiv_rn(1.0f, scale);
        const int vec_end = len & ~7;  // elements handled by 8-wide steps
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            uint32_t w = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int e = 8 * j + l;
                uint32_t b = Q4 ? 8u : 0u;  // value 0
                if (e < len) {
                    const float p = __fmul_rn(v[e], inv);
                    const int32_t qi = e < vec_end ? cvt_rne_indefinite(p) : cvt_lround_int(p);
                    b = Q4 ? (uint32_t)((qi < -8 ? -8 : (qi > 7 ? 7 : qi)) + 8) : clamp127_byte(qi);
                }
                w |= b << (8 * j);
            }
            words[l] = w;
        }
    } else {
#pragma unroll
        for (int l = 0; l < 8; ++l) words[l] = Q4 ? 0x08080808u : 0u;
    }
    if (blk < nb_pad) scales[(int64_t)row * nb_pad + blk] = scale;

    uint32_t* pw = reinterpret_cast<uint32_t*>(packed[warp]);
    if (Q4) {
        // Segment = 8 chunks x 64 bytes. Blocks 2p (low nibbles) and 2p + 1
        // (high nibbles) of a chunk share lane slice word p.
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t partner = __shfl_xor_sync(0xffffffffu, words[l], 1);
            if ((lane & 1) == 0) pw[(lane >> 2) * 16 + l * 2 + ((lane & 3) >> 1)] = words[l] | (partner << 4);
        }
    } else {
        // Packed position inside this segment's 1 KB: chunk (lane/4), lane l, block lane%4.
#pragma unroll
        for (int l = 0; l < 8; ++l) pw[(lane >> 2) * 32 + l * 4 + (lane & 3)] = words[l];
    }
    __syncwarp();

    // 8 chunks of 128 (int8) or 64 (int4) bytes; the segment may stop short
    // of 8 chunks at the row end.
    constexpr int CB = Q4 ? 64 : 128;
    const int chunks = min(8, nb_pad / 4 - seg * 8);
    uint4* dst = reinterpret_cast<uint4*>(q + (int64_t)row * (k_pad / kChunk) * CB + (int64_t)seg * 8 * CB);
    const uint4* s4 = reinterpret_cast<const uint4*>(packed[warp]);
    for (int i = lane; i < chunks * (CB / 16); i += 32) dst[i] = s4[i];
}

}  // namespace

cudaError_t launch_quantize_pack(const void* src, int dtype, int64_t src_stride, int rows, int k, uint8_t* q,
                                 float* scales, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    const int k_pad = packed_k(k);
    const int nseg = (k_pad / kBlock + 31) / 32;
    const int64_t warps = (int64_t)rows * nseg;
    const int64_t ctas = (warps + kWarpsPerCta - 1) / kWarpsPerCta;
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
    quantize_pack_kernel<false><<<(unsigned)ctas, kWarpsPerCta * 32, 0, stream>>>(src, dtype, src_stride, rows, k,
                                                                                   k_pad, q, scales);
    return cudaGetLastError();
}

cudaError_t launch_quantize_pack_q4(const void* src, int dtype, int64_t src_stride, int rows, int k, uint8_t* q,
                                    float* scales, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    const int k_pad = packed_k(k);
    const int nseg = (k_pad / kBlock + 31) / 32;
    const int64_t warps = (int64_t)rows * nseg;
    const int64_t ctas = (warps + kWarpsPerCta - 1) / kWarpsPerCta;
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
    quantize_pack_kernel<true><<<(unsigned)ctas, kWarpsPerCta * 32, 0, stream>>>(src, dtype, src_stride, rows, k,
                                                                                  k_pad, q, scales);
    return cudaGetLastError();
}

namespace {

// One thread per (row, 128-element chunk, lane l): the 16 int8 bytes (or 8
// int4 bytes) lane l of the GEMV reads from the chunk, gathered from the row-
// major codes; lanes 0..3 also move the chunk's four scales.
template <bool Q4>
__global__ void repack_kernel(const uint8_t* __restrict__ codes, int64_t code_stride, const float* __restrict__ sin,
                              int64_t s_stride, int rows, int k, int k_pad, uint8_t* __restrict__ q,
                              float* __restrict__ sout) {
    const int nck = k_pad / kChunk, nb = (k + kBlock - 1) / kBlock, nb_pad = k_pad / kBlock;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (int64_t)rows * nck * 8) return;
    const int l = (int)(t & 7);
    const int64_t rc = t >> 3;
    const int c = (int)(rc % nck);
    const int64_t row = rc / nck;
    const uint8_t* src = codes + row * code_stride;
    const int k0 = c * kChunk + l;
    if (!Q4) {
        uint32_t w[4];
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
            uint32_t v = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kk = k0 + 32 * bb + 8 * j;
                v |= (uint32_t)(kk < k ? src[kk] : 0u) << (8 * j);
            }
            w[bb] = v;
        }
        *reinterpret_cast<uint4*>(q + (row * nck + c) * kChunk + l * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        auto nib = [&](int kk) -> uint32_t { return kk < k ? (uint32_t)(src[kk >> 1] >> ((kk & 1) * 4)) & 0xFu : 8u; };
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            lo |= (nib(k0 + 8 * j) | nib(k0 + 32 + 8 * j) << 4) << (8 * j);
            hi |= (nib(k0 + 64 + 8 * j) | nib(k0 + 96 + 8 * j) << 4) << (8 * j);
        }
        *reinterpret_cast<uint2*>(q + (row * nck + c) * (kChunk / 2) + l * 8) = make_uint2(lo, hi);
    }
    if (l < 4) {
        const int blk = 4 * c + l;
        sout[row * nb_pad + blk] = blk < nb ? sin[row * s_stride + blk] : 0.0f;
    }
}

}  // namespace

cudaError_t launch_repack(const uint8_t* codes, int64_t code_stride, const float* scales, int64_t scale_stride,
                          int rows, int k, bool q4, uint8_t* q, float* s, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    const int k_pad = packed_k(k);
    const int64_t threads = (int64_t)rows * (k_pad / kChunk) * 8;
    const int64_t ctas = (threads + 255) / 256;
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
    if (q4)
        repack_kernel<true><<<(unsigned)ctas, 256, 0, stream>>>(codes, code_stride, scales, scale_stride, rows, k,
                                                                k_pad, q, s);
    else
        repack_kernel<false><<<(unsigned)ctas, 256, 0, stream>>>(codes, code_stride, scales, scale_stride, rows, k,
                                                                 k_pad, q, s);
    return cudaGetLastError();
}

}  // namespace qlm
