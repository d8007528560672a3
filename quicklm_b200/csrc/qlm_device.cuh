// qlm_device.cuh — device-side helpers shared by the sm_100a kernels.
//
// Packed int8 weight layout in HBM ("P128"), chosen for the decode GEMV:
//   k_pad  = round_up(k, 128), nb_pad = k_pad / 32
//   q      : uint8 [rows][k_pad]; element k of row r lives at byte
//            r*k_pad + (k/128)*128 + (k%8)*16 + ((k/32)%4)*4 + (k%32)/8
//   scales : fp32  [rows][nb_pad]; scale of block b of row r at r*nb_pad + b
// Inside one 128-element chunk, the 16 bytes at offset l*16 are exactly the
// elements "lane" l of the reference kernel consumes from the chunk's four
// 32-blocks (k = 32*bb + 8*j + l, byte bb*4 + j): one 128-bit load per lane per
// chunk, and the 8 lanes of a row read one contiguous 128-byte line.
// Padding bytes are 0 and padding scales are 0; kernels never fold them in.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace qlm {

constexpr int kBlock = 32;   // Tensor::INT8_BLOCK_SIZE
constexpr int kChunk = 128;  // elements per packed chunk (4 blocks)

__host__ __device__ inline int round_up(int v, int m) { return (v + m - 1) / m * m; }
__host__ __device__ inline int packed_k(int k) { return round_up(k, kChunk); }

// Byte offset of element k within a packed row.
__host__ __device__ inline int packed_offset(int k) {
    return (k & ~(kChunk - 1)) + (k & 7) * 16 + ((k >> 5) & 3) * 4 + ((k >> 3) & 3);
}

// int4 packing ("P128/4"): k_pad / 2 bytes per row; inside one 128-element
// chunk (64 bytes) the 8 bytes at l*8 are lane l's: bytes 0..3 hold steps
// j = 0..3 of blocks 0 (low nibble) and 1 (high nibble), bytes 4..7 those of
// blocks 2 and 3. A nibble is value + 8 (QuickLM's Q4_0 bias). Byte offset of
// element k within a packed row, and the shift of its nibble in that byte:
__host__ __device__ inline int packed_offset_q4(int k) {
    return ((k & ~(kChunk - 1)) >> 1) + (k & 7) * 8 + (((k >> 5) & 3) >> 1) * 4 + ((k >> 3) & 3);
}
__host__ __device__ inline int packed_shift_q4(int k) { return ((k >> 5) & 1) * 4; }

// Position of x[k] in the permuted activation staging used by the GEMV:
// chunk c, block bb, lane l, j -> c*128 + bb*32 + l*4 + j, so lane l reads
// the four x values of block bb as one float4 (conflict-free across lanes).
__host__ __device__ inline int xperm_offset(int k) {
    return (k & ~(kChunk - 1)) + ((k >> 5) & 3) * 32 + (k & 7) * 4 + ((k >> 3) & 3);
}

// Exact int8 -> fp32 for the 4 signed bytes of w: byte j (0..3) is biased to
// u = q + 128 and placed in the low mantissa of 2^23, so the float is exactly
// 2^23 + u; subtracting 2^23 + 128 is exact. Returns q_j as fp32 in f[j].
__device__ __forceinline__ void s8x4_to_f32(uint32_t w, float f[4]) {
    const uint32_t u = w ^ 0x80808080u;
    const float bias = 8388736.0f;  // 2^23 + 128
    f[0] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)), bias);
    f[1] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)), bias);
    f[2] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)), bias);
    f[3] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)), bias);
}

// Streaming 128-bit load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float4 ldg_f4(const void* p) {
    float4 r;
    asm volatile("ld.global.nc.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p));
    return r;
}

// 1-D bulk copy global -> shared (no multicast), completing on an mbarrier.
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// Bring `bytes` (a multiple of 16) of global memory at `src` (16-byte
// aligned) into L2 without a destination: the copy engine fetches it while
// the issuing thread goes on.
__device__ __forceinline__ void prefetch_l2_bulk(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// Order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) writes to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Paired fp32 arithmetic (sm_100): two IEEE binary32 ops, each rounded to
// nearest-even, in one instruction.
__device__ __forceinline__ unsigned long long f2pack(float a, float b) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
// Pair two 32-bit registers (lo, hi) without arithmetic.
__device__ __forceinline__ unsigned long long u2pack(uint32_t lo, uint32_t hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ void f2unpack(unsigned long long v, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2mul(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long f2add(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long f2fma(unsigned long long a, unsigned long long b,
                                                    unsigned long long c) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ unsigned long long f2sub(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// Exact int8 -> fp32 for the 4 signed bytes of w, as two float pairs:
// lo = (q0, q1), hi = (q2, q3). Same bias construction as s8x4_to_f32.
__device__ __forceinline__ void s8x4_to_f32x2(uint32_t w, unsigned long long& lo, unsigned long long& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const unsigned long long bias = 0x4B0000804B000080ull;  // (2^23 + 128, 2^23 + 128)
    const uint32_t b0 = __byte_perm(u, 0x4B000000u, 0x7540), b1 = __byte_perm(u, 0x4B000000u, 0x7541);
    const uint32_t b2 = __byte_perm(u, 0x4B000000u, 0x7542), b3 = __byte_perm(u, 0x4B000000u, 0x7543);
    lo = f2sub(((unsigned long long)b1 << 32) | b0, bias);
    hi = f2sub(((unsigned long long)b3 << 32) | b2, bias);
}

// Release/acquire fence at system scope (orders this thread's, and by
// cumulativity its CTA's barrier-ordered, memory accesses for peer GPUs).
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// System-scope release store / acquire load (flags shared with peer GPUs).
__device__ __forceinline__ void st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// 64-bit relaxed accesses at system scope (single-copy atomic: a reader sees
// a whole word written by a peer GPU or none of it; never served from L1).
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int ld_relaxed_sys_i32(const int* p) {
    int v;
    asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Nanoseconds of the GPU's global timer (for wait limits given in time).
__device__ __forceinline__ long long globaltimer_ns() {
    long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Programmatic dependent launch (sm_90+): let the next kernel in the stream
// start launching, and wait until the previous kernel's results are visible.
// Both are no-ops when the launch did not opt in.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launch `kern` in stream s; with pdl, as a programmatic-dependent secondary
// of the previous kernel in the stream: it may start while that kernel still
// runs, so it must call pdl_wait() before touching data another kernel writes,
// and read such data through L2 (its L1 may hold lines from before the
// producer's stores).
template <typename... P, typename... A>
inline cudaError_t launch_pdl(bool pdl, void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              A&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<A&&>(args)...);
}

}  // namespace qlm
