// qlm_argmax.cu — greedy token selection over lm_head logits on the device,
// replacing DecoderModel::sample(logits, 0, 0) (QuickLM src/model/model.cpp:
// 259-272): a scan from index 0 that keeps the first strictly larger logit.
// Equivalently: 0 if logits[0] is NaN, otherwise the lowest index holding the
// maximum of the non-NaN logits (NaN never compares larger; equal values,
// +0 and -0 included, keep the lower index).
//
// One CTA reduces this rank's shard with a commutative, associative choice
// (larger value, then lower index; NaN candidates excluded). With a row-
// sharded lm_head the ranks then exchange one 64-bit word each instead of the
// logits: (tag << 56) | (global index << 32) | value bits, tag = 0x80 | the
// call epoch's low 7 bits (never zero), stored with a single-copy-atomic 8-byte
// store into every rank's exchange header (halves by epoch parity, like the
// gathered GEMV's words). Every rank combines the words in rank order (shards
// are contiguous, so rank order is index order) and clears its own slots after
// reading them, so a slot only ever holds a word of the call that reads it:
// its next writer is a peer's call e + 2, which starts only after this rank's
// call e + 1 — and therefore this kernel — has completed.
#include "qlm_device.cuh"
#include "qlm_kernels.h"

#include <cstdint>

namespace qlm {
namespace {

constexpr int kThreads = 1024;
constexpr int kStatusArgmaxTimeout = 0x203;
constexpr uint32_t kIdxNone = 0xFFFFFFu;     // no non-NaN logit in the shard
constexpr uint32_t kIdxFirstNan = 0xFFFFFEu;  // global logit 0 is NaN: the answer is 0

struct Cand {
    float v;
    int i;  // -1: none
};

__device__ __forceinline__ Cand pick(Cand a, Cand b) {
    if (a.i < 0) return b;
    if (b.i < 0) return a;
    if (b.v > a.v) return b;
    if (a.v > b.v) return a;
    return b.i < a.i ? b : a;
}

__device__ __forceinline__ Cand shfl_pick(Cand c) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Cand d;
        d.v = __shfl_xor_sync(0xffffffffu, c.v, o);
        d.i = __shfl_xor_sync(0xffffffffu, c.i, o);
        c = pick(c, d);
    }
    return c;
}

__global__ void __launch_bounds__(kThreads) argmax_kernel(const float* __restrict__ y, int n, int col0, ArgmaxArgs a,
                                                          int* out_idx, float* out_val) {
    __shared__ Cand warp_best[kThreads / 32];
    __shared__ Cand rank_best[kMaxRanks];
    __shared__ int rank_first_nan[kMaxRanks];
    pdl_wait();  // the logits come from the previous kernel
    pdl_launch_dependents();
    Cand c{0.0f, -1};
    for (int base = 0; base < n; base += 8 * kThreads) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = base + u * kThreads + (int)threadIdx.x;
            v[u] = i < n ? y[i] : __int_as_float(0x7fc00000);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = base + u * kThreads + (int)threadIdx.x;
            if (!isnan(v[u])) c = pick(c, Cand{v[u], i});
        }
    }
    c = shfl_pick(c);
    if ((threadIdx.x & 31) == 0) warp_best[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x < 32) {
        c = warp_best[threadIdx.x];
        c = shfl_pick(c);
    }
    // c (thread 0): this shard's best non-NaN logit, local index
    const bool first_nan = col0 == 0 && n > 0 && isnan(y[0]);
    if (a.nranks == 0) {
        if (threadIdx.x == 0) {
            if (first_nan) {
                *out_idx = 0;
                *out_val = y[0];
            } else {
                *out_idx = c.i < 0 ? -1 : col0 + c.i;
                *out_val = c.i < 0 ? __int_as_float(0x7fc00000) : c.v;
            }
        }
        return;
    }
    // A failed communicator (a bounded wait gave up earlier): do nothing.
    if (a.status && *reinterpret_cast<volatile const int*>(a.status) != 0) return;
    const int e = *reinterpret_cast<volatile const int*>(a.epochs) + 1;
    const unsigned long long* mine = a.peer_words[a.rank] + (e & 1) * kMaxRanks;
    if (threadIdx.x == 0) {
        const uint32_t idx = first_nan ? kIdxFirstNan : (c.i < 0 ? kIdxNone : (uint32_t)(col0 + c.i));
        const unsigned long long word = ((unsigned long long)(0x80 | (e & 0x7F)) << 56) |
                                        ((unsigned long long)(idx & 0xFFFFFFu) << 32) |
                                        (c.i < 0 ? 0u : __float_as_uint(c.v));
#pragma unroll 1
        for (int r = 0; r < a.nranks; ++r) st_relaxed_sys_u64(a.peer_words[r] + (e & 1) * kMaxRanks + a.rank, word);
    }
    if ((int)threadIdx.x < a.nranks) {
        const int r = threadIdx.x;
        const long long t0 = globaltimer_ns();
        unsigned long long w = ld_relaxed_sys_u64(mine + r);
        bool ok = true;
        while ((int)(w >> 56) != (0x80 | (e & 0x7F))) {
            if (globaltimer_ns() - t0 > a.wait_ns) {
                ok = false;
                if (a.status) atomicCAS(a.status, 0, kStatusArgmaxTimeout);
                break;
            }
            __nanosleep(32);
            w = ld_relaxed_sys_u64(mine + r);
        }
        const uint32_t idx = (uint32_t)(w >> 32) & 0xFFFFFFu;
        st_relaxed_sys_u64(const_cast<unsigned long long*>(mine) + r, 0ull);  // consumed
        rank_first_nan[r] = ok && idx == kIdxFirstNan;
        rank_best[r] = (!ok || idx >= kIdxFirstNan) ? Cand{0.0f, -1} : Cand{__uint_as_float((uint32_t)w), (int)idx};
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int first = 0;
        Cand best{0.0f, -1};
        for (int r = 0; r < a.nranks; ++r) {
            first |= rank_first_nan[r];
            best = pick(best, rank_best[r]);
        }
        if (first) {
            *out_idx = 0;
            *out_val = __int_as_float(0x7fc00000);
        } else {
            *out_idx = best.i;
            *out_val = best.i < 0 ? __int_as_float(0x7fc00000) : best.v;
        }
        if (*reinterpret_cast<volatile const int*>(a.status) == 0)
            for (int s = 0; s < a.nepochs; ++s) reinterpret_cast<volatile int*>(a.epochs)[s] = e;
    }
}

}  // namespace

cudaError_t launch_argmax(const float* y, int n, int col0, const ArgmaxArgs& a, int* out_idx, float* out_val,
                          cudaStream_t stream, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, argmax_kernel, y, n, col0, a, out_idx, out_val);
}

}  // namespace qlm
