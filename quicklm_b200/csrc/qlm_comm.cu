// qlm_comm.cu — row-sharded int8 linear with a fused NVLink all-gather.
//
// QuickLM runs on one CPU; the B200 build shards weight matrices by output
// rows across the GPUs of a box (column-parallel lm_head / MLP / projections).
// Row sharding preserves the reference's bits: each output element is still
// computed by exactly one thread with the reference's sequence
// (src/ops/math_ops.cpp:874-894), only on a different GPU.
//
// Exchange: every rank owns one exchange buffer (two halves of the gathered
// output, as 64-bit words (epoch << 32) | value) shared with the other ranks
// through CUDA IPC. A call is ONE kernel: the thread that computes an output
// row stores its word into every rank's buffer (plain 8-byte peer stores over
// NVLink; no multicast, no fences, no separate flags: the epoch travels with
// the value), then every CTA waits (bounded) until the words of its slice of
// the gathered row carry this call's epoch and copies their values into y.
// The epoch lives on the device, so a sequence of calls can be captured in a
// CUDA graph and replayed. Halves alternate by epoch parity: a rank can start
// call e + 1 only after every rank has stored all of call e, which each rank
// does only after its call e - 1 kernel (the last reader of that half) ended.
#include "../../include/qlm_b200.h"
#include "qlm_device.cuh"
#include "qlm_handle.h"
#include "qlm_kernels.h"
#include "qlm_prof.h"

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>

struct qlm_comm {
    int device = -1, rank = 0, nranks = 0, sm_count = 0;
    long long max_out = 0;             // gathered-width capacity (floats)
    long long stride = 0;              // 64-bit words per output half
    char* base = nullptr;              // local exchange buffer
    char* peers[qlm::kMaxRanks] = {};  // every rank's buffer as seen from this device
    bool opened[qlm::kMaxRanks] = {};
    int* state = nullptr;              // [0] CTA counter, [1] epoch, [2] status
    long long wait_ns = 2000000000LL;  // bounded waits for peers give up after this long
    bool failed = false;               // a wait gave up: every later call is refused
};

namespace qlm_internal {
void set_last_error(const std::string& msg);
}

namespace {

constexpr size_t kHeaderBytes = 256;  // greedy-choice words; keeps the gathered words 256-byte aligned
// Device state words: [2] the sticky status, [8, 8 + kEpochWords) the epoch
// words (qlm::GatherArgs), one per CTA index of a gather launch (at most one
// CTA per SM).
constexpr int kEpochOffset = 8;
constexpr int kEpochWords = 256;
static_assert(2 * qlm::kMaxRanks * sizeof(unsigned long long) <= kHeaderBytes, "argmax words fit the header");

int fail(int code, const char* fmt, ...) {
    char buf[384];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    qlm_internal::set_last_error(buf);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(e == cudaErrorMemoryAllocation ? QLM_ERR_OUT_OF_MEMORY : QLM_ERR_CUDA, "%s: %s", what,
                cudaGetErrorString(e));
}

struct Dev {
    int prev = -1;
    bool ok = false;
    explicit Dev(int d) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        ok = cudaSetDevice(d) == cudaSuccess;
    }
    ~Dev() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" {

int qlm_comm_create(int device, int rank, int nranks, int64_t max_out, qlm_comm** out, void* handle_out) {
    if (!out || !handle_out) return fail(QLM_ERR_INVALID_ARG, "NULL argument");
    *out = nullptr;
    if (nranks < 1 || nranks > qlm::kMaxRanks) return fail(QLM_ERR_INVALID_ARG, "nranks %d not in [1, %d]", nranks, qlm::kMaxRanks);
    if (rank < 0 || rank >= nranks) return fail(QLM_ERR_INVALID_ARG, "rank %d not in [0, %d)", rank, nranks);
    if (max_out <= 0) return fail(QLM_ERR_INVALID_ARG, "max_out must be positive");
    Dev g(device);
    if (!g.ok) return fail(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    qlm_comm* c = new (std::nothrow) qlm_comm();
    if (!c) return fail(QLM_ERR_OUT_OF_MEMORY, "host allocation failed");
    c->device = device;
    c->rank = rank;
    c->nranks = nranks;
    c->max_out = max_out;
    c->stride = (max_out + 1) & ~1LL;  // both halves start 16-byte aligned
    cudaError_t e = cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device);
    const size_t bytes = kHeaderBytes + 2 * (size_t)c->stride * sizeof(unsigned long long);
    if (e == cudaSuccess) e = cudaMalloc(&c->base, bytes);
    if (e == cudaSuccess) e = cudaMemset(c->base, 0, bytes);
    if (e == cudaSuccess && c->sm_count > kEpochWords) e = cudaErrorNotSupported;
    if (e == cudaSuccess) e = cudaMalloc(&c->state, (kEpochOffset + kEpochWords) * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->state, 0, (kEpochOffset + kEpochWords) * sizeof(int));
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->base);
    if (e != cudaSuccess) {
        if (c->base) cudaFree(c->base);
        if (c->state) cudaFree(c->state);
        delete c;
        return cuda_fail(e, "exchange buffer");
    }
    std::memcpy(handle_out, &h, sizeof(h));
    c->peers[rank] = c->base;
    *out = c;
    return QLM_OK;
}

int qlm_comm_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int qlm_comm_set_timeout_us(qlm_comm* c, int64_t us) {
    if (!c) return fail(QLM_ERR_INVALID_ARG, "NULL communicator");
    if (us < 1 || us > 600000000LL) return fail(QLM_ERR_INVALID_ARG, "timeout %lld us not in [1, 6e8]", (long long)us);
    c->wait_ns = (long long)us * 1000LL;
    return QLM_OK;
}

int qlm_comm_status(qlm_comm* c) {
    if (!c) return fail(QLM_ERR_INVALID_ARG, "NULL communicator");
    if (c->failed) return fail(QLM_ERR_TIMEOUT, "the communicator failed earlier (a peer did not answer); free and recreate it");
    Dev g(c->device);
    if (!g.ok) return fail(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    int code = 0;
    const cudaError_t e = cudaMemcpy(&code, c->state + 2, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "read status");
    if (code) {
        c->failed = true;
        return fail(QLM_ERR_TIMEOUT, "a bounded wait for peer ranks gave up (code 0x%x); free and recreate the communicator", code);
    }
    return QLM_OK;
}

int qlm_comm_connect(qlm_comm* c, const void* all_handles) {
    if (!c || !all_handles) return fail(QLM_ERR_INVALID_ARG, "NULL argument");
    Dev g(c->device);
    if (!g.ok) return fail(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    for (int r = 0; r < c->nranks; ++r) {
        if (r == c->rank || c->opened[r]) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const char*>(all_handles) + (size_t)r * sizeof(h), sizeof(h));
        void* ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle (peer exchange buffer)");
        c->peers[r] = static_cast<char*>(ptr);
        c->opened[r] = true;
    }
    return QLM_OK;
}

void qlm_comm_free(qlm_comm* c) {
    if (!c) return;
    Dev g(c->device);
    for (int r = 0; r < c->nranks; ++r)
        if (c->opened[r]) cudaIpcCloseMemHandle(c->peers[r]);
    if (c->base) cudaFree(c->base);
    if (c->state) cudaFree(c->state);
    delete c;
}

int qlm_linear_int8_allgather(const float* x, int M, int k, int64_t ldx, const qlm_w8* w, qlm_comm* c, float* y,
                              int64_t ldy, int flags, void* stream) {
    if (!x || !w || !c || !y) return fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (M != 1) return fail(QLM_ERR_UNSUPPORTED, "the fused all-gather serves decode (M = 1); got M=%d", M);
    if (k != w->k || ldx < k) return fail(QLM_ERR_INVALID_ARG, "k=%d does not match the weight's k=%d", k, w->k);
    if (ldy < w->n_total) return fail(QLM_ERR_INVALID_ARG, "ldy %lld < gathered width %d", (long long)ldy, w->n_total);
    if (w->device != c->device) return fail(QLM_ERR_INVALID_ARG, "weight and communicator on different devices");
    if (w->n_total > c->max_out) return fail(QLM_ERR_INVALID_ARG, "gathered width %d > exchange capacity %lld", w->n_total, c->max_out);
    if (flags & ~QLM_LINEAR_SYNC) return fail(QLM_ERR_INVALID_ARG, "only QLM_LINEAR_SYNC is accepted (device pointers)");
    for (int r = 0; r < c->nranks; ++r)
        if (!c->peers[r]) return fail(QLM_ERR_INVALID_ARG, "communicator not connected (rank %d)", r);
    if (c->failed) return fail(QLM_ERR_TIMEOUT, "the communicator failed earlier (a peer did not answer); free and recreate it");
    Dev g(c->device);
    if (!g.ok) return fail(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    qlm_internal::ProfScope prof("qlm_linear_int8_allgather", M, w->n_total, k, s);

    qlm::GatherArgs ga{};
    ga.wait_ns = c->wait_ns;
    for (int r = 0; r < c->nranks; ++r) {
        ga.peer_slots[r] = reinterpret_cast<unsigned long long*>(c->peers[r] + kHeaderBytes);
    }
    ga.epochs = c->state + kEpochOffset;
    ga.nepochs = kEpochWords;
    ga.out_stride = c->stride;
    ga.nranks = c->nranks;
    ga.rank = c->rank;
    ga.col0 = w->row_begin;
    ga.n_total = w->n_total;
    cudaError_t e = qlm::launch_gemv_exact(x, ldx, 1, w->q, w->s, w->gmaps, w->rows, k, y, ldy, c->state + 2,
                                           c->sm_count, s, true, &ga, w->bits == 4);
    if (e != cudaSuccess) return cuda_fail(e, "fused GEMV + all-gather launch");
    e = qlm::launch_gather_collect(ga, y, c->state + 2, c->sm_count, s, true);
    if (e != cudaSuccess) return cuda_fail(e, "all-gather collect launch");
    prof.stop();
    if (flags & QLM_LINEAR_SYNC) {
        e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
        int code = 0;
        e = cudaMemcpy(&code, c->state + 2, sizeof(int), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return cuda_fail(e, "read status");
        if (code) {
            c->failed = true;  // the status word stays set: later kernels on c do nothing
            return fail(QLM_ERR_TIMEOUT, "a bounded wait for peer ranks gave up (code 0x%x); free and recreate the communicator", code);
        }
    }
    return QLM_OK;
}

int qlm_argmax_f32(const float* logits, int n, int64_t col0, qlm_comm* c, int* out_index, float* out_value, int flags,
                   void* stream) {
    if (!logits || !out_index || !out_value) return fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (n <= 0) return fail(QLM_ERR_INVALID_ARG, "n=%d must be >= 1", n);
    if (col0 < 0 || col0 + n > 0xFFFFFD)
        return fail(QLM_ERR_INVALID_ARG, "global logit indices [%lld, %lld) exceed 2^24 - 2", (long long)col0,
                    (long long)(col0 + n));
    if (flags & ~QLM_LINEAR_SYNC) return fail(QLM_ERR_INVALID_ARG, "only QLM_LINEAR_SYNC is accepted (device pointers)");
    qlm::ArgmaxArgs a{};
    int device = -1;
    if (c) {
        for (int r = 0; r < c->nranks; ++r)
            if (!c->peers[r]) return fail(QLM_ERR_INVALID_ARG, "communicator not connected (rank %d)", r);
        if (c->failed) return fail(QLM_ERR_TIMEOUT, "the communicator failed earlier (a peer did not answer); free and recreate it");
        for (int r = 0; r < c->nranks; ++r) a.peer_words[r] = reinterpret_cast<unsigned long long*>(c->peers[r]);
        a.wait_ns = c->wait_ns;
        a.epochs = c->state + kEpochOffset;
        a.nepochs = kEpochWords;
        a.status = c->state + 2;
        a.nranks = c->nranks;
        a.rank = c->rank;
        device = c->device;
    } else {
        cudaError_t e = cudaGetDevice(&device);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    }
    Dev g(device);
    if (!g.ok) return fail(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = qlm::launch_argmax(logits, n, (int)col0, a, out_index, out_value, s, true);
    if (e != cudaSuccess) return cuda_fail(e, "argmax launch");
    if (flags & QLM_LINEAR_SYNC) {
        e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
        if (c) {
            int code = 0;
            e = cudaMemcpy(&code, c->state + 2, sizeof(int), cudaMemcpyDeviceToHost);
            if (e != cudaSuccess) return cuda_fail(e, "read status");
            if (code) {
                c->failed = true;
                return fail(QLM_ERR_TIMEOUT, "a bounded wait for peer ranks gave up (code 0x%x); free and recreate the communicator", code);
            }
        }
    }
    return QLM_OK;
}

}  // extern "C"
