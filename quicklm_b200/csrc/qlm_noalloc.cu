// qlm_noalloc.cu — tensor-core prefill GEMM entry point that allocates nothing.
//
// Who needs it: a host engine that reserves all device memory for its own pool
// at start-up and forbids later allocations, or a latency-critical decode loop
// where cudaMalloc/cudaFree would synchronise the device and stall other
// streams. qlm_linear_int8(QLM_LINEAR_TENSOR) grows per-device scratch buffers
// with cudaMalloc on demand; this entry point instead uses one fixed array in
// the library's own static device memory, so it never allocates.
//
// The scratch: kNoAllocScratchBytes (8 MiB) of static __device__ memory per
// GPU that loads the library, held until the process exits. It holds the fp16
// activation staging (M * round_up(k, 128) * 2 bytes), the per-row activation
// exponents (M ints) and a status word. Requests that do not fit are rejected.
// Every call on a device shares the same array: calls whose work can overlap
// on the GPU (different streams, no ordering between them) race on it.
#include "../../include/qlm_b200.h"
#include "qlm_device.cuh"
#include "qlm_handle.h"
#include "qlm_kernels.h"

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;
constexpr size_t kStatusOffset = kNoAllocScratchBytes - 256;      // one int, own 256-byte slot
constexpr size_t kExpOffset = kStatusOffset - 64 * 1024;          // activation exponents
constexpr int kMaxRows = (int)((64 * 1024) / sizeof(int));        // 16384 activation rows
constexpr size_t kActBytes = kExpOffset;                          // fp16 activation staging

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_setup_mu;

thread_local std::string g_err_local;

int fail(int code, const char* fmt, ...) {
    char buf[384];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err_local = buf;
    return code;
}

// Device address of the static scratch on `dev` (which must be current).
// The host-side name g_noalloc_scratch is only a stand-in; the address comes
// from cudaGetSymbolAddress, once per device.
int scratch_for(int dev, unsigned char** out) {
    if (dev < 0 || dev >= kMaxDevices) return fail(QLM_ERR_INVALID_ARG, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_scratch_addr[dev]) {
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr)
            return fail(QLM_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
        g_scratch_addr[dev] = ptr;
    }
    *out = static_cast<unsigned char*>(g_scratch_addr[dev]);
    return QLM_OK;
}

}  // namespace

// Defined in qlm_capi.cu: records the message for qlm_last_error().
namespace qlm_internal {
void set_last_error(const std::string& msg);
}

extern "C" int qlm_linear_int8_tc_noalloc(const float* x, int M, int k, int64_t ldx, const qlm_w8* w, float* y,
                                          int64_t ldy, int flags, void* stream) {
    int rc = QLM_OK;
    do {
        if (!x || !y || !w) {
            rc = fail(QLM_ERR_INVALID_ARG, "NULL argument");
            break;
        }
        if (M <= 0 || k != w->k || ldx < k || ldy < w->rows) {
            rc = fail(QLM_ERR_INVALID_ARG, "bad shape: M=%d k=%d (weight k=%d) ldx=%lld ldy=%lld rows=%d", M, k, w->k,
                      (long long)ldx, (long long)ldy, w->rows);
            break;
        }
        if (w->bits != 8) {
            rc = fail(QLM_ERR_UNSUPPORTED, "the tensor-core path serves int8 weights; this handle is int4");
            break;
        }
        if (flags & ~QLM_LINEAR_SYNC) {
            rc = fail(QLM_ERR_INVALID_ARG, "only QLM_LINEAR_SYNC is accepted here (device pointers only)");
            break;
        }
        const size_t act_bytes = (size_t)M * (size_t)w->k_pad * 2;
        if (M > kMaxRows || act_bytes > kActBytes) {
            rc = fail(QLM_ERR_INVALID_ARG,
                      "M=%d x k=%d needs %zu bytes of activation staging; the static scratch holds %zu bytes and "
                      "%d rows",
                      M, k, act_bytes, kActBytes, kMaxRows);
            break;
        }
        int prev = -1;
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (cudaSetDevice(w->device) != cudaSuccess) {
            rc = fail(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", w->device);
            break;
        }
        unsigned char* base = nullptr;
        rc = scratch_for(w->device, &base);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (rc == QLM_OK) {
            qlm::TcMaps maps;  // on the stack: encoding a tensor map allocates nothing
            cudaError_t e = qlm::tc_make_weight_maps(w->q, w->s, w->rows, w->k_pad, &maps);
            int* status = reinterpret_cast<int*>(base + kStatusOffset);
            if (e == cudaSuccess) e = cudaMemsetAsync(status, 0, sizeof(int), s);  // must start at zero
            if (e == cudaSuccess)
                e = qlm::launch_gemm_tc(maps, w->ew, w->rows, k, x, ldx, M, base, reinterpret_cast<int*>(base + kExpOffset),
                                        y, ldy, status, s, false);
            if (e == cudaSuccess && (flags & QLM_LINEAR_SYNC)) {
                e = cudaStreamSynchronize(s);
                int code = 0;
                if (e == cudaSuccess) e = cudaMemcpy(&code, status, sizeof(int), cudaMemcpyDeviceToHost);
                if (e == cudaSuccess && code != 0)
                    rc = fail(QLM_ERR_TIMEOUT, "a device-side wait gave up (code 0x%x)", code);
            }
            if (e != cudaSuccess) rc = fail(QLM_ERR_CUDA, "tensor-core GEMM (static scratch): %s", cudaGetErrorString(e));
        }
        if (prev >= 0) cudaSetDevice(prev);
    } while (0);
    if (rc != QLM_OK) qlm_internal::set_last_error(g_err_local);
    return rc;
}
