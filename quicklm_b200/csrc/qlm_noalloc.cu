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
//
// The status word is sticky: the array is zero when the module loads and no
// call clears the word, so a device-side wait that gave up in an asynchronous
// call (flags = 0) stays visible until qlm_device_status(device, reset != 0)
// or a QLM_LINEAR_SYNC call of this entry point reads and clears it.
#include "../../include/qlm_b200.h"
#include "qlm_device.cuh"
#include "qlm_handle.h"
#include "qlm_kernels.h"
#include "qlm_prof.h"

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>

namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;
constexpr size_t kStatusOffset = kNoAllocScratchBytes - 256;      // one int, own 256-byte slot
constexpr size_t kExpOffset = kStatusOffset - 64 * 1024;          // activation exponents
constexpr int kMaxRows = (int)((64 * 1024) / sizeof(int));        // 16384 activation rows
constexpr size_t kActBytes = kExpOffset;                          // fp16 activation staging

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
// Devices on which this entry point has run (so the status check below never
// loads the module, and with it the 8 MiB array, on a device that never used it).
std::atomic<bool> g_used[kMaxDevices];

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

// Device address of the static scratch on the current device. The host-side
// name g_noalloc_scratch is only a stand-in for it. The address is looked up
// on every call (cheap once the module is loaded), so a context that was
// reset and reloaded never sees a stale pointer. The first lookup on a device
// loads the library's device code there, which is when the array is
// allocated: make one call at start-up, before any stream capture.
cudaError_t scratch_here(unsigned char** out) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e == cudaSuccess && !ptr) return cudaErrorInvalidSymbol;
    *out = static_cast<unsigned char*>(ptr);
    return e;
}

}  // namespace

// Defined in qlm_capi.cu: records the message for qlm_last_error().
namespace qlm_internal {
void set_last_error(const std::string& msg);

// Status word of this entry point on `device` (which must be current): 0, or
// the code of a device-side wait that gave up; cleared when reset != 0.
// Reads nothing on a device where the entry point never ran.
cudaError_t noalloc_status(int device, int reset, int* code) {
    *code = 0;
    if (device < 0 || device >= kMaxDevices || !g_used[device].load()) return cudaSuccess;
    unsigned char* base = nullptr;
    cudaError_t e = scratch_here(&base);
    if (e != cudaSuccess) return e;
    int* status = reinterpret_cast<int*>(base + kStatusOffset);
    e = cudaMemcpy(code, status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && *code != 0 && reset) e = cudaMemset(status, 0, sizeof(int));
    return e;
}
}  // namespace qlm_internal

extern "C" int qlm_linear_int8_tc_noalloc(const float* x, int M, int k, int64_t ldx, const qlm_w8* w, float* y,
                                          int64_t ldy, int flags, void* stream) {
    qlm_internal::NvtxRange range("qlm_linear_int8_tc_noalloc");
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
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        cudaError_t e = scratch_here(&base);
        if (e != cudaSuccess) {
            rc = fail(QLM_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
        } else {
            if (w->device >= 0 && w->device < kMaxDevices) g_used[w->device].store(true);
            qlm::TcMaps maps;  // on the stack: encoding a tensor map allocates nothing
            e = qlm::tc_make_weight_maps(w->q, w->s, w->rows, w->k_pad, &maps);
            int* status = reinterpret_cast<int*>(base + kStatusOffset);  // sticky: never cleared here
            if (e == cudaSuccess)
                e = qlm::launch_gemm_tc(maps, w->ew, w->rows, k, x, ldx, M, base, reinterpret_cast<int*>(base + kExpOffset),
                                        y, ldy, status, s, false);
            if (e == cudaSuccess && (flags & QLM_LINEAR_SYNC)) {
                e = cudaStreamSynchronize(s);
                int code = 0;
                if (e == cudaSuccess) e = cudaMemcpy(&code, status, sizeof(int), cudaMemcpyDeviceToHost);
                if (e == cudaSuccess && code != 0) {
                    e = cudaMemset(status, 0, sizeof(int));
                    if (e == cudaSuccess)
                        rc = fail(QLM_ERR_TIMEOUT, "a device-side wait gave up (code 0x%x); results are invalid",
                                  code);
                }
            }
            if (e != cudaSuccess) rc = fail(QLM_ERR_CUDA, "tensor-core GEMM (static scratch): %s", cudaGetErrorString(e));
        }
        if (prev >= 0) cudaSetDevice(prev);
    } while (0);
    if (rc != QLM_OK) qlm_internal::set_last_error(g_err_local);
    return rc;
}
