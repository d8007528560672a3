// qlm_capi.cu — the C ABI declared in include/qlm_b200.h.
//
// Host-side responsibilities: argument validation (the reference's
// math::matmul validates nothing; here a bad shape is an error code, never
// undefined behaviour), device selection, weight handles, host<->device
// staging for QLM_LINEAR_HOST_IO, and dispatch to the kernels. No call throws
// across the ABI; every failure leaves a message for qlm_last_error().
#include "../../include/qlm_b200.h"
#include "qlm_device.cuh"
#include "qlm_handle.h"
#include "qlm_kernels.h"
#include "qlm_prof.h"

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>


namespace {

thread_local std::string g_err;

int set_err(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

int cuda_err(cudaError_t e, const char* what) {
    if (e == cudaErrorMemoryAllocation)
        return set_err(QLM_ERR_OUT_OF_MEMORY, "%s: %s", what, cudaGetErrorString(e));
    return set_err(QLM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define QLM_CUDA(call, what)                         \
    do {                                             \
        cudaError_t _e = (call);                     \
        if (_e != cudaSuccess) return cuda_err(_e, what); \
    } while (0)

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

constexpr int kMaxDevices = 64;

struct DeviceState {
    int sm_count = 0;
    float* x_buf = nullptr;  // HOST_IO staging
    size_t x_cap = 0;
    float* y_buf = nullptr;
    size_t y_cap = 0;
    void* x16 = nullptr;     // tensor-core path: fp16 activations
    size_t x16_cap = 0;
    int* ea = nullptr;       // tensor-core path: activation row exponents
    size_t ea_cap = 0;
    int* status = nullptr;   // device status word written by kernels on a timeout
    void* xpair = nullptr;   // exact small-M product: activations in its pair layout
    size_t xpair_cap = 0;
    cudaEvent_t done = nullptr;  // HOST_IO: marks the end of a call's work on its stream
    float* pin_x = nullptr;      // HOST_IO: pinned, mapped staging of small pageable inputs
    size_t pin_x_cap = 0;
    float* pin_y = nullptr;      // ... and outputs
    size_t pin_y_cap = 0;
};
DeviceState g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_state(int dev, DeviceState** out) {
    if (dev < 0 || dev >= kMaxDevices) return set_err(QLM_ERR_INVALID_ARG, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DeviceState& st = g_dev[dev];
    if (st.sm_count == 0) {
        int sms = 0;
        QLM_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
        int prev = -1;
        QLM_CUDA(cudaGetDevice(&prev), "cudaGetDevice");
        QLM_CUDA(cudaSetDevice(dev), "cudaSetDevice");
        cudaError_t e = cudaMalloc(&st.status, sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(st.status, 0, sizeof(int));
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&st.done, cudaEventDisableTiming);
        cudaSetDevice(prev);
        if (e != cudaSuccess) return cuda_err(e, "device status word");
        st.sm_count = sms;
    }
    *out = &st;
    return QLM_OK;
}

// QLM_HOSTIO_SPIN=0 makes synchronous host-buffer calls block in
// cudaStreamSynchronize instead of polling their completion event (for
// comparisons).
bool hostio_spin() {
    static const bool on = [] {
        const char* e = std::getenv("QLM_HOSTIO_SPIN");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Device address of a pinned, mapped host buffer (nullptr for any other
// memory). A small output of a synchronous host-buffer call is stored there by
// the kernel itself, which saves a device-to-host copy and its dependency gap.
float* mapped_host_ptr(void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();  // an unregistered pointer is an answer here, not an error
        return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? static_cast<float*>(a.devicePointer) : nullptr;
}
constexpr size_t kZeroCopyMaxBytes = 1 << 20;

// The input rows of a synchronous call from a pinned, mapped host buffer into
// device memory, read by the device itself. It lets the GEMV that follows (a
// programmatic-launch secondary) start at once, so the GEMV's weight copies
// from HBM overlap the transfer of x; the GEMV reads x after its dependency
// wait, when this kernel has completed.
__global__ void __launch_bounds__(256) host_rows_in_kernel(const float* __restrict__ src, int64_t lds, int M, int k,
                                                          float* __restrict__ dst) {
    qlm::pdl_launch_dependents();
    const int64_t n = (int64_t)M * k;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / k, c = i - m * k;
        dst[i] = src[m * lds + c];
    }
}
constexpr size_t kHostReadMaxBytes = 64 << 10;

// Waits for the work queued on s so far. The synchronous host-buffer call
// (math::matmul's contract) returns as soon as its copy-out lands: polling an
// event avoids the wake-up latency of a blocking synchronisation, which is
// several microseconds against a kernel of a few. After ~50 ms of polling it
// falls back to the blocking wait, so a long queue costs no more CPU than that.
cudaError_t wait_stream(cudaStream_t s, cudaEvent_t ev) {
    if (!hostio_spin() || !ev) return cudaStreamSynchronize(s);
    cudaError_t e = cudaEventRecord(ev, s);
    if (e != cudaSuccess) return e;
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        e = cudaEventQuery(ev);
        if (e != cudaErrorNotReady) break;
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(50)) {
            e = cudaEventSynchronize(ev);
            break;
        }
    }
    // "not ready" is an answer, not an error: leave no trace of it for the
    // launch checks that read the runtime's last error.
    if (cudaPeekAtLastError() == cudaErrorNotReady) cudaGetLastError();
    return e;
}

// Pinned, mapped host staging (cudaHostAlloc), grown on demand.
int ensure_pinned(float** buf, size_t* cap, size_t bytes) {
    if (*cap >= bytes) return QLM_OK;
    if (*buf) cudaFreeHost(*buf);
    *buf = nullptr;
    *cap = 0;
    QLM_CUDA(cudaHostAlloc(reinterpret_cast<void**>(buf), bytes, cudaHostAllocMapped), "cudaHostAlloc(staging)");
    *cap = bytes;
    return QLM_OK;
}

template <typename T>
int ensure_buf(T** buf, size_t* cap, size_t bytes) {
    if (*cap >= bytes) return QLM_OK;
    if (*buf) cudaFree(*buf);
    *buf = nullptr;
    *cap = 0;
    QLM_CUDA(cudaMalloc(reinterpret_cast<void**>(buf), bytes), "cudaMalloc(scratch)");
    *cap = bytes;
    return QLM_OK;
}

// The exact product for 9..64 activation rows per launch streams W once
// (qlm_gemm_exact.cu); QLM_GEMM_EXACT=0 runs such M as launches of up to 8
// rows instead, =2 uses the one-launch kernel whatever the row count (both
// for comparisons).
int exact_gemm_mode() {
    static const int mode = [] {
        const char* e = std::getenv("QLM_GEMM_EXACT");
        return e && e[0] == '0' ? 0 : (e && e[0] == '2' ? 2 : 1);
    }();
    return mode;
}
bool exact_gemm_enabled() { return exact_gemm_mode() != 0; }
constexpr int kExactGemmMin = 9;  // from this M on, one launch per 64 rows
// ... for matrices up to this many rows: every pass of that kernel restages
// all activation rows of its chunks, which outweighs the single weight stream
// for a vocabulary head. Measured with QLM_GEMM_EXACT=2 against launches of 8
// rows: lm_head [151936, 2560] at M = 16/32/64 0.64/1.24/2.42 ms vs
// 0.53/1.06/2.11 ms, its half [75968, 2560] 0.34/0.64/1.23 vs 0.29/0.58/1.15
// ms; [2560, 9728] at M = 64: 0.22 vs 1.29 ms.
constexpr int kExactGemmMaxRows = 65536;

bool pdl_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("QLM_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

int alloc_weight(int device, int n_total, int k, int row_begin, int row_end, qlm_w8** out, int bits = 8) {
    qlm_w8* w = new (std::nothrow) qlm_w8();
    if (!w) return set_err(QLM_ERR_OUT_OF_MEMORY, "host allocation failed");
    w->device = device;
    w->n_total = n_total;
    w->k = k;
    w->k_pad = qlm::packed_k(k);
    w->nb_pad = w->k_pad / QLM_BLOCK;
    w->row_begin = row_begin;
    w->row_end = row_end;
    w->rows = row_end - row_begin;
    w->bits = bits;
    cudaError_t e = cudaMalloc(&w->q, (size_t)w->rows * w->k_pad * bits / 8);
    if (e == cudaSuccess) e = cudaMalloc(&w->s, (size_t)w->rows * w->nb_pad * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&w->ew, (size_t)w->rows * sizeof(int));
    const char* what = "cudaMalloc(weight)";
    if (e == cudaSuccess) {
        e = qlm::gemv_make_maps(w->q, w->s, w->rows, k, bits == 4, &w->gmaps);
        what = "GEMV tensor maps";
    }
    if (e != cudaSuccess) {
        if (w->q) cudaFree(w->q);
        if (w->s) cudaFree(w->s);
        if (w->ew) cudaFree(w->ew);
        delete w;
        return cuda_err(e, what);
    }
    *out = w;
    return QLM_OK;
}

int check_shard(int n_total, int k, int row_begin, int row_end) {
    if (n_total <= 0 || k <= 0) return set_err(QLM_ERR_INVALID_ARG, "shape [%d, %d] must be positive", n_total, k);
    if (row_begin < 0 || row_end > n_total || row_begin >= row_end)
        return set_err(QLM_ERR_INVALID_ARG, "row range [%d, %d) invalid for %d rows", row_begin, row_end, n_total);
    if (qlm::packed_k(k) < k) return set_err(QLM_ERR_INVALID_ARG, "k=%d too large", k);
    return QLM_OK;
}

}  // namespace

namespace qlm_internal {
void set_last_error(const std::string& msg) { g_err = msg; }
// qlm_noalloc.cu: the allocation-free entry point's status word.
cudaError_t noalloc_status(int device, int reset, int* code);
}  // namespace qlm_internal

extern "C" {

int qlm_abi_version(void) { return QLM_ABI_VERSION; }

const char* qlm_last_error(void) { return g_err.c_str(); }

}  // extern "C"

namespace {

// Shared body of the int8 and int4 uploads.
int quantize_upload(const void* src, int src_dtype, int64_t src_row_stride, int n_total, int k, int row_begin,
                    int row_end, int device, void* stream, qlm_w8** out, int bits) {
    if (!out) return set_err(QLM_ERR_INVALID_ARG, "out is NULL");
    *out = nullptr;
    if (!src) return set_err(QLM_ERR_INVALID_ARG, "src is NULL");
    if (src_dtype != QLM_SRC_F32 && src_dtype != QLM_SRC_BF16)
        return set_err(QLM_ERR_INVALID_ARG, "unsupported source dtype %d (F32=0, BF16=1 only)", src_dtype);
    int rc = check_shard(n_total, k, row_begin, row_end);
    if (rc) return rc;
    if (src_row_stride < k) return set_err(QLM_ERR_INVALID_ARG, "row stride %lld < k %d", (long long)src_row_stride, k);
    DeviceState* st;
    if ((rc = device_state(device, &st))) return rc;
    DeviceGuard g(device);
    if (!g.ok) return set_err(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    const size_t elem = src_dtype == QLM_SRC_BF16 ? 2 : 4;
    cudaPointerAttributes attr;
    bool on_device = false;
    if (cudaPointerGetAttributes(&attr, src) == cudaSuccess)
        on_device = attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
    else
        cudaGetLastError();  // clear: plain host pointers may report an error on old drivers

    qlm_w8* w = nullptr;
    if ((rc = alloc_weight(device, n_total, k, row_begin, row_end, &w, bits))) return rc;
    auto pack = bits == 4 ? qlm::launch_quantize_pack_q4 : qlm::launch_quantize_pack;
    const size_t q_row_bytes = (size_t)w->k_pad * bits / 8;

    cudaError_t e = cudaSuccess;
    if (on_device) {
        const char* base = static_cast<const char*>(src) + (size_t)row_begin * src_row_stride * elem;
        e = pack(base, src_dtype, src_row_stride, w->rows, k, w->q, w->s, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    } else {
        // Stage host rows through a bounded device buffer (<= 64 MB per pass).
        const size_t row_bytes = (size_t)k * elem;
        int chunk = (int)((64u << 20) / row_bytes);
        if (chunk < 1) chunk = 1;
        if (chunk > w->rows) chunk = w->rows;
        void* stage = nullptr;
        e = cudaMalloc(&stage, (size_t)chunk * row_bytes);
        for (int r = 0; e == cudaSuccess && r < w->rows; r += chunk) {
            const int nr = (w->rows - r) < chunk ? (w->rows - r) : chunk;
            const char* hsrc = static_cast<const char*>(src) + ((size_t)(row_begin + r) * src_row_stride) * elem;
            e = cudaMemcpy2DAsync(stage, row_bytes, hsrc, (size_t)src_row_stride * elem, row_bytes, nr,
                                  cudaMemcpyHostToDevice, s);
            if (e == cudaSuccess)
                e = pack(stage, src_dtype, k, nr, k, w->q + (size_t)r * q_row_bytes, w->s + (size_t)r * w->nb_pad, s);
        }
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (stage) cudaFree(stage);
    }
    if (e == cudaSuccess && bits == 8) e = qlm::launch_weight_exponents(w->s, w->rows, k, w->ew, s);  // tensor-core path only
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        qlm_weight_free(w);
        return cuda_err(e, "quantize/upload");
    }
    *out = w;
    return QLM_OK;
}

// Shared body of the int8 and int4 imports: codes in the reference Tensor's
// layout (int8 [n_total][k]; int4 [n_total][(k+1)/2] bytes) and scales
// [n_total][ceil(k/32)], host or device memory. Rows [row_begin, row_end) are
// moved (host memory through a bounded device staging buffer) and repacked on
// the device.
int import_quantized(const void* codes, const float* scales, int n_total, int k, int row_begin, int row_end,
                     int device, void* stream, qlm_w8** out, int bits) {
    if (!out) return set_err(QLM_ERR_INVALID_ARG, "out is NULL");
    *out = nullptr;
    if (!codes || !scales) return set_err(QLM_ERR_INVALID_ARG, "codes/scales is NULL");
    int rc = check_shard(n_total, k, row_begin, row_end);
    if (rc) return rc;
    DeviceState* st;
    if ((rc = device_state(device, &st))) return rc;
    DeviceGuard g(device);
    if (!g.ok) return set_err(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    const int nb = (k + QLM_BLOCK - 1) / QLM_BLOCK;
    const size_t code_row = bits == 8 ? (size_t)k : (size_t)(k + 1) / 2;
    auto on_device = [](const void* p) {
        cudaPointerAttributes attr;
        if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        return attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
    };
    const bool dev_codes = on_device(codes), dev_scales = on_device(scales);

    qlm_w8* w = nullptr;
    if ((rc = alloc_weight(device, n_total, k, row_begin, row_end, &w, bits))) return rc;
    const size_t q_row_bytes = (size_t)w->k_pad * bits / 8;
    const uint8_t* csrc = static_cast<const uint8_t*>(codes) + (size_t)row_begin * code_row;
    const float* ssrc = scales + (size_t)row_begin * nb;

    cudaError_t e = cudaSuccess;
    if (dev_codes && dev_scales) {
        e = qlm::launch_repack(csrc, (int64_t)code_row, ssrc, nb, w->rows, k, bits == 4, w->q, w->s, s);
    } else {
        // <= 64 MB of rows per pass through one staging buffer (codes, then scales).
        const size_t row_bytes = code_row + (size_t)nb * sizeof(float);
        int chunk = (int)((64u << 20) / row_bytes);
        if (chunk < 1) chunk = 1;
        if (chunk > w->rows) chunk = w->rows;
        uint8_t* stage = nullptr;
        const size_t scale_off = ((size_t)chunk * code_row + 15) / 16 * 16;
        e = cudaMalloc(&stage, scale_off + (size_t)chunk * nb * sizeof(float));
        for (int r = 0; e == cudaSuccess && r < w->rows; r += chunk) {
            const int nr = (w->rows - r) < chunk ? (w->rows - r) : chunk;
            float* sstage = reinterpret_cast<float*>(stage + scale_off);
            e = cudaMemcpyAsync(stage, csrc + (size_t)r * code_row, (size_t)nr * code_row, cudaMemcpyDefault, s);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(sstage, ssrc + (size_t)r * nb, (size_t)nr * nb * sizeof(float),
                                    cudaMemcpyDefault, s);
            if (e == cudaSuccess)
                e = qlm::launch_repack(stage, (int64_t)code_row, sstage, nb, nr, k, bits == 4,
                                       w->q + (size_t)r * q_row_bytes, w->s + (size_t)r * w->nb_pad, s);
        }
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (stage) cudaFree(stage);
    }
    if (e == cudaSuccess && bits == 8) e = qlm::launch_weight_exponents(w->s, w->rows, k, w->ew, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        qlm_weight_free(w);
        return cuda_err(e, "import upload");
    }
    *out = w;
    return QLM_OK;
}

}  // namespace

extern "C" {

int qlm_weight_quantize_upload(const void* src, int src_dtype, int64_t src_row_stride, int n_total, int k,
                               int row_begin, int row_end, int device, void* stream, qlm_w8** out) {
    return quantize_upload(src, src_dtype, src_row_stride, n_total, k, row_begin, row_end, device, stream, out, 8);
}

int qlm_weight_quantize_upload_q4(const void* src, int src_dtype, int64_t src_row_stride, int n_total, int k,
                                  int row_begin, int row_end, int device, void* stream, qlm_w8** out) {
    return quantize_upload(src, src_dtype, src_row_stride, n_total, k, row_begin, row_end, device, stream, out, 4);
}

int qlm_weight_import_int8(const int8_t* q, const float* scales, int n_total, int k, int row_begin, int row_end,
                           int device, void* stream, qlm_w8** out) {
    return import_quantized(q, scales, n_total, k, row_begin, row_end, device, stream, out, 8);
}

int qlm_weight_import_int4(const uint8_t* packed, const float* scales, int n_total, int k, int row_begin,
                           int row_end, int device, void* stream, qlm_w8** out) {
    return import_quantized(packed, scales, n_total, k, row_begin, row_end, device, stream, out, 4);
}

int qlm_weight_export_int8(const qlm_w8* w, int8_t* q, float* scales) {
    if (!w || !q || !scales) return set_err(QLM_ERR_INVALID_ARG, "NULL argument");
    if (w->bits != 8) return set_err(QLM_ERR_INVALID_ARG, "the handle holds int4 weights (qlm_weight_export_int4)");
    DeviceGuard g(w->device);
    if (!g.ok) return set_err(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", w->device);
    const int nb = (w->k + QLM_BLOCK - 1) / QLM_BLOCK;
    std::vector<uint8_t> hq;
    std::vector<float> hs;
    try {
        hq.resize((size_t)w->rows * w->k_pad);
        hs.resize((size_t)w->rows * w->nb_pad);
    } catch (...) {
        return set_err(QLM_ERR_OUT_OF_MEMORY, "host staging allocation failed");
    }
    QLM_CUDA(cudaMemcpy(hq.data(), w->q, hq.size(), cudaMemcpyDeviceToHost), "export q");
    QLM_CUDA(cudaMemcpy(hs.data(), w->s, hs.size() * sizeof(float), cudaMemcpyDeviceToHost), "export scales");
    for (int r = 0; r < w->rows; ++r) {
        const uint8_t* src = hq.data() + (size_t)r * w->k_pad;
        int8_t* dst = q + (size_t)r * w->k;
        for (int kk = 0; kk < w->k; ++kk) dst[kk] = (int8_t)src[qlm::packed_offset(kk)];
        std::memcpy(scales + (size_t)r * nb, hs.data() + (size_t)r * w->nb_pad, nb * sizeof(float));
    }
    return QLM_OK;
}

int qlm_weight_export_int4(const qlm_w8* w, uint8_t* packed, float* scales) {
    if (!w || !packed || !scales) return set_err(QLM_ERR_INVALID_ARG, "NULL argument");
    if (w->bits != 4) return set_err(QLM_ERR_INVALID_ARG, "the handle holds int8 weights (qlm_weight_export_int8)");
    DeviceGuard g(w->device);
    if (!g.ok) return set_err(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", w->device);
    const int nb = (w->k + QLM_BLOCK - 1) / QLM_BLOCK;
    const size_t dev_row = (size_t)w->k_pad / 2, ref_row = (size_t)(w->k + 1) / 2;
    std::vector<uint8_t> hq;
    std::vector<float> hs;
    try {
        hq.resize((size_t)w->rows * dev_row);
        hs.resize((size_t)w->rows * w->nb_pad);
    } catch (...) {
        return set_err(QLM_ERR_OUT_OF_MEMORY, "host staging allocation failed");
    }
    QLM_CUDA(cudaMemcpy(hq.data(), w->q, hq.size(), cudaMemcpyDeviceToHost), "export q");
    QLM_CUDA(cudaMemcpy(hs.data(), w->s, hs.size() * sizeof(float), cudaMemcpyDeviceToHost), "export scales");
    for (int r = 0; r < w->rows; ++r) {
        const uint8_t* src = hq.data() + (size_t)r * dev_row;
        uint8_t* dst = packed + (size_t)r * ref_row;
        std::memset(dst, 0x88, ref_row);  // a missing odd partner is nibble 8 (value 0), as the reference writes
        for (int kk = 0; kk < w->k; ++kk) {
            const uint8_t nib = (uint8_t)((src[qlm::packed_offset_q4(kk)] >> qlm::packed_shift_q4(kk)) & 0xF);
            uint8_t& b = dst[kk / 2];
            b = (kk & 1) ? (uint8_t)((b & 0x0F) | (nib << 4)) : (uint8_t)((b & 0xF0) | nib);
        }
        std::memcpy(scales + (size_t)r * nb, hs.data() + (size_t)r * w->nb_pad, nb * sizeof(float));
    }
    return QLM_OK;
}

int qlm_weight_bits(const qlm_w8* w) { return w ? w->bits : -1; }

int qlm_weight_shape(const qlm_w8* w, int* rows, int* k, int* row_begin, int* row_end, int* n_total) {
    if (!w) return set_err(QLM_ERR_INVALID_ARG, "NULL handle");
    if (rows) *rows = w->rows;
    if (k) *k = w->k;
    if (row_begin) *row_begin = w->row_begin;
    if (row_end) *row_end = w->row_end;
    if (n_total) *n_total = w->n_total;
    return QLM_OK;
}

int64_t qlm_weight_bytes(const qlm_w8* w) {
    if (!w) return 0;
    return (int64_t)w->rows * w->k_pad * w->bits / 8 + (int64_t)w->rows * w->nb_pad * (int64_t)sizeof(float);
}

void qlm_weight_free(qlm_w8* w) {
    if (!w) return;
    DeviceGuard g(w->device);
    if (w->q) cudaFree(w->q);
    if (w->s) cudaFree(w->s);
    if (w->ew) cudaFree(w->ew);
    if (w->gmaps.dev) cudaFree(w->gmaps.dev);
    delete w->maps;
    delete w;
}

int qlm_linear_int8(const float* x, int M, int k, int64_t ldx, const qlm_w8* w, float* y, int64_t ldy, int flags,
                    void* stream) {
    if (!x || !y || !w) return set_err(QLM_ERR_INVALID_ARG, "NULL argument");
    if (M <= 0) return set_err(QLM_ERR_INVALID_ARG, "M=%d must be >= 1", M);
    if (k != w->k) return set_err(QLM_ERR_INVALID_ARG, "k=%d does not match the weight's k=%d", k, w->k);
    if (ldx < k) return set_err(QLM_ERR_INVALID_ARG, "ldx %lld < k %d", (long long)ldx, k);
    if (ldy < w->rows) return set_err(QLM_ERR_INVALID_ARG, "ldy %lld < rows %d", (long long)ldy, w->rows);
    if (flags & ~(QLM_LINEAR_TENSOR | QLM_LINEAR_HOST_IO | QLM_LINEAR_SYNC))
        return set_err(QLM_ERR_INVALID_ARG, "unknown flags 0x%x", flags);
    const bool tensor = (flags & QLM_LINEAR_TENSOR) != 0;
    const bool q4 = w->bits == 4;
    if (tensor && q4) return set_err(QLM_ERR_UNSUPPORTED, "the tensor-core path serves int8 weights; this handle is int4");
    DeviceState* st;
    int rc = device_state(w->device, &st);
    if (rc) return rc;
    DeviceGuard g(w->device);
    if (!g.ok) return set_err(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", w->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    qlm_internal::ProfScope prof("qlm_linear_int8", M, w->rows, k, s);

    // Exact path: rows of x per launch (all activations of a launch live in
    // shared memory next to the weight slots).
    int mm = 8;
    while (mm > 1 && !qlm::gemv_supported(mm, w->rows, k, st->sm_count, q4)) --mm;
    if (!tensor && !qlm::gemv_supported(mm, w->rows, k, st->sm_count, q4))
        return set_err(QLM_ERR_UNSUPPORTED, "k=%d exceeds the exact path's shared-memory staging limit", k);
    if (tensor) {
        std::lock_guard<std::mutex> lk(g_dev_mu);
        if (!w->maps) {
            qlm::TcMaps* maps = new (std::nothrow) qlm::TcMaps();
            if (!maps) return set_err(QLM_ERR_OUT_OF_MEMORY, "host allocation failed");
            cudaError_t e = qlm::tc_make_weight_maps(w->q, w->s, w->rows, w->k_pad, maps);
            if (e != cudaSuccess) {
                delete maps;
                return cuda_err(e, "tensor map encode (weights)");
            }
            const_cast<qlm_w8*>(w)->maps = maps;
        }
        if ((rc = ensure_buf(&st->x16, &st->x16_cap, (size_t)M * w->k_pad * 2))) return rc;
        if ((rc = ensure_buf(&st->ea, &st->ea_cap, (size_t)M * sizeof(int)))) return rc;
    }

    const float* dx = x;
    float* dy = y;
    int64_t dldx = ldx, dldy = ldy;
    const bool host_io = (flags & QLM_LINEAR_HOST_IO) != 0;
    bool y_direct = false, y_staged = false;
    if (host_io) {
        std::lock_guard<std::mutex> lk(g_dev_mu);
        if ((rc = ensure_buf(&st->x_buf, &st->x_cap, (size_t)M * k * sizeof(float)))) return rc;
        if ((rc = ensure_buf(&st->y_buf, &st->y_cap, (size_t)M * w->rows * sizeof(float)))) return rc;
        const bool small_x = (size_t)M * k * sizeof(float) <= kHostReadMaxBytes;
        const float* mx = small_x ? mapped_host_ptr(const_cast<float*>(x)) : nullptr;
        int64_t mldx = ldx;
        if (small_x && !mx) {
            // A small pageable input (QuickLM's own activations): a host copy
            // into pinned staging, which the device then reads itself.
            if ((rc = ensure_pinned(&st->pin_x, &st->pin_x_cap, (size_t)M * k * sizeof(float)))) return rc;
            for (int m = 0; m < M; ++m)
                std::memcpy(st->pin_x + (size_t)m * k, x + (size_t)m * ldx, (size_t)k * sizeof(float));
            mx = mapped_host_ptr(st->pin_x);
            mldx = k;
        }
        if (mx) {
            const int64_t n = (int64_t)M * k;
            // one element per thread: every read is in flight at once
            host_rows_in_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(mx, mldx, M, k, st->x_buf);
            QLM_CUDA(cudaGetLastError(), "read x from the pinned host buffer");
        } else if (ldx == k || M == 1)
            QLM_CUDA(cudaMemcpyAsync(st->x_buf, x, (size_t)M * k * sizeof(float), cudaMemcpyHostToDevice, s),
                     "copy x to device");
        else
            QLM_CUDA(cudaMemcpy2DAsync(st->x_buf, (size_t)k * sizeof(float), x, (size_t)ldx * sizeof(float),
                                       (size_t)k * sizeof(float), M, cudaMemcpyHostToDevice, s),
                     "copy x to device");
        dx = st->x_buf;
        dldx = k;
        const bool small_y = (size_t)M * ldy * sizeof(float) <= kZeroCopyMaxBytes;
        float* my = small_y ? mapped_host_ptr(y) : nullptr;
        if (my) {
            dy = my;  // the kernel stores into the caller's pinned buffer
            dldy = ldy;
            y_direct = true;
        } else if (small_y && (rc = ensure_pinned(&st->pin_y, &st->pin_y_cap,
                                                  (size_t)M * w->rows * sizeof(float))) == QLM_OK &&
                   (my = mapped_host_ptr(st->pin_y)) != nullptr) {
            dy = my;  // pinned staging, copied into the caller's pageable buffer after the wait
            dldy = w->rows;
            y_direct = true;
            y_staged = true;
        } else {
            if (rc) return rc;
            dy = st->y_buf;
            dldy = w->rows;
        }
    }
    if (tensor) {
        QLM_CUDA(qlm::launch_gemm_tc(*w->maps, w->ew, w->rows, k, dx, dldx, M, st->x16, st->ea, dy, dldy, st->status,
                                     s, pdl_enabled()),
                 "tensor-core GEMM launch");
    } else if (M >= kExactGemmMin && exact_gemm_enabled() &&
               (w->rows <= kExactGemmMaxRows || exact_gemm_mode() == 2)) {
        {
            std::lock_guard<std::mutex> lk(g_dev_mu);
            if ((rc = ensure_buf(&st->xpair, &st->xpair_cap, qlm::gemm_exact_scratch_bytes(64, k)))) return rc;
        }
        for (int m0 = 0; m0 < M; m0 += 64) {
            const int g_rows = (M - m0) < 64 ? (M - m0) : 64;
            if (g_rows >= 2) {
                QLM_CUDA(qlm::launch_gemm_exact(dx + (int64_t)m0 * dldx, dldx, g_rows, w->q, w->s, w->rows, k, q4,
                                                dy + (int64_t)m0 * dldy, dldy, st->xpair, st->sm_count, s),
                         "exact small-M launch");
            } else {
                QLM_CUDA(qlm::launch_gemv_exact(dx + (int64_t)m0 * dldx, dldx, 1, w->q, w->s, w->gmaps, w->rows, k,
                                                dy + (int64_t)m0 * dldy, dldy, st->status, st->sm_count, s,
                                                pdl_enabled(), nullptr, q4),
                         "gemv launch");
            }
        }
    } else {
        for (int m0 = 0; m0 < M; m0 += mm) {
            const int g_rows = (M - m0) < mm ? (M - m0) : mm;
            QLM_CUDA(qlm::launch_gemv_exact(dx + (int64_t)m0 * dldx, dldx, g_rows, w->q, w->s, w->gmaps, w->rows, k,
                                            dy + (int64_t)m0 * dldy, dldy, st->status, st->sm_count, s,
                                            pdl_enabled(), nullptr, q4),
                     "gemv launch");
        }
    }
    if (host_io && !y_direct) {
        if (ldy == w->rows || M == 1)
            QLM_CUDA(cudaMemcpyAsync(y, dy, (size_t)M * w->rows * sizeof(float), cudaMemcpyDeviceToHost, s),
                     "copy y to host");
        else
            QLM_CUDA(cudaMemcpy2DAsync(y, (size_t)ldy * sizeof(float), dy, (size_t)w->rows * sizeof(float),
                                       (size_t)w->rows * sizeof(float), M, cudaMemcpyDeviceToHost, s),
                     "copy y to host");
    }
    prof.stop();
    if (host_io || (flags & QLM_LINEAR_SYNC)) {
        QLM_CUDA(host_io ? wait_stream(s, st->done) : cudaStreamSynchronize(s), "stream synchronize");
        if (y_staged)
            for (int m = 0; m < M; ++m)
                std::memcpy(y + (size_t)m * ldy, st->pin_y + (size_t)m * w->rows, (size_t)w->rows * sizeof(float));
        if (tensor || (flags & QLM_LINEAR_SYNC)) return qlm_device_status(w->device, 1);
    }
    return QLM_OK;
}

int qlm_linear_int8_grouped(const float* x, int M, int k, int64_t ldx, const qlm_w8* const* ws, int nw,
                            float* const* ys, const int64_t* ldys, int flags, void* stream) {
    if (!x || !ws || !ys || !ldys) return set_err(QLM_ERR_INVALID_ARG, "NULL argument");
    if (nw < 1 || nw > qlm::kMaxGroup) return set_err(QLM_ERR_INVALID_ARG, "nw=%d not in [1, %d]", nw, qlm::kMaxGroup);
    if (M <= 0) return set_err(QLM_ERR_INVALID_ARG, "M=%d must be >= 1", M);
    if (ldx < k) return set_err(QLM_ERR_INVALID_ARG, "ldx %lld < k %d", (long long)ldx, k);
    if (flags & ~QLM_LINEAR_SYNC) return set_err(QLM_ERR_INVALID_ARG, "only QLM_LINEAR_SYNC is accepted (device pointers)");
    qlm::GemvWeight gw[qlm::kMaxGroup];
    int rows_total = 0;
    for (int g = 0; g < nw; ++g) {
        const qlm_w8* w = ws[g];
        if (!w || !ys[g]) return set_err(QLM_ERR_INVALID_ARG, "NULL weight or output %d", g);
        if (w->k != k) return set_err(QLM_ERR_INVALID_ARG, "weight %d has k=%d, expected %d", g, w->k, k);
        if (w->device != ws[0]->device) return set_err(QLM_ERR_INVALID_ARG, "weights on different devices");
        if (w->bits != ws[0]->bits) return set_err(QLM_ERR_INVALID_ARG, "int8 and int4 weights in one group");
        if (ldys[g] < w->rows) return set_err(QLM_ERR_INVALID_ARG, "ldy %lld < rows %d (weight %d)", (long long)ldys[g], w->rows, g);
        gw[g] = qlm::GemvWeight{w->q, w->s, &w->gmaps, w->rows, ys[g], ldys[g]};
        rows_total += w->rows;
    }
    DeviceState* st;
    int rc = device_state(ws[0]->device, &st);
    if (rc) return rc;
    DeviceGuard g(ws[0]->device);
    if (!g.ok) return set_err(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", ws[0]->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    qlm_internal::ProfScope prof("qlm_linear_int8_grouped", M, rows_total, k, s);
    int mm = 8;
    const bool q4 = ws[0]->bits == 4;
    while (mm > 1 && !qlm::gemv_supported(mm, rows_total, k, st->sm_count, q4)) --mm;
    if (!qlm::gemv_supported(mm, rows_total, k, st->sm_count, q4))
        return set_err(QLM_ERR_UNSUPPORTED, "k=%d exceeds the exact path's shared-memory staging limit", k);
    if (M >= kExactGemmMin && exact_gemm_enabled()) {
        // one exact small-M launch per weight and 64 activation rows
        {
            std::lock_guard<std::mutex> lk(g_dev_mu);
            if ((rc = ensure_buf(&st->xpair, &st->xpair_cap, qlm::gemm_exact_scratch_bytes(64, k)))) return rc;
        }
        for (int m0 = 0; m0 < M; m0 += 64) {
            const int g_rows = (M - m0) < 64 ? (M - m0) : 64;
            for (int g = 0; g < nw; ++g) {
                if (g_rows >= 2) {
                    QLM_CUDA(qlm::launch_gemm_exact(x + (int64_t)m0 * ldx, ldx, g_rows, gw[g].q, gw[g].s, gw[g].rows,
                                                    k, q4, gw[g].y + (int64_t)m0 * gw[g].ldy, gw[g].ldy, st->xpair, st->sm_count, s),
                             "exact small-M launch");
                } else {
                    QLM_CUDA(qlm::launch_gemv_exact(x + (int64_t)m0 * ldx, ldx, 1, gw[g].q, gw[g].s, *gw[g].maps,
                                                    gw[g].rows, k, gw[g].y + (int64_t)m0 * gw[g].ldy, gw[g].ldy,
                                                    st->status, st->sm_count, s, pdl_enabled(), nullptr, q4),
                             "gemv launch");
                }
            }
        }
        prof.stop();
        if (flags & QLM_LINEAR_SYNC) {
            QLM_CUDA(cudaStreamSynchronize(s), "stream synchronize");
            return qlm_device_status(ws[0]->device, 1);
        }
        return QLM_OK;
    }
    for (int m0 = 0; m0 < M; m0 += mm) {
        const int rows_m = (M - m0) < mm ? (M - m0) : mm;
        qlm::GemvWeight gm[qlm::kMaxGroup];
        for (int i = 0; i < nw; ++i) {
            gm[i] = gw[i];
            gm[i].y = gw[i].y + (int64_t)m0 * gw[i].ldy;
        }
        QLM_CUDA(qlm::launch_gemv_grouped(x + (int64_t)m0 * ldx, ldx, rows_m, gm, nw, k, st->status, st->sm_count, s,
                                          pdl_enabled(), nullptr, q4),
                 "grouped gemv launch");
    }
    prof.stop();
    if (flags & QLM_LINEAR_SYNC) {
        QLM_CUDA(cudaStreamSynchronize(s), "stream synchronize");
        return qlm_device_status(ws[0]->device, 1);
    }
    return QLM_OK;
}

int qlm_device_status(int device, int reset) {
    DeviceState* st;
    int rc = device_state(device, &st);
    if (rc) return rc;
    DeviceGuard g(device);
    if (!g.ok) return set_err(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    int code = 0;
    if (st->status) {
        QLM_CUDA(cudaMemcpy(&code, st->status, sizeof(int), cudaMemcpyDeviceToHost), "read status");
        if (code != 0 && reset) QLM_CUDA(cudaMemset(st->status, 0, sizeof(int)), "reset status");
    }
    // The allocation-free entry point keeps its own (sticky) word in its static scratch.
    int code_na = 0;
    QLM_CUDA(qlm_internal::noalloc_status(device, reset, &code_na), "read no-alloc status");
    if (code == 0) code = code_na;
    if (code == 0) return QLM_OK;
    return set_err(QLM_ERR_TIMEOUT, "a device-side wait gave up (code 0x%x); results of that call are invalid", code);
}

int qlm_stream_sync(void* stream) {
    QLM_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize");
    return QLM_OK;
}

}  // extern "C"
