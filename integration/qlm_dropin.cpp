// qlm_dropin.cpp — QuickLM's int8 matmul path moved onto the B200.
//
// Linked into QuickLM in place of two reference definitions (which the build
// renames, see integration/Makefile):
//   * SafetensorsLoader::get_tensor_keep_int8 (src/io/safetensors.cpp:517-585):
//     quantizes and packs the weight on the GPU straight from the memory-mapped
//     F32/BF16 bytes (bit-identical bytes and scales) and keeps it resident in
//     HBM; the returned Tensor's int8 storage holds the device handle itself
//     (a tag and the handle pointer; its deleter frees the device weight).
//   * math::matmul (src/ops/math_ops.hpp:92, src/ops/math_ops.cpp:820-900):
//     int8 B operands run on the device through the C ABI (bit-identical by
//     default); every other operand type goes to the reference's own code.
// The model code (src/model, src/arch) is unchanged and still calls
// math::matmul at every projection and the lm_head.
//
// Environment: QLM_DEVICE (CUDA ordinal, default 0); QLM_TENSOR_MIN_M (if set,
// products with at least that many activation rows use the tensor-core GEMM,
// which is within relative L2 2e-3 instead of bit-identical; default off).
#include "math_ops.hpp"
#include "qlm_b200.h"
#include "safetensors.hpp"

#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

namespace math {
// The reference's own matmul, renamed when math_ops.cpp is compiled for this build.
void qlm_reference_matmul_cpu(const Tensor& A, const Tensor& B, Tensor& C, bool transpose_B);
}  // namespace math

namespace {

// Weights quantized on the CPU, imported once: host address -> device weight.
struct Registry {
    std::mutex mu;
    std::unordered_map<const int8_t*, qlm_w8*> handles;
    ~Registry() {
        for (auto& kv : handles) qlm_weight_free(kv.second);
    }
};

Registry& registry() {
    static Registry r;
    return r;
}

int device_ordinal() {
    static const int dev = [] {
        const char* e = std::getenv("QLM_DEVICE");
        return e ? std::atoi(e) : 0;
    }();
    return dev;
}

int tensor_min_m() {
    static const int m = [] {
        const char* e = std::getenv("QLM_TENSOR_MIN_M");
        return e ? std::atoi(e) : 0;
    }();
    return m;
}

[[noreturn]] void raise(const char* what) {
    throw std::runtime_error(std::string(what) + ": " + qlm_last_error());
}

// A device-resident weight travels in the Tensor's own int8 storage (the
// reference Tensor has no field for it, and its sources stay unchanged): 8
// tag bytes, then the handle pointer. The storage's deleter frees the weight.
constexpr char kDeviceTag[8] = {'q', 'l', 'm', 'b', '2', '0', '0', 'w'};

std::shared_ptr<std::vector<int8_t>> device_storage(qlm_w8* h) {
    auto* v = new std::vector<int8_t>(sizeof(kDeviceTag) + sizeof(qlm_w8*));
    std::memcpy(v->data(), kDeviceTag, sizeof(kDeviceTag));
    std::memcpy(v->data() + sizeof(kDeviceTag), &h, sizeof(h));
    return std::shared_ptr<std::vector<int8_t>>(v, [h](std::vector<int8_t>* p) {
        qlm_weight_free(h);
        delete p;
    });
}

qlm_w8* stored_handle(const Tensor& B) {
    const std::vector<int8_t>* v = B.int8_owner.get();
    if (!v || v->size() != sizeof(kDeviceTag) + sizeof(qlm_w8*) || B.int8_data != v->data() ||
        std::memcmp(v->data(), kDeviceTag, sizeof(kDeviceTag)) != 0)
        return nullptr;
    qlm_w8* h = nullptr;
    std::memcpy(&h, v->data() + sizeof(kDeviceTag), sizeof(h));
    return h;
}

// Device handle for an int8 B: carried by the Tensor (quantized on the device
// at load), or imported once from the reference's host int8 layout if the
// Tensor was quantized on the CPU (kept in a registry by host address).
qlm_w8* device_weight(const Tensor& B, int N, int K) {
    if (qlm_w8* h = stored_handle(B)) return h;
    Registry& r = registry();
    std::lock_guard<std::mutex> lk(r.mu);
    auto it = r.handles.find(B.int8_data);
    if (it != r.handles.end()) return it->second;
    if (!B.int8_scales) throw std::runtime_error("int8 weight without scales");
    qlm_w8* h = nullptr;
    if (qlm_weight_import_int8(B.int8_data, B.int8_scales->data(), N, K, 0, N, device_ordinal(), nullptr, &h) != QLM_OK)
        raise("qlm_weight_import_int8");
    r.handles.emplace(B.int8_data, h);
    return h;
}

}  // namespace

Tensor SafetensorsLoader::get_tensor_keep_int8(const std::string& name) {
    auto it = tensor_infos.find(name);
    if (it == tensor_infos.end()) throw std::runtime_error("Tensor not found in safetensors file: " + name);
    const auto& info = it->second;
    if (info.dtype != "F32" && info.dtype != "BF16") {
        throw std::runtime_error("Unsupported tensor datatype for '" + name + "': " + info.dtype +
                                 " (only F32 and BF16 supported for int8 quantization)");
    }
    const size_t abs_start = binary_start_offset + info.start_offset;
    const size_t abs_end = binary_start_offset + info.end_offset;
    if (abs_end > mapped_file->file_size)
        throw std::runtime_error("Tensor '" + name + "' offset goes out of file boundaries");

    const int rows = info.shape.empty() ? 1 : info.shape[0];
    const int K = info.shape.empty() ? 0 : info.shape.back();
    const void* src = static_cast<const char*>(mapped_file->mapped_data) + abs_start;
    const int dtype = info.dtype == "BF16" ? QLM_SRC_BF16 : QLM_SRC_F32;
    qlm_w8* h = nullptr;
    if (qlm_weight_quantize_upload(src, dtype, K, rows, K, 0, rows, device_ordinal(), nullptr, &h) != QLM_OK)
        raise(("qlm_weight_quantize_upload(" + name + ")").c_str());

    Tensor t;
    t.shape = info.shape;
    t.compute_strides();
    // The int8 codes and scales live only in HBM; the Tensor carries the handle.
    t.int8_owner = device_storage(h);
    t.int8_data = t.int8_owner->data();
    t.int8_scales = std::make_shared<std::vector<float>>(1, 0.0f);
    return t;
}

namespace math {

void matmul(const Tensor& A, const Tensor& B, Tensor& C, bool transpose_B) {
    if (B.int8_data && transpose_B) {
        const int M = (A.shape.size() > 1) ? A.shape[0] : 1;
        const int K = A.shape.back();
        const int N = B.shape[0];
        // Rows of C are C.strides[0] apart (the reference writes row m at
        // C.data + m * C.strides[0]); with one row, N contiguous floats.
        const int64_t ldc = (M == 1 || C.strides.empty()) ? N : C.strides[0];
        qlm_w8* h = device_weight(B, N, K);
        int flags = QLM_LINEAR_HOST_IO;
        if (tensor_min_m() > 0 && M >= tensor_min_m()) flags |= QLM_LINEAR_TENSOR;
        if (qlm_linear_int8(A.data, M, K, K, h, C.data, ldc, flags, nullptr) != QLM_OK) raise("qlm_linear_int8");
        return;
    }
    qlm_reference_matmul_cpu(A, B, C, transpose_B);
}

}  // namespace math
