// qlm_kernels.h — internal launch interface between the C ABI and the kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace qlm {

// Quantize `rows` rows of k F32 (dtype 0) or BF16 (dtype 1) device values with
// row stride src_stride into the packed layout: q [rows][packed_k(k)],
// scales [rows][packed_k(k)/32].
cudaError_t launch_quantize_pack(const void* src, int dtype, int64_t src_stride, int rows, int k, uint8_t* q,
                                 float* scales, cudaStream_t stream);

// Bit-exact y[m][0:rows] = x[m][0:k] . W^T for m < mm (1..8), W packed.
cudaError_t launch_gemv_exact(const float* x, int64_t ldx, int mm, const uint8_t* q, const float* s, int rows,
                              int k, float* y, int64_t ldy, int sm_count, cudaStream_t stream, bool pdl);

// Dynamic shared memory the exact GEMV needs for mm activation rows.
size_t gemv_smem_bytes(int mm, int k);

}  // namespace qlm
