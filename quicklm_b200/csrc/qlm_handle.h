// qlm_handle.h — layout of the opaque qlm_w8 weight handle (internal).
#pragma once

#include <cstdint>

#include "qlm_kernels.h"

struct qlm_w8 {
    int device = -1;
    int rows = 0, k = 0, k_pad = 0, nb_pad = 0;
    int row_begin = 0, row_end = 0, n_total = 0;
    int bits = 8;          // 8: int8 P128 layout; 4: int4 P128/4 layout (qlm_device.cuh)
    uint8_t* q = nullptr;  // packed [rows][k_pad * bits / 8]
    float* s = nullptr;    // [rows][nb_pad]
    int* ew = nullptr;     // [rows] range exponents for the tensor-core path
    qlm::GemvMaps gmaps;           // TMA descriptors of the exact GEMV, built at allocation
    qlm::TcMaps* maps = nullptr;  // TMA descriptors, built on first tensor-core use
};
