// qlm_prof.h — per-matmul device timing inside the library.
//
// The counterpart of QuickLM's QUICKLM_PROF: the reference adds the wall time
// of every math::matmul call to one accumulator when the variable is set
// (src/ops/math_ops.cpp:151-159, 821-823, 896-899) and prints the total at exit
// (src/main.cpp:706-709). Here each linear entry point brackets its work with
// two CUDA events on the caller's stream, so the figure is the device span of
// the call (its copies and kernels) and costs no synchronisation; events are
// folded into per-(entry, M, N, K) totals when the host asks. Every scope also
// opens an NVTX range named after the entry point, for nsys/ncu timelines.
#pragma once

#include <cuda_runtime.h>

namespace qlm_internal {

// True when QUICKLM_PROF or QLM_PROF is set, or after qlm_prof_enable(1).
bool prof_on();

class ProfScope {
public:
    // `kind` must be a string literal (kept by pointer). Records the start
    // event on `s` when profiling is on and `s` is not being captured.
    ProfScope(const char* kind, int M, int N, int K, cudaStream_t s);
    // Records the end event (call before a synchronisation, so host latency
    // does not enter the span); later calls do nothing.
    void stop();
    ~ProfScope();
    ProfScope(const ProfScope&) = delete;
    ProfScope& operator=(const ProfScope&) = delete;

private:
    const char* kind_;
    int M_, N_, K_;
    cudaStream_t s_;
    cudaEvent_t a_ = nullptr;
    bool nvtx_ = false;
};

// An NVTX range only (no events), for calls that are not matmuls.
class NvtxRange {
public:
    explicit NvtxRange(const char* name);
    ~NvtxRange();
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

}  // namespace qlm_internal
