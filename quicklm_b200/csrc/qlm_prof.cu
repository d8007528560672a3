// qlm_prof.cu — per-matmul device timing (QUICKLM_PROF counterpart) and the
// qlm_prof_* C ABI. See qlm_prof.h for what is measured.
//
// Events come from a per-device pool and are recorded on the caller's stream;
// a finished call leaves one (start, end) pair pending. Pairs are folded into
// the per-(entry, M, N, K) totals when the host asks (qlm_prof_matmul_ms /
// qlm_prof_report, which wait for the pending end events), or, oldest half
// first, once 4096 pairs are pending. No cudaEventQuery is used: a not-ready
// answer would be the only status this file leaves behind for the caller.
#include "../../include/qlm_b200.h"
#include "qlm_prof.h"

#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <utility>
#include <vector>

namespace qlm_internal {
void set_last_error(const std::string& msg);
}

namespace {

constexpr size_t kMaxPending = 4096;

struct Stat {
    long long calls = 0;
    double ms = 0.0;
};

struct Pending {
    cudaEvent_t a, b;
    int dev;
    const char* kind;
    int M, N, K;
};

using Key = std::tuple<std::string, int, int, int>;

struct Prof {
    std::mutex mu;
    std::vector<Pending> pending;
    std::vector<std::pair<int, cudaEvent_t>> pool;  // (device, idle event)
    std::map<Key, Stat> stats;
};

// Never destroyed: events may still be pending when static destructors run.
Prof& prof() {
    static Prof* p = new Prof();
    return *p;
}

std::atomic<int> g_enabled{-1};  // -1: not yet read from the environment

cudaEvent_t take_event(Prof& P, int dev) {
    for (size_t i = P.pool.size(); i-- > 0;) {
        if (P.pool[i].first == dev) {
            cudaEvent_t e = P.pool[i].second;
            P.pool[i] = P.pool.back();
            P.pool.pop_back();
            return e;
        }
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) {
        cudaGetLastError();  // the failure is ours; leave no status for the caller's launch checks
        return nullptr;
    }
    return e;
}

// Folds pending[0, n) into the totals (waits for each end event). Returns the
// first CUDA error met; every pair is released either way.
cudaError_t fold(Prof& P, size_t n) {
    cudaError_t first = cudaSuccess;
    for (size_t i = 0; i < n; ++i) {
        Pending& p = P.pending[i];
        float ms = 0.f;
        cudaError_t e = cudaEventSynchronize(p.b);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, p.a, p.b);
        if (e == cudaSuccess) {
            Stat& s = P.stats[Key(p.kind, p.M, p.N, p.K)];
            s.calls += 1;
            s.ms += ms;
        } else if (first == cudaSuccess) {
            first = e;
        }
        P.pool.emplace_back(p.dev, p.a);
        P.pool.emplace_back(p.dev, p.b);
    }
    P.pending.erase(P.pending.begin(), P.pending.begin() + (ptrdiff_t)n);
    return first;
}

}  // namespace

namespace qlm_internal {

bool prof_on() {
    int v = g_enabled.load(std::memory_order_relaxed);
    if (v < 0) {
        v = (std::getenv("QUICKLM_PROF") || std::getenv("QLM_PROF")) ? 1 : 0;
        int expect = -1;
        g_enabled.compare_exchange_strong(expect, v);
        v = g_enabled.load();
    }
    return v == 1;
}

ProfScope::ProfScope(const char* kind, int M, int N, int K, cudaStream_t s)
    : kind_(kind), M_(M), N_(N), K_(K), s_(s) {
    nvtxRangePushA(kind);
    nvtx_ = true;
    if (!prof_on()) return;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    if (cs != cudaStreamCaptureStatusNone) return;  // events in a graph time nothing useful
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    Prof& P = prof();
    std::lock_guard<std::mutex> lk(P.mu);
    cudaEvent_t a = take_event(P, dev);
    if (!a) return;
    if (cudaEventRecord(a, s) != cudaSuccess) {
        cudaGetLastError();
        P.pool.emplace_back(dev, a);
        return;
    }
    a_ = a;
}

void ProfScope::stop() {
    if (a_) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) cudaGetLastError();
        Prof& P = prof();
        std::lock_guard<std::mutex> lk(P.mu);
        cudaEvent_t b = take_event(P, dev);
        if (b && cudaEventRecord(b, s_) == cudaSuccess) {
            P.pending.push_back(Pending{a_, b, dev, kind_, M_, N_, K_});
            if (P.pending.size() >= kMaxPending) fold(P, kMaxPending / 2);
        } else {
            if (b) {
                cudaGetLastError();
                P.pool.emplace_back(dev, b);
            }
            P.pool.emplace_back(dev, a_);
        }
        a_ = nullptr;
    }
    if (nvtx_) {
        nvtxRangePop();
        nvtx_ = false;
    }
}

ProfScope::~ProfScope() { stop(); }

NvtxRange::NvtxRange(const char* name) { nvtxRangePushA(name); }
NvtxRange::~NvtxRange() { nvtxRangePop(); }

}  // namespace qlm_internal

extern "C" {

int qlm_prof_enable(int on) {
    const int before = qlm_internal::prof_on() ? 1 : 0;
    if (on == 0 || on == 1) g_enabled.store(on);
    return before;
}

int qlm_prof_matmul_ms(double* ms, int64_t* calls) {
    Prof& P = prof();
    std::lock_guard<std::mutex> lk(P.mu);
    cudaError_t e = fold(P, P.pending.size());
    double t = 0.0;
    long long n = 0;
    for (const auto& kv : P.stats) {
        t += kv.second.ms;
        n += kv.second.calls;
    }
    if (ms) *ms = t;
    if (calls) *calls = n;
    if (e != cudaSuccess) {
        qlm_internal::set_last_error(std::string("profiling events: ") + cudaGetErrorString(e));
        return QLM_ERR_CUDA;
    }
    return QLM_OK;
}

int qlm_prof_reset(void) {
    Prof& P = prof();
    std::lock_guard<std::mutex> lk(P.mu);
    cudaError_t e = fold(P, P.pending.size());
    P.stats.clear();
    if (e != cudaSuccess) {
        qlm_internal::set_last_error(std::string("profiling events: ") + cudaGetErrorString(e));
        return QLM_ERR_CUDA;
    }
    return QLM_OK;
}

int qlm_prof_report(char* buf, int64_t cap, int64_t* needed) {
    Prof& P = prof();
    std::string out;
    cudaError_t e;
    {
        std::lock_guard<std::mutex> lk(P.mu);
        e = fold(P, P.pending.size());
        std::vector<std::pair<Key, Stat>> rows(P.stats.begin(), P.stats.end());
        std::sort(rows.begin(), rows.end(),
                  [](const std::pair<Key, Stat>& x, const std::pair<Key, Stat>& y) { return x.second.ms > y.second.ms; });
        char line[256];
        for (const auto& r : rows) {
            snprintf(line, sizeof(line), "%s\t%d\t%d\t%d\t%lld\t%.6f\n", std::get<0>(r.first).c_str(),
                     std::get<1>(r.first), std::get<2>(r.first), std::get<3>(r.first), r.second.calls, r.second.ms);
            out += line;
        }
    }
    if (needed) *needed = (int64_t)out.size() + 1;
    if (buf && cap > 0) {
        const size_t n = std::min<size_t>(out.size(), (size_t)cap - 1);
        out.copy(buf, n);
        buf[n] = '\0';
    }
    if (e != cudaSuccess) {
        qlm_internal::set_last_error(std::string("profiling events: ") + cudaGetErrorString(e));
        return QLM_ERR_CUDA;
    }
    return QLM_OK;
}

}  // extern "C"
