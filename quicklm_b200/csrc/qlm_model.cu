// qlm_model.cu — a device-resident decode step for QuickLM's Qwen3.5 hybrid
// decoder (linear-attention gated-delta-net layers and gated GQA layers).
//
// QuickLM's DecoderModel::forward (src/model/model.cpp:151-199) keeps every
// activation in host memory and runs each layer's ops on the CPU between its
// int8 matmuls. This file runs the same step with the activations in HBM from
// the token id to the greedy choice: the embedding row, every layer
// (DecoderLayer::forward, src/model/modules.hpp:210-241, with the reference's
// default un-fused add + RMSNorm and SiLU + multiply), the final norm, the
// lm_head and DecoderModel::sample(logits, 0, 0) (model.cpp:259-272). Only the
// next token id crosses to the host. The per-layer ops are the library's
// device kernels (qlm_layer.cu), each restating the reference function it
// replaces; the matmuls are the bit-exact int8 GEMV (weights quantized on the
// device at load exactly as get_tensor_keep_int8 does, so the int8 bytes and
// scales equal the reference's).
//
// Numerics: every matmul, norm, RoPE rotation, conv step, delta-rule update
// and attention score is bit-identical to the reference's given the same
// inputs. The reference also calls the host's libm exp/log1p (SiLU, the
// gated-delta-net gates, softmax, the sigmoid output gate); the device
// evaluates these in double and rounds once, which agrees with the host's
// expf except in rare last-bit cases. So the logits agree to within a few ulp
// rather than bit for bit, and a greedy token can only differ where the top
// two logits are that close.
//
// Loading reads QuickLM's checkpoint directory as the reference does
// (src/model/model.cpp:40-131, src/arch/qwen3_5.cpp): config.json, the
// safetensors tensors (F32 or BF16) under the canonical names or their
// "model.language_model." variants, a tied lm_head when lm_head.weight is
// absent, and the conv kernel transposed tap-major
// (src/model/attention.cpp:393-407).
#include <dirent.h>

#include <algorithm>
#include <cmath>
#include <new>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <string>
#include <vector>

#include "../../include/qlm_b200.h"
#include "qlm_device.cuh"
#include "qlm_handle.h"
#include "qlm_kernels.h"
#include "qlm_prof.h"
#include "qlm_safetensors.h"

namespace qlm_internal {
void set_last_error(const std::string& msg);
}

namespace {

constexpr int kEmbThreads = 256;

// x[b][i] = the embedding row of tokens[b] (BF16 upcast exactly, or F32
// copied); one CTA row per sequence b.
__global__ void embed_rows_kernel(const void* table, int bf16, const int* __restrict__ tokens, int hidden, float* x) {
    const int t = tokens[blockIdx.y];
    float* xr = x + (int64_t)blockIdx.y * hidden;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x) {
        if (bf16) {
            const uint16_t h = static_cast<const uint16_t*>(table)[(int64_t)t * hidden + i];
            xr[i] = __uint_as_float((uint32_t)h << 16);
        } else {
            xr[i] = static_cast<const float*>(table)[(int64_t)t * hidden + i];
        }
    }
}

// DecoderModel::sample(logits, 0, 0) (src/model/model.cpp:259-272) for each
// of the rows: the scan keeps the first strictly larger logit starting from
// logit 0, i.e. 0 if logit 0 is NaN, else the lowest index of the largest
// non-NaN logit (0 when no other logit is a number). One CTA per row.
__global__ void __launch_bounds__(1024) greedy_rows_kernel(const float* __restrict__ logits, int n, int* out) {
    qlm::pdl_wait();  // the logits come from the lm_head GEMV (read through L2)
    const float* l = logits + (int64_t)blockIdx.x * n;
    float best = 0.0f;
    int bi = -1;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = __ldcg(l + i);
        if (v == v && (bi < 0 || v > best)) {  // indices ascend per thread: ties keep the first
            best = v;
            bi = i;
        }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    auto better = [](float v, int i, float bv, int b) {  // (v, i) beats (bv, b)?
        if (i < 0) return false;
        if (b < 0) return true;
        return v > bv || (v == bv && i < b);
    };
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, best, o);
        const int i = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(v, i, best, bi)) {
            best = v;
            bi = i;
        }
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (lane == 0) {
        sv[w] = best;
        si[w] = bi;
    }
    __syncthreads();
    if (w == 0) {
        best = lane < nw ? sv[lane] : 0.0f;
        bi = lane < nw ? si[lane] : -1;
        for (int o = 16; o > 0; o >>= 1) {
            const float v = __shfl_xor_sync(0xffffffffu, best, o);
            const int i = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(v, i, best, bi)) {
                best = v;
                bi = i;
            }
        }
        if (lane == 0) {
            const float l0 = __ldcg(l);
            out[blockIdx.x] = (l0 != l0 || bi < 0) ? 0 : bi;
        }
    }
}

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    qlm_internal::set_last_error(buf);
    return code;
}

struct Layer {
    bool full_attn = false;
    // gated delta net, batched: in_proj_qkv as three row ranges (q, k, v), so
    // each part of every sequence is contiguous ([part][B][lin]); the conv runs
    // over those 3*B*lin channels with its kernel replicated per sequence
    qlm_w8 *qkv_q = nullptr, *qkv_k = nullptr, *qkv_v = nullptr;
    float* in_norm = nullptr;    // input_layernorm [hidden] (zero-centred)
    float* post_norm = nullptr;  // post_attention_layernorm [hidden]
    qlm_w8 *gate = nullptr, *up = nullptr, *down = nullptr;
    // gated GQA
    qlm_w8 *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
    float *q_norm = nullptr, *k_norm = nullptr;  // [head_dim] each
    float *k_cache = nullptr, *v_cache = nullptr;  // [max_seq][B][kv_heads][head_dim]
    // gated delta net
    qlm_w8 *z = nullptr, *b = nullptr, *a = nullptr, *out = nullptr;
    float* conv_wt = nullptr;     // [kernel][3][B][lin] (tap-major, replicated per sequence)
    float* conv_state = nullptr;  // [kernel - 1][3][B][lin]
    float *gdn_norm = nullptr, *A_log = nullptr, *dt_bias = nullptr;
    float* rstate = nullptr;      // [B][lin_heads][lin_dim][lin_dim]
};

}  // namespace

struct qlm_model {
    int device = -1;
    // configuration (src/model/config.hpp, parsed as src/arch/qwen3_5.cpp:11-72)
    int vocab = 0, hidden = 0, inter = 0, layers_n = 0, heads = 0, kv_heads = 0, head_dim = 0;
    int lin_heads = 0, lin_dim = 0, rotary_dim = 0, conv_kernel = 0, max_seq = 0;
    int batch = 1;  // sequences decoded in lockstep (one position for all)
    float eps = 1e-6f, rope_theta = 1000000.0f;
    std::vector<Layer> layers;
    void* embed = nullptr;  // [vocab][hidden], BF16 or F32 as stored
    int embed_bf16 = 1;
    float* final_norm = nullptr;
    qlm_w8* lm_head = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;  // [max_seq][rotary_dim / 2]
    // activations and scratch (device)
    float *x = nullptr, *h = nullptr, *t1 = nullptr, *t2 = nullptr, *t3 = nullptr, *t4 = nullptr, *t5 = nullptr;
    float *gate_buf = nullptr, *up_buf = nullptr, *logits = nullptr, *scores = nullptr;
    // The step's control words [B tokens][position][conv ring position],
    // uploaded with one copy; the greedy choices come back in the token words.
    int* d_tokens = nullptr;  // device [B + 2]
    int* h_tokens = nullptr;  // pinned host [B + 2]
    int ring = 0;             // oldest tap of every gated-delta-net conv ring (all advance together)
    // The step captured once as a CUDA graph (after one eager step has sized
    // every scratch buffer) and replayed at every position.
    bool use_graph = true;
    bool pdl = true;  // step kernels launched as programmatic-dependent secondaries (QLM_PDL=0: not)
    int eager_steps = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    cudaStream_t stream = nullptr;
    std::vector<void*> allocs;
    std::vector<qlm_w8*> weights;
};

namespace {

using qlm_st::JValue;

// The checkpoint: every .safetensors file of the directory (ModelWeights::
// load_from_dir, src/model/weights.cpp:6-21) and the name lookup with the
// architecture's fallback remap (model.* -> model.language_model.*).
struct Checkpoint {
    std::vector<std::unique_ptr<qlm_st::Store>> files;
    const qlm_st::TensorRef* find(const std::string& name, const qlm_st::Store** in) const {
        for (const auto& f : files) {
            auto it = f->tensors.find(name);
            if (it != f->tensors.end()) {
                *in = f.get();
                return &it->second;
            }
        }
        if (name.rfind("model.", 0) == 0) {
            const std::string alt = "model.language_model." + name.substr(6);
            for (const auto& f : files) {
                auto it = f->tensors.find(alt);
                if (it != f->tensors.end()) {
                    *in = f.get();
                    return &it->second;
                }
            }
        }
        return nullptr;
    }
};

const JValue* member(const JValue& o, const char* key) {
    if (o.kind != JValue::Obj) return nullptr;
    auto it = o.obj.find(key);
    return it == o.obj.end() ? nullptr : &it->second;
}

// A number of config.json read as the reference does (strtod, then the
// member's own type).
bool number(const JValue& o, const char* key, double* out) {
    const JValue* v = member(o, key);
    if (!v || v->kind != JValue::Num) return false;
    char* end = nullptr;
    const double d = std::strtod(v->str.c_str(), &end);
    if (!end || end == v->str.c_str()) return false;
    *out = d;
    return true;
}

struct Loader {
    qlm_model* m;
    Checkpoint ck;
    cudaStream_t s;

    int dev_alloc(void** p, size_t bytes) {
        const cudaError_t e = cudaMalloc(p, bytes);
        if (e != cudaSuccess) return fail(QLM_ERR_OUT_OF_MEMORY, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
        m->allocs.push_back(*p);
        return QLM_OK;
    }
    template <typename T>
    int zeros(T** p, size_t n) {
        int rc = dev_alloc(reinterpret_cast<void**>(p), n * sizeof(T));
        if (rc) return rc;
        if (cudaMemsetAsync(*p, 0, n * sizeof(T), s) != cudaSuccess) return fail(QLM_ERR_CUDA, "cudaMemset failed");
        return QLM_OK;
    }
    const qlm_st::TensorRef* tensor(const std::string& name, const qlm_st::Store** in, size_t numel) {
        const qlm_st::TensorRef* t = ck.find(name, in);
        if (!t) {
            fail(QLM_ERR_INVALID_ARG, "checkpoint has no tensor '%s'", name.c_str());
            return nullptr;
        }
        size_t n = 1;
        for (int64_t d : t->shape) n *= (size_t)d;
        const size_t esz = t->dtype == "F32" ? 4 : t->dtype == "BF16" ? 2 : 0;
        if (!esz) {
            fail(QLM_ERR_INVALID_ARG, "tensor '%s' has dtype %s (F32 or BF16 expected)", name.c_str(), t->dtype.c_str());
            return nullptr;
        }
        if ((numel && n != numel) || t->end - t->begin != n * esz) {
            fail(QLM_ERR_INVALID_ARG, "tensor '%s' has %zu elements / %llu bytes, expected %zu elements", name.c_str(),
                 n, (unsigned long long)(t->end - t->begin), numel);
            return nullptr;
        }
        return t;
    }
    // The values on the host only (BF16 upcast exactly).
    int host_f32(const std::string& name, size_t numel, std::vector<float>& h) {
        const qlm_st::Store* st = nullptr;
        const qlm_st::TensorRef* t = tensor(name, &st, numel);
        if (!t) return QLM_ERR_INVALID_ARG;
        h.resize(numel);
        const uint8_t* src = static_cast<const uint8_t*>(st->m.base) + t->begin;
        if (t->dtype == "F32") {
            std::memcpy(h.data(), src, numel * 4);
        } else {
            for (size_t i = 0; i < numel; ++i) {
                uint16_t b;
                std::memcpy(&b, src + 2 * i, 2);
                const uint32_t bits = (uint32_t)b << 16;
                std::memcpy(&h[i], &bits, 4);
            }
        }
        return QLM_OK;
    }
    // An F32 copy on the device (ModelWeights::get_tensor: BF16 upcast exactly).
    int f32(const std::string& name, size_t numel, float** out, std::vector<float>* host = nullptr) {
        const qlm_st::Store* st = nullptr;
        const qlm_st::TensorRef* t = tensor(name, &st, numel);
        if (!t) return QLM_ERR_INVALID_ARG;
        std::vector<float> h(numel);
        const uint8_t* src = static_cast<const uint8_t*>(st->m.base) + t->begin;
        if (t->dtype == "F32") {
            std::memcpy(h.data(), src, numel * 4);
        } else {
            for (size_t i = 0; i < numel; ++i) {
                uint16_t b;
                std::memcpy(&b, src + 2 * i, 2);
                const uint32_t bits = (uint32_t)b << 16;
                std::memcpy(&h[i], &bits, 4);
            }
        }
        if (host) *host = h;
        int rc = dev_alloc(reinterpret_cast<void**>(out), numel * 4);
        if (rc) return rc;
        if (cudaMemcpy(*out, h.data(), numel * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return fail(QLM_ERR_CUDA, "upload of '%s' failed", name.c_str());
        return QLM_OK;
    }
    // Rows [rb, re) (all when re < 0) of an int8 matmul weight [rows, k],
    // quantized on the device from the mapped bytes (ModelWeights::get_weight
    // at Precision::Int8 -> get_tensor_keep_int8; the quantizer is row-local,
    // so a row range holds exactly those rows' bytes and scales).
    int weight(const std::string& name, int rows, int k, qlm_w8** out, int rb = 0, int re = -1) {
        const qlm_st::Store* st = nullptr;
        const qlm_st::TensorRef* t = tensor(name, &st, (size_t)rows * k);
        if (!t) return QLM_ERR_INVALID_ARG;
        if (t->shape.size() != 2 || t->shape[0] != rows || t->shape[1] != k)
            return fail(QLM_ERR_INVALID_ARG, "weight '%s' is not [%d, %d]", name.c_str(), rows, k);
        const void* src = static_cast<const uint8_t*>(st->m.base) + t->begin;
        const int rc = qlm_weight_quantize_upload(src, t->dtype == "F32" ? QLM_SRC_F32 : QLM_SRC_BF16, k, rows, k, rb,
                                                  re < 0 ? rows : re, m->device, s, out);
        if (rc == QLM_OK) m->weights.push_back(*out);
        return rc;
    }
};

int parse_config(const std::string& dir, qlm_model* m) {
    const std::string path = dir + "/config.json";
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return fail(QLM_ERR_INVALID_ARG, "cannot open %s", path.c_str());
    std::string text;
    char buf[65536];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof buf, f)) > 0 && text.size() < (16u << 20)) text.append(buf, n);
    std::fclose(f);
    qlm_st::JParser jp{text.data(), text.data() + text.size(), {}};
    JValue root;
    if (!jp.value(root, 0) || root.kind != JValue::Obj)
        return fail(QLM_ERR_INVALID_ARG, "%s: not a JSON object (%s)", path.c_str(), jp.err.c_str());
    const JValue* tc = member(root, "text_config");
    const JValue& c = tc && tc->kind == JValue::Obj ? *tc : root;
    const JValue* mt = member(c, "model_type");
    if (!mt) mt = member(root, "model_type");
    if (!mt || mt->kind != JValue::Str || mt->str.rfind("qwen3_5", 0) != 0)
        return fail(QLM_ERR_UNSUPPORTED, "%s: model_type %s is not a Qwen3.5 hybrid", path.c_str(),
                    mt && mt->kind == JValue::Str ? mt->str.c_str() : "(missing)");
    double v = 0;
    auto need = [&](const char* key, int* out) {
        if (!number(c, key, &v) || v <= 0 || v > 1e9) return false;
        *out = (int)v;
        return true;
    };
    if (!need("vocab_size", &m->vocab) || !need("hidden_size", &m->hidden) ||
        !need("intermediate_size", &m->inter) || !need("num_hidden_layers", &m->layers_n) ||
        !need("num_attention_heads", &m->heads))
        return fail(QLM_ERR_INVALID_ARG, "%s: missing or bad sizes", path.c_str());
    if (!need("num_key_value_heads", &m->kv_heads)) m->kv_heads = m->heads;
    if (number(c, "rms_norm_eps", &v)) m->eps = (float)v;
    double partial = 1.0;
    if (number(c, "rope_theta", &v)) {
        m->rope_theta = (float)v;
    } else if (const JValue* rp = member(c, "rope_parameters")) {
        if (number(*rp, "rope_theta", &v)) m->rope_theta = (float)v;
        if (number(*rp, "partial_rotary_factor", &v)) partial = v;
    }
    if (number(c, "partial_rotary_factor", &v)) partial = v;
    if (!need("head_dim", &m->head_dim)) m->head_dim = m->hidden / m->heads;
    need("linear_num_key_heads", &m->lin_heads);
    need("linear_key_head_dim", &m->lin_dim);
    // static_cast<int>(head_dim * partial_rotary_factor), the factor a float
    m->rotary_dim = (int)((float)m->head_dim * (float)partial);
    m->layers.assign(m->layers_n, Layer{});
    const JValue* lt = member(c, "layer_types");
    for (int i = 0; i < m->layers_n; ++i) {
        bool full = i % 4 == 3;  // the reference's default 3:1 pattern
        if (lt && lt->kind == JValue::Arr) {
            if ((int)lt->arr.size() <= i || lt->arr[i].kind != JValue::Str)
                return fail(QLM_ERR_INVALID_ARG, "%s: layer_types too short", path.c_str());
            full = lt->arr[i].str == "full_attention";
        }
        m->layers[i].full_attn = full;
    }
    return QLM_OK;
}

}  // namespace

namespace {

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

#define QLM_TRY(x)                   \
    do {                             \
        const int _rc = (x);         \
        if (_rc != QLM_OK) return _rc; \
    } while (0)

int launch_ok(const char* what) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QLM_OK : fail(QLM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int load_all(const std::string& dir, qlm_model* m) {
    Loader L{m, {}, m->stream};
    // every .safetensors file of the directory, in name order
    std::vector<std::string> names;
    if (DIR* d = opendir(dir.c_str())) {
        while (dirent* e = readdir(d)) {
            const std::string n = e->d_name;
            if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) names.push_back(n);
        }
        closedir(d);
    }
    std::sort(names.begin(), names.end());
    if (names.empty()) return fail(QLM_ERR_INVALID_ARG, "no .safetensors files in %s", dir.c_str());
    for (const std::string& n : names) {
        auto st = std::make_unique<qlm_st::Store>();
        std::string err;
        if (qlm_st::open_store((dir + "/" + n).c_str(), *st, err)) return fail(QLM_ERR_INVALID_ARG, "%s", err.c_str());
        L.ck.files.push_back(std::move(st));
    }
    const int H = m->hidden;
    // embedding table as stored (only the looked-up row is upcast, as the reference does)
    {
        const qlm_st::Store* st = nullptr;
        const qlm_st::TensorRef* t = L.ck.find("model.embed_tokens.weight", &st);
        if (!t || t->shape.size() != 2 || t->shape[1] != H || (t->dtype != "BF16" && t->dtype != "F32"))
            return fail(QLM_ERR_INVALID_ARG, "embedding model.embed_tokens.weight missing or not [*, %d] F32/BF16", H);
        m->embed_bf16 = t->dtype == "BF16";
        const size_t bytes = t->end - t->begin;
        QLM_TRY(L.dev_alloc(&m->embed, bytes));
        if (cudaMemcpy(m->embed, static_cast<const uint8_t*>(st->m.base) + t->begin, bytes, cudaMemcpyHostToDevice) !=
            cudaSuccess)
            return fail(QLM_ERR_CUDA, "embedding upload failed");
        m->vocab = (int)t->shape[0];
    }
    int conv_dim_max = 0;
    for (int i = 0; i < m->layers_n; ++i) {
        Layer& ly = m->layers[i];
        const std::string p = "model.layers." + std::to_string(i) + ".";
        QLM_TRY(L.f32(p + "input_layernorm.weight", H, &ly.in_norm));
        QLM_TRY(L.f32(p + "post_attention_layernorm.weight", H, &ly.post_norm));
        QLM_TRY(L.weight(p + "mlp.gate_proj.weight", m->inter, H, &ly.gate));
        QLM_TRY(L.weight(p + "mlp.up_proj.weight", m->inter, H, &ly.up));
        QLM_TRY(L.weight(p + "mlp.down_proj.weight", H, m->inter, &ly.down));
        if (ly.full_attn) {
            const int hd = m->head_dim, qd = 2 * hd;
            const qlm_st::Store* st = nullptr;
            if (L.ck.find(p + "self_attn.q_proj.bias", &st))
                return fail(QLM_ERR_UNSUPPORTED, "attention projection biases are not supported");
            QLM_TRY(L.weight(p + "self_attn.q_proj.weight", m->heads * qd, H, &ly.q));  // [query | gate] per head
            QLM_TRY(L.weight(p + "self_attn.k_proj.weight", m->kv_heads * hd, H, &ly.k));
            QLM_TRY(L.weight(p + "self_attn.v_proj.weight", m->kv_heads * hd, H, &ly.v));
            QLM_TRY(L.weight(p + "self_attn.o_proj.weight", H, m->heads * hd, &ly.o));
            if (!L.ck.find(p + "self_attn.q_norm.weight", &st))
                return fail(QLM_ERR_UNSUPPORTED, "attention without QK-norm is not supported");
            QLM_TRY(L.f32(p + "self_attn.q_norm.weight", hd, &ly.q_norm));
            QLM_TRY(L.f32(p + "self_attn.k_norm.weight", hd, &ly.k_norm));
            QLM_TRY(L.zeros(&ly.k_cache, (size_t)m->max_seq * m->batch * m->kv_heads * hd));
            QLM_TRY(L.zeros(&ly.v_cache, (size_t)m->max_seq * m->batch * m->kv_heads * hd));
        } else {
            const int lin = m->lin_heads * m->lin_dim;
            if (lin <= 0) return fail(QLM_ERR_INVALID_ARG, "linear-attention layer %d without linear head sizes", i);
            const int conv_dim = 3 * lin;
            const std::string qkv = p + "linear_attn.in_proj_qkv.weight";
            QLM_TRY(L.weight(qkv, conv_dim, H, &ly.qkv_q, 0, lin));
            QLM_TRY(L.weight(qkv, conv_dim, H, &ly.qkv_k, lin, 2 * lin));
            QLM_TRY(L.weight(qkv, conv_dim, H, &ly.qkv_v, 2 * lin, 3 * lin));
            QLM_TRY(L.weight(p + "linear_attn.in_proj_z.weight", lin, H, &ly.z));
            QLM_TRY(L.weight(p + "linear_attn.in_proj_b.weight", m->lin_heads, H, &ly.b));
            QLM_TRY(L.weight(p + "linear_attn.in_proj_a.weight", m->lin_heads, H, &ly.a));
            QLM_TRY(L.weight(p + "linear_attn.out_proj.weight", H, lin, &ly.out));
            const qlm_st::Store* st = nullptr;
            const qlm_st::TensorRef* cw = L.ck.find(p + "linear_attn.conv1d.weight", &st);
            if (!cw || cw->shape.size() != 3 || cw->shape[0] != conv_dim || cw->shape[1] != 1 || cw->shape[2] < 2)
                return fail(QLM_ERR_INVALID_ARG, "conv1d weight of layer %d is not [%d, 1, kernel]", i, conv_dim);
            const int kernel = (int)cw->shape[2];
            if (m->conv_kernel && m->conv_kernel != kernel) return fail(QLM_ERR_UNSUPPORTED, "conv kernels differ");
            m->conv_kernel = kernel;
            std::vector<float> w;
            QLM_TRY(L.host_f32(p + "linear_attn.conv1d.weight", (size_t)conv_dim * kernel, w));
            // tap-major (attention.cpp:402-407), channels ordered [part][sequence][c]
            const int B = m->batch;
            std::vector<float> wt((size_t)kernel * 3 * B * lin);
            for (int k = 0; k < kernel; ++k)
                for (int part = 0; part < 3; ++part)
                    for (int b = 0; b < B; ++b)
                        for (int c = 0; c < lin; ++c)
                            wt[(size_t)k * 3 * B * lin + ((size_t)part * B + b) * lin + c] =
                                w[(size_t)(part * lin + c) * kernel + k];
            QLM_TRY(L.dev_alloc(reinterpret_cast<void**>(&ly.conv_wt), wt.size() * 4));
            if (cudaMemcpy(ly.conv_wt, wt.data(), wt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
                return fail(QLM_ERR_CUDA, "conv weight upload failed");
            QLM_TRY(L.zeros(&ly.conv_state, (size_t)(kernel - 1) * 3 * B * lin));
            QLM_TRY(L.f32(p + "linear_attn.norm.weight", m->lin_dim, &ly.gdn_norm));
            QLM_TRY(L.f32(p + "linear_attn.A_log", m->lin_heads, &ly.A_log));
            QLM_TRY(L.f32(p + "linear_attn.dt_bias", m->lin_heads, &ly.dt_bias));
            QLM_TRY(L.zeros(&ly.rstate, (size_t)m->batch * m->lin_heads * m->lin_dim * m->lin_dim));
            conv_dim_max = conv_dim > conv_dim_max ? conv_dim : conv_dim_max;
        }
    }
    QLM_TRY(L.f32("model.norm.weight", H, &m->final_norm));
    {
        const qlm_st::Store* st = nullptr;
        const std::string lm = L.ck.find("lm_head.weight", &st) ? "lm_head.weight" : "model.embed_tokens.weight";
        const qlm_st::TensorRef* t = L.ck.find(lm, &st);
        QLM_TRY(L.weight(lm, (int)t->shape[0], H, &m->lm_head));
        m->vocab = (int)t->shape[0];  // the effective vocabulary: lm_head's rows (model.cpp:127)
    }
    if (m->rotary_dim < 2 || m->rotary_dim > m->head_dim || (m->rotary_dim & 1))
        return fail(QLM_ERR_UNSUPPORTED, "rotary_dim %d not in [2, head_dim] and even", m->rotary_dim);
    {
        const int half = m->rotary_dim / 2;
        std::vector<float> c((size_t)m->max_seq * half), sn((size_t)m->max_seq * half);
        QLM_TRY(qlm_rope_neox_tables(0, m->max_seq, m->rope_theta, m->rotary_dim, c.data(), sn.data()));
        QLM_TRY(L.dev_alloc(reinterpret_cast<void**>(&m->rope_cos), c.size() * 4));
        QLM_TRY(L.dev_alloc(reinterpret_cast<void**>(&m->rope_sin), c.size() * 4));
        if (cudaMemcpy(m->rope_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return fail(QLM_ERR_CUDA, "RoPE table upload failed");
    }
    size_t big = (size_t)H;
    const size_t cands[] = {(size_t)conv_dim_max, (size_t)2 * m->heads * m->head_dim, (size_t)m->inter,
                            (size_t)m->lin_heads * m->lin_dim, (size_t)2 * m->lin_heads + 16};
    for (size_t c : cands) big = c > big ? c : big;
    const size_t B = (size_t)m->batch;
    float** bufs[] = {&m->x, &m->h, &m->t1, &m->t2, &m->t3, &m->t4, &m->t5};
    for (float** b : bufs) QLM_TRY(L.zeros(b, B * big));
    QLM_TRY(L.zeros(&m->gate_buf, B * m->inter));
    QLM_TRY(L.zeros(&m->up_buf, B * m->inter));
    QLM_TRY(L.zeros(&m->logits, B * m->vocab));
    QLM_TRY(L.zeros(&m->scores, B * m->heads * m->max_seq));
    QLM_TRY(L.zeros(&m->d_tokens, B + 2));
    if (cudaMallocHost(reinterpret_cast<void**>(&m->h_tokens), (B + 2) * sizeof(int)) != cudaSuccess)
        return fail(QLM_ERR_OUT_OF_MEMORY, "pinned host words");
    bool any_attn = false;
    for (const Layer& ly : m->layers) any_attn = any_attn || ly.full_attn;
    if (any_attn && qlm::gqa_dev_smem_bytes(m->max_seq - 1) > 200 * 1024)
        return fail(QLM_ERR_UNSUPPORTED, "max_seq %d too long for the attention kernels", m->max_seq);
    {
        const char* e = std::getenv("QLM_MODEL_GRAPH");
        m->use_graph = !(e && e[0] == '0');
        const char* p = std::getenv("QLM_PDL");
        m->pdl = !(p && p[0] == '0');
    }
    if (cudaStreamSynchronize(m->stream) != cudaSuccess) return fail(QLM_ERR_CUDA, "load synchronize failed");
    return QLM_OK;
}

void release(qlm_model* m) {
    if (!m) return;
    Dev g(m->device >= 0 ? m->device : 0);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->graph_exec) cudaGraphExecDestroy(m->graph_exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    for (qlm_w8* w : m->weights) qlm_weight_free(w);
    for (void* p : m->allocs) cudaFree(p);
    if (m->h_tokens) cudaFreeHost(m->h_tokens);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

}  // namespace

namespace {

// One layer's gated-delta-net step (Qwen3_5GatedDeltaNet::forward,
// src/model/attention.cpp:414-591) for the B sequences on m->h [B][hidden];
// result in m->t5 [B][hidden]. Heads of all sequences run as B * lin_heads heads.
int gdn_step(qlm_model* m, Layer& ly) {
    cudaStream_t s = m->stream;
    const int B = m->batch, H = m->hidden, lh = m->lin_heads, ld = m->lin_dim, lin = lh * ld;
    const int channels = 3 * B * lin;  // conv channels: [part][sequence][c]
    float* qkv = m->t1;                // [3][B][lin]
    float* conv = m->t2;               // same layout, after the conv
    float* z = m->t3;                  // [B][lin]
    float* b_raw = m->t4;              // [B][lh]
    float* a_raw = m->t4 + (size_t)B * lh;
    const qlm_w8* ws[6] = {ly.qkv_q, ly.qkv_k, ly.qkv_v, ly.z, ly.b, ly.a};
    float* ys[6] = {qkv, qkv + (size_t)B * lin, qkv + (size_t)2 * B * lin, z, b_raw, a_raw};
    const int64_t lds[6] = {lin, lin, lin, lin, lh, lh};
    QLM_TRY(qlm_linear_int8_grouped(m->h, B, H, H, ws, 6, ys, lds, 0, s));                      // 1. projections
    if (qlm::launch_conv1d_silu_dev(qkv, ly.conv_state, m->d_tokens + B + 1, ly.conv_wt, conv, channels,
                                    m->conv_kernel, s, m->pdl) != cudaSuccess)
        return launch_ok("conv step + SiLU");                                                     // 2.-4. conv, SiLU
    float *q = conv, *k = conv + (size_t)B * lin, *v = conv + (size_t)2 * B * lin;
    float* out = qkv;  // the projections are consumed
    if (qlm::launch_gdn_recurrence_fused(ly.rstate, q, k, v, a_raw, b_raw, ly.A_log, ly.dt_bias, lh, 1e-6f, out,
                                         B * lh, ld, s, m->pdl) != cudaSuccess)
        return launch_ok("L2 norms + gates + delta rule");                                        // 5.-7.
    if (qlm::launch_head_norm_gate(out, ly.gdn_norm, z, B * lh, ld, 1e-6f, s, m->pdl) != cudaSuccess)
        return launch_ok("head norm + output gate");                                              // 8.-9.
    return qlm_linear_int8(z, B, lin, lin, ly.out, m->t5, H, 0, s);                               // 10. out_proj
}

// One layer's gated GQA step (Qwen3_5Attention::forward,
// src/model/attention.cpp:138-235) for the B sequences at the position held
// in the step's control words (device memory, so a captured step replays at
// every position); result in m->t5. Sequence b's query head h is head
// b * heads + h, its KV head b * kv_heads + h / group: the cache
// [T][B][kv_heads][d] reads as B * kv_heads heads.
int attn_step(qlm_model* m, Layer& ly) {
    cudaStream_t s = m->stream;
    const int B = m->batch, H = m->hidden, hd = m->head_dim, qd = 2 * hd, nh = m->heads, kvh = m->kv_heads;
    const int kv = kvh * hd;
    float *q = m->t1, *k = m->t2, *v = m->t3, *att = m->t4;
    const qlm_w8* ws[3] = {ly.q, ly.k, ly.v};
    float* ys[3] = {q, k, v};
    const int64_t lds[3] = {(int64_t)nh * qd, kv, kv};
    QLM_TRY(qlm_linear_int8_grouped(m->h, B, H, H, ws, 3, ys, lds, 0, s));                // 1. projections
    if (qlm::launch_qk_norm(q, qd, ly.q_norm, B * nh, k, hd, ly.k_norm, B * kvh, hd, 1e-6f, s, m->pdl) !=
        cudaSuccess)
        return launch_ok("QK-norm");                                                          // 2. QK-norm
    const int* d_pos = m->d_tokens + B;  // q: the query half of each [query | gate] row
    if (qlm::launch_rope_append(q, qd, B * nh, k, v, B * kvh, hd, m->rotary_dim, m->rope_cos, m->rope_sin, d_pos,
                                ly.k_cache, ly.v_cache, s, m->pdl) != cudaSuccess)
        return launch_ok("RoPE + KV cache write");                                           // 3.-4.
    if (qlm::launch_gqa_attend_dev(q, qd, ly.k_cache, ly.v_cache, att, d_pos, m->max_seq - 1, B * nh, B * kvh, hd,
                                   m->scores, q + hd, qd, s, m->pdl) != cudaSuccess)                 // 5.-6. attention,
        return launch_ok("attention");                                                       // output gate
    return qlm_linear_int8(att, B, nh * hd, nh * hd, ly.o, m->t5, H, 0, s);                 // 7. o_proj
}

}  // namespace

namespace {

// The step's device work, from the upload of the control words to the
// read-back of the greedy choices (DecoderModel::forward + sample,
// src/model/model.cpp:151-199, 259-272). Enqueued eagerly or into a capture.
int enqueue_step(qlm_model* m) {
    const int B = m->batch;
    cudaStream_t s = m->stream;
    const int H = m->hidden;
    if (cudaMemcpyAsync(m->d_tokens, m->h_tokens, (size_t)(B + 2) * sizeof(int), cudaMemcpyHostToDevice, s) !=
        cudaSuccess)
        return fail(QLM_ERR_CUDA, "token upload failed");
    embed_rows_kernel<<<dim3((H + kEmbThreads - 1) / kEmbThreads, B), kEmbThreads, 0, s>>>(m->embed, m->embed_bf16,
                                                                                           m->d_tokens, H, m->x);
    QLM_TRY(launch_ok("embedding"));
    // Each residual add is fused with the norm that follows it (post-attention
    // norm, the next layer's input norm, the final norm): same bits as
    // elementwise_add + rms_norm (modules.hpp:228-231, 239-240).
    const size_t nl = m->layers.size();
    if (qlm::launch_rms_norm(m->x, nl ? m->layers[0].in_norm : m->final_norm, m->h, B, H, m->eps, s, m->pdl) !=
        cudaSuccess)
        return launch_ok("input norm");
    for (size_t l = 0; l < nl; ++l) {
        Layer& ly = m->layers[l];
        QLM_TRY(ly.full_attn ? attn_step(m, ly) : gdn_step(m, ly));
        if (qlm::launch_add_then_rms_norm(m->x, m->t5, ly.post_norm, m->h, B, H, m->eps, s, m->pdl) != cudaSuccess)
            return launch_ok("residual add + post-attention norm");
        const qlm_w8* ws[2] = {ly.gate, ly.up};
        float* ys[2] = {m->gate_buf, m->up_buf};
        const int64_t lds[2] = {m->inter, m->inter};
        QLM_TRY(qlm_linear_int8_grouped(m->h, B, H, H, ws, 2, ys, lds, 0, s));
        if (qlm::launch_silu_mul(m->gate_buf, m->up_buf, (int64_t)B * m->inter, s, m->pdl) != cudaSuccess)
            return launch_ok("SiLU * up");
        QLM_TRY(qlm_linear_int8(m->gate_buf, B, m->inter, m->inter, ly.down, m->t5, H, 0, s));
        const float* next_norm = l + 1 < nl ? m->layers[l + 1].in_norm : m->final_norm;
        if (qlm::launch_add_then_rms_norm(m->x, m->t5, next_norm, m->h, B, H, m->eps, s, m->pdl) != cudaSuccess)
            return launch_ok("residual add + norm");
    }
    QLM_TRY(qlm_linear_int8(m->h, B, H, H, m->lm_head, m->logits, m->vocab, 0, s));
    if (qlm::launch_pdl(m->pdl, greedy_rows_kernel, dim3(B), dim3(1024), 0, s, (const float*)m->logits, m->vocab,
                        m->d_tokens) != cudaSuccess)
        return launch_ok("greedy choice");
    if (cudaMemcpyAsync(m->h_tokens, m->d_tokens, (size_t)B * sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return fail(QLM_ERR_CUDA, "token read-back failed");
    return QLM_OK;
}

// Captures the step into m->graph_exec; on any failure the model stays on
// eager steps (the result is the same, only slower).
void capture_step(qlm_model* m) {
    cudaStream_t s = m->stream;
    if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        m->use_graph = false;
        return;
    }
    const int rc = enqueue_step(m);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(s, &g);
    if (rc != QLM_OK || e != cudaSuccess || !g ||
        cudaGraphInstantiate(&m->graph_exec, g, 0) != cudaSuccess) {
        cudaGetLastError();
        if (g) cudaGraphDestroy(g);
        m->graph_exec = nullptr;
        m->use_graph = false;
        return;
    }
    m->graph = g;
}

int decode_step(qlm_model* m, const int* tokens, int pos, int* next_tokens, float* logits) {
    const int B = m->batch;
    for (int b = 0; b < B; ++b)
        if (tokens[b] < 0 || tokens[b] >= m->vocab)
            return fail(QLM_ERR_INVALID_ARG, "token %d (sequence %d) not in [0, %d)", tokens[b], b, m->vocab);
    if (pos < 0 || pos >= m->max_seq)
        return fail(QLM_ERR_INVALID_ARG, "position %d not in [0, max_seq %d)", pos, m->max_seq);
    Dev g(m->device);
    if (!g.ok) return fail(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", m->device);
    cudaStream_t s = m->stream;
    std::memcpy(m->h_tokens, tokens, (size_t)B * sizeof(int));
    m->h_tokens[B] = pos;
    m->h_tokens[B + 1] = m->ring;
    // While per-matmul timing is on the step runs eagerly, so every linear
    // call is timed (calls replayed inside a graph are not).
    const bool graph = m->use_graph && !qlm_internal::prof_on();
    if (graph && !m->graph_exec && m->eager_steps > 0) capture_step(m);
    if (graph && m->graph_exec) {
        if (cudaGraphLaunch(m->graph_exec, s) != cudaSuccess) return launch_ok("decode step graph");
    } else {
        QLM_TRY(enqueue_step(m));
        ++m->eager_steps;
    }
    if (logits &&
        cudaMemcpyAsync(logits, m->logits, (size_t)B * m->vocab * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return fail(QLM_ERR_CUDA, "logits read-back failed");
    if (cudaStreamSynchronize(s) != cudaSuccess) return launch_ok("decode step");
    if (m->conv_kernel > 1) m->ring = (m->ring + 1) % (m->conv_kernel - 1);
    QLM_TRY(qlm_device_status(m->device, 1));
    std::memcpy(next_tokens, m->h_tokens, (size_t)B * sizeof(int));
    return QLM_OK;
}

}  // namespace

extern "C" {

int qlm_model_load_batch(const char* dir, int device, int max_seq, int batch, qlm_model** out) {
    if (!dir || !out) return fail(QLM_ERR_INVALID_ARG, "NULL argument");
    *out = nullptr;
    if (max_seq < 1 || max_seq > (1 << 20)) return fail(QLM_ERR_INVALID_ARG, "max_seq %d not in [1, 2^20]", max_seq);
    if (batch < 1 || batch > 1024) return fail(QLM_ERR_INVALID_ARG, "batch %d not in [1, 1024]", batch);
    qlm_model* m = new (std::nothrow) qlm_model();
    if (!m) return fail(QLM_ERR_OUT_OF_MEMORY, "host allocation failed");
    m->device = device;
    m->max_seq = max_seq;
    m->batch = batch;
    int rc = parse_config(dir, m);
    Dev g(device);
    if (rc == QLM_OK && !g.ok) rc = fail(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    if (rc == QLM_OK && cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess)
        rc = fail(QLM_ERR_CUDA, "cudaStreamCreate failed");
    if (rc == QLM_OK) rc = load_all(dir, m);
    if (rc != QLM_OK) {
        release(m);
        return rc;
    }
    *out = m;
    return QLM_OK;
}

int qlm_model_load(const char* dir, int device, int max_seq, qlm_model** out) {
    return qlm_model_load_batch(dir, device, max_seq, 1, out);
}

int qlm_model_reset(qlm_model* m) {
    if (!m) return fail(QLM_ERR_INVALID_ARG, "NULL model");
    Dev g(m->device);
    if (!g.ok) return fail(QLM_ERR_CUDA, "cudaSetDevice(%d) failed", m->device);
    const size_t B = (size_t)m->batch;
    for (Layer& ly : m->layers) {
        const size_t kv = (size_t)m->max_seq * B * m->kv_heads * m->head_dim * 4;
        const size_t lin = (size_t)m->lin_heads * m->lin_dim;
        cudaError_t e = cudaSuccess;
        if (ly.full_attn) {
            e = cudaMemsetAsync(ly.k_cache, 0, kv, m->stream);
            if (e == cudaSuccess) e = cudaMemsetAsync(ly.v_cache, 0, kv, m->stream);
        } else {
            e = cudaMemsetAsync(ly.conv_state, 0, (size_t)(m->conv_kernel - 1) * 3 * B * lin * 4, m->stream);
            if (e == cudaSuccess) e = cudaMemsetAsync(ly.rstate, 0, B * lin * m->lin_dim * 4, m->stream);
        }
        if (e != cudaSuccess) return fail(QLM_ERR_CUDA, "state reset failed");
    }
    m->ring = 0;
    return cudaStreamSynchronize(m->stream) == cudaSuccess ? QLM_OK : fail(QLM_ERR_CUDA, "synchronize failed");
}

int qlm_model_info(const qlm_model* m, int* vocab, int* hidden, int* layers, int* max_seq, int* batch) {
    if (!m) return fail(QLM_ERR_INVALID_ARG, "NULL model");
    if (vocab) *vocab = m->vocab;
    if (hidden) *hidden = m->hidden;
    if (layers) *layers = m->layers_n;
    if (max_seq) *max_seq = m->max_seq;
    if (batch) *batch = m->batch;
    return QLM_OK;
}

int qlm_model_decode(qlm_model* m, int token, int pos, int* next_token, float* logits) {
    if (!m || !next_token) return fail(QLM_ERR_INVALID_ARG, "NULL argument");
    if (m->batch != 1) return fail(QLM_ERR_INVALID_ARG, "the model decodes %d sequences: use qlm_model_decode_batch", m->batch);
    qlm_internal::NvtxRange range("qlm_model_decode");
    return decode_step(m, &token, pos, next_token, logits);
}

int qlm_model_decode_batch(qlm_model* m, const int* tokens, int pos, int* next_tokens, float* logits) {
    if (!m || !tokens || !next_tokens) return fail(QLM_ERR_INVALID_ARG, "NULL argument");
    qlm_internal::NvtxRange range("qlm_model_decode_batch");
    return decode_step(m, tokens, pos, next_tokens, logits);
}

void* qlm_model_stream(const qlm_model* m) { return m ? static_cast<void*>(m->stream) : nullptr; }

void qlm_model_free(qlm_model* m) { release(m); }

}  // extern "C"
