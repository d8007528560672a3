// qlm_kernels.h — internal launch interface between the C ABI and the kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

namespace qlm {

// Quantize `rows` rows of k F32 (dtype 0) or BF16 (dtype 1) device values with
// row stride src_stride into the packed layout: q [rows][packed_k(k)],
// scales [rows][packed_k(k)/32].
cudaError_t launch_quantize_pack(const void* src, int dtype, int64_t src_stride, int rows, int k, uint8_t* q,
                                 float* scales, cudaStream_t stream);

// The int4 (Q4_0-style) counterpart: scale = max|v| / 8, values in [-8, 7],
// q [rows][packed_k(k) / 2] in the P128/4 layout (qlm_device.cuh).
cudaError_t launch_quantize_pack_q4(const void* src, int dtype, int64_t src_stride, int rows, int k, uint8_t* q,
                                    float* scales, cudaStream_t stream);

// Move already-quantized codes from the reference Tensor's layouts (int8
// [rows][k] with row stride code_stride bytes; int4 [rows][(k+1)/2] bytes, low
// nibble = even column) and their scales [rows][ceil(k/32)] (row stride
// scale_stride floats) into the packed layout and padded scales. Device
// pointers.
cudaError_t launch_repack(const uint8_t* codes, int64_t code_stride, const float* scales, int64_t scale_stride,
                          int rows, int k, bool q4, uint8_t* q, float* s, cudaStream_t stream);

constexpr int kMaxRanks = 8;

// Peer pointers for the fused GEMV + all-gather (M = 1). peer_slots[r] is
// rank r's exchange area: two halves of out_stride 64-bit words, picked by
// the parity of the call's epoch; a word holds (epoch << 32) | float bits of
// one gathered output, so a reader knows from the word alone whether it
// belongs to the current call. Device-resident state of this rank: the
// communicator's last completed call (its epoch), kept in nepochs equal
// words, one per CTA index. The GEMV's CTA b reads word b; the collect
// kernel's CTA b reads word b and, at its end, writes the new epoch into words
// b, b + grid, b + 2 grid, ..., so every word advances once per call for any
// grid size, with no cross-CTA counter.
struct GatherArgs {
    unsigned long long* peer_slots[kMaxRanks];
    int* epochs;
    int nepochs;
    long long out_stride;
    int n_total; // gathered width copied into y
    int nranks;  // 0 = no gather
    int rank;
    int col0;    // this shard's first output column
    long long wait_ns;  // give up waiting for peers after this long (status 0x202)
};

// Greedy selection across ranks: peer_words[r] is rank r's exchange header
// (two halves of kMaxRanks 64-bit words, by epoch parity). nranks = 0: this
// launch reduces its logits alone.
struct ArgmaxArgs {
    unsigned long long* peer_words[kMaxRanks];
    int* epochs;        // the communicator's epoch words (GatherArgs); this one-CTA launch advances all
    int nepochs;
    int* status;        // the communicator's: non-zero = failed, the kernel does nothing
    int nranks;
    int rank;
    long long wait_ns;  // give up waiting for peers after this long
};

// out_idx / out_val (device) = the reference's greedy choice over the logits
// y[0:n], whose first element is global logit col0; with a.nranks > 0 the
// choice is over every rank's shard (each rank passes its own).
cudaError_t launch_argmax(const float* y, int n, int col0, const ArgmaxArgs& a, int* out_idx, float* out_val,
                          cudaStream_t stream, bool pdl);

// TMA descriptors through which the exact GEMV reads a packed weight: the
// codes as a 2-D tensor of 8-byte elements [rows][row bytes / 8], the scales
// as [rows][k_pad / 32]. One load brings a unit of 4R rows x `sc` chunks (one
// work item) into shared memory in the [row][chunk][bytes] order the
// arithmetic reads; index r - 1 serves R = r rows per thread. The kernel
// reads them from `dev`, a device copy of q[0], q[1], s[0], s[1] (kept out of
// the kernel parameters, which every launch copies).
struct GemvMaps {
    alignas(64) CUtensorMap q[2];
    alignas(64) CUtensorMap s[2];
    int sc;                         // chunks per box: the segment length the GEMV plans for this k
    CUtensorMap* dev = nullptr;     // device copy (owned by the weight handle)
};

// Build the GEMV descriptors of a packed weight and their device copy
// (allocates out->dev; the caller frees it with cudaFree).
cudaError_t gemv_make_maps(const uint8_t* q, const float* s, int rows, int k, bool q4, GemvMaps* out);

// Bit-exact y[m][0:rows] = x[m][0:k] . W^T for m < mm (1..8), W packed.
// status: device int set non-zero if a bounded wait gave up. With gather
// (mm == 1 only) the rows are stored into every rank's exchange buffer
// instead of y, and launch_gather_collect, next in the stream, completes the
// call.
cudaError_t launch_gemv_exact(const float* x, int64_t ldx, int mm, const uint8_t* q, const float* s,
                              const GemvMaps& maps, int rows, int k, float* y, int64_t ldy, int* status, int sm_count,
                              cudaStream_t stream, bool pdl, const GatherArgs* gather = nullptr, bool q4 = false);

// Completes a gather call: waits (bounded, ga.wait_ns; status 0x202 on a
// give-up) for every rank's words of the call in this rank's exchange buffer,
// writes y[0:ga.n_total] and advances the epoch words. Does nothing when
// *status is non-zero.
cudaError_t launch_gather_collect(const GatherArgs& ga, float* y, int* status, int sm_count, cudaStream_t stream,
                                  bool pdl);

// One weight of a grouped exact launch (packed q, scales, their descriptors,
// rows, output).
constexpr int kMaxGroup = 8;
struct GemvWeight {
    const uint8_t* q;
    const float* s;
    const GemvMaps* maps;
    int rows;
    float* y;
    int64_t ldy;
};

// Bit-exact y_g[m][0:rows_g] = x[m][0:k] . W_g^T for nw <= kMaxGroup weights
// that share x, in one launch (each output identical to a single-weight
// launch). Gather requires nw == 1 and mm == 1.
cudaError_t launch_gemv_grouped(const float* x, int64_t ldx, int mm, const GemvWeight* ws, int nw, int k,
                                int* status, int sm_count, cudaStream_t stream, bool pdl,
                                const GatherArgs* gather = nullptr, bool q4 = false);

// Whether the exact GEMV can stage mm activation rows of length k.
bool gemv_supported(int mm, int rows, int k, int sm_count, bool q4 = false);

// Decode (M = 1) form of the exact GEMV (qlm_gemv_decode.cu): producer warps
// form block sums with the activations in registers, chain warps run the
// ordered FMA chains; bit-identical outputs. Serves k up to 12 * 8 * 128.
bool gemv_decode_supported(int rows_total, int nw, int k, int sm_count, bool q4);
cudaError_t launch_gemv_decode(const float* x, const GemvWeight* ws, int nw, int k, int* status, int sm_count,
                               cudaStream_t stream, bool pdl, bool q4);

// x += delta (stored), then y = rms_norm(x) with rms_norm's own accumulation
// order (zero-centred gain): the decoder layer's unfused residual add and the
// next norm in one launch, bit-identical to the two (qlm_layer.cu).
cudaError_t launch_add_then_rms_norm(float* x, const float* delta, const float* w, float* y, int rows, int size,
                                     float eps, cudaStream_t stream, bool pdl);
// math::rms_norm (zero-centred gain) and math::silu_mul, launched from the
// decode step (qlm_layer.cu).
cudaError_t launch_rms_norm(const float* x, const float* w, float* y, int rows, int size, float eps,
                            cudaStream_t stream, bool pdl);
cudaError_t launch_silu_mul(float* a, const float* b, int64_t n, cudaStream_t stream, bool pdl);

// Decode-step forms (pdl: launched as programmatic-dependent secondaries; the
// kernels wait and read through L2) that read the position (and the conv ring
// position) from device memory, so one captured step replays at every position
// (qlm_layer.cu). launch_gqa_attend_dev: the three-launch attention with grids
// and shared memory sized for positions up to max_pos; scratch holds
// heads * (max_pos + 1) floats; gqa_v_kernel takes gqa_dev_smem_bytes(max_pos)
// of shared memory (at most 200 KB); gate (optional, row stride gate_ld): the
// sigmoid output gate applied to each output in the same launch.
// The conv step followed by SiLU on every output channel, in one launch.
cudaError_t launch_conv1d_silu_dev(const float* input, float* state, const int* d_oldest, const float* weight_t,
                                   float* output, int conv_dim, int kernel_size, cudaStream_t stream, bool pdl);
// Partial NeoX RoPE of nq query heads (in place, head stride q_ld) and nk key
// heads at position *d_pos, the rotated keys and the values written to row
// *d_pos of the caches ([T][nk * head_dim]); one launch, the arithmetic of
// the separate RoPE and append.
cudaError_t launch_rope_append(float* q, int q_ld, int nq, const float* k, const float* v, int nk, int head_dim,
                               int rotary_dim, const float* cos_all, const float* sin_all, const int* d_pos,
                               float* k_cache, float* v_cache, cudaStream_t stream, bool pdl);
// The attention's q and k head norms (zero-centred gain) in one launch, in
// place: nq query rows of stride q_ld with wq, nk key rows of stride k_ld with
// wk; bit-identical to the two separate rms_norm launches.
cudaError_t launch_qk_norm(float* q, int q_ld, const float* wq, int nq, float* k, int k_ld, const float* wk, int nk,
                           int size, float eps, cudaStream_t stream, bool pdl);
// Per head row: o = rms_norm with plain gain w (not stored), then
// z = silu(z) * o — the gated-delta-net's head norm and output gate in one
// launch, bit-identical to qlm_rms_norm_gain + qlm_silu_mul.
cudaError_t launch_head_norm_gate(const float* x, const float* w, float* z, int rows, int size, float eps,
                                  cudaStream_t stream, bool pdl);
// The delta-rule recurrence with the gates and the q/k L2 norms folded in:
// each head's decay and beta computed in the recurrence's CTAs from the raw
// gate inputs (parameters repeating every `per` heads), q and k normalized in
// shared memory (eps norm_eps); the separate steps' arithmetic. pdl: launched
// as a programmatic-dependent secondary.
cudaError_t launch_gdn_recurrence_fused(float* state, const float* q, const float* k, const float* v,
                                        const float* a_raw, const float* b_raw, const float* A_log,
                                        const float* dt_bias, int per, float norm_eps, float* out, int heads,
                                        int head_dim, cudaStream_t stream, bool pdl);
size_t gqa_dev_smem_bytes(int max_pos);
cudaError_t launch_gqa_attend_dev(const float* q, int q_stride, const float* k_cache, const float* v_cache,
                                  float* out, const int* d_pos, int max_pos, int heads, int kv_heads, int head_dim,
                                  float* scratch, const float* gate, int gate_ld, cudaStream_t stream, bool pdl);

// Bit-exact y[m][0:rows] = x[m][0:k] . W^T for 2 <= M <= 64 activation rows
// in one launch that streams W once (qlm_gemm_exact.cu): a pre-pass writes the
// activations into `scratch` (gemm_exact_scratch_bytes) in the kernel's pair
// layout; one CTA per SM (sm_count) works a balanced range of rows. Outputs
// bit-identical to the GEMV for every m.
bool gemm_exact_supported(int M, int k);
size_t gemm_exact_scratch_bytes(int M, int k);
cudaError_t launch_gemm_exact(const float* x, int64_t ldx, int M, const uint8_t* q, const float* s, int rows, int k,
                              bool q4, float* y, int64_t ldy, void* scratch, int sm_count, cudaStream_t stream);

// ---- tensor-core prefill GEMM (qlm_gemm_tc.cu) ----
struct TcMaps {
    alignas(64) CUtensorMap w;  // packed int8 rows, 128 x 128-byte boxes
    alignas(64) CUtensorMap s;  // fp32 scales
};

// The driver's tensor-map encoder (nullptr if the driver lacks it).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// TMA descriptors for a packed weight (built once per weight).
cudaError_t tc_make_weight_maps(const uint8_t* q, const float* s, int rows, int k_pad, TcMaps* out);

// Per-row weight exponents ew[rows] used to range-scale the fp16 weight tile.
cudaError_t launch_weight_exponents(const float* s, int rows, int k, int* ew, cudaStream_t stream);

// Token-tile width (multiple of 16, <= 256) the GEMM uses for M activation
// rows against a weight of `rows` rows on a GPU with sm_count SMs.
int tc_pick_bn(int M, int rows, int sm_count);

// y[M][rows] = x[M][k] . W^T on tensor cores. Scratch: x16 >= M*packed_k(k)
// fp16 and ea >= M ints; status: device int set non-zero on a timeout.
cudaError_t launch_gemm_tc(const TcMaps& maps, const int* ew, int rows, int k, const float* x, int64_t ldx, int M,
                           void* x16_scratch, int* ea_scratch, float* y, int64_t ldy, int* status,
                           cudaStream_t stream, bool pdl);

}  // namespace qlm
