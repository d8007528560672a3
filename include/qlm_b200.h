/*
 * qlm_b200.h — C ABI of the B200 (sm_100a) int8 quantized-matmul path for
 * QuickLM. Plain pointers and sizes only; every entry point returns a
 * qlm_status and never throws. qlm_last_error() gives the message of the most
 * recent failure on the calling thread.
 *
 * The path this replaces in QuickLM (paths inside its source tree):
 *   - load-time quantization: SafetensorsLoader::get_tensor_keep_int8
 *     (src/io/safetensors.cpp:517-585) with st_quantize_row_f32/_bf16
 *     (src/io/safetensors.cpp:296-391);
 *   - the int8 weight storage in Tensor (src/tensor/tensor.hpp:30-43);
 *   - the int8 branch of math::matmul (src/ops/math_ops.hpp:92,
 *     src/ops/math_ops.cpp:820-900) and its kernels int8_gemv_range /
 *     dot8/dot4/dot_avx2_int8 (src/ops/math_ops.cpp:403-579).
 *
 * Numerics: the default (exact) linear path reproduces the reference's
 * per-element arithmetic bit for bit, for any M. QLM_LINEAR_TENSOR selects the
 * tcgen05 tensor-core GEMM for prefill, which is within relative L2 2e-3.
 *
 * Threading: like math::matmul, calls for one device are expected from one
 * host thread at a time (the library keeps per-device scratch buffers).
 */
#ifndef QLM_B200_H
#define QLM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QLM_ABI_VERSION 1

/* Scale granularity: one fp32 scale per 32 consecutive elements of a row
 * (Tensor::INT8_BLOCK_SIZE, src/tensor/tensor.hpp:32). */
#define QLM_BLOCK 32

typedef enum qlm_status {
    QLM_OK = 0,
    QLM_ERR_INVALID_ARG = 1, /* bad shape, null pointer, stride, range       */
    QLM_ERR_CUDA = 2,        /* a CUDA runtime call failed                    */
    QLM_ERR_OUT_OF_MEMORY = 3,
    QLM_ERR_UNSUPPORTED = 4, /* valid request this build/device cannot serve  */
    QLM_ERR_TIMEOUT = 5,     /* a bounded device-side wait gave up            */
    QLM_ERR_NCCL = 6,        /* a NCCL call failed                            */
    QLM_ERR_INTERNAL = 7
} qlm_status;

/* Source element type of the weights handed to qlm_weight_quantize_upload,
 * the two dtypes get_tensor_keep_int8 accepts (src/io/safetensors.cpp:524-527). */
typedef enum qlm_src_dtype { QLM_SRC_F32 = 0, QLM_SRC_BF16 = 1 } qlm_src_dtype;

/* Flags for qlm_linear_int8. */
#define QLM_LINEAR_EXACT 0x0   /* bit-exact CUDA-core path (default)            */
#define QLM_LINEAR_TENSOR 0x1  /* tcgen05 tensor-core GEMM (prefill, M >= 64)   */
#define QLM_LINEAR_HOST_IO 0x2 /* x and y are HOST pointers; the call copies x  */
                               /* in, runs, copies y out and returns with y     */
                               /* complete (math::matmul's synchronous contract) */
#define QLM_LINEAR_SYNC 0x4    /* device pointers, but synchronize before return */

/* A device-resident int8 weight: rows [row_begin, row_end) of an [n_total, k]
 * matrix, packed for the decode GEMV, with its per-32-block fp32 scales.
 * Owns its device memory; release with qlm_weight_free. */
typedef struct qlm_w8 qlm_w8;

/* ABI version of the loaded library (QLM_ABI_VERSION). */
int qlm_abi_version(void);

/* Message for the most recent failing call on this thread ("" if none). */
const char* qlm_last_error(void);

/* Quantize + pack + upload. Replaces get_tensor_keep_int8
 * (src/io/safetensors.cpp:517-585): per 32-block absmax/127 scale, RN-even
 * rounding, clamp to [-127, 127], bit-identical to st_quantize_row_f32/_bf16
 * (src/io/safetensors.cpp:296-391), computed on the device.
 *   src:            [n_total, k] row-major F32 or BF16 values, row stride
 *                   src_row_stride elements (>= k); host memory (e.g. the
 *                   safetensors mmap) or device memory (detected).
 *   row_begin/end:  the output-row shard this device keeps (0, n_total for all).
 *   device:         CUDA ordinal that will hold the weight.
 *   stream:         cudaStream_t (NULL = the legacy default stream).
 * On success *out holds a new handle; the call returns after the upload. */
int qlm_weight_quantize_upload(const void* src, int src_dtype, int64_t src_row_stride, int n_total, int k,
                               int row_begin, int row_end, int device, void* stream, qlm_w8** out);

/* Int4 (Q4_0) variant of qlm_weight_quantize_upload, same arguments.
 * Replaces get_tensor_keep_int4 (src/io/safetensors.cpp:587-656): per
 * 32-block scale absmax/8, RN-even rounding, clamp to [-8, 7], bit-identical
 * to st_quantize_row_f32_int4/_bf16_int4 (src/io/safetensors.cpp:393-515).
 * The handle holds 4-bit codes (half the device bytes of int8) and is served
 * by the exact decode GEMV only: qlm_linear_int8 with QLM_LINEAR_TENSOR on an
 * int4 handle returns QLM_ERR_UNSUPPORTED. Products are bit-identical to the
 * reference int4 matmul (src/ops/math_ops.cpp:581-794, 837-854). */
int qlm_weight_quantize_upload_q4(const void* src, int src_dtype, int64_t src_row_stride, int n_total, int k,
                                  int row_begin, int row_end, int device, void* stream, qlm_w8** out);

/* Upload an already-quantized weight given in the reference Tensor's int8
 * layout (src/tensor/tensor.hpp:34-41): q [n_total, k] int8 row-major and
 * scales [n_total, ceil(k/32)] fp32; host pointers. Keeps rows
 * [row_begin, row_end). */
int qlm_weight_import_int8(const int8_t* q, const float* scales, int n_total, int k, int row_begin,
                           int row_end, int device, void* stream, qlm_w8** out);

/* Int4 counterpart of qlm_weight_import_int8: packed [n_total, (k+1)/2] bytes
 * in the reference Tensor's int4 layout (src/tensor/tensor.hpp:45-61: value + 8,
 * low nibble = even column) and scales [n_total, ceil(k/32)]. Both imports
 * take host or device pointers and repack on the device. */
int qlm_weight_import_int4(const uint8_t* packed, const float* scales, int n_total, int k, int row_begin,
                           int row_end, int device, void* stream, qlm_w8** out);

/* Copy a handle's rows back into the reference layout (host pointers):
 * q [rows, k] int8 and scales [rows, ceil(k/32)] fp32, rows = row_end - row_begin. */
int qlm_weight_export_int8(const qlm_w8* w, int8_t* q, float* scales);

/* Int4 counterpart of qlm_weight_export_int8 in the reference Tensor's int4
 * layout (src/tensor/tensor.hpp:45-61): packed [rows, (k+1)/2] bytes, low
 * nibble = even column, nibble = value + 8, and scales [rows, ceil(k/32)]. */
int qlm_weight_export_int4(const qlm_w8* w, uint8_t* packed, float* scales);

/* Bits per stored weight code: 8 (int8 handle) or 4 (int4 handle); -1 for NULL. */
int qlm_weight_bits(const qlm_w8* w);

/* Shape of a handle. Any output pointer may be NULL. */
int qlm_weight_shape(const qlm_w8* w, int* rows, int* k, int* row_begin, int* row_end, int* n_total);

/* Device bytes read by one M=1 product with this weight: packed codes plus
 * scales, the "weight bytes" of the decode roofline. */
int64_t qlm_weight_bytes(const qlm_w8* w);

/* Pre-quantized weights on disk: a standard safetensors file holding, per
 * weight, its codes in the reference Tensor's layout (dtype "I8" [rows, k], or
 * "U8" [rows, (k+1)/2] for int4), "<name>.qscale" F32 [rows, ceil(k/32)], and
 * "__metadata__" entry "qlm.<name>" = "int8 k=<k>" | "int4 k=<k>". Loading
 * skips quantization, which QuickLM's loader always performs because it
 * accepts only F32/BF16 tensors (src/io/safetensors.cpp:524-527).
 *   qlm_store_save: write n handles (their rows) under the given names.
 *   qlm_store_load: map the file, check the header (offsets inside the file,
 *                   sizes matching shapes) and upload rows [row_begin,
 *                   row_end) of `name` (row_end < 0: all rows).
 *   qlm_store_info: code width (8 or 4), rows and k of `name`; host only. */
int qlm_store_save(const char* path, int n, const char* const* names, const qlm_w8* const* weights);
int qlm_store_load(const char* path, const char* name, int row_begin, int row_end, int device, void* stream,
                   qlm_w8** out);
int qlm_store_info(const char* path, const char* name, int* bits, int64_t* rows, int64_t* k);

/* Per-layer ops on device-resident fp32 activations (device pointers,
 * asynchronous on `stream`), so a decoder layer's activations can stay in HBM
 * between its projections:
 *   qlm_rms_norm      y = rms_norm(x) per row of `size`, zero-centred gain
 *                     (1 + w): math::rms_norm (src/ops/math_ops.cpp:1055-1074).
 *                     x and y may be the same buffer. Bit-identical.
 *   qlm_add_rms_norm  residual += delta; out = rms_norm(residual):
 *                     math::add_rms_norm (math_ops.cpp:1133-1174). Bit-identical.
 *   qlm_add_then_rms_norm  the decoder layer's unfused residual step
 *                     (src/model/modules.hpp:228-231, 239-240, the default):
 *                     math::elementwise_add(residual, delta), then
 *                     math::rms_norm(residual) into out, in one launch;
 *                     bit-identical to the two (whose accumulation order
 *                     differs from math::add_rms_norm's).
 *   qlm_silu_mul      a = silu(a) * b: math::silu_mul (math_ops.cpp:1122-1131);
 *                     within 2 ulp (exp in double, rounded once, vs host expf).
 *   qlm_rope_neox     partial NeoX RoPE of t [num_tokens][num_heads][head_dim]
 *                     (first rotary_dim dims per head) with per-token cos/sin
 *                     tables [num_tokens][rotary_dim/2] in device memory:
 *                     math::apply_rope_neox (math_ops.cpp:1237-1291). Bit-identical
 *                     with tables from qlm_rope_neox_tables.
 *   qlm_rope_neox_tables  host: cos/sin for positions pos0 .. pos0+num_tokens-1,
 *                     computed with the reference's own float expressions and
 *                     libm calls (math_ops.cpp:1256-1271).
 *   qlm_silu          x = x / (1 + exp(-x)): math::silu (math_ops.cpp:1076-1084)
 *                     and the gated-delta-net conv activation (model/attention.cpp
 *                     :452-457); within 2 ulp, like qlm_silu_mul.
 *   qlm_conv1d_update_tapmajor  one depthwise causal-conv step on a tap-major
 *                     ring: math::causal_conv1d_update_tapmajor (math_ops.cpp
 *                     :1321-1366); the caller advances oldest_tap as the model
 *                     does (attention.cpp:444-448). Bit-identical.
 *   qlm_l2norm_heads  x_h /= sqrt(sumsq(x_h) + eps) per head row: the q/k
 *                     normalisation of the gated-delta-net step (attention.cpp
 *                     :462-470). Bit-identical.
 *   qlm_gdn_gates     per-head decay exp(-exp(A_log) softplus(a + dt_bias)) and
 *                     write gate sigmoid(b) (attention.cpp:472-482); libm calls
 *                     evaluated in double and rounded once (a few ulp).
 *   qlm_gdn_recurrence the gated delta rule for all heads: state [heads][d][d]
 *                     updated in place, out [heads][d] (attention.cpp:498-560).
 *                     Bit-identical given the same inputs.
 *   qlm_rms_norm_gain rms_norm with a plain gain w (the head-wise output norm,
 *                     attention.cpp:573-577). Bit-identical.
 *   qlm_gqa_attend    GQA attention of one decode token over cached positions
 *                     0..pos: q [heads][q_stride] (query in the first head_dim),
 *                     caches [T][kv_heads][head_dim], out [heads][head_dim]
 *                     (attention.cpp:17-81, 202-213). Scores, sums and the V
 *                     accumulation in the reference's order; exp in double, so
 *                     within a few ulp. Contexts up to ~50K positions. With a
 *                     device scratch of heads * (pos + 1) floats the work is
 *                     spread over three launches — scores over (head, position
 *                     block) CTAs, the softmax per head, V over (head, 32
 *                     outputs) CTAs — with the same results; NULL: one CTA per
 *                     head. */
int qlm_rms_norm(const float* x, const float* w, float* y, int rows, int size, float eps, void* stream);
int qlm_add_rms_norm(float* residual, const float* delta, const float* w, float* out, int rows, int size, float eps,
                     void* stream);
int qlm_add_then_rms_norm(float* residual, const float* delta, const float* w, float* out, int rows, int size,
                          float eps, void* stream);
int qlm_silu_mul(float* a, const float* b, int64_t n, void* stream);
int qlm_rope_neox(float* t, int num_tokens, int num_heads, int head_dim, int rotary_dim, const float* cos_tab,
                  const float* sin_tab, void* stream);
int qlm_rope_neox_tables(int pos0, int num_tokens, float rope_theta, int rotary_dim, float* cos_out, float* sin_out);
int qlm_silu(float* x, int64_t n, void* stream);
int qlm_conv1d_update_tapmajor(const float* input, float* state, int oldest_tap, const float* weight_t,
                               float* output, int conv_dim, int kernel_size, void* stream);
int qlm_l2norm_heads(float* x, int heads, int head_dim, float eps, void* stream);
int qlm_gdn_gates(const float* a_raw, const float* b_raw, const float* A_log, const float* dt_bias, float* decay,
                  float* beta, int heads, void* stream);
int qlm_gdn_recurrence(float* state, const float* q, const float* k, const float* v, const float* decay,
                       const float* beta, float* out, int heads, int head_dim, void* stream);
int qlm_rms_norm_gain(const float* x, const float* w, float* y, int rows, int size, float eps, void* stream);
int qlm_gqa_attend(const float* q, int q_stride, const float* k_cache, const float* v_cache, float* out, int pos,
                   int heads, int kv_heads, int head_dim, float* scratch, void* stream);

/* ---- A device-resident decode step for a whole model ----------------------
 * QuickLM's Qwen3.5 hybrid decoder (gated-delta-net and gated GQA layers)
 * run with every activation in HBM: DecoderModel::forward + sample(logits, 0,
 * 0) (src/model/model.cpp:151-199, 259-272; layers src/model/modules.hpp:
 * 210-241, src/model/attention.cpp:138-235, 414-591), where the reference keeps
 * activations on the host and calls math::matmul per projection. Built from
 * this library's kernels: matmuls bit-exact int8 (weights quantized on the
 * device at load as get_tensor_keep_int8 does), norms, RoPE, conv and delta
 * rule bit-identical given their inputs; the libm exp/log1p of SiLU, the
 * gates and softmax evaluated in double and rounded once (within a few ulp of
 * the host's), so logits agree to a few ulp, not bit for bit.
 *   qlm_model_load:   read a checkpoint directory as DecoderModel::load does
 *                     (config.json + *.safetensors, F32/BF16; src/model/
 *                     model.cpp:34-131, src/arch/qwen3_5.cpp) onto `device`,
 *                     with KV caches for max_seq positions.
 *   qlm_model_reset:  clear the KV caches and the recurrent/conv states
 *                     (DecoderModel::reset_states).
 *   qlm_model_decode: one step at position pos for input token `token`:
 *                     *next_token = the greedy choice over the logits; logits
 *                     (optional HOST pointer, vocab floats) receives them.
 *                     Prefill = one call per prompt token, pos 0, 1, ...
 *                     (the reference's chunked prefill computes the same).
 *   qlm_model_info:   vocab (lm_head rows), hidden size, layers, max_seq,
 *                     batch (any output pointer may be NULL).
 * Batched decode (no counterpart in the reference, which decodes one sequence
 * per DecoderModel): qlm_model_load_batch keeps `batch` independent sequences
 * (own KV caches, conv and recurrent states) that advance in lockstep, one
 * position for all; qlm_model_decode_batch takes their `batch` input tokens
 * (host array) and returns their greedy choices, logits [batch][vocab]
 * optional. Every op is row- or head-independent, so each sequence's logits
 * are bit-identical to decoding it alone. qlm_model_load / qlm_model_decode
 * are the batch = 1 forms.
 * Execution: the first step runs eagerly; the next one captures the step into
 * a CUDA graph (the position and conv ring position travel in device memory
 * with the tokens) that every later step replays, with the same results.
 * QLM_MODEL_GRAPH=0 in the environment at load keeps every step eager.
 * max_seq * 4 bytes must fit the attention kernels' 200 KB of shared memory
 * (max_seq <= 51200) when the model has attention layers. */
typedef struct qlm_model qlm_model;
int qlm_model_load(const char* dir, int device, int max_seq, qlm_model** out);
int qlm_model_load_batch(const char* dir, int device, int max_seq, int batch, qlm_model** out);
int qlm_model_reset(qlm_model* m);
int qlm_model_decode(qlm_model* m, int token, int pos, int* next_token, float* logits);
int qlm_model_decode_batch(qlm_model* m, const int* tokens, int pos, int* next_tokens, float* logits);
int qlm_model_info(const qlm_model* m, int* vocab, int* hidden, int* layers, int* max_seq, int* batch);
/* The cudaStream_t every step of the model runs on (for timing with events). */
void* qlm_model_stream(const qlm_model* m);
void qlm_model_free(qlm_model* m);

/* Release a handle and its device memory (NULL is a no-op). */
void qlm_weight_free(qlm_w8* w);

/* y[m, 0:rows] = x[m, 0:k] . W^T, for m in [0, M). Replaces the int8 branch of
 * math::matmul(A, B, C, transpose_B=true) (src/ops/math_ops.cpp:820-900):
 *   x:    [M, k] fp32, row stride ldx (>= k)
 *   y:    [M, rows] fp32, row stride ldy (>= rows); overwritten, not accumulated
 *   flags QLM_LINEAR_*; device pointers unless QLM_LINEAR_HOST_IO.
 * Both paths accept any M >= 1 and any k (the exact path up to k = 51200).
 * QLM_LINEAR_TENSOR is never substituted silently: the caller chooses it.
 * An int4 handle (qlm_weight_quantize_upload_q4 / import_int4) runs the exact
 * int4 product (the int4 branch of math::matmul, math_ops.cpp:837-854);
 * QLM_LINEAR_TENSOR on an int4 handle returns QLM_ERR_UNSUPPORTED.
 * Asynchronous on `stream` unless HOST_IO/SYNC. */
int qlm_linear_int8(const float* x, int M, int k, int64_t ldx, const qlm_w8* w, float* y, int64_t ldy, int flags,
                    void* stream);

/* y_g[m, 0:rows_g] = x[m, 0:k] . W_g^T for nw (1..8) weights that share the
 * activations (q/k/v, gate/up, GDN qkv/z/b/a): one exact launch per group of
 * up to 8 activation rows streams all the weights, instead of one launch per
 * weight; every output is bit-identical to qlm_linear_int8's exact path. The
 * int8 counterpart of math::matmul_batched (src/ops/math_ops.cpp:902-954),
 * which QuickLM runs for bf16 weights only. ws: handles on one device with the
 * same k and the same code width (all int8 or all int4); ys / ldys: device
 * outputs [M, rows_g] with row strides >= rows_g.
 * flags: 0 or QLM_LINEAR_SYNC (device pointers). */
int qlm_linear_int8_grouped(const float* x, int M, int k, int64_t ldx, const qlm_w8* const* ws, int nw,
                            float* const* ys, const int64_t* ldys, int flags, void* stream);

/* The tensor-core GEMM of qlm_linear_int8(QLM_LINEAR_TENSOR), for callers that
 * must not allocate device memory once running: an engine that hands all of
 * device memory to its own pool at start-up, or a decode loop that cannot
 * afford cudaMalloc's device-wide synchronisation. No counterpart in the
 * reference. It allocates nothing: its scratch (fp16 activations, row
 * exponents, a status word) lives in 8 MiB of static device memory that every
 * GPU loading this library holds until exit.
 *   x, y:  DEVICE pointers, shapes as qlm_linear_int8.
 *   Limit: M <= 16384 and M * round_up(k, 128) * 2 bytes <= 8 MiB - 64 KiB - 256;
 *          larger requests return QLM_ERR_INVALID_ARG.
 *   flags: 0, or QLM_LINEAR_SYNC to wait and report device-side timeouts.
 *   int4 handles return QLM_ERR_UNSUPPORTED (the tensor-core path is int8).
 * Every call looks up the array's device address (cudaGetSymbolAddress) with
 * the weight's device current. The first call on a device loads the library's
 * device code there, which is when the array itself is allocated: make one
 * call at start-up, before any stream capture. All calls on a device share
 * the array and keep the last call's contents, so calls that may overlap on
 * the GPU (unordered streams) race; order them. Device-side timeouts set a
 * sticky status word in the array; qlm_device_status(device, reset) reports
 * (and with reset != 0 clears) it, as does this call with QLM_LINEAR_SYNC. */
int qlm_linear_int8_tc_noalloc(const float* x, int M, int k, int64_t ldx, const qlm_w8* w, float* y, int64_t ldy,
                               int flags, void* stream);

/* ---- Row-sharded weights across the GPUs of one box (NVLink) ----------------
 * No counterpart in the reference (QuickLM is single-process); the sharded
 * product keeps the reference's bits, since each output element is still
 * computed by exactly one thread with the reference's sequence
 * (src/ops/math_ops.cpp:874-894), on the GPU that owns its row. */
typedef struct qlm_comm qlm_comm;

/* Bytes of one rank's exchange handle (a CUDA IPC handle). */
int qlm_comm_handle_bytes(void);

/* This rank's exchange buffer on `device` for gathered outputs of up to
 * max_out floats; writes its handle (qlm_comm_handle_bytes() bytes) to
 * handle_out. The caller exchanges the handles between ranks (any transport)
 * and passes all of them, in rank order, to qlm_comm_connect. */
int qlm_comm_create(int device, int rank, int nranks, int64_t max_out, qlm_comm** out, void* handle_out);
int qlm_comm_connect(qlm_comm* c, const void* all_handles);
void qlm_comm_free(qlm_comm* c);

/* Failure detection for the row-sharded calls below (no counterpart in the
 * reference, which is single-process). Every wait of this rank's kernels for a
 * peer's data is bounded: after `us` microseconds (default 2 s) the kernel gives
 * up, records a status code and returns. From then on the communicator is
 * failed: its kernels do nothing and every call on it returns
 * QLM_ERR_TIMEOUT; free it and create a new one on every rank (new exchange
 * buffers and epochs) to go on.
 *   qlm_comm_set_timeout_us: the wait limit for later calls (1 us .. 600 s).
 *   qlm_comm_status:         QLM_OK, or QLM_ERR_TIMEOUT if a wait of this
 *                            rank's calls gave up (reads the device status;
 *                            synchronous). SYNC calls check it themselves. */
int qlm_comm_set_timeout_us(qlm_comm* c, int64_t us);
int qlm_comm_status(qlm_comm* c);

/* y[0, 0:n_total] = x[0, 0:k] . W^T for a row-sharded W: this rank's shard w
 * (rows [row_begin, row_end) of n_total) is computed and stored into every
 * rank's exchange buffer over NVLink by the GEMV kernel itself; a second,
 * small kernel then waits (bounded) for the other ranks' rows and copies the
 * gathered row into y (device pointer, n_total floats), while the next kernel
 * in the stream already starts its weight copies. M must be 1 (decode). All
 * ranks must make the same sequence of calls. */
int qlm_linear_int8_allgather(const float* x, int M, int k, int64_t ldx, const qlm_w8* w, qlm_comm* c, float* y,
                              int64_t ldy, int flags, void* stream);

/* Greedy token choice over device logits, as DecoderModel::sample(logits, 0, 0)
 * (src/model/model.cpp:259-272): 0 if logit 0 is NaN, else the lowest index of
 * the largest non-NaN logit. logits: this rank's n logits (device pointer),
 * the first of which is global logit col0 (0 without sharding). c: NULL on one
 * GPU (the current device); or the communicator of a row-sharded lm_head, in
 * which case every rank passes its own shard and all receive the choice over
 * all shards (one 8-byte word per rank crosses NVLink instead of the logits;
 * all ranks must make the same sequence of calls on c). out_index / out_value:
 * device pointers (-1 / NaN when no logit is a number). Global indices must be
 * below 2^24 - 2. flags: 0 or QLM_LINEAR_SYNC. */
int qlm_argmax_f32(const float* logits, int n, int64_t col0, qlm_comm* c, int* out_index, float* out_value, int flags,
                   void* stream);

/* Status of bounded device-side waits on `device`: QLM_OK, or QLM_ERR_TIMEOUT
 * if a kernel gave up waiting since the last reset (reset != 0 clears it).
 * Covers every entry point, qlm_linear_int8_tc_noalloc's status word included.
 * Synchronous calls check this themselves. */
int qlm_device_status(int device, int reset);

/* Block until all work queued on `stream` is done (reports async errors). */
int qlm_stream_sync(void* stream);

/* ---- Per-matmul timing (replaces QUICKLM_PROF's matmul accumulator) -------
 * Replaces math::get_matmul_ms / reset_matmul_ms (src/ops/math_ops.hpp:85-87;
 * accumulation at src/ops/math_ops.cpp:151-159, 821-823, 896-899; the total is
 * printed by src/main.cpp:706-709). On when QUICKLM_PROF or QLM_PROF is set in
 * the environment, or after qlm_prof_enable(1). While on, qlm_linear_int8,
 * qlm_linear_int8_grouped and qlm_linear_int8_allgather record two CUDA events
 * on their stream around their work (host copies included for
 * QLM_LINEAR_HOST_IO), so the figure is device time and adds no
 * synchronisation; calls issued while their stream is being captured into a
 * CUDA graph are not timed (qlm_model_decode[_batch] therefore runs its step
 * eagerly while timing is on). qlm_linear_int8_tc_noalloc is never timed (event
 * pools allocate). Every linear entry point, qlm_model_decode and
 * qlm_model_decode_batch also open an NVTX range named after the entry point,
 * whether or not timing is on.
 *
 * qlm_prof_enable: on = 1 / 0 switches timing on / off, -1 only asks; returns
 * the state before the call (1 on, 0 off). */
int qlm_prof_enable(int on);

/* Cumulative device milliseconds and number of timed calls since the last
 * reset (waits for the calls still in flight). Either pointer may be NULL. */
int qlm_prof_matmul_ms(double* ms, int64_t* calls);

/* Zero the totals (waits for calls still in flight). */
int qlm_prof_reset(void);

/* Per-(entry point, M, N, K) totals as text, one line each, largest total
 * first: "<entry>\t<M>\t<N>\t<K>\t<calls>\t<ms>\n". Writes at most cap bytes
 * (always NUL-terminated when cap > 0) and sets *needed to the full size
 * including the NUL. */
int qlm_prof_report(char* buf, int64_t cap, int64_t* needed);

#ifdef __cplusplus
}
#endif

#endif /* QLM_B200_H */
