/*
 * gdsq — C ABI of the B200 (sm_100a) fused dequantize + GEMV library.
 *
 * Plain pointers and sizes only: no torch, no CUDA types.  Every pointer
 * argument is a device pointer unless stated otherwise; `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream).  Every entry
 * point is asynchronous with respect to the host, returns GDSQ_OK or an error
 * code, and never aborts the process.  The text of the last error on the
 * calling thread is available from gdsq_last_error().
 *
 * Weight layouts are the reference's packed layouts, unchanged:
 *   GGUF Q4_0  [N][K/32] blocks of 18 B: fp16 d, 16 bytes of nibbles;
 *              w[j] = d*((qs[j] & 15) - 8), w[j+16] = d*((qs[j] >> 4) - 8)
 *              (gdsllm/runtime/gguf_dequant.cu:96-107)
 *   GGUF Q8_0  [N][K/32] blocks of 34 B: fp16 d, 32 int8; w[i] = d*qs[i]
 *              (gdsllm/runtime/gguf_dequant.cu:52-57)
 *   affine Q4  weight uint32 [N][K/8] (8 nibbles, LSB first), fp16 scales and
 *              biases [N][K/group]; w = fma(nibble, scale, bias)
 *              (gdsllm/runtime/affine_q4_dequant.cu:54-56, .h:3-12)
 *
 * Activations x are fp16 [batch][K] (row-major, contiguous), outputs y are
 * fp16 [batch][N].  batch = 1 reproduces the reference's batch-1 ops; the
 * reference has no batch > 1 form.
 */
#ifndef GDSQ_H
#define GDSQ_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GDSQ_API __attribute__((visibility("default")))
#else
#define GDSQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum gdsq_status {
  GDSQ_OK = 0,
  GDSQ_ERR_INVALID_VALUE = 1, /* null pointer, bad shape or size */
  GDSQ_ERR_MISALIGNED = 2,    /* pointer alignment the format needs is missing */
  GDSQ_ERR_UNSUPPORTED = 3,   /* valid input this build has no kernel for */
  GDSQ_ERR_CUDA = 4,          /* a CUDA runtime call failed (see gdsq_last_error) */
};

#define GDSQ_MAX_BATCH 16

/* Library version, major*10000 + minor*100 + patch. */
GDSQ_API int gdsq_version(void);

/* Static description of a status code. */
GDSQ_API const char* gdsq_status_string(int status);

/* Detail of the last failing call on this host thread ("" if none). */
GDSQ_API const char* gdsq_last_error(void);

/* Reads the device-side error word of `device` (bit 1: a bounded wait on an
 * async copy gave up; bit 2: a kernel rejected its arguments; bit 4: an index
 * read from device memory, a MoE expert id, was out of range).  Synchronises
 * the device.  clear != 0 resets the word afterwards. */
GDSQ_API int gdsq_device_error(int device, int clear, int* out_bits);

/* Programmatic dependent launch for the GEMV kernels (default off).  When on,
 * a GEMV launched right after another kernel may start streaming its WEIGHTS
 * before that kernel finishes; activations and outputs are only touched
 * after it completes.  Turn it on only when no earlier kernel in the stream
 * writes weight memory. */
GDSQ_API int gdsq_set_pdl(int enable);

/* Upper bound, in nanoseconds, of every device-side wait for another GPU
 * (gdsq_allreduce_sum_f16, gdsq_allreduce_sum_words and the finishers of
 * gdsq_fused_gemv_allreduce) in launches made after the call; 0 restores
 * the default of 1 s.  A wait that runs out sets device error bit 1 and the
 * call returns without writing its output.  Returns the previous bound.  No
 * reference counterpart (the reference runs one GPU). */
GDSQ_API unsigned long long gdsq_set_peer_wait_limit_ns(unsigned long long ns);

/* ---- Dequantization to fp16 ------------------------------------------- */

/* Replaces launch_dequant_q4_0 (gdsllm/runtime/gguf_dequant.h:26-27).
 * src: num_blocks * 18 bytes (2-byte aligned); dst: num_blocks * 32 fp16. */
GDSQ_API int gdsq_dequant_q4_0(const void* src, void* dst, uint64_t num_blocks, void* stream);

/* Replaces launch_dequant_q8_0 (gdsllm/runtime/gguf_dequant.h:19-20).
 * src: num_blocks * 34 bytes (2-byte aligned); dst: num_blocks * 32 fp16. */
GDSQ_API int gdsq_dequant_q8_0(const void* src, void* dst, uint64_t num_blocks, void* stream);

/* dst[t][:] = the fp16 dequantization of row ids[t] of a GGUF Q4_0 / Q8_0
 * table [rows][cols] (gguf_type GDSQ_TYPE_Q4_0 / GDSQ_TYPE_Q8_0), the same
 * bits as dequantizing the whole table and gathering the rows.  Replaces the
 * embedding lookup of the reference's callers, which dequantize the full
 * table per call (gdsllm/runtime/scheduler.py:22-45, no single launcher).
 * ids: num_ids int64 on the device (8-byte aligned); dst: num_ids * cols fp16.
 * An id outside 0..rows-1 gives a zero row and sets device error bit 4. */
GDSQ_API int gdsq_dequant_rows_gguf(int gguf_type, const void* table, long long rows, int cols,
                                    const long long* ids, long long num_ids, void* dst, void* stream);

/* Replaces launch_dequant_affine_q4 (gdsllm/runtime/affine_q4_dequant.h:29-32).
 * weight: num_elements/8 uint32 (4-byte aligned); scales, biases:
 * num_elements/group_size fp16; dst: num_elements fp16.  in_dim must be a
 * multiple of group_size and group_size a multiple of 8. */
GDSQ_API int gdsq_dequant_affine_q4(const void* weight, const void* scales, const void* biases, void* dst,
                           uint64_t num_elements, int in_dim, int group_size, void* stream);

/* ---- Fused dequantize + matrix-vector product ------------------------- */

/* Replaces launch_fused_q4_0_gemv (gdsllm/runtime/fused_gemv.h:23-25).
 * y[b][n] = fp16( sum_k W[n][k] * x[b][k] ) for b < batch (1..16).
 * in_dim % 32 == 0; weight 2-byte aligned (16-byte aligned with
 * in_dim % 256 == 0 takes the bulk-copy fast path). */
GDSQ_API int gdsq_fused_q4_0_gemv(const void* weight, const void* x, void* y, int out_dim, int in_dim,
                         int batch, void* stream);

/* Replaces launch_fused_q8_0_gemv (gdsllm/runtime/fused_gemv.h:29-31). */
GDSQ_API int gdsq_fused_q8_0_gemv(const void* weight, const void* x, void* y, int out_dim, int in_dim,
                         int batch, void* stream);

/* Replaces launch_fused_affine_q4_gemv (gdsllm/runtime/affine_q4_dequant.h:41-44).
 * weight [out_dim][in_dim/8] uint32, scales/biases [out_dim][in_dim/group_size]. */
GDSQ_API int gdsq_fused_affine_q4_gemv(const void* weight, const void* scales, const void* biases,
                              const void* x, void* y, int out_dim, int in_dim, int group_size,
                              int batch, void* stream);

/* Several GGUF matrices that read the same x (LLaMA's q, k, v; gate, up) in
 * one launch: ys[m][b][n] = fp16( sum_k W_m[n][k] * x[b][k] ).  Host arrays
 * `weights`, `out_dims`, `ys` of `count` (1..4) entries; gguf_type
 * GDSQ_TYPE_Q4_0 or GDSQ_TYPE_Q8_0.  No single reference launcher: the
 * reference calls launch_fused_*_gemv once per matrix (llama.py:122-141).
 * Shapes the fast path cannot take (in_dim % 256, alignment, batch > 4) run
 * as one launch per matrix with the same results. */
#define GDSQ_TYPE_Q4_0 0
#define GDSQ_TYPE_Q8_0 1
GDSQ_API int gdsq_fused_gemv_group(int gguf_type, int count, const void* const* weights, const int* out_dims,
                                   void* const* ys, const void* x, int in_dim, int batch, void* stream);

/* ---- Mixture-of-experts gather (affine-Q4 experts, decode) ------------- */

/* No single reference launcher: these two calls replace the decode loop of
 * moe_mlp_selective (gdsllm/runtime/qwen_moe.py:453-474), which per top-k slot
 * reads the expert id to the host and calls launch_fused_affine_q4_gemv
 * (affine_q4_dequant.h:41-44) three times with torch SiLU / mul / add between.
 *
 * Experts are stacked: *_weight [expert_count][rows][cols/8] uint32,
 * *_scales / *_biases [expert_count][rows][cols/group_size] fp16, holding the
 * experts expert_first .. expert_first+expert_count-1 of expert_total.
 * expert_ids [num_tokens][top_k] int32 in device memory; slots whose expert is
 * not resident are skipped (expert parallelism), ids outside 0..expert_total-1
 * set device error bit 4 and are skipped.  top_k <= 64. */

/* h[t][k][i] = fp16(silu(fp16(gate_e x_t)[i]) * fp16(up_e x_t)[i]), e = ids[t][k].
 * gate/up rows = inter_dim, cols = hidden_dim; x [num_tokens][hidden_dim] fp16;
 * h [num_tokens][S][inter_dim] fp16 with S = top_k, or top_k + 1 when the
 * shared expert is given (its six shared_* pointers: [1][rows][cols/8] words,
 * [1][rows][cols/group_size] scales and biases; all six null = none); slot
 * top_k is then the shared expert (qwen_moe.py:497-503).  Entries of
 * non-resident slots are left unwritten. */
GDSQ_API int gdsq_moe_affine_q4_gate_up(const void* gate_weight, const void* gate_scales,
                                        const void* gate_biases, const void* up_weight,
                                        const void* up_scales, const void* up_biases,
                                        const void* shared_gate_weight, const void* shared_gate_scales,
                                        const void* shared_gate_biases, const void* shared_up_weight,
                                        const void* shared_up_scales, const void* shared_up_biases,
                                        const void* x, const int32_t* expert_ids, void* h, int num_tokens,
                                        int top_k, int inter_dim, int hidden_dim, int group_size,
                                        int expert_first, int expert_count, int expert_total, void* stream);

#define GDSQ_MOE_OUT_F32 1    /* y is fp32 instead of fp16 */
#define GDSQ_MOE_ACCUMULATE 2 /* y += result instead of y = result */
#define GDSQ_MOE_CLAMP 4      /* clamp to +-65504 before storing (qwen_moe.py:514) */

/* y[t][j] = sum over resident slots k of route_weights[t][k] * (down_e h[t][k])[j]
 * (+ shared_weights[t] * (shared_down h[t][top_k])[j] when the shared expert's
 * three shared_down_* pointers and shared_weights [num_tokens] fp16 are
 * given), summed in fp32.  down rows = hidden_dim, cols = inter_dim;
 * route_weights [num_tokens][top_k] fp16; y [num_tokens][hidden_dim].  h must
 * have been produced with the same shared-expert choice. */
GDSQ_API int gdsq_moe_affine_q4_down(const void* down_weight, const void* down_scales,
                                     const void* down_biases, const void* shared_down_weight,
                                     const void* shared_down_scales, const void* shared_down_biases,
                                     const void* h, const int32_t* expert_ids, const void* route_weights,
                                     const void* shared_weights, void* y, int num_tokens, int top_k,
                                     int hidden_dim, int inter_dim, int group_size, int expert_first,
                                     int expert_count, int expert_total, int flags, void* stream);

/* gdsq_moe_affine_q4_down with fp16 y = residual + fp16(result), added in
 * fp16 (the caller's `x + moe(x)` residual add in the same two roundings;
 * residual fp16 [num_tokens][hidden_dim], may be y itself).  flags may not
 * hold GDSQ_MOE_OUT_F32 or GDSQ_MOE_ACCUMULATE. */
GDSQ_API int gdsq_moe_affine_q4_down_residual(const void* down_weight, const void* down_scales,
                                              const void* down_biases, const void* shared_down_weight,
                                              const void* shared_down_scales, const void* shared_down_biases,
                                              const void* h, const int32_t* expert_ids, const void* route_weights,
                                              const void* shared_weights, void* y, int num_tokens, int top_k,
                                              int hidden_dim, int inter_dim, int group_size, int expert_first,
                                              int expert_count, int expert_total, int flags, const void* residual,
                                              void* stream);

/* gdsq_moe_affine_q4_gate_up then gdsq_moe_affine_q4_down (same arguments,
 * same results) with the intermediate h kept in a fixed 4 MiB array of the
 * library's static device memory instead of a caller buffer, so the call
 * allocates nothing.  No reference counterpart.  Limits: num_tokens *
 * (top_k + 1 if the shared expert is given, else top_k) * inter_dim <=
 * 2097152 fp16 elements, otherwise GDSQ_ERR_INVALID_VALUE before any CUDA
 * call.  The array is shared by every call on a device: calls on different
 * streams (or host threads) at the same time overwrite each other's h, so
 * serialise them or use the two-call form with your own buffer.  The first
 * call on a device looks up the array's address (cudaGetSymbolAddress) and
 * must happen before any stream capture that records a later call; a first
 * call on a capturing stream returns GDSQ_ERR_INVALID_VALUE.  The shared
 * expert's nine tensors and shared_weights are all given or all null
 * (GDSQ_ERR_INVALID_VALUE otherwise, before any CUDA call). */
GDSQ_API int gdsq_moe_affine_q4_noalloc(const void* gate_weight, const void* gate_scales, const void* gate_biases,
                                        const void* up_weight, const void* up_scales, const void* up_biases,
                                        const void* down_weight, const void* down_scales, const void* down_biases,
                                        const void* shared_gate_weight, const void* shared_gate_scales,
                                        const void* shared_gate_biases, const void* shared_up_weight,
                                        const void* shared_up_scales, const void* shared_up_biases,
                                        const void* shared_down_weight, const void* shared_down_scales,
                                        const void* shared_down_biases, const void* x, const int32_t* expert_ids,
                                        const void* route_weights, const void* shared_weights, void* y,
                                        int num_tokens, int top_k, int hidden_dim, int inter_dim, int group_size,
                                        int expert_first, int expert_count, int expert_total, int flags,
                                        void* stream);

/* ---- Tensor-parallel exchange ----------------------------------------- */

/* out[i] = sum over ranks r (in rank order, fp32) of in_r[i], fp16, over
 * NVLink peer memory: a one-shot all-reduce for the row-split projections'
 * partial outputs (no reference counterpart: the reference runs one GPU).
 * bufs / flags: host arrays of `world` device pointers, entry r = rank r's
 * data buffer (2 * cap fp16, 16-byte aligned) and flag array (32 * 8 int32,
 * zero-initialised), mapped into this process (CUDA IPC); entry `rank` is
 * this rank's own.  Every rank must make the same sequence of calls.  n %
 * 8 == 0, n <= cap, n <= 32768.  A peer that does not arrive within 1 s sets
 * device error bit 1 and the call returns without a result. */
GDSQ_API int gdsq_allreduce_sum_f16(const void* in, void* out, int n, const void* const* bufs, void* const* flags,
                                    int cap, int rank, int world, void* stream);

#define GDSQ_ELEM_F16 0
#define GDSQ_ELEM_F32 1
#define GDSQ_ELEM_F32_TO_F16 2 /* fp32 in; out fp16 of the sum clamped to +-65504 (qwen_moe.py:514) */

/* out[i] = sum over ranks r (in rank order, fp32) of in_r[i], fp16 or fp32
 * (elem_type GDSQ_ELEM_F16 / GDSQ_ELEM_F32; GDSQ_ELEM_F32_TO_F16 adds fp32
 * and writes the clamped fp16 result), over NVLink peer memory: every
 * rank stores each element with the call's epoch as one 64-bit word into
 * every rank's buffer and waits only on its own buffer (no flags).  The
 * expert-parallel exchange of the MoE partial sums (no reference
 * counterpart: the reference runs one GPU).  bufs: host array of `world`
 * device pointers, entry r = rank r's buffer (2 * world * cap 64-bit words,
 * 8-byte aligned, zero-initialised) mapped into this process (CUDA IPC);
 * epochs: this rank's own 32 int32 (zero-initialised, not shared).  n <= cap,
 * n <= 32768.  Every rank must make the same sequence of calls.  A peer that
 * does not arrive within 1 s sets device error bit 1 and the call leaves its
 * output unwritten. */
GDSQ_API int gdsq_allreduce_sum_words(int elem_type, const void* in, void* out, int n, const void* const* bufs,
                                      void* epochs, int cap, int rank, int world, void* stream);

/* The same with elem_type GDSQ_ELEM_F32_TO_F16 and out = residual + the
 * clamped fp16 sum, added in fp16 (the caller's `x + moe(x)` of the
 * expert-parallel layer in the same roundings); residual fp16 [n], may be
 * out itself. */
GDSQ_API int gdsq_allreduce_sum_words_residual(int elem_type, const void* in, void* out, int n,
                                               const void* const* bufs, void* epochs, int cap, int rank, int world,
                                               const void* residual, void* stream);

/* A row-split (K-sharded) Q4_0 / Q8_0 GEMV whose output rows are summed over
 * the tensor-parallel ranks inside the kernel: y = sum over ranks r of
 * W_r . x_r, fp32 sums added in rank order (identical on every rank), fp16
 * out.  Batch 1.  bufs / flags: host arrays of `world` device pointers, entry
 * r = rank r's exchange buffer (2 * world * rows_cap 64-bit words, 8-byte
 * aligned, zero-initialised: every rank stores its partial rows, each with
 * the call's epoch, into every rank's buffer) and flags (64 int32,
 * zero-initialised), mapped into this process (CUDA IPC).  rows_cap >=
 * out_dim rounded up to 32, out_dim <= 32768.  Every rank must make the same
 * sequence of calls with the same shapes.  No reference counterpart. */
GDSQ_API int gdsq_fused_gemv_allreduce(int gguf_type, const void* weight, const void* x, void* y, int out_dim,
                                       int in_dim, const void* const* bufs, void* const* flags, int rows_cap, int rank,
                                       int world, void* stream);

/* The routing tail of moe_route (qwen_moe.py:407-413) on router logits fp16
 * [num_tokens][num_experts] (the output of F.linear(x, W_router)): expert_ids
 * int32 [num_tokens][top_k] of the top_k largest logits, largest first (equal
 * logits: lower expert index first), route_weights fp16 = softmax of those
 * logits in fp32.  With shared_gate fp16 [hidden_dim] (and x fp16
 * [num_tokens][hidden_dim], 16-byte aligned) also shared_weights fp16
 * [num_tokens] = sigmoid(fp16(x . shared_gate)) (qwen_moe.py:505-509).
 * num_experts <= 4096, top_k <= 64. */
GDSQ_API int gdsq_moe_route(const void* logits, int num_tokens, int num_experts, int top_k, const void* x,
                            const void* shared_gate, int hidden_dim, int32_t* expert_ids, void* route_weights,
                            void* shared_weights, void* stream);

/* The router's F.linear and gdsq_moe_route in one launch (qwen_moe.py:
 * 386-416, 505-509): logits [num_tokens][num_experts + 1] fp16 = x .
 * router_weight^T (fp32 sums of the fp16 products, rounded once; column
 * num_experts holds x . shared_gate when shared_gate is given), then the
 * top_k ids, softmax weights and the shared gate's sigmoid as
 * gdsq_moe_route writes them.  The CTAs count themselves done on `counter`
 * (one zero-initialised uint32 per call sequence on a stream; the last CTA
 * routes and sets it back to 0).  num_tokens <= 16, num_experts <= 512,
 * top_k <= 32, hidden_dim % 512 == 0; x, router_weight [num_experts]
 * [hidden_dim] and shared_gate [hidden_dim] fp16, 16-byte aligned. */
GDSQ_API int gdsq_moe_router(const void* x, int num_tokens, int hidden_dim, const void* router_weight,
                             int num_experts, const void* shared_gate, int top_k, void* logits,
                             int32_t* expert_ids, void* route_weights, void* shared_weights, unsigned int* counter,
                             void* stream);

/* ---- Decode step (batch 1, position in device memory) --------------------
 * The work of one LLaMA decode position around the fused GEMVs, so that a
 * whole token can be captured as one CUDA graph.  No reference launcher:
 * these replace the torch code of llama.py's transformer_block at decode,
 * in the same arithmetic order.  pos points to one int64 on the device;
 * a position outside [0, max_seq) sets device error bit 4 and nothing is
 * written. */

/* h_out = h_in + delta (fp16 add; skipped when delta is NULL), then
 * x_out = fp16(fp16(h * rsqrt(mean(h^2) + eps)) * weight) per row of
 * `hidden` elements (llama.py:17-23, 285-293).  hidden % 8 == 0, <= 16384;
 * 16-byte aligned pointers; h_out may equal h_in. */
GDSQ_API int gdsq_add_rmsnorm_f16(const void* h_in, const void* delta, void* h_out, const void* weight, void* x_out,
                                  int rows, int hidden, float eps, void* stream);

/* RoPE (llama.py:83-105) of q [num_heads][head_dim] into q_out and of k
 * [num_kv_heads][head_dim] into k_cache at *pos, v copied into v_cache at
 * *pos (KVCache.update, kv_cache.py:44-67).  freqs: float pairs
 * [max_seq][head_dim/2] (view_as_real of precompute_freqs_cis); caches of
 * one layer [num_kv_heads][max_seq][head_dim] fp16. */
GDSQ_API int gdsq_rope_kv_f16(const void* q, const void* k, const void* v, void* q_out, const void* freqs,
                              const long long* pos, void* k_cache, void* v_cache, int num_heads, int num_kv_heads,
                              int head_dim, int max_seq, void* stream);

/* out [num_heads][head_dim] = softmax(fp16(fp16(q.K^T) * scale)) V over the
 * positions [0, *pos] of the layer's caches (llama.py:228-242), query head h
 * reading KV head h / (num_heads / num_kv_heads).  scale is the fp32
 * reciprocal torch uses for `scores / sqrt(head_dim)`:
 * 1.0f / (float)sqrt(head_dim).  head_dim 64 or 128. */
GDSQ_API int gdsq_attention_decode_f16(const void* q, const void* k_cache, const void* v_cache, const long long* pos,
                                       void* out, int num_heads, int num_kv_heads, int head_dim, int max_seq,
                                       float scale, void* stream);

/* The same attention with the RoPE and cache write of gdsq_rope_kv_f16
 * folded in: q [num_heads][head_dim], k and v [num_kv_heads][head_dim] are
 * the projections before RoPE; k (rotated) and v are written into the
 * caches at *pos and attended to in the same launch. */
GDSQ_API int gdsq_attention_decode_rope_f16(const void* q, const void* k, const void* v, const void* freqs,
                                            const long long* pos, void* k_cache, void* v_cache, void* out,
                                            int num_heads, int num_kv_heads, int head_dim, int max_seq, float scale,
                                            void* stream);

/* out = fp16(silu(gate)) * up, n elements (llama.py:248-252). */
GDSQ_API int gdsq_silu_mul_f16(const void* gate, const void* up, void* out, long long n, void* stream);

/* *token = the first index of the largest of n fp16 logits (torch.argmax);
 * then *pos += 1 when pos is not NULL. */
GDSQ_API int gdsq_argmax_f16(const void* logits, int n, long long* token, long long* pos, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GDSQ_H */
