/*
 * The reference's C++ launcher ABI, served by libgdsq.so.
 *
 * These are the exact declarations of GdsLLM's kernel launchers (C++
 * linkage, same parameter types), so the reference binding
 * gdsllm/runtime/gds_bindings.cpp links against libgdsq.so unchanged in place
 * of fused_gemv.cu, gguf_dequant.cu and affine_q4_dequant.cu.  Each forwards
 * to the C entry point in gdsq.h with batch = 1.  Like the reference, they
 * return nothing; a failure is printed to stderr and left in
 * gdsq_last_error() (the reference printed launch errors only,
 * gdsllm/runtime/fused_gemv.cu:129-134).
 */
#ifndef GDSQ_REFERENCE_ABI_H
#define GDSQ_REFERENCE_ABI_H

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "gdsq.h"

/* gdsllm/runtime/fused_gemv.h:23-25 */
GDSQ_API void launch_fused_q4_0_gemv(const void* weight, const __half* x, __half* y, int out_dim,
                                     int in_dim, cudaStream_t stream);
/* gdsllm/runtime/fused_gemv.h:29-31 */
GDSQ_API void launch_fused_q8_0_gemv(const void* weight, const __half* x, __half* y, int out_dim,
                                     int in_dim, cudaStream_t stream);
/* gdsllm/runtime/gguf_dequant.h:19-20 */
GDSQ_API void launch_dequant_q8_0(const void* src, __half* dst, size_t num_blocks,
                                  cudaStream_t stream = 0);
/* gdsllm/runtime/gguf_dequant.h:26-27 */
GDSQ_API void launch_dequant_q4_0(const void* src, __half* dst, size_t num_blocks,
                                  cudaStream_t stream = 0);
/* gdsllm/runtime/affine_q4_dequant.h:29-32 */
GDSQ_API void launch_dequant_affine_q4(const uint32_t* weight, const __half* scales,
                                       const __half* biases, __half* dst, size_t num_elements,
                                       int in_dim, int group_size, cudaStream_t stream = 0);
/* gdsllm/runtime/affine_q4_dequant.h:41-44 */
GDSQ_API void launch_fused_affine_q4_gemv(const uint32_t* weight, const __half* scales,
                                          const __half* biases, const __half* x, __half* y,
                                          int out_dim, int in_dim, int group_size,
                                          cudaStream_t stream);

#endif /* GDSQ_REFERENCE_ABI_H */
