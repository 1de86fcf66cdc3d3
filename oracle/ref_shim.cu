// TEST INFRASTRUCTURE ONLY.  A C-ABI shim over GdsLLM's own CUDA launchers so
// that tests can run the reference kernels, compiled unchanged from the
// reference tree for sm_100a, on the same device buffers as gdsq.
//
// Built by oracle/build.py together with the reference sources
//   gdsllm/runtime/fused_gemv.cu, gguf_dequant.cu, affine_q4_dequant.cu
// into oracle/_ref/libref_kernels.so.  Each wrapper returns the CUDA error
// state after the launch (cudaPeekAtLastError).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "affine_q4_dequant.h"
#include "fused_gemv.h"
#include "gguf_dequant.h"

#define REF_API extern "C" __attribute__((visibility("default")))

REF_API int ref_fused_q4_0_gemv(const void* w, const void* x, void* y, int out_dim, int in_dim,
                                void* stream) {
  launch_fused_q4_0_gemv(w, static_cast<const __half*>(x), static_cast<__half*>(y), out_dim, in_dim,
                         static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaPeekAtLastError());
}

REF_API int ref_fused_q8_0_gemv(const void* w, const void* x, void* y, int out_dim, int in_dim,
                                void* stream) {
  launch_fused_q8_0_gemv(w, static_cast<const __half*>(x), static_cast<__half*>(y), out_dim, in_dim,
                         static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaPeekAtLastError());
}

REF_API int ref_fused_affine_q4_gemv(const void* w, const void* s, const void* b, const void* x,
                                     void* y, int out_dim, int in_dim, int group_size,
                                     void* stream) {
  launch_fused_affine_q4_gemv(static_cast<const uint32_t*>(w), static_cast<const __half*>(s),
                              static_cast<const __half*>(b), static_cast<const __half*>(x),
                              static_cast<__half*>(y), out_dim, in_dim, group_size,
                              static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaPeekAtLastError());
}

REF_API int ref_dequant_q4_0(const void* src, void* dst, uint64_t num_blocks, void* stream) {
  launch_dequant_q4_0(src, static_cast<__half*>(dst), num_blocks, static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaPeekAtLastError());
}

REF_API int ref_dequant_q8_0(const void* src, void* dst, uint64_t num_blocks, void* stream) {
  launch_dequant_q8_0(src, static_cast<__half*>(dst), num_blocks, static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaPeekAtLastError());
}

REF_API int ref_dequant_affine_q4(const void* w, const void* s, const void* b, void* dst,
                                  uint64_t num_elements, int in_dim, int group_size, void* stream) {
  launch_dequant_affine_q4(static_cast<const uint32_t*>(w), static_cast<const __half*>(s),
                           static_cast<const __half*>(b), static_cast<__half*>(dst), num_elements,
                           in_dim, group_size, static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaPeekAtLastError());
}
