// Block dequantization to dense fp16: GGUF Q4_0, GGUF Q8_0, affine Q4.
//
// Reference kernels replaced (bit-identical outputs):
//   kernel_dequant_q4_0       gdsllm/runtime/gguf_dequant.cu:76-108
//   kernel_dequant_q8_0       gdsllm/runtime/gguf_dequant.cu:32-58
//   kernel_dequant_affine_q4  gdsllm/runtime/affine_q4_dequant.cu:28-59
//
// These are write-bound streams (Q4_0 reads 18 B and writes 64 B per block).
// One thread produces 8 consecutive fp16 outputs and writes them with one
// 16-byte store, so a warp writes 512 contiguous bytes per instruction.
// Rounding matches the reference exactly:
//   Q4_0 / Q8_0: the fp32 product d*q is exact, then round-to-nearest-even.
//   affine: fmaf(nibble, scale, bias), then RNE to fp16.  nibble*scale is
//   exact in fp32, so this is the reference's `nibble * scale + bias` with or
//   without FMA contraction: one rounding at the add.
#pragma once

#include "common.cuh"

namespace gdsq {

template <bool kVecStore>
__device__ __forceinline__ void store8(__half* dst, const float (&v)[8]) {
  if constexpr (kVecStore) {
    uint4 o;
    o.x = h2_as_u32(__floats2half2_rn(v[0], v[1]));
    o.y = h2_as_u32(__floats2half2_rn(v[2], v[3]));
    o.z = h2_as_u32(__floats2half2_rn(v[4], v[5]));
    o.w = h2_as_u32(__floats2half2_rn(v[6], v[7]));
    *reinterpret_cast<uint4*>(dst) = o;
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) dst[k] = __float2half_rn(v[k]);
  }
}

// Unit u covers outputs [8u, 8u+8) of block u/4; quarter t = u%4 takes
//   t=0: low nibbles of qs[0..7]   (outputs 0..7)
//   t=1: low nibbles of qs[8..15]  (outputs 8..15)
//   t=2: high nibbles of qs[0..7]  (outputs 16..23)
//   t=3: high nibbles of qs[8..15] (outputs 24..31)
template <bool kVecStore>
__global__ void __launch_bounds__(256)
    dequant_q4_0_kernel(const uint8_t* __restrict__ src, __half* __restrict__ dst, uint64_t units) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t u = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += stride) {
    const uint64_t blk = u >> 2;
    const int t = static_cast<int>(u & 3);
    const uint16_t* bp = reinterpret_cast<const uint16_t*>(src + blk * 18);
    const float d = __half2float(__ushort_as_half(__ldg(bp)));
    const uint16_t* qp = bp + 1 + 4 * (t & 1);
    const uint32_t lo = (uint32_t)__ldg(qp) | ((uint32_t)__ldg(qp + 1) << 16);
    const uint32_t hi = (uint32_t)__ldg(qp + 2) | ((uint32_t)__ldg(qp + 3) << 16);
    const int sh = (t >> 1) * 4;
    float v[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[k] = d * float((int)((lo >> (8 * k + sh)) & 15u) - 8);
      v[k + 4] = d * float((int)((hi >> (8 * k + sh)) & 15u) - 8);
    }
    store8<kVecStore>(dst + u * 8, v);
  }
}

// Unit u covers outputs [8u, 8u+8) of block u/4: qs[8t .. 8t+7], t = u%4.
template <bool kVecStore>
__global__ void __launch_bounds__(256)
    dequant_q8_0_kernel(const uint8_t* __restrict__ src, __half* __restrict__ dst, uint64_t units) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t u = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += stride) {
    const uint64_t blk = u >> 2;
    const int t = static_cast<int>(u & 3);
    const uint16_t* bp = reinterpret_cast<const uint16_t*>(src + blk * 34);
    const float d = __half2float(__ushort_as_half(__ldg(bp)));
    const uint16_t* qp = bp + 1 + 4 * t;
    float v[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t two = __ldg(qp + k);
      v[2 * k] = d * float(static_cast<int8_t>(two & 0xFFu));
      v[2 * k + 1] = d * float(static_cast<int8_t>(two >> 8));
    }
    store8<kVecStore>(dst + u * 8, v);
  }
}

// Row gather: out[t][:] = the dequantized row ids[t] of a [rows][cols]
// GGUF table (F: kFmtQ4_0 = 0 or kFmtQ8_0 = 1), the same bits as a full
// dequantization followed by F.embedding, which the reference's callers do
// for the embedding (gdsllm/runtime/scheduler.py:22-45).  Unit u covers 8
// outputs of token u / (4 * blocks_per_row), in the order of the kernels
// above.  An id outside 0..rows-1 sets device error bit 4 and yields zeros.
template <int F, bool kVecStore>
__global__ void __launch_bounds__(256)
    dequant_rows_kernel(const uint8_t* __restrict__ src, const long long* __restrict__ ids, long long rows,
                        int blocks_per_row, __half* __restrict__ dst, uint64_t units) {
  constexpr int kBlockBytes = F == 0 ? 18 : 34;
  pdl_launch_dependents();
  pdl_wait_primary();
  const uint64_t per_token = (uint64_t)blocks_per_row * 4;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t u = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += stride) {
    const uint64_t tok = u / per_token;
    const uint64_t r = u - tok * per_token;
    const long long id = __ldg(ids + tok);
    float v[8];
    if (id < 0 || id >= rows) {
      if (r == 0) record_device_error(kDevErrBadIndex);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = 0.f;
    } else {
      const uint64_t blk = (uint64_t)id * blocks_per_row + (r >> 2);
      const int t = static_cast<int>(r & 3);
      const uint16_t* bp = reinterpret_cast<const uint16_t*>(src + blk * kBlockBytes);
      const float d = __half2float(__ushort_as_half(__ldg(bp)));
      if constexpr (F == 0) {
        const uint16_t* qp = bp + 1 + 4 * (t & 1);
        const uint32_t lo = (uint32_t)__ldg(qp) | ((uint32_t)__ldg(qp + 1) << 16);
        const uint32_t hi = (uint32_t)__ldg(qp + 2) | ((uint32_t)__ldg(qp + 3) << 16);
        const int sh = (t >> 1) * 4;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          v[k] = d * float((int)((lo >> (8 * k + sh)) & 15u) - 8);
          v[k + 4] = d * float((int)((hi >> (8 * k + sh)) & 15u) - 8);
        }
      } else {
        const uint16_t* qp = bp + 1 + 4 * t;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t two = __ldg(qp + k);
          v[2 * k] = d * float(static_cast<int8_t>(two & 0xFFu));
          v[2 * k + 1] = d * float(static_cast<int8_t>(two >> 8));
        }
      }
    }
    store8<kVecStore>(dst + u * 8, v);
  }
}

// Unit u = packed word u (8 nibbles, LSB first) -> outputs [8u, 8u+8).
template <bool kVecStore>
__global__ void __launch_bounds__(256)
    dequant_affine_q4_kernel(const uint32_t* __restrict__ w, const __half* __restrict__ scales,
                             const __half* __restrict__ biases, __half* __restrict__ dst,
                             uint64_t units, int group) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t u = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += stride) {
    const uint64_t g = (u * 8) / (uint64_t)group;
    const float s = __half2float(__ldg(scales + g));
    const float b = __half2float(__ldg(biases + g));
    const uint32_t packed = __ldg(w + u);
    float v[8];
#pragma unroll
    for (int n = 0; n < 8; ++n) v[n] = __fmaf_rn(float((packed >> (4 * n)) & 15u), s, b);
    store8<kVecStore>(dst + u * 8, v);
  }
}

}  // namespace gdsq
