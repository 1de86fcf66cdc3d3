// Fused dequantize + GEMV kernels for GGUF Q4_0, GGUF Q8_0 and affine-Q4
// weights, batch 1..16.
//
// Reference kernels replaced (same math, different schedule):
//   kernel_fused_q4_0_gemv       gdsllm/runtime/fused_gemv.cu:27-105
//   kernel_fused_q8_0_gemv       gdsllm/runtime/fused_gemv.cu:142-205
//   kernel_fused_affine_q4_gemv  gdsllm/runtime/affine_q4_dequant.cu:79-158
//
// Fast path (weights 16-byte aligned, K % 256 == 0):
//   * A CTA owns 32 consecutive output rows and 4 warps.  Lane l of every
//     warp works on row (row0 + l); the warps split the row's 256-column
//     "chunks" round-robin.
//   * Each warp streams its chunks through a private ring of shared-memory
//     stages.  A stage holds one chunk of all 32 rows; every lane issues one
//     1-D bulk copy (cp.async.bulk) of its own row's chunk bytes, and lane 0
//     arms the stage's mbarrier with the stage's byte count.  No register or
//     LSU work is spent moving weights.
//   * The activations are copied once per CTA into shared memory, permuted so
//     that the pair order matches the order in which the dequantizer produces
//     weight pairs.  All 32 lanes then read the same activation address, so
//     each 16-byte shared load is a broadcast.
//   * Nibbles become exact fp16 (q - 8) with the magic-number trick; products
//     are summed in fp16 pairs over at most 16 terms per 32-column block and
//     then in fp32 across blocks.  Q8_0 is dequantized straight to fp32 and
//     summed in fp32.
//   * Partial sums of the 4 warps meet in shared memory; one fp16 store per
//     (batch row, output row).
//
// Generic path: any K % 32 == 0 (group_size % 8 == 0 for affine) and 2-byte
// (4-byte for affine words) alignment; one warp per row, plain loads.
#pragma once

#include "common.cuh"

namespace gdsq {

enum WeightFormat : int { kFmtQ4_0 = 0, kFmtQ8_0 = 1, kFmtAffineQ4 = 2 };

constexpr int kGemvWarps = 4;
constexpr int kChunkCols = 256;

template <int F>
struct GemvFormat;

template <>
struct GemvFormat<kFmtQ4_0> {
  static constexpr int kChunkBytes = 144;  // 8 blocks x 18 B
  static constexpr int kSlotStride = 144;  // 36 words = 4 (mod 32): LDS.128 conflict-free
  static constexpr int kStages = 4;
  static constexpr int kXBytes = 2;        // activations kept as permuted fp16
};

template <>
struct GemvFormat<kFmtQ8_0> {
  static constexpr int kChunkBytes = 272;  // 8 blocks x 34 B
  static constexpr int kSlotStride = 272;  // 68 words = 4 (mod 32)
  static constexpr int kStages = 2;
  static constexpr int kXBytes = 4;        // activations kept as fp32
};

template <>
struct GemvFormat<kFmtAffineQ4> {
  static constexpr int kChunkBytes = 128;  // 32 words of 8 nibbles
  static constexpr int kSlotStride = 144;  // padded from 128 B to avoid bank conflicts
  static constexpr int kStages = 4;
  static constexpr int kXBytes = 2;
};

struct GemvParams {
  const uint8_t* w;       // packed weights, row-major
  const __half* scales;   // affine only: [N][K/group]
  const __half* biases;   // affine only
  const __half* x;        // [nb][K]
  __half* y;              // [nb][N]
  int N;
  int K;
  int nb;                 // batch rows actually present (<= template B)
  int group;              // affine group size
  long long row_bytes;    // packed bytes per weight row
};

// Shared-memory carve-up of the fast kernel, identical on host and device.
struct GemvSmemLayout {
  int ring;   // byte offsets from the dynamic smem base
  int xs;
  int xsum;
  int sb;
  int sb_stride;  // words per row of the (scale, bias) table
  int red;
  int total;
};

template <int F>
__host__ __device__ inline GemvSmemLayout gemv_smem_layout(int B, int K, int group) {
  using T = GemvFormat<F>;
  GemvSmemLayout L;
  int off = 128;  // mbarriers: kGemvWarps * kStages * 8 <= 128 bytes
  L.ring = off;
  off += kGemvWarps * T::kStages * 32 * T::kSlotStride;
  L.xs = off;
  off += B * K * T::kXBytes;
  L.xsum = off;
  L.sb = off;
  L.sb_stride = 0;
  if (F == kFmtAffineQ4) {
    const int G = K / group;
    off += B * G * 4;
    L.sb = off;
    L.sb_stride = G | 1;  // odd word stride: conflict-free per-lane reads
    off += 32 * L.sb_stride * 4;
  }
  L.red = off;
  off += kGemvWarps * B * 32 * 4;
  L.total = off;
  return L;
}

// ---------------------------------------------------------------------------
// Activation staging (runs after the programmatic-dependency wait).

// Q4_0: per 32-column block, 16 half2 in the order the dequantizer emits:
// for qs word i (bytes 4i..4i+3):
//   (x[4i], x[4i+2]), (x[16+4i], x[18+4i]), (x[4i+1], x[4i+3]), (x[17+4i], x[19+4i])
__device__ __forceinline__ void stage_x_q4_0(const __half* __restrict__ x, uint8_t* xs, int nb,
                                             int B, int K) {
  const int nblk = K / 32;
  for (int u = threadIdx.x; u < B * nblk; u += blockDim.x) {
    const int b = u / nblk;
    const int blk = u - b * nblk;
    uint4* dst = reinterpret_cast<uint4*>(xs) + (size_t)u * 4;
    if (b >= nb) {
      const uint4 z = make_uint4(0, 0, 0, 0);
      dst[0] = z; dst[1] = z; dst[2] = z; dst[3] = z;
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)b * K + blk * 32);
    uint32_t h[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = src[j];
      h[4 * j] = v.x; h[4 * j + 1] = v.y; h[4 * j + 2] = v.z; h[4 * j + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 o;
      o.x = __byte_perm(h[2 * i], h[2 * i + 1], 0x5410);          // x[4i],    x[4i+2]
      o.y = __byte_perm(h[8 + 2 * i], h[9 + 2 * i], 0x5410);      // x[16+4i], x[18+4i]
      o.z = __byte_perm(h[2 * i], h[2 * i + 1], 0x7632);          // x[4i+1],  x[4i+3]
      o.w = __byte_perm(h[8 + 2 * i], h[9 + 2 * i], 0x7632);      // x[17+4i], x[19+4i]
      dst[i] = o;
    }
  }
}

// Q8_0: plain fp32 copy of x.
__device__ __forceinline__ void stage_x_f32(const __half* __restrict__ x, uint8_t* xs, int nb,
                                            int B, int K) {
  const int n8 = K / 8;
  for (int u = threadIdx.x; u < B * n8; u += blockDim.x) {
    const int b = u / n8;
    float4* dst = reinterpret_cast<float4*>(xs) + (size_t)u * 2;
    if (b >= nb) {
      dst[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      dst[1] = dst[0];
      continue;
    }
    const uint4 v = *reinterpret_cast<const uint4*>(x + (size_t)u * 8);
    const float2 a = __half22float2(u32_as_h2(v.x));
    const float2 c = __half22float2(u32_as_h2(v.y));
    const float2 e = __half22float2(u32_as_h2(v.z));
    const float2 g = __half22float2(u32_as_h2(v.w));
    dst[0] = make_float4(a.x, a.y, c.x, c.y);
    dst[1] = make_float4(e.x, e.y, g.x, g.y);
  }
}

// Affine: per 8-column word, (x0,x4),(x1,x5),(x2,x6),(x3,x7); plus the fp32
// sum of x over each quantization group (needed for the bias term).
template <int GS>
__device__ __forceinline__ void stage_x_affine(const __half* __restrict__ x, uint8_t* xs,
                                               float* xsum, int nb, int B, int K) {
  constexpr int kLanesPerGroup = GS / 8;  // 4..32, divides 32
  const int n8 = K / 8;
  const int total = B * n8;
  for (int base = threadIdx.x & ~31; base < total; base += blockDim.x) {
    const int u = base + (threadIdx.x & 31);
    float s = 0.f;
    if (u < total) {
      const int b = u / n8;
      uint4 o = make_uint4(0, 0, 0, 0);
      if (b < nb) {
        const uint4 v = *reinterpret_cast<const uint4*>(x + (size_t)u * 8);
        o.x = __byte_perm(v.x, v.z, 0x5410);  // x0, x4
        o.y = __byte_perm(v.x, v.z, 0x7632);  // x1, x5
        o.z = __byte_perm(v.y, v.w, 0x5410);  // x2, x6
        o.w = __byte_perm(v.y, v.w, 0x7632);  // x3, x7
        const float2 a = __half22float2(u32_as_h2(v.x));
        const float2 c = __half22float2(u32_as_h2(v.y));
        const float2 e = __half22float2(u32_as_h2(v.z));
        const float2 g = __half22float2(u32_as_h2(v.w));
        s = ((a.x + a.y) + (c.x + c.y)) + ((e.x + e.y) + (g.x + g.y));
      }
      reinterpret_cast<uint4*>(xs)[u] = o;
    }
#pragma unroll
    for (int m = 1; m < kLanesPerGroup; m <<= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
    if (u < total && (u % kLanesPerGroup) == 0) xsum[u / kLanesPerGroup] = s;
  }
}

// ---------------------------------------------------------------------------
// Per-chunk compute: one lane, one row, 256 columns.

template <int B>
__device__ __forceinline__ void chunk_q4_0(const uint8_t* slot, const uint8_t* xs, int K, int c,
                                           float (&acc)[B]) {
  uint32_t w[36];
  const uint4* s4 = reinterpret_cast<const uint4*>(slot);
#pragma unroll
  for (int j = 0; j < 9; ++j) {
    const uint4 v = s4[j];
    w[4 * j] = v.x; w[4 * j + 1] = v.y; w[4 * j + 2] = v.z; w[4 * j + 3] = v.w;
  }
  const uint4* xc = reinterpret_cast<const uint4*>(xs) + (size_t)c * (kChunkCols / 8);
#pragma unroll
  for (int blk = 0; blk < 8; ++blk) {
    const int o = 18 * blk;  // byte offset of the block inside the chunk
    uint32_t d16, q[4];
    if ((blk & 1) == 0) {
      const int wi = o / 4;
      d16 = w[wi] & 0xFFFFu;
#pragma unroll
      for (int i = 0; i < 4; ++i) q[i] = __funnelshift_r(w[wi + i], w[wi + i + 1], 16);
    } else {
      const int wi = (o - 2) / 4;
      d16 = w[wi] >> 16;
#pragma unroll
      for (int i = 0; i < 4; ++i) q[i] = w[wi + 1 + i];
    }
    const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(d16)));
    __half2 wv[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) unpack_nibbles_minus8(q[i], &wv[4 * i]);
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const uint4* xr = xc + (size_t)b * (K / 8) + blk * 4;
      __half2 a0 = u32_as_h2(0u), a1 = u32_as_h2(0u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 xv = xr[i];
        a0 = __hfma2(wv[4 * i + 0], u32_as_h2(xv.x), a0);
        a1 = __hfma2(wv[4 * i + 1], u32_as_h2(xv.y), a1);
        a0 = __hfma2(wv[4 * i + 2], u32_as_h2(xv.z), a0);
        a1 = __hfma2(wv[4 * i + 3], u32_as_h2(xv.w), a1);
      }
      const float2 f = __half22float2(__hadd2(a0, a1));
      acc[b] = fmaf(d, f.x + f.y, acc[b]);
    }
  }
}

template <int B>
__device__ __forceinline__ void chunk_q8_0(const uint8_t* slot, const uint8_t* xs, int K, int c,
                                           float (&acc)[B]) {
  uint32_t w[68];
  const uint4* s4 = reinterpret_cast<const uint4*>(slot);
#pragma unroll
  for (int j = 0; j < 17; ++j) {
    const uint4 v = s4[j];
    w[4 * j] = v.x; w[4 * j + 1] = v.y; w[4 * j + 2] = v.z; w[4 * j + 3] = v.w;
  }
  const float4* xc = reinterpret_cast<const float4*>(xs) + (size_t)c * (kChunkCols / 4);
  constexpr float kBias = 8388736.0f;  // 2^23 + 128
#pragma unroll
  for (int blk = 0; blk < 8; ++blk) {
    const int o = 34 * blk;
    uint32_t d16, q[8];
    if ((blk & 1) == 0) {
      const int wi = o / 4;
      d16 = w[wi] & 0xFFFFu;
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = __funnelshift_r(w[wi + i], w[wi + i + 1], 16);
    } else {
      const int wi = (o - 2) / 4;
      d16 = w[wi] >> 16;
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = w[wi + 1 + i];
    }
    const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(d16)));
    float wf[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t u = q[i] ^ 0x80808080u;  // int8 -> excess-128
#pragma unroll
      for (int k = 0; k < 4; ++k)
        wf[4 * i + k] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650 + k)) - kBias;
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const float4* xr = xc + (size_t)b * (K / 4) + blk * 8;
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 xv = xr[i];
        s0 = fmaf(wf[4 * i + 0], xv.x, s0);
        s1 = fmaf(wf[4 * i + 1], xv.y, s1);
        s0 = fmaf(wf[4 * i + 2], xv.z, s0);
        s1 = fmaf(wf[4 * i + 3], xv.w, s1);
      }
      acc[b] = fmaf(d, s0 + s1, acc[b]);
    }
  }
}

// Affine: sum_k (n_k*s + b) x_k = s * sum_k (n_k - 8) x_k + (b + 8 s) * sum_k x_k
// over each group; the (n - 8) form keeps the fp16 partial sums small.
template <int B, int GS>
__device__ __forceinline__ void chunk_affine(const uint8_t* slot, const uint8_t* xs,
                                             const float* xsum, const uint32_t* sb_row, int K,
                                             int c, float (&acc)[B]) {
  uint32_t w[32];
  const uint4* s4 = reinterpret_cast<const uint4*>(slot);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4 v = s4[j];
    w[4 * j] = v.x; w[4 * j + 1] = v.y; w[4 * j + 2] = v.z; w[4 * j + 3] = v.w;
  }
  constexpr int kGroupsPerChunk = kChunkCols / GS;
  constexpr int kWordsPerGroup = GS / 8;
  const uint4* xc = reinterpret_cast<const uint4*>(xs) + (size_t)c * (kChunkCols / 8);
  const int G = K / GS;
#pragma unroll
  for (int gi = 0; gi < kGroupsPerChunk; ++gi) {
    float P[B];
#pragma unroll
    for (int b = 0; b < B; ++b) P[b] = 0.f;
#pragma unroll
    for (int sub = 0; sub < kWordsPerGroup / 4; ++sub) {
      __half2 wv[16];
#pragma unroll
      for (int t = 0; t < 4; ++t) unpack_nibbles_minus8(w[gi * kWordsPerGroup + sub * 4 + t], &wv[4 * t]);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const uint4* xr = xc + (size_t)b * (K / 8) + gi * kWordsPerGroup + sub * 4;
        __half2 a0 = u32_as_h2(0u), a1 = u32_as_h2(0u);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint4 xv = xr[t];
          a0 = __hfma2(wv[4 * t + 0], u32_as_h2(xv.x), a0);
          a1 = __hfma2(wv[4 * t + 1], u32_as_h2(xv.y), a1);
          a0 = __hfma2(wv[4 * t + 2], u32_as_h2(xv.z), a0);
          a1 = __hfma2(wv[4 * t + 3], u32_as_h2(xv.w), a1);
        }
        const float2 f = __half22float2(__hadd2(a0, a1));
        P[b] += f.x + f.y;
      }
    }
    const int g = c * kGroupsPerChunk + gi;
    const float2 sbf = __half22float2(u32_as_h2(sb_row[g]));
    const float s = sbf.x;
    const float b8 = fmaf(8.f, s, sbf.y);
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = fmaf(s, P[b], fmaf(b8, xsum[b * G + g], acc[b]));
  }
}

// ---------------------------------------------------------------------------

template <int F, int B, int GS>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_fast_kernel(const GemvParams p) {
  using T = GemvFormat<F>;
  extern __shared__ __align__(128) uint8_t smem[];
  const GemvSmemLayout L = gemv_smem_layout<F>(B, p.K, GS);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int K = p.K;
  const int nchunks = K / kChunkCols;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * T::kStages;
  uint8_t* ring = smem + L.ring + warp * (T::kStages * 32 * T::kSlotStride);
  uint8_t* xs = smem + L.xs;
  float* xsum = reinterpret_cast<float*>(smem + L.xsum);
  uint32_t* sb = reinterpret_cast<uint32_t*>(smem + L.sb);
  float* red = reinterpret_cast<float*>(smem + L.red);

  const int row0 = blockIdx.x * 32;
  const int nvalid = min(32, p.N - row0);
  const bool valid = lane < nvalid;
  const uint8_t* wrow = p.w + (size_t)(row0 + (valid ? lane : 0)) * p.row_bytes;
  const uint32_t stage_bytes = static_cast<uint32_t>(nvalid * T::kChunkBytes);
  const int nmine = warp < nchunks ? (nchunks - warp + kGemvWarps - 1) / kGemvWarps : 0;
  const uint64_t policy = l2_policy_evict_first();

  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < T::kStages; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncwarp();

  auto issue = [&](int stage, int chunk) {
    if (lane == 0) mbar_arrive_expect_tx(&bars[stage], stage_bytes);
    __syncwarp();
    if (valid)
      bulk_copy_g2s_hint(ring + stage * (32 * T::kSlotStride) + lane * T::kSlotStride,
                         wrow + (size_t)chunk * T::kChunkBytes, T::kChunkBytes, &bars[stage],
                         policy);
  };

  // Weights do not depend on the previous kernel: start streaming them now.
  const int npro = min(T::kStages, nmine);
  for (int i = 0; i < npro; ++i) issue(i, warp + i * kGemvWarps);
  pdl_launch_dependents();

  if constexpr (F == kFmtAffineQ4) {
    const int G = K / GS;
    for (int idx = threadIdx.x; idx < 32 * G; idx += blockDim.x) {
      const int r = idx / G;
      const int g = idx - r * G;
      uint32_t v = 0;
      if (r < nvalid) {
        const size_t gi = (size_t)(row0 + r) * G + g;
        const uint32_t s = __half_as_ushort(p.scales[gi]);
        const uint32_t b = __half_as_ushort(p.biases[gi]);
        v = s | (b << 16);
      }
      sb[r * L.sb_stride + g] = v;
    }
  }

  pdl_wait_primary();  // activations are produced by the previous kernel
  if constexpr (F == kFmtQ4_0) stage_x_q4_0(p.x, xs, p.nb, B, K);
  else if constexpr (F == kFmtQ8_0) stage_x_f32(p.x, xs, p.nb, B, K);
  else stage_x_affine<GS>(p.x, xs, xsum, p.nb, B, K);
  __syncthreads();

  float acc[B];
#pragma unroll
  for (int b = 0; b < B; ++b) acc[b] = 0.f;

  const uint32_t* sb_row = sb + lane * L.sb_stride;
  int i = 0;
  for (; i < nmine; ++i) {
    const int s = i % T::kStages;
    const uint32_t parity = (i / T::kStages) & 1;
    if (!mbar_wait(&bars[s], parity)) break;
    const int c = warp + i * kGemvWarps;
    const uint8_t* slot = ring + s * (32 * T::kSlotStride) + lane * T::kSlotStride;
    if constexpr (F == kFmtQ4_0) chunk_q4_0<B>(slot, xs, K, c, acc);
    else if constexpr (F == kFmtQ8_0) chunk_q8_0<B>(slot, xs, K, c, acc);
    else chunk_affine<B, GS>(slot, xs, xsum, sb_row, K, c, acc);
    __syncwarp();
    const int inext = i + T::kStages;
    if (inext < nmine) {
      fence_proxy_async_smem();
      issue(s, warp + inext * kGemvWarps);
    }
  }
  if (i < nmine) {
    // A copy never completed.  Record it and wait (bounded) for the copies
    // that are still in flight into this warp's ring before leaving.
    if (lane == 0) record_device_error(kDevErrBarrierTimeout);
    for (int j = i; j < min(nmine, i + T::kStages); ++j)
      (void)mbar_wait(&bars[j % T::kStages], (j / T::kStages) & 1);
  }

#pragma unroll
  for (int b = 0; b < B; ++b) red[(warp * B + b) * 32 + lane] = acc[b];
  __syncthreads();
  for (int t = threadIdx.x; t < B * 32; t += blockDim.x) {
    const int b = t >> 5;
    const int l = t & 31;
    if (b < p.nb && l < nvalid) {
      float sum = 0.f;
#pragma unroll
      for (int wv = 0; wv < kGemvWarps; ++wv) sum += red[(wv * B + b) * 32 + l];
      p.y[(size_t)b * p.N + row0 + l] = __float2half_rn(sum);
    }
  }
}

// ---------------------------------------------------------------------------
// Generic fallback: one warp per output row, 8 rows per CTA.

template <int F>
__global__ void __launch_bounds__(256) gemv_generic_kernel(const GemvParams p) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  pdl_launch_dependents();
  pdl_wait_primary();
  if (row >= p.N) return;
  const uint8_t* wrow = p.w + (size_t)row * p.row_bytes;
  const int K = p.K;
  for (int b = 0; b < p.nb; ++b) {
    const __half* xb = p.x + (size_t)b * K;
    float acc = 0.f;
    if constexpr (F == kFmtQ4_0) {
      for (int blk = lane; blk < K / 32; blk += 32) {
        const uint16_t* bp = reinterpret_cast<const uint16_t*>(wrow + (size_t)blk * 18);
        const float d = __half2float(__ushort_as_half(bp[0]));
        const __half* xk = xb + blk * 32;
        float s = 0.f;
#pragma unroll
        for (int j2 = 0; j2 < 8; ++j2) {
          const uint32_t two = bp[1 + j2];
          const int b0 = two & 0xFF, b1 = two >> 8;
          s = fmaf(float((b0 & 15) - 8), __half2float(xk[2 * j2]), s);
          s = fmaf(float((b0 >> 4) - 8), __half2float(xk[2 * j2 + 16]), s);
          s = fmaf(float((b1 & 15) - 8), __half2float(xk[2 * j2 + 1]), s);
          s = fmaf(float((b1 >> 4) - 8), __half2float(xk[2 * j2 + 17]), s);
        }
        acc = fmaf(d, s, acc);
      }
    } else if constexpr (F == kFmtQ8_0) {
      for (int blk = lane; blk < K / 32; blk += 32) {
        const uint16_t* bp = reinterpret_cast<const uint16_t*>(wrow + (size_t)blk * 34);
        const float d = __half2float(__ushort_as_half(bp[0]));
        const __half* xk = xb + blk * 32;
        float s = 0.f;
#pragma unroll
        for (int j2 = 0; j2 < 16; ++j2) {
          const uint32_t two = bp[1 + j2];
          s = fmaf(float(static_cast<int8_t>(two & 0xFF)), __half2float(xk[2 * j2]), s);
          s = fmaf(float(static_cast<int8_t>(two >> 8)), __half2float(xk[2 * j2 + 1]), s);
        }
        acc = fmaf(d, s, acc);
      }
    } else {
      const uint32_t* ww = reinterpret_cast<const uint32_t*>(wrow);
      const int G = K / p.group;
      for (int wd = lane; wd < K / 8; wd += 32) {
        const int g = (wd * 8) / p.group;
        const float s = __half2float(p.scales[(size_t)row * G + g]);
        const float bb = __half2float(p.biases[(size_t)row * G + g]);
        const uint32_t packed = ww[wd];
        const __half* xk = xb + wd * 8;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const float val = fmaf(float((packed >> (4 * n)) & 15u), s, bb);
          acc = fmaf(val, __half2float(xk[n]), acc);
        }
      }
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    if (lane == 0) p.y[(size_t)b * p.N + row] = __float2half_rn(acc);
  }
}

}  // namespace gdsq
