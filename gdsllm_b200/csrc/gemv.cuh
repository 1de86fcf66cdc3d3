// Fused dequantize + GEMV kernels for GGUF Q4_0, GGUF Q8_0 and affine-Q4
// weights, batch 1..16.
//
// Reference kernels replaced (same math, different schedule):
//   kernel_fused_q4_0_gemv       gdsllm/runtime/fused_gemv.cu:27-105
//   kernel_fused_q8_0_gemv       gdsllm/runtime/fused_gemv.cu:142-205
//   kernel_fused_affine_q4_gemv  gdsllm/runtime/affine_q4_dequant.cu:79-158
//
// Fast path (weights 16-byte aligned, K % 256 == 0):
//   * Work item = 32 consecutive output rows ("row group").  Lane l of every
//     warp computes row (row0 + l).
//   * K is split across a thread-block cluster of `cs` CTAs: CTA rank r owns
//     256-column chunks [C*r/cs, C*(r+1)/cs).  Inside a CTA, each of the 4
//     warps owns a contiguous run of those chunks.
//   * Each warp streams its chunks through a private ring of shared-memory
//     stages.  A stage holds 1 or 2 chunks (plan) of all 32 rows, each
//     chunk one 2-D TMA box (32 rows x chunk bytes) of the weight matrix's
//     tensor map, issued by lane 0, which also arms the stage's mbarrier.
//     Rows past N arrive as zeros.  Copies for the next stages are in flight
//     while the current one is computed, and the ring keeps streaming across
//     row groups when a cluster owns several.
//   * The activations of the CTA's K slice are staged once in shared memory,
//     permuted so that pair order matches the dequantizer's output order; all
//     32 lanes read the same address, so activation loads are broadcasts.
//   * Arithmetic is fp32 throughout, as in the reference: every product of a
//     quantized value and an activation is exact in fp32 and every sum is an
//     fp32 sum (see "Exact fp32 products" below for how the packed values
//     reach the FMA without a conversion instruction each).
//   * Per row group: warps meet in shared memory; with cs > 1 every CTA writes
//     its partial sums into the cluster leader's shared memory (distributed
//     shared memory), and after a cluster barrier the leader adds the cs
//     partials in rank order and stores fp16 y.
//
// Generic path: any K % 32 == 0 (group_size % 8 == 0 for affine) and 2-byte
// (4-byte for affine words) alignment; one warp per row, plain loads.
#pragma once

#include "common.cuh"

namespace gdsq {

enum WeightFormat : int { kFmtQ4_0 = 0, kFmtQ8_0 = 1, kFmtAffineQ4 = 2 };

constexpr int kGemvWarps = 4;
constexpr int kChunkCols = 256;
constexpr int kMaxStages = 8;
constexpr int kMaxCluster = 8;

template <int F>
struct GemvFormat;

// One chunk of 32 rows lands in shared memory as a dense [32][kChunkBytes]
// box.  For Q4_0 and Q8_0 the row pitch is 36 or 68 words (= 4 mod 32), so
// 16-byte loads of 8 consecutive lanes hit 8 distinct bank groups.  The
// affine pitch is 128 bytes, so its boxes use the 128-byte swizzle (16-byte
// unit u of row r is stored at unit u ^ (r % 8)).
// Activations are staged as scaled fp32 (kXBytes per column) in the order the
// dequantizer emits its values, plus one fp32 per 32-column block (GGUF
// formats: the block's offset term) or per quantization group (affine: the
// group's activation sum).
template <>
struct GemvFormat<kFmtQ4_0> {
  static constexpr int kChunkBytes = 144;  // 8 blocks x 18 B
  static constexpr int kMaxCopyChunks = 2;  // chunks (TMA boxes) per ring stage, at most
  static constexpr bool kSwizzle = false;
  static constexpr int kXBytes = 4;
};

template <>
struct GemvFormat<kFmtQ8_0> {
  static constexpr int kChunkBytes = 272;  // 8 blocks x 34 B
  static constexpr int kMaxCopyChunks = 1;
  static constexpr bool kSwizzle = false;
  static constexpr int kXBytes = 4;
};

template <>
struct GemvFormat<kFmtAffineQ4> {
  static constexpr int kChunkBytes = 128;  // 32 words of 8 nibbles
  static constexpr int kMaxCopyChunks = 2;
  static constexpr bool kSwizzle = true;
  static constexpr int kXBytes = 4;
};

// ---------------------------------------------------------------------------
// Exact fp32 products from packed integers.
//
// A field of a 32-bit word masked in place, v << s with v < 2^m and
// s + m <= 23, read as fp32 bits is the subnormal v * 2^(s - 149): an exact
// value, produced by one LOP3 and consumed by the FMA at full rate (this
// library is built without flush-to-zero).  The staging code multiplies the
// activation that meets field position s by 2^(110 - s), so every product is
// exactly v * x * 2^-39 and the running sums are ordinary fp32 sums in units
// of 2^-39; the epilogue multiplies by 2^39, which is exact.  Range: fp16
// |x| <= 65504 < 2^16 keeps x * 2^110 below 2^126, and the smallest nonzero
// product (x = 2^-24, v = 1) is 2^-63, a normal fp32.
//
// Nibble words (Q4_0 and affine) give 4 fp32 pairs per word, the FFMA2
// operand pairs: (bits 0-3, 4-7), (8-11, 12-15), (16-19, 20-23), (24-27,
// 28-31), built as q & 0xF, q & 0xF0, q & 0xF00, q & 0xF000, q & 0xF0000,
// (q >> 16) & 0xF0, (q >> 16) & 0xF00, q >> 28 — field shifts s = 0, 4, 8,
// 12, 16, 4, 8, 0.  Byte words (Q8_0, excess-128) give 2 pairs: u & 0xFF,
// u & 0xFF00, (u >> 16) & 0xFF, (u >> 16) & 0xFF00 — shifts 0, 8, 0, 8.
constexpr float kUnscale = 0x1p39f;

// Activation scale for each of the 8 nibble fields of a word, in word order.
__device__ __forceinline__ float nib_xscale(int k) {
  return k == 0 || k == 7 ? 0x1p110f : k == 1 || k == 5 ? 0x1p106f : k == 2 || k == 6 ? 0x1p102f
         : k == 3 ? 0x1p98f : 0x1p94f;
}

__device__ __forceinline__ void nib_fields(uint32_t q, float2 (&f)[4]) {
  const uint32_t h = q >> 16;
  f[0] = make_float2(__uint_as_float(q & 0xFu), __uint_as_float(q & 0xF0u));
  f[1] = make_float2(__uint_as_float(q & 0xF00u), __uint_as_float(q & 0xF000u));
  f[2] = make_float2(__uint_as_float(q & 0xF0000u), __uint_as_float(h & 0xF0u));
  f[3] = make_float2(__uint_as_float(h & 0xF00u), __uint_as_float(q >> 28));
}

// Signed bytes as excess-128 fields (value + 128).
__device__ __forceinline__ void byte_fields(uint32_t q, float2 (&f)[2]) {
  const uint32_t u = q ^ 0x80808080u;
  const uint32_t h = u >> 16;
  f[0] = make_float2(__uint_as_float(u & 0xFFu), __uint_as_float(u & 0xFF00u));
  f[1] = make_float2(__uint_as_float(h & 0xFFu), __uint_as_float(h & 0xFF00u));
}

__device__ __forceinline__ float2 lo2(float4 v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(float4 v) { return make_float2(v.z, v.w); }

// Bytes of one ring stage holding `copy` chunks of 32 rows.
template <int F>
__host__ __device__ constexpr int stage_bytes(int copy) {
  return copy * 32 * GemvFormat<F>::kChunkBytes;
}

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
  int cs;                 // CTAs per cluster (K slices)
  int stages;             // ring stages per warp (1..kMaxStages)
  int copy;               // chunks per ring stage (1..kMaxCopyChunks)
  int num_rg;             // row groups = ceil(N / 32) (summed over the group)
  // Grouped launch (GGUF formats): up to 4 matrices with the same K and x,
  // their 32-row groups laid end to end; matrix m owns row groups
  // [rg_start[m], rg_start[m + 1]), writes ys[m] and has ns[m] rows.
  // count == 1 for a plain launch (ys[0] = y, ns[0] = N).
  int count;
  int rg_start[5];
  __half* ys[4];
  int ns[4];
  // Tensor-parallel row split (the TP instantiation; batch 1, count 1,
  // tp_world > 1): each output row is summed over the ranks inside the kernel (tp_publish /
  // tp_finish_cta).  tp_bufs[r] = rank r's exchange buffer [2][world]
  // [tp_rows] of (fp32 value, epoch) words, tp_flags[r] = its flags
  // [kTpFlagInts]; both mapped into every rank.
  int tp_world;
  int tp_rank;
  int tp_rows;
  unsigned long long* tp_bufs[8];
  int* tp_flags[8];
  unsigned long long* tp_own_buf;  // tp_bufs[tp_rank]
  int* tp_own_flags;               // tp_flags[tp_rank]
  unsigned long long tp_wait_ns;   // bound of the finishers' wait for the peers' rows
};

constexpr int kMaxGroup = 4;
constexpr int kTpMaxRanks = 8;
constexpr int kTpMaxRowGroups = 1024;

// Tensor-parallel exchange of the row-split GEMV (batch 1, one matrix).
// Per rank: a buffer [2 slots][world][tp_rows] of 64-bit words, each the
// fp32 bits of one partial output row (low half) and the call epoch (high
// half), and an int array [kTpFlagInts] (local only: [kTpEpoch] = the last
// call finished, [kTpFinCount] = finishers done in the current call); both
// mapped into every rank.  Call epoch E = [kTpEpoch] + 1, slot E & 1.
//   tp_publish (the CTA that computed a row group, warp 0): one 64-bit store
//     of (row value, E) into row `rank` of slot E & 1 of every rank's buffer
//     (remote ones over NVLink).  The value travels with its epoch in one
//     single-copy-atomic word, so no fence or flag is needed, and publishing
//     never waits.
//   tp_finish_cta (the leaders of the first nf clusters, after their own row
//     groups): poll (bounded) this rank's own buffer until each row of the
//     finisher's share carries E for every rank, add the world values in
//     rank order (fp32, identical bits on every rank) and store fp16.  The
//     last finisher to count itself done records E in [kTpEpoch].
// Every finisher reads E before it counts itself, and every publisher reads
// E before its rows appear, which some finisher waits for; so [kTpEpoch]
// changes only after every CTA of the call has read it.  The next call's
// CTAs read it only after this grid completed (programmatic dependent launch
// waits).  All CTAs but the finishers leave right after publishing.  Two
// slots suffice: rank A writes slot E & 1 of rank B again in call E + 2,
// which starts after A's call E + 1 saw B's rows of E + 1, which B writes
// only after its call E (the last reader of the slot) completed.
constexpr int kTpFlagInts = 64;
constexpr int kTpEpoch = 1;
constexpr int kTpFinCount = 2;
constexpr int kTpFinishers = 8;

__device__ __forceinline__ int tp_call_epoch(const int* own_flags) {
  return *reinterpret_cast<const volatile int*>(own_flags + kTpEpoch) + 1;
}

__device__ __forceinline__ size_t tp_word(int e, int world, int rows_cap, int src, int row) {
  return ((size_t)(e & 1) * world + src) * rows_cap + row;
}

__device__ __forceinline__ void tp_publish(const GemvParams& p, int e, int rg, int lane, float v) {
  const unsigned long long w = ((unsigned long long)(unsigned)e << 32) | __float_as_uint(v);
  const size_t i = tp_word(e, p.tp_world, p.tp_rows, p.tp_rank, rg * 32 + lane);
#pragma unroll
  for (int r = 0; r < kTpMaxRanks; ++r)  // constant indices keep the parameter array in place
    if (r < p.tp_world) st_volatile_u64(p.tp_bufs[r] + i, w);
}

// Every thread of finisher f of nf.  Scalar arguments only, so the kernel's
// parameter block is never copied to local memory for the call.  Returns
// false if a wait expired.
__device__ __noinline__ bool tp_finish_cta(const unsigned long long* buf, int* own, __half* y, int N, int num_rg,
                                           int world, int rows_cap, int e, int f, int nf,
                                           unsigned long long wait_ns) {
  __shared__ int s_fail;
  constexpr int kRows = 8;  // rows per thread per pass
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  const int rows = num_rg * 32;
  const int per = (rows + nf - 1) / nf;
  const int lo = f * per;
  const int hi = min(rows, lo + per);
  bool ok = true;
  for (int base = lo + threadIdx.x; base < hi; base += blockDim.x * kRows) {
    float sum[kRows];
#pragma unroll
    for (int j = 0; j < kRows; ++j) sum[j] = 0.f;
    for (int q = 0; q < world; ++q) {
      unsigned long long w[kRows];
      const size_t i0 = tp_word(e, world, rows_cap, q, 0);
#pragma unroll
      for (int j = 0; j < kRows; ++j) {
        const int row = base + j * blockDim.x;
        w[j] = row < hi ? ld_volatile_u64(buf + i0 + row) : ((unsigned long long)(unsigned)e << 32);
      }
      unsigned long long t0 = 0;
#pragma unroll
      for (int j = 0; j < kRows; ++j) {
        const int row = base + j * blockDim.x;
        while (ok && (int)(w[j] >> 32) != e) {
          if (t0 == 0) t0 = global_timer_ns();
          else if (global_timer_ns() - t0 > wait_ns) {
            record_device_error(kDevErrBarrierTimeout);
            ok = false;
            break;
          }
          w[j] = ld_volatile_u64(buf + i0 + row);
        }
        sum[j] += __uint_as_float((unsigned)w[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
      const int row = base + j * blockDim.x;
      if (ok && row < hi && row < N) y[row] = __float2half_rn(sum[j]);
    }
  }
  if (!ok) s_fail = 1;
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(own + kTpFinCount, 1) == nf - 1) {
      own[kTpFinCount] = 0;
      *reinterpret_cast<volatile int*>(own + kTpEpoch) = e;
    }
  }
  return s_fail == 0;
}

// Shared-memory carve-up of the fast kernel, identical on host and device.
struct GemvSmemLayout {
  int ring;       // byte offsets from the dynamic smem base
  int xs;
  int xsum;
  int sb;
  int sb_stride;  // words per row of the (scale, bias) table
  int red;
  int slots;
  int total;
  int kslice;     // columns of the largest K slice
};

template <int F>
__host__ __device__ inline GemvSmemLayout gemv_smem_layout(int B, int K, int group, int cs,
                                                           int stages, int copy) {
  using T = GemvFormat<F>;
  GemvSmemLayout L;
  const int C = K / kChunkCols;
  (void)sizeof(T);
  L.kslice = (C + cs - 1) / cs * kChunkCols;
  int off = 1024;  // mbarriers (kGemvWarps * kMaxStages * 8 bytes); ring 1024-aligned
  L.ring = off;
  off += kGemvWarps * stages * stage_bytes<F>(copy);
  L.xs = off;
  off += B * L.kslice * T::kXBytes;
  L.xsum = off;  // one fp32 per block (GGUF) or per group (affine) and batch row
  L.sb_stride = 0;
  if (F != kFmtAffineQ4) {
    off += B * (L.kslice / 32) * 4;
    L.sb = off;
  } else {
    const int gs = L.kslice / group;
    off += B * gs * 4;
    L.sb = off;
    L.sb_stride = gs | 1;  // odd word stride: conflict-free per-lane reads
    off += 32 * L.sb_stride * 4;
  }
  L.red = off;
  off += 2 * kGemvWarps * B * 32 * 4;
  L.slots = off;
  if (cs > 1) off += 2 * cs * B * 32 * 4;
  L.total = off + 1024;  // slack to align the base to 1024 bytes at run time
  return L;
}

// ---------------------------------------------------------------------------
// Activation staging: columns [col0, col0 + ncols) of x into shared memory,
// row stride ncols_max.  Runs after the programmatic-dependency wait.

// Every staging function works in units of 8 columns (one thread each, a
// warp's units consecutive) and writes, per unit, 8 scaled fp32 activations
// as two 16-byte stores; `ld` is the staged row stride in columns.  Units of
// batch rows >= nb are zero.

__device__ __forceinline__ void store_x8(uint8_t* xs, size_t col, const float (&v)[8]) {
  float4* dst = reinterpret_cast<float4*>(xs + col * 4);
  dst[0] = make_float4(v[0], v[1], v[2], v[3]);
  dst[1] = make_float4(v[4], v[5], v[6], v[7]);
}

__device__ __forceinline__ void h8_to_f32(uint2 a, uint2 b, float (&v)[8]) {
  const float2 p0 = __half22float2(u32_as_h2(a.x)), p1 = __half22float2(u32_as_h2(a.y));
  const float2 p2 = __half22float2(u32_as_h2(b.x)), p3 = __half22float2(u32_as_h2(b.y));
  v[0] = p0.x; v[1] = p0.y; v[2] = p1.x; v[3] = p1.y;
  v[4] = p2.x; v[5] = p2.y; v[6] = p3.x; v[7] = p3.y;
}

// Q4_0: unit (b, block, i) stages the 8 columns that meet qs word i (bytes
// 4i..4i+3) in field order: x[4i], x[4i+16], x[4i+1], x[4i+17], x[4i+2],
// x[4i+18], x[4i+3], x[4i+19], each times nib_xscale(field).  xc[b][block] =
// -8 * sum(x over the block) * 2^-39, the (q - 8) offset of the block in the
// units of the partial sums.
__device__ __forceinline__ void stage_x_q4_0(const __half* __restrict__ x, uint8_t* xs, float* xc,
                                             int nb, int B, int K, int col0, int ncols, int ld) {
  const int nblk = ncols / 32;
  const int total = B * nblk * 4;
  for (int base = threadIdx.x & ~31; base < total; base += blockDim.x) {
    const int u = base + (threadIdx.x & 31);
    float s = 0.f;
    int b = 0, blk = 0, i = 0;
    if (u < total) {
      i = u & 3;
      blk = (u >> 2) % nblk;
      b = (u >> 2) / nblk;
      float v[8];
      if (b < nb) {
        const __half* xb = x + (size_t)b * K + col0 + blk * 32 + 4 * i;
        float lo[8];
        h8_to_f32(*reinterpret_cast<const uint2*>(xb), *reinterpret_cast<const uint2*>(xb + 16), lo);
        // lo = x[4i..4i+3], x[4i+16..4i+19]
        const float o[8] = {lo[0], lo[4], lo[1], lo[5], lo[2], lo[6], lo[3], lo[7]};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          v[k] = o[k] * nib_xscale(k);
          s += o[k];
        }
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = 0.f;
      }
      store_x8(xs, (size_t)b * ld + blk * 32 + 8 * i, v);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (u < total && i == 0) xc[b * (ld / 32) + blk] = s * (-8.0f * 0x1p-39f);
  }
}

// Q8_0: unit (b, j) stages columns 8j..8j+7 in order, scaled 2^110, 2^102
// alternately (byte fields at shifts 0 and 8); xc[b][block] = -128 *
// sum(x over the block) * 2^-39 (the excess-128 offset).
__device__ __forceinline__ void stage_x_q8_0(const __half* __restrict__ x, uint8_t* xs, float* xc,
                                             int nb, int B, int K, int col0, int ncols, int ld) {
  const int n8 = ncols / 8;
  const int total = B * n8;
  for (int base = threadIdx.x & ~31; base < total; base += blockDim.x) {
    const int u = base + (threadIdx.x & 31);
    float s = 0.f;
    int b = 0, j = 0;
    if (u < total) {
      b = u / n8;
      j = u - b * n8;
      float v[8];
      if (b < nb) {
        const uint4 h = *reinterpret_cast<const uint4*>(x + (size_t)b * K + col0 + j * 8);
        h8_to_f32(make_uint2(h.x, h.y), make_uint2(h.z, h.w), v);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          s += v[k];
          v[k] *= (k & 1) ? 0x1p102f : 0x1p110f;
        }
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = 0.f;
      }
      store_x8(xs, (size_t)b * ld + j * 8, v);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (u < total && (j & 3) == 0) xc[b * (ld / 32) + j / 4] = s * (-128.0f * 0x1p-39f);
  }
}

// Affine: unit (b, j) stages word j's columns 8j..8j+7 in order, each times
// nib_xscale(field); xsum[b][group] = sum(x over the group) * 2^-39 (the
// bias term, in the units of the partial sums).
template <int GS>
__device__ __forceinline__ void stage_x_affine(const __half* __restrict__ x, uint8_t* xs,
                                               float* xsum, int nb, int B, int K, int col0,
                                               int ncols, int ld) {
  constexpr int kLanesPerGroup = GS / 8;  // 4..32, divides 32
  const int n8 = ncols / 8;
  const int total = B * n8;
  for (int base = threadIdx.x & ~31; base < total; base += blockDim.x) {
    const int u = base + (threadIdx.x & 31);
    float s = 0.f;
    int b = 0, j = 0;
    if (u < total) {
      b = u / n8;
      j = u - b * n8;
      float v[8];
      if (b < nb) {
        const uint4 h = *reinterpret_cast<const uint4*>(x + (size_t)b * K + col0 + j * 8);
        h8_to_f32(make_uint2(h.x, h.y), make_uint2(h.z, h.w), v);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          s += v[k];
          v[k] *= nib_xscale(k);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = 0.f;
      }
      store_x8(xs, (size_t)b * ld + j * 8, v);
    }
#pragma unroll
    for (int m = 1; m < kLanesPerGroup; m <<= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
    if (u < total && (j % kLanesPerGroup) == 0) xsum[b * (ld / GS) + j / kLanesPerGroup] = s * 0x1p-39f;
  }
}

// ---------------------------------------------------------------------------
// Per-chunk compute: one lane, one row, 256 columns.  `src` is the shared
// address of this lane's chunk bytes, `xa` the shared address of the staged
// activations of this chunk for batch row 0 and `xb` the byte distance
// between batch rows; `xc` / `xcb` likewise for the per-block offset terms
// (GGUF formats).  acc[] accumulates in units of 2^-39.

// This lane's row of a Q4_0 chunk (8 blocks, 144 bytes) into registers.
__device__ __forceinline__ void load_chunk_q4_0(uint32_t src, uint32_t (&w)[36]) {
#pragma unroll
  for (int j = 0; j < 9; ++j) {
    const uint4 v = lds128(src + 16 * j);
    w[4 * j] = v.x; w[4 * j + 1] = v.y; w[4 * j + 2] = v.z; w[4 * j + 3] = v.w;
  }
}

template <int B>
__device__ __forceinline__ void chunk_q4_0_regs(const uint32_t (&w)[36], uint32_t xa, uint32_t xb, uint32_t xc,
                                                uint32_t xcb, float (&acc)[B]) {
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
    float2 f[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) nib_fields(q[i], f[i]);
#pragma unroll
    for (int b = 0; b < B; ++b) {
      // sum of n * x over the block (two fp32 FFMA2 chains), then the -8 offset
      float2 s0 = make_float2(0.f, 0.f), s1 = make_float2(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t xw = xa + b * xb + (blk * 32 + i * 8) * 4;
        const float4 x0 = lds128f(xw);
        const float4 x1 = lds128f(xw + 16);
        s0 = __ffma2_rn(f[i][0], lo2(x0), s0);
        s1 = __ffma2_rn(f[i][1], hi2(x0), s1);
        s0 = __ffma2_rn(f[i][2], lo2(x1), s0);
        s1 = __ffma2_rn(f[i][3], hi2(x1), s1);
      }
      const float sum = ((s0.x + s0.y) + (s1.x + s1.y)) + lds32f(xc + b * xcb + blk * 4);
      acc[b] = fmaf(d, sum, acc[b]);
    }
  }
}

template <int B>
__device__ __forceinline__ void chunk_q4_0(uint32_t src, uint32_t xa, uint32_t xb, uint32_t xc,
                                           uint32_t xcb, float (&acc)[B]) {
  uint32_t w[36];
  load_chunk_q4_0(src, w);
  chunk_q4_0_regs<B>(w, xa, xb, xc, xcb, acc);
}

template <int B>
__device__ __forceinline__ void chunk_q8_0(uint32_t src, uint32_t xa, uint32_t xb, uint32_t xc,
                                           uint32_t xcb, float (&acc)[B]) {
  // Two blocks (68 bytes) at a time: words [17*pr, 17*pr + 17) of the chunk.
#pragma unroll
  for (int pr = 0; pr < 4; ++pr) {
    uint32_t w[20];
    const int w0 = 17 * pr;       // first word of the pair
    const int u0 = w0 / 4;        // first 16-byte unit covering it
#pragma unroll
    for (int u = 0; u < 5; ++u) {
      const uint4 v = lds128(src + 16 * (u0 + u));
      w[4 * u] = v.x; w[4 * u + 1] = v.y; w[4 * u + 2] = v.z; w[4 * u + 3] = v.w;
    }
    const int sh = w0 - 4 * u0;  // 0..3
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int blk = 2 * pr + half;
      uint32_t d16, q[8];
      if (half == 0) {
        d16 = w[sh] & 0xFFFFu;
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = __funnelshift_r(w[sh + i], w[sh + i + 1], 16);
      } else {
        d16 = w[sh + 8] >> 16;
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = w[sh + 9 + i];
      }
      const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(d16)));
      float2 f[8][2];
#pragma unroll
      for (int i = 0; i < 8; ++i) byte_fields(q[i], f[i]);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        // sum of (v + 128) * x over the block, then the -128 offset
        float2 s0 = make_float2(0.f, 0.f), s1 = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 xv = lds128f(xa + b * xb + (blk * 8 + i) * 16);
          if (i & 1) {
            s1 = __ffma2_rn(f[i][0], lo2(xv), s1);
            s1 = __ffma2_rn(f[i][1], hi2(xv), s1);
          } else {
            s0 = __ffma2_rn(f[i][0], lo2(xv), s0);
            s0 = __ffma2_rn(f[i][1], hi2(xv), s0);
          }
        }
        const float sum = ((s0.x + s0.y) + (s1.x + s1.y)) + lds32f(xc + b * xcb + blk * 4);
        acc[b] = fmaf(d, sum, acc[b]);
      }
    }
  }
}

// Affine: sum_k (n_k*s + b) x_k = s * sum_k n_k x_k + b * sum_k x_k over each
// group, both sums fp32.  `sb_row` (shared address of this lane's (scale,
// bias) row) and `xsum` are indexed by the group's position in the K slice,
// starting at g0.


// This lane's row of an affine chunk (32 words, a 128-byte swizzled box row)
// into registers.
__device__ __forceinline__ void load_chunk_affine(uint32_t src, uint32_t swz, uint32_t (&w)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4 v = lds128(src + 16 * (j ^ swz));
    w[4 * j] = v.x; w[4 * j + 1] = v.y; w[4 * j + 2] = v.z; w[4 * j + 3] = v.w;
  }
}

template <int B, int GS>
__device__ __forceinline__ void chunk_affine_regs(const uint32_t (&w)[32], uint32_t xa, uint32_t xb, uint32_t xsum,
                                                  uint32_t xsum_b, uint32_t sb_row, int g0, float (&acc)[B]) {
  constexpr int kGroupsPerChunk = kChunkCols / GS;
  constexpr int kWordsPerGroup = GS / 8;
#pragma unroll
  for (int gi = 0; gi < kGroupsPerChunk; ++gi) {
    float2 s0[B], s1[B];
#pragma unroll
    for (int b = 0; b < B; ++b) s0[b] = s1[b] = make_float2(0.f, 0.f);
#pragma unroll
    for (int t = 0; t < kWordsPerGroup; ++t) {
      float2 f[4];
      nib_fields(w[gi * kWordsPerGroup + t], f);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const uint32_t xw = xa + b * xb + (gi * GS + t * 8) * 4;
        const float4 x0 = lds128f(xw);
        const float4 x1 = lds128f(xw + 16);
        s0[b] = __ffma2_rn(f[0], lo2(x0), s0[b]);
        s1[b] = __ffma2_rn(f[1], hi2(x0), s1[b]);
        s0[b] = __ffma2_rn(f[2], lo2(x1), s0[b]);
        s1[b] = __ffma2_rn(f[3], hi2(x1), s1[b]);
      }
    }
    const int g = g0 + gi;
    const float2 sbf = __half22float2(u32_as_h2(lds32(sb_row + 4 * g)));
#pragma unroll
    for (int b = 0; b < B; ++b)
      acc[b] = fmaf(sbf.x, (s0[b].x + s0[b].y) + (s1[b].x + s1[b].y),
                    fmaf(sbf.y, lds32f(xsum + b * xsum_b + 4 * g), acc[b]));
  }
}

template <int B, int GS>
__device__ __forceinline__ void chunk_affine(uint32_t src, uint32_t swz, uint32_t xa, uint32_t xb,
                                             uint32_t xsum, uint32_t xsum_b, uint32_t sb_row,
                                             int g0, float (&acc)[B]) {
  uint32_t w[32];
  load_chunk_affine(src, swz, w);
  chunk_affine_regs<B, GS>(w, xa, xb, xsum, xsum_b, sb_row, g0, acc);
}

// ---------------------------------------------------------------------------
// Cluster helpers (distributed shared memory).

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Split form: an early relaxed arrive only announces "this CTA is running";
// the matching wait, just before the first distributed-shared-memory store,
// then costs nothing when every peer started long ago.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of `local` (a shared::cta address in this CTA's window) in the
// shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(const void* local, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_addr(local)), "r"(rank));
  return out;
}

__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// ---------------------------------------------------------------------------

// TP: the tensor-parallel row split (batch 1, one matrix, tp_world > 1):
// the epilogue publishes the rows to the ranks and the first few leader CTAs
// finish the cross-rank sums (tp_publish / tp_finish_cta).  A separate
// instantiation, so the plain kernels carry none of its code or registers.
template <int F, int B, int GS, bool TP = false>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_fast_kernel(const GemvParams p, const __grid_constant__ CUtensorMap wmap,
                     const __grid_constant__ CUtensorMap wmap1, const __grid_constant__ CUtensorMap wmap2,
                     const __grid_constant__ CUtensorMap wmap3) {
  using T = GemvFormat<F>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // TMA destinations (the 128-byte swizzle in particular) need a 1024-byte
  // aligned base; the layout reserves the slack.
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int cs = p.cs;
  const int S = p.stages;
  const int CP = p.copy;
  const GemvSmemLayout L = gemv_smem_layout<F>(B, p.K, GS, cs, S, CP);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int K = p.K;
  const int C = K / kChunkCols;

  const int crank = cs > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int cluster = blockIdx.x / cs;
  const int nclusters = gridDim.x / cs;
  const int nitems = cluster < p.num_rg ? (p.num_rg - 1 - cluster) / nclusters + 1 : 0;

  // This CTA's K slice and this warp's contiguous chunks inside it.
  const int c0 = (C * crank) / cs;
  const int cslice = (C * (crank + 1)) / cs - c0;
  const int per_warp = (cslice + kGemvWarps - 1) / kGemvWarps;
  const int wc0 = min(cslice, warp * per_warp);            // slice-local
  const int mw = min(cslice, wc0 + per_warp) - wc0;        // chunks per item
  const int nsteps = (mw + CP - 1) / CP;
  const int total = nitems * nsteps;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * kMaxStages;
  uint8_t* ring = smem + L.ring + warp * (S * stage_bytes<F>(CP));
  uint8_t* xs = smem + L.xs;
  float* xsum = reinterpret_cast<float*>(smem + L.xsum);
  uint32_t* sb = reinterpret_cast<uint32_t*>(smem + L.sb);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* slots = reinterpret_cast<float*>(smem + L.slots);
  const uint32_t ring_a = smem_addr(ring) + lane * T::kChunkBytes;  // this lane's row, stage 0, chunk 0
  const uint64_t policy = l2_policy_evict_first();

  // Cluster reduction barriers (after the per-warp stage barriers): the
  // leader's red_full[item & 1] counts the peers' partial-sum stores, a
  // peer's red_empty[item & 1] the leader's release of that slot buffer.
  uint64_t* red_full = reinterpret_cast<uint64_t*>(smem) + kGemvWarps * kMaxStages;
  uint64_t* red_empty = red_full + 2;
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    if (warp == 0 && cs > 1) {
      for (int d = 0; d < 2; ++d) {
        mbar_init(&red_full[d], (cs - 1) * B * 32);
        mbar_init(&red_empty[d], B * 32);
      }
    }
    fence_barrier_init();
    if (warp == 0) {
      prefetch_tensor_map(&wmap);
      if (p.count > 1) prefetch_tensor_map(&wmap1);
      if (p.count > 2) prefetch_tensor_map(&wmap2);
      if (p.count > 3) prefetch_tensor_map(&wmap3);
    }
  }
  __syncwarp();
  if (cs > 1) cluster_arrive_relaxed();  // waited for before the first DSMEM store

  // Matrix of a global row group and the group's first row inside it.
  auto locate = [&](int rg, int* m, int* lrow0) {
    int mm = 0;
    if (p.count > 1) mm = (rg >= p.rg_start[1]) + (rg >= p.rg_start[2]) + (rg >= p.rg_start[3]);
    *m = mm;
    *lrow0 = (rg - p.rg_start[mm]) * 32;
  };

  // Producer cursor: the next (item, step) to copy and the stage it goes to.
  int p_item = 0, p_step = 0, p_stage = 0, issued = 0;
  auto issue_next = [&]() {
    if (lane == 0) {
      int m, row0;
      locate(cluster + p_item * nclusters, &m, &row0);
      const CUtensorMap* map = m == 0 ? &wmap : m == 1 ? &wmap1 : m == 2 ? &wmap2 : &wmap3;
      const int chunk = c0 + wc0 + p_step * CP;
      const int nch = min(CP, mw - p_step * CP);
      uint8_t* dst = ring + p_stage * stage_bytes<F>(CP);
      mbar_arrive_expect_tx(&bars[p_stage], static_cast<uint32_t>(nch * 32 * T::kChunkBytes));
      for (int j = 0; j < nch; ++j)
        tma_load_2d(dst + j * (32 * T::kChunkBytes), map, (chunk + j) * (T::kChunkBytes / 8), row0,
                    &bars[p_stage], policy);
    }
    ++issued;
    if (++p_step == nsteps) { p_step = 0; ++p_item; }
    if (++p_stage == S) p_stage = 0;
  };

  // Weights do not depend on the previous kernel: start streaming them now.
  const int npro = min(S, total);
  for (int t = 0; t < npro; ++t) issue_next();
  pdl_launch_dependents();

  const int gslice = F == kFmtAffineQ4 ? cslice * kChunkCols / GS : 0;
  auto load_sb = [&](int row0) {
    if constexpr (F == kFmtAffineQ4) {
      const int G = K / GS;
      const int nvalid = min(32, p.N - row0);
      for (int idx = threadIdx.x; idx < 32 * gslice; idx += blockDim.x) {
        const int r = idx / gslice;
        const int g = idx - r * gslice;
        uint32_t v = 0;
        if (r < nvalid) {
          const size_t gi = (size_t)(row0 + r) * G + c0 * (kChunkCols / GS) + g;
          v = (uint32_t)__half_as_ushort(p.scales[gi]) | ((uint32_t)__half_as_ushort(p.biases[gi]) << 16);
        }
        sb[r * L.sb_stride + g] = v;
      }
    }
  };
  if (nitems > 0) load_sb(cluster * 32);

  pdl_wait_primary();  // activations are produced by the previous kernel
  // Tensor-parallel exchange: the call's epoch (read after the previous
  // call's grid completed) and the finisher count (each has a row group).
  const int tp_e = TP && crank == 0 ? tp_call_epoch(p.tp_own_flags) : 0;
  const int ld = L.kslice;  // staged row stride, in elements
  if constexpr (F == kFmtQ4_0) stage_x_q4_0(p.x, xs, xsum, p.nb, B, K, c0 * kChunkCols, cslice * kChunkCols, ld);
  else if constexpr (F == kFmtQ8_0) stage_x_q8_0(p.x, xs, xsum, p.nb, B, K, c0 * kChunkCols, cslice * kChunkCols, ld);
  else stage_x_affine<GS>(p.x, xs, xsum, p.nb, B, K, c0 * kChunkCols, cslice * kChunkCols, ld);
  __syncthreads();

  const uint32_t xs_a = smem_addr(xs);
  const uint32_t xb = static_cast<uint32_t>(ld * T::kXBytes);   // bytes between batch rows
  const uint32_t xsum_a = smem_addr(xsum);
  const uint32_t sb_a = smem_addr(sb) + lane * L.sb_stride * 4;
  bool ok = true;
  int fail_stage = 0, fail_pending = 0;
  uint32_t fail_phase = 0;
  int consumed = 0;
  int stage = 0;
  uint32_t phase = 0;
  for (int item = 0; item < nitems; ++item) {
    int m, row0;
    locate(cluster + item * nclusters, &m, &row0);
    const int Nm = p.ns[m];
    __half* ym = p.ys[m];
    const int nvalid = min(32, Nm - row0);
    if (F == kFmtAffineQ4 && item > 0) {
      __syncthreads();
      load_sb(row0);
      __syncthreads();
    }
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.f;

    for (int st = 0; st < nsteps; ++st) {
      if (ok && !mbar_wait(&bars[stage], phase)) {
        ok = false;
        fail_stage = stage;
        fail_phase = phase;
        fail_pending = issued - consumed;  // copies issued and not yet consumed
      }
      ++consumed;
      if (F == kFmtQ4_0 && CP == 1) {
        // One chunk per stage: the lane's row goes to registers first, and
        // the stage is refilled before the arithmetic, so the next copy
        // overlaps it (an extra stage of buffering in registers).
        if (ok) {
          const uint32_t slot = ring_a + stage * stage_bytes<F>(1);
          const int cl = wc0 + st;
          uint32_t w[36];
          load_chunk_q4_0(slot, w);
          __syncwarp();
          if (issued < total) {
            if (lane == 0) fence_proxy_async_smem();  // the reads above before the copy's writes
            issue_next();
          }
          chunk_q4_0_regs<B>(w, xs_a + cl * (kChunkCols * 4), xb, xsum_a + cl * 32, (ld / 32) * 4, acc);
        }
        __syncwarp();
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
        continue;
      }
      if (ok) {
        const uint32_t slot = ring_a + stage * stage_bytes<F>(CP);
        const int cl0 = wc0 + st * CP;  // slice-local chunk
        const int nch = min(CP, mw - st * CP);
#pragma unroll
        for (int j = 0; j < T::kMaxCopyChunks; ++j) {
          if (j < nch) {
            const int cl = cl0 + j;
            const uint32_t src = slot + j * (32 * T::kChunkBytes);
            if constexpr (F == kFmtQ4_0) {
              chunk_q4_0<B>(src, xs_a + cl * (kChunkCols * 4), xb, xsum_a + cl * 32, (ld / 32) * 4, acc);
            } else if constexpr (F == kFmtQ8_0) {
              chunk_q8_0<B>(src, xs_a + cl * (kChunkCols * 4), xb, xsum_a + cl * 32, (ld / 32) * 4, acc);
            } else {
              chunk_affine<B, GS>(src, lane & 7, xs_a + cl * (kChunkCols * 4), xb, xsum_a,
                                  (ld / GS) * 4, sb_a, cl * (kChunkCols / GS), acc);
            }
          }
        }
      }
      __syncwarp();
      if (ok && issued < total) issue_next();
      if (++stage == S) {
        stage = 0;
        phase ^= 1;
      }
    }

    // Reduce the 4 warps, then the cs CTAs of the cluster.
    float* rd = red + (item & 1) * (kGemvWarps * B * 32);
#pragma unroll
    for (int b = 0; b < B; ++b) rd[(warp * B + b) * 32 + lane] = acc[b] * kUnscale;
    if (cs > 1 && item == 0) cluster_wait();  // every peer is running: DSMEM stores are safe
    __syncthreads();
    // Peers push their partial sums into the leader's slot buffer and arrive
    // on its barrier; only the leader waits (no cluster-wide barrier).
    float* sl = slots + (item & 1) * (cs * B * 32);
    const uint32_t par = (item >> 1) & 1;
    for (int idx = threadIdx.x; idx < B * 32; idx += blockDim.x) {  // one arrival per (b, l)
      const int b = idx >> 5;
      const int l = idx & 31;
      float v = 0.f;
#pragma unroll
      for (int wv = 0; wv < kGemvWarps; ++wv) v += rd[(wv * B + b) * 32 + l];
      if (cs == 1) {
        if constexpr (TP) tp_publish(p, tp_e, cluster + item * nclusters, l, v);  // batch 1: warp 0
        else if (b < p.nb && l < nvalid) ym[(size_t)b * Nm + row0 + l] = __float2half_rn(v);
      } else if (crank != 0) {
        if (item >= 2 && ok && !mbar_wait_cluster(&red_empty[item & 1], par ^ 1)) {
          ok = false;
          record_device_error(kDevErrBarrierTimeout);
        }
        st_cluster_f32(map_to_rank(sl + (crank * B + b) * 32 + l, 0), v);
        mbar_arrive_cluster(map_to_rank(&red_full[item & 1], 0));
      } else {
        if (ok && !mbar_wait_cluster(&red_full[item & 1], par)) {
          ok = false;
          record_device_error(kDevErrBarrierTimeout);
        }
        for (int r = 1; r < cs; ++r) v += sl[(r * B + b) * 32 + l];
        if constexpr (TP) tp_publish(p, tp_e, cluster + item * nclusters, l, v);  // batch 1: warp 0
        else if (b < p.nb && l < nvalid) ym[(size_t)b * Nm + row0 + l] = __float2half_rn(v);
        if (item + 2 < nitems) {
          for (int r = 1; r < cs; ++r) mbar_arrive_cluster(map_to_rank(&red_empty[item & 1], r));
        }
      }
    }
  }

  if (cs > 1 && nitems == 0) cluster_wait();  // pairs the early arrive
  if constexpr (TP) {
    // The cross-rank sums (one matrix, batch 1), by the first few leaders.
    const int tp_nf = min(min(nclusters, p.num_rg), kTpFinishers);
    if (crank == 0 && cluster < tp_nf &&
        !tp_finish_cta(p.tp_own_buf, p.tp_own_flags, p.y, p.N, p.num_rg, p.tp_world, p.tp_rows, tp_e, cluster,
                       tp_nf, p.tp_wait_ns))
      ok = false;
  }
  if (!ok) {
    // A copy never completed.  Record it and wait (bounded) for the copies
    // still in flight into this warp's ring (at most S, starting with the one
    // that timed out) before leaving.
    if (lane == 0) record_device_error(kDevErrBarrierTimeout);
    // The copies in flight were issued in ring order starting at the stage
    // that timed out.
    uint32_t ph = fail_phase;
    int sidx = fail_stage;
    for (int j = 0; j < fail_pending; ++j) {
      (void)mbar_wait(&bars[sidx], ph);
      if (++sidx == S) {
        sidx = 0;
        ph ^= 1;
      }
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
