// Tensor-core (tcgen05) fused dequantize + GEMV for batches of activations
// (B = 2..16 rows of x), GGUF Q4_0 / Q8_0 and affine-Q4 weights.
//
// The reference runs a batch through dequant_* then F.linear (cuBLAS, fp32
// accumulation) whenever x has more than one row (gdsllm/runtime/llama.py:
// 144-166, qwen_moe.py:58-73).  This kernel computes the same product without
// writing the fp16 weights to memory:
//
//   y[b][r] = fp16( sum_k W16[r][k] * x[b][k] )
//
// where W16 is the fp16 dequantized weight: Q4_0 / Q8_0 give exactly the
// values of the reference's dequant kernels (fp16(d * q), an exact product
// rounded once); affine-Q4 gives fp16(n * s + b) with one rounding (the
// reference rounds to fp32 first, which can move a value by one fp16 ulp in
// rare ties).  Products and sums are fp32 on the tensor core.
//
// One CTA per SM (all 512 TMEM columns): 128 output rows (the MMA's M, one
// TMEM lane each) and a K slice; K is split over a cluster of cs CTAs whose
// partial sums meet in the leader's shared memory.  Warp roles:
//   warp 16      TMA producer: per 256-column chunk, one 2-D box of the
//                weight matrix (128 rows x chunk bytes) into a ring stage.
//   warps 0-15   dequantizers in 4 groups of 4 (one warp per TMEM lane
//                quarter, lane = row): group g turns quarter g (64 columns)
//                of every chunk into 32 fp16-pair TMEM columns (tcgen05.st),
//                alternating between its two A buffers, and copies the same
//                64 columns of x (16 rows, rows >= B zero) into the stage as
//                the MMA's K-major core matrices (one 16-byte load per
//                thread, fetched a chunk ahead).  Group 0 also runs the
//                epilogue of each row tile: tcgen05.ld of the fp32 D tiles,
//                cluster reduction, fp16 y.
//   warp 17      TMEM allocation and the MMA issuer: per chunk and group, 4 x
//                tcgen05.mma (M=128, N=16, K=16, A from TMEM, B = x from
//                shared memory) into one of two D buffers; tcgen05.commit
//                frees A buffers and the x half of the ring stage and, per
//                tile, publishes D.  An N=16 MMA is short, so consecutive
//                MMAs into one accumulator would wait on each other: a D
//                buffer holds 8 accumulators, the chunk's 16 MMAs rotate
//                over them, and the epilogue adds the 8 partial tiles.
// Every wait is bounded; a failed wait raises a CTA-wide abort flag so that
// every role skips its remaining waits, and the device error word is set.
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace gdsq {

constexpr int kTbRows = 128;                       // MMA M, TMEM lanes
constexpr int kTbN = 16;                           // MMA N: batch rows, zero-padded
constexpr int kTbGroups = 4;                       // dequantizer groups (one quarter each)
constexpr int kTbDequantWarps = 4 * kTbGroups;
constexpr int kTbThreads = (kTbDequantWarps + 2) * 32;  // + producer + MMA warp
constexpr int kTbACols = 32;                       // TMEM columns of one A buffer (64 fp16 of K)
constexpr int kTbDCol = kTbGroups * 2 * kTbACols;  // 256: two D buffers from here
constexpr int kTbAcc = 8;                          // independent accumulators per D buffer
constexpr int kTbDCols = kTbAcc * kTbN;            // 128 columns per D buffer
constexpr int kTbTmemCols = 512;
constexpr int kTbXChunkBytes = kTbN * kChunkCols * 2;  // 8192
constexpr int kTbMaxCluster = 8;
constexpr int kTbMaxStages = 6;
constexpr int kTbMinSmem = 116 * 1024;             // > half an SM: one CTA (512 TMEM columns) per SM

// kind::f16 instruction descriptor: D F32, A = B = F16, both K-major,
// N = 16 (bits 17-22 = N >> 3), M = 128 (bits 24-28 = M >> 4).
constexpr uint32_t kTbIdesc = (1u << 4) | (2u << 17) | (8u << 24);

template <int F>
__host__ __device__ constexpr int tb_stage_bytes() {
  return kTbRows * GemvFormat<F>::kChunkBytes + kTbXChunkBytes;  // multiples of 1024
}

struct TbLayout {
  int ring;
  int slots;
  int total;
};

// Barriers and flags live in the first 1024 bytes.
template <int F, int B>
__host__ __device__ inline TbLayout tb_layout(int cs, int stages) {
  TbLayout L;
  int off = 1024;
  L.ring = off;
  off += stages * tb_stage_bytes<F>();
  L.slots = off;
  if (cs > 1) off += 2 * (cs - 1) * B * kTbRows * 4;
  off += 1024;  // slack to align the base at run time
  // Never two CTAs on one SM, so that tcgen05.alloc of all 512 columns
  // never has to wait.
  L.total = off < kTbMinSmem ? kTbMinSmem : off;
  return L;
}

// ---- dequantizers: one 64-column quarter q of a row's 256-column chunk into
// 32 TMEM columns of fp16 pairs (column c = K positions 2c, 2c+1 of the
// quarter).  `src` is the shared address of the row's chunk bytes.

__device__ __forceinline__ void tb_q4_0_quarter(uint32_t src, int q, uint32_t (&o)[32]) {
  // Blocks 2q and 2q+1 occupy bytes [36q, 36q + 36); load the 16-byte
  // aligned 48-byte window that covers them.
  uint32_t w[12];
  const uint32_t base = src + ((36 * q) & ~15);
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const uint4 v = lds128(base + 16 * j);
    w[4 * j] = v.x; w[4 * j + 1] = v.y; w[4 * j + 2] = v.z; w[4 * j + 3] = v.w;
  }
  const int sh = q & 3;  // (36q mod 16) / 4
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t d16, qs[4];
    if (half == 0) {
      d16 = w[sh] & 0xFFFFu;
#pragma unroll
      for (int i = 0; i < 4; ++i) qs[i] = __funnelshift_r(w[sh + i], w[sh + i + 1], 16);
    } else {
      d16 = w[sh + 4] >> 16;
#pragma unroll
      for (int i = 0; i < 4; ++i) qs[i] = w[sh + 5 + i];
    }
    const __half2 d2 = u32_as_h2(d16 | (d16 << 16));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // bytes (b0, b2, b1, b3): the unpacker then yields natural K pairs
      __half2 r[4];
      unpack_nibbles_minus8(__byte_perm(qs[i], 0, 0x3120), r);
      o[16 * half + 2 * i] = h2_as_u32(__hmul2(r[0], d2));      // w[4i],    w[4i+1]
      o[16 * half + 2 * i + 1] = h2_as_u32(__hmul2(r[2], d2));  // w[4i+2],  w[4i+3]
      o[16 * half + 8 + 2 * i] = h2_as_u32(__hmul2(r[1], d2));  // w[16+4i], w[17+4i]
      o[16 * half + 9 + 2 * i] = h2_as_u32(__hmul2(r[3], d2));  // w[18+4i], w[19+4i]
    }
  }
}

__device__ __forceinline__ void tb_q8_0_quarter(uint32_t src, int q, uint32_t (&o)[32]) {
  // Blocks 2q and 2q+1: bytes [68q, 68q + 68), inside the 80-byte aligned
  // window starting at (68q & ~15), shifted by q words.
  uint32_t w[20];
  const uint32_t base = src + ((68 * q) & ~15);
#pragma unroll
  for (int j = 0; j < 5; ++j) {
    const uint4 v = lds128(base + 16 * j);
    w[4 * j] = v.x; w[4 * j + 1] = v.y; w[4 * j + 2] = v.z; w[4 * j + 3] = v.w;
  }
  const int sh = q & 3;
  const __half2 k1152 = u32_as_h2(0x64806480u);  // 1024 + 128
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t d16, qs[8];
    if (half == 0) {
      d16 = w[sh] & 0xFFFFu;
#pragma unroll
      for (int i = 0; i < 8; ++i) qs[i] = __funnelshift_r(w[sh + i], w[sh + i + 1], 16);
    } else {
      d16 = w[sh + 8] >> 16;
#pragma unroll
      for (int i = 0; i < 8; ++i) qs[i] = w[sh + 9 + i];
    }
    const __half2 d2 = u32_as_h2(d16 | (d16 << 16));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t t = qs[i] ^ 0x80808080u;  // int8 -> excess-128 bytes
      const __half2 lo = __hsub2(u32_as_h2(__byte_perm(t, 0x64646464u, 0x4140)), k1152);
      const __half2 hi = __hsub2(u32_as_h2(__byte_perm(t, 0x64646464u, 0x4342)), k1152);
      o[16 * half + 2 * i] = h2_as_u32(__hmul2(lo, d2));
      o[16 * half + 2 * i + 1] = h2_as_u32(__hmul2(hi, d2));
    }
  }
}

// Affine: words 8q .. 8q+7 of the row's 32-word chunk (128-byte swizzled
// box row, 16-byte unit u stored at u ^ swz).  sbw[j] = (scale, bias) fp16
// pair of the group of word j.
__device__ __forceinline__ void tb_affine_quarter(uint32_t src, uint32_t swz, int q,
                                                  const uint32_t (&sbw)[8], uint32_t (&o)[32]) {
  const uint4 v0 = lds128(src + 16 * ((2 * q) ^ swz));
  const uint4 v1 = lds128(src + 16 * ((2 * q + 1) ^ swz));
  const uint32_t wd[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  const __half2 kMul = u32_as_h2(0x2C003C00u);   // (1, 1/16)
  const __half2 kSub = u32_as_h2(0xD400E400u);   // (-1024, -64)
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const __half2 s2 = u32_as_h2(__byte_perm(sbw[j], 0, 0x1010));  // (s, s)
    const __half2 b2 = u32_as_h2(__byte_perm(sbw[j], 0, 0x3232));  // (b, b)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      // byte jj holds columns 2jj (low nibble) and 2jj+1 (high nibble)
      const uint32_t t = __byte_perm(wd[j], 0, jj * 0x1111);
      const __half2 v = u32_as_h2(lop3_and_or(t, 0x00F0000Fu, 0x64006400u));  // (1024+lo, 1024+16hi)
      const __half2 n = __hfma2(v, kMul, kSub);                                // (lo, hi), exact
      o[4 * j + jj] = h2_as_u32(__hfma2(n, s2, b2));
    }
  }
}

// ---------------------------------------------------------------------------

// Quarter Q of a chunk, dequantized into the 32 TMEM columns at `ta`.
template <int F, int GS, int Q>
__device__ __forceinline__ void tb_quarter(uint32_t src, uint32_t swz, const uint32_t (&sbv)[2], uint32_t ta) {
  uint32_t o[32];
  if constexpr (F == kFmtQ4_0) {
    tb_q4_0_quarter(src, Q, o);
  } else if constexpr (F == kFmtQ8_0) {
    tb_q8_0_quarter(src, Q, o);
  } else {
    uint32_t sbw[8];  // word j of the quarter covers quarter columns 8j .. 8j+7
#pragma unroll
    for (int j = 0; j < 8; ++j) sbw[j] = sbv[GS == 32 ? (j >= 4 ? 1 : 0) : 0];
    tb_affine_quarter(src, swz, Q, sbw, o);
  }
  uint32_t lo[16], hi[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    lo[j] = o[j];
    hi[j] = o[16 + j];
  }
  tmem_st16(ta, lo);
  tmem_st16(ta + 16, hi);
}

template <int F, int B, int GS>
__global__ void __launch_bounds__(kTbThreads, 1)
    gemv_tcb_kernel(const GemvParams p, const __grid_constant__ CUtensorMap wmap) {
  constexpr int CB = GemvFormat<F>::kChunkBytes;
  constexpr int SB = tb_stage_bytes<F>();
  constexpr int kProducerWarp = kTbDequantWarps;
  constexpr int kMmaWarp = kTbDequantWarps + 1;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int cs = p.cs;
  const int S = p.stages;
  const TbLayout L = tb_layout<F, B>(cs, S);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int crank = cs > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int cluster = blockIdx.x / cs;
  const int nclusters = gridDim.x / cs;
  const int nitems = cluster < p.num_rg ? (p.num_rg - 1 - cluster) / nclusters + 1 : 0;
  const int C = p.K / kChunkCols;
  const int c0 = (C * crank) / cs;
  const int cslice = (C * (crank + 1)) / cs - c0;
  const int total = nitems * cslice;

  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* full_w = bar;                  // [kTbMaxStages]
  uint64_t* empty_w = bar + 8;             // [kTbMaxStages]
  uint64_t* full_a = bar + 16;             // [group][2]
  uint64_t* empty_a = bar + 24;            // [group][2]
  uint64_t* d_full = bar + 32;             // [2]
  uint64_t* d_empty = bar + 34;            // [2]
  uint64_t* red_full = bar + 36;           // [2] leader: partial sums arrived
  uint64_t* red_empty = bar + 38;          // [2] others: leader consumed the buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 40);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar + 41);
  uint8_t* ring = smem + L.ring;
  float* slots = reinterpret_cast<float*>(smem + L.slots);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_w[s], 1);
      mbar_init(&empty_w[s], kTbDequantWarps + 1);  // dequant warps + the MMA commit (x half)
    }
    for (int a = 0; a < 2 * kTbGroups; ++a) {
      mbar_init(&full_a[a], 4);
      mbar_init(&empty_a[a], 1);
    }
    for (int d = 0; d < 2; ++d) {
      mbar_init(&d_full[d], 1);
      mbar_init(&d_empty[d], 4);
      mbar_init(&red_full[d], (cs - 1) * kTbRows);
      mbar_init(&red_empty[d], kTbRows);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTbTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  if (cs > 1) cluster_sync_all();  // peers' barriers exist before any remote arrive

  bool ok = true;
  auto fail_now = [&]() {
    ok = false;
    *abort_flag = 1;
    record_device_error(kDevErrBarrierTimeout);
  };
  auto wait = [&](uint64_t* b, uint32_t parity) {
    if (!ok) return;
    if (*abort_flag || !mbar_wait(b, parity)) fail_now();
  };

  if (warp == kProducerWarp) {
    // ---------------- TMA producer (weights only) ----------------
    if (lane == 0) {
      prefetch_tensor_map(&wmap);
      const uint64_t pol_w = l2_policy_evict_first();
      for (int t = 0; t < total && ok; ++t) {
        const int s = t % S;
        if (t >= S) wait(&empty_w[s], ((t / S) & 1) ^ 1);
        if (!ok) break;
        const int ii = t / cslice;
        const int row0 = (cluster + ii * nclusters) * kTbRows;
        const int chunk = c0 + (t - ii * cslice);
        mbar_arrive_expect_tx(&full_w[s], kTbRows * CB);
        tma_load_2d(ring + s * SB, &wmap, chunk * (CB / 8), row0, &full_w[s], pol_w);
      }
      // Copies still in flight must land before the CTA may exit.
      for (int t = max(0, total - S); t < total; ++t) (void)mbar_wait(&full_w[t % S], (t / S) & 1);
    }
    pdl_launch_dependents();
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int t = 0;
      for (int ii = 0; ii < nitems && ok; ++ii) {
        const int db = ii & 1;
        wait(&d_empty[db], ((ii >> 1) & 1) ^ 1);
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem + kTbDCol + kTbDCols * db;
        for (int cc = 0; cc < cslice && ok; ++cc, ++t) {
          const int s = t % S;
          const int j = t & 1;
          wait(&full_w[s], (t / S) & 1);
          const uint32_t xs = smem_addr(ring + s * SB + kTbRows * CB);
          for (int g = 0; g < kTbGroups && ok; ++g) {
            wait(&full_a[2 * g + j], (t >> 1) & 1);
            if (!ok) break;
            tc_fence_after_sync();
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int kk = g * 64 + k * 16;  // K offset in the chunk
              const uint64_t bdesc = smem_desc_kmajor(xs + (kk / 8) * 256, 256, 128);
              // accumulator (4g + k) % 8: its first MMA of the tile is at cc == 0, g < 2
              tc_mma_f16_ts(d_tmem + ((4 * g + k) & (kTbAcc - 1)) * kTbN, tmem + (2 * g + j) * kTbACols + k * 8,
                            bdesc, kTbIdesc, (cc > 0 || g >= 2) ? 1u : 0u);
            }
            tc_commit(&empty_a[2 * g + j]);
          }
          tc_commit(&empty_w[s]);
        }
        tc_commit(&d_full[db]);
      }
      // The last commit covers every MMA issued: wait for it before the
      // CTA may free its tensor memory.
      if (nitems > 0) (void)mbar_wait(&d_full[(nitems - 1) & 1], ((nitems - 1) >> 1) & 1);
    }
    pdl_launch_dependents();
  } else {
    // ---------------- dequantizers (warps 0-15) + epilogue (group 0) -------
    pdl_launch_dependents();
    const int group = warp >> 2;
    const int quad = warp & 3;
    const int rl = quad * 32 + lane;  // row within the tile = TMEM lane
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const int G = F == kFmtAffineQ4 ? p.K / GS : 0;
    pdl_wait_primary();  // x (and, for y, its readers) belong to the previous kernel
    // This thread's 16-byte unit of the group's x quarter: batch row xr,
    // 8-column group xg of the quarter.
    const int xu = quad * 32 + lane;
    const int xr = xu & 15;
    const int xg = xu >> 4;
    const __half* xsrc = p.x + (size_t)xr * p.K + group * 64 + xg * 8;
    const uint32_t xdst = (uint32_t)((group * 8 + xg) * 256 + xr * 16);
    auto load_x = [&](int cc) -> uint4 {
      if (xr >= p.nb) return make_uint4(0, 0, 0, 0);
      return __ldg(reinterpret_cast<const uint4*>(xsrc + (size_t)(c0 + cc) * kChunkCols));
    };
    uint4 xv = total > 0 ? load_x(0) : make_uint4(0, 0, 0, 0);
    int t = 0;
    for (int ii = 0; ii < nitems; ++ii) {
      const int row0 = (cluster + ii * nclusters) * kTbRows;
      const int row = row0 + rl;
      for (int cc = 0; cc < cslice; ++cc, ++t) {
        const int s = t % S;
        const int j = t & 1;
        const uint4 xnext = t + 1 < total ? load_x(cc + 1 == cslice ? 0 : cc + 1) : make_uint4(0, 0, 0, 0);
        // (scale, bias) of this group's quarter: one group, or two for GS = 32
        uint32_t sbv[2] = {0u, 0u};
        if constexpr (F == kFmtAffineQ4) {
          if (row < p.N) {
            const int gq = ((c0 + cc) * kChunkCols + group * 64) / GS;
#pragma unroll
            for (int h = 0; h < (GS == 32 ? 2 : 1); ++h) {
              const size_t gi = (size_t)row * G + gq + h;
              sbv[h] = (uint32_t)__half_as_ushort(p.scales[gi]) | ((uint32_t)__half_as_ushort(p.biases[gi]) << 16);
            }
          }
        }
        wait(&full_w[s], (t / S) & 1);
        wait(&empty_a[2 * group + j], ((t >> 1) & 1) ^ 1);
        tc_fence_after_sync();
        if (ok) {
          // x quarter for the tensor core: generic stores, then a proxy fence
          const uint32_t xa = smem_addr(ring + s * SB + kTbRows * CB) + xdst;
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(xa), "r"(xv.x), "r"(xv.y), "r"(xv.z),
                       "r"(xv.w)
                       : "memory");
          fence_proxy_async_smem();
          const uint32_t src = smem_addr(ring + s * SB) + rl * CB;
          const uint32_t ta = tmem + lane_base + (2 * group + j) * kTbACols;
          switch (group) {
            case 0: tb_quarter<F, GS, 0>(src, lane & 7, sbv, ta); break;
            case 1: tb_quarter<F, GS, 1>(src, lane & 7, sbv, ta); break;
            case 2: tb_quarter<F, GS, 2>(src, lane & 7, sbv, ta); break;
            default: tb_quarter<F, GS, 3>(src, lane & 7, sbv, ta); break;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty_w[s]);  // this warp is done with the weight bytes
          tmem_wait_st();
        }
        tc_fence_before_sync();
        __syncwarp();
        if (ok && lane == 0) mbar_arrive(&full_a[2 * group + j]);
        xv = xnext;
      }
      if (group != 0) continue;

      // ---- epilogue of row tile ii (group 0) ----
      const int db = ii & 1;
      wait(&d_full[db], (ii >> 1) & 1);
      tc_fence_after_sync();
      float acc[B];
#pragma unroll
      for (int b = 0; b < B; ++b) acc[b] = 0.f;
      if (ok) {
#pragma unroll
        for (int h = 0; h < kTbAcc / 2; ++h) {  // two accumulators per load
          uint32_t dv[32];
          tmem_ld32(tmem + lane_base + kTbDCol + kTbDCols * db + 32 * h, dv);
          tmem_wait_ld();
#pragma unroll
          for (int b = 0; b < B; ++b) acc[b] += __uint_as_float(dv[b]) + __uint_as_float(dv[16 + b]);
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&d_empty[db]);
      float* sl = slots + db * ((cs - 1) * B * kTbRows);
      if (cs > 1 && crank != 0) {
        if (ok && (*abort_flag || !mbar_wait_cluster(&red_empty[db], ((ii >> 1) & 1) ^ 1))) fail_now();
#pragma unroll
        for (int b = 0; b < B; ++b)
          st_cluster_f32(map_to_rank(sl + ((crank - 1) * B + b) * kTbRows + rl, 0), acc[b]);
        mbar_arrive_cluster(map_to_rank(&red_full[db], 0));
      } else {
        if (cs > 1) {
          if (ok && (*abort_flag || !mbar_wait_cluster(&red_full[db], (ii >> 1) & 1))) fail_now();
          for (int r = 1; r < cs; ++r) {
#pragma unroll
            for (int b = 0; b < B; ++b) acc[b] += sl[((r - 1) * B + b) * kTbRows + rl];
          }
          if (ii + 2 < nitems) {
            for (int r = 1; r < cs; ++r) mbar_arrive_cluster(map_to_rank(&red_empty[db], r));
          }
        }
        if (row < p.N) {
#pragma unroll
          for (int b = 0; b < B; ++b)
            if (b < p.nb) p.y[(size_t)b * p.N + row] = __float2half_rn(acc[b]);
        }
      }
    }
  }

  // Teardown: every role has finished (all waits are bounded).
  tc_fence_before_sync();
  __syncthreads();
  if (cs > 1) cluster_sync_all();
  if (warp == kMmaWarp) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kTbTmemCols);
  }
}

}  // namespace gdsq
