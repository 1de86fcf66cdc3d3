// Tensor-core (tcgen05) fused dequantize + GEMV for GGUF Q4_0, batch 1.
//
// Same result as kernel_fused_q4_0_gemv (gdsllm/runtime/fused_gemv.cu:27-105):
// y[r] = fp16( sum_b d[r][b] * sum_{j<32} (q[r][b][j] - 8) * x[32b + j] ),
// with fp32 accumulation.
//
// The CUDA cores only unpack nibbles; the multiply-accumulate runs on the
// tensor core:
//   * A operand (tensor memory): one CTA covers 128 output rows (TMEM lanes,
//     one warp per 32-lane quarter).  Each nibble pair becomes an exact fp16
//     pair with one LOP3: (1024 + n) for low nibbles, (1024 + 16 n) for high
//     nibbles (fp16's ulp in [1024, 2048) is 1).  A 32-weight block is 16
//     32-bit TMEM columns, written by tcgen05.st.
//   * B operand (shared memory, "block diagonal"): for the 8 blocks of a
//     256-column chunk, block j's activations sit in N-row j of a 16-row B
//     tile (other rows zero), high-nibble positions pre-scaled by 1/16.  One
//     fp32 D tile of 16 TMEM columns therefore collects the 8 per-block sums
//     D_j = sum (1024 + n) x_lo + sum (1024 + 16 n) x_hi / 16 in columns 0..7.
//   * Epilogue per block: sum (n - 8) x = D_j - (1032 X_lo + 72 X_hi), where
//     X_lo / X_hi are the fp32 sums of the block's activations at low / high
//     nibble positions (precomputed with the B tiles); then acc += d * (...).
// Activations and weights keep the reference's exact values; products are
// exact in fp32 and accumulate in fp32.
//
// Pipeline per CTA: a ring of weight stages (one 128-row x 144-byte TMA box
// per 256-column chunk, issued by thread 0, plus the chunk's 4 KB of B tiles);
// per chunk four pairs of blocks, each pair dequantized into one of two TMEM A
// buffers, then 4 MMAs (M=128, N=16, K=16) issued by thread 0 and committed to
// an mbarrier; the D tile of chunk c-1 is read while chunk c is processed.
// 128 TMEM columns per CTA (up to 4 CTAs per SM).  K is split across a
// cluster of cs CTAs; partial sums meet in the leader's shared memory.
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace gdsq {

constexpr int kTcRows = 128;                        // output rows per CTA (TMEM lanes)
constexpr int kTcThreads = 128;                     // 4 warps, one per lane quarter
constexpr int kTcTmemCols = 128;                    // allocation per CTA (<= 4 CTAs per SM)
constexpr int kTcACol = 0;                          // A: 2 buffers x 32 columns (a pair of blocks each)
constexpr int kTcDCol = 64;                         // D: 2 buffers x 16 columns (one chunk each)
constexpr int kTcChunkBytes = 144;                  // one Q4_0 row chunk (8 blocks)
constexpr int kTcStageBytes = kTcRows * kTcChunkBytes;  // 18432, a multiple of 128
constexpr int kTcBChunkBytes = 8 * 2 * 2 * 128;    // B tiles per chunk: 8 blocks x 2 MMAs x 2 core matrices
constexpr int kTcMinSmem = 46 * 1024;               // 5 CTAs never fit: at most 4 x 128 TMEM columns per SM

// Instruction descriptor, kind::f16: D = F32 (bits 4-5 = 1), A = B = F16
// (bits 7-9, 10-12 = 0), both K-major (bits 15, 16 = 0), N = 16 (bits 17-22
// = N >> 3 = 2), M = 128 (bits 24-28 = M >> 4 = 8).
constexpr uint32_t kTcIdesc = (1u << 4) | (2u << 17) | (8u << 24);

struct TcLayout {
  int ring;    // weight stages
  int btile;   // B tiles, one 4 KB set per stage
  int bzero;   // 256 zero bytes (the unused 8-row group of every B tile)
  int xc;      // compact staged activations of the K slice: 64 B per block
  int corr;    // per-block correction 1032 X_lo + 72 X_hi
  int slots;   // cluster partial sums (leader)
  int total;   // bytes to request (>= kTcMinSmem)
  int cmax;    // largest chunk count of a K slice
};

__host__ __device__ inline TcLayout tc_layout(int K, int cs, int stages) {
  TcLayout L;
  const int C = K / kChunkCols;
  L.cmax = (C + cs - 1) / cs;
  int off = 1024;  // mbarriers, TMEM address slot
  L.ring = off;
  off += stages * kTcStageBytes;
  L.btile = off;
  off += stages * kTcBChunkBytes;
  L.bzero = off;
  off += 256;
  L.xc = off;
  off += L.cmax * 8 * 64;
  L.corr = off;
  off += L.cmax * 8 * 4;
  L.slots = off;
  if (cs > 1) off += cs * kTcRows * 4;
  off += 1024;  // slack to align the base at run time
  L.total = off < kTcMinSmem ? kTcMinSmem : off;
  return L;
}

// Stage the CTA's K slice of x compactly (64 B per 32-column block: for qs
// word i, 16 bytes = (x[4i], x[4i+2]), (x[16+4i], x[18+4i]) / 16,
// (x[4i+1], x[4i+3]), (x[17+4i], x[19+4i]) / 16 -- the dequantizer's pair
// order, high-nibble positions scaled by 1/16) and the per-block corrections;
// zero the B tiles and the zero block.
__device__ __forceinline__ void tc_stage_x(const __half* __restrict__ x, uint8_t* xc, float* corr,
                                           uint8_t* btile, int btile_bytes, uint8_t* bzero, int col0,
                                           int nchunks) {
  uint4* z = reinterpret_cast<uint4*>(btile);
  for (int i = threadIdx.x; i < btile_bytes / 16; i += blockDim.x) z[i] = make_uint4(0, 0, 0, 0);
  uint4* zz = reinterpret_cast<uint4*>(bzero);
  if (threadIdx.x < 16) zz[threadIdx.x] = make_uint4(0, 0, 0, 0);
  const __half2 k16th = __floats2half2_rn(0.0625f, 0.0625f);
  const int nblk = nchunks * 8;
  for (int jb = threadIdx.x; jb < nblk; jb += blockDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(x + col0 + jb * 32);
    uint32_t h[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = src[j];
      h[4 * j] = v.x; h[4 * j + 1] = v.y; h[4 * j + 2] = v.z; h[4 * j + 3] = v.w;
    }
    float xlo = 0.f, xhi = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 a = __half22float2(u32_as_h2(h[k]));
      const float2 b = __half22float2(u32_as_h2(h[8 + k]));
      xlo += a.x + a.y;
      xhi += b.x + b.y;
    }
    corr[jb] = fmaf(1032.f, xlo, 72.f * xhi);
    uint4* dst = reinterpret_cast<uint4*>(xc + jb * 64);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 o;
      o.x = __byte_perm(h[2 * i], h[2 * i + 1], 0x5410);
      o.y = h2_as_u32(__hmul2(u32_as_h2(__byte_perm(h[8 + 2 * i], h[9 + 2 * i], 0x5410)), k16th));
      o.z = __byte_perm(h[2 * i], h[2 * i + 1], 0x7632);
      o.w = h2_as_u32(__hmul2(u32_as_h2(__byte_perm(h[8 + 2 * i], h[9 + 2 * i], 0x7632)), k16th));
      dst[i] = o;
    }
  }
}

// B tile of one 256-column chunk: core matrix (block j, MMA half kk, K unit
// u) at ((j * 2 + kk) * 2 + u) * 128; its row j holds unit (word 2 kk + u) of
// block j, the other rows stay zero.  Warp-wide: lane = block * 4 + word.
__device__ __forceinline__ void tc_fill_btile(uint32_t btile_a, uint32_t xc_a, int chunk, int lane) {
  const int j = lane >> 2;
  const int i = lane & 3;
  const uint4 v = lds128(xc_a + (chunk * 8 + j) * 64 + i * 16);
  const uint32_t dst = btile_a + ((j * 2 + (i >> 1)) * 2 + (i & 1)) * 128 + 16 * j;
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__global__ void __launch_bounds__(kTcThreads, 1)
    gemv_tc_q4_0_kernel(const GemvParams p, const __grid_constant__ CUtensorMap wmap) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int cs = p.cs;
  const int S = p.stages;
  const TcLayout L = tc_layout(p.K, cs, S);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int crank = cs > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int row0 = (blockIdx.x / cs) * kTcRows;
  const int C = p.K / kChunkCols;
  const int c0 = (C * crank) / cs;
  const int nc = (C * (crank + 1)) / cs - c0;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [kMaxStages]
  uint64_t* mma_done = full + kMaxStages;               // [2], one per A buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 2);
  uint8_t* ring = smem + L.ring;
  float* corr = reinterpret_cast<float*>(smem + L.corr);
  float* slots = reinterpret_cast<float*>(smem + L.slots);
  const uint64_t policy = l2_policy_evict_first();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
    mbar_init(&mma_done[0], 1);
    mbar_init(&mma_done[1], 1);
    fence_barrier_init();
    prefetch_tensor_map(&wmap);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  // Weights do not depend on the previous kernel: start streaming them now.
  int issued = 0;
  auto issue = [&](int c) {  // thread 0 only
    const int st = c % S;
    mbar_arrive_expect_tx(&full[st], kTcStageBytes);
    tma_load_2d(ring + st * kTcStageBytes, &wmap, (c0 + c) * (kTcChunkBytes / 8), row0, &full[st], policy);
  };
  if (threadIdx.x == 0)
    for (; issued < min(S, nc); ++issued) issue(issued);
  pdl_launch_dependents();

  pdl_wait_primary();  // activations are produced by the previous kernel
  tc_stage_x(p.x, smem + L.xc, corr, smem + L.btile, S * kTcBChunkBytes, smem + L.bzero,
             c0 * kChunkCols, nc);
  if (cs > 1) cluster_sync_all();
  __syncthreads();

  const uint32_t lane_tm = tmem + (static_cast<uint32_t>(warp * 32) << 16);  // this warp's lane quarter
  const uint32_t ring_a = smem_addr(ring) + (warp * 32 + lane) * kTcChunkBytes;
  const uint32_t btile_a = smem_addr(smem + L.btile);
  const uint32_t bzero_a = smem_addr(smem + L.bzero);
  const uint32_t xc_a = smem_addr(smem + L.xc);

  float acc = 0.f;
  float dprev[8];
  bool ok = true;
  int stage = 0;
  uint32_t phase = 0;

  auto readout = [&](int c) {  // D tile of chunk c -> acc (all threads)
    uint32_t dv[8];
    tmem_ld8(lane_tm + kTcDCol + (c & 1) * 16, dv);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 8; ++j) acc = fmaf(dprev[j], __uint_as_float(dv[j]) - corr[c * 8 + j], acc);
  };
  auto wait_mma = [&](int buf, uint32_t parity) {
    if (!mbar_wait(&mma_done[buf], parity)) {
      ok = false;
      record_device_error(kDevErrBarrierTimeout);
    }
    tc_fence_after_sync();
  };

  for (int c = 0; c < nc; ++c) {
    if (ok && !mbar_wait(&full[stage], phase)) {
      ok = false;
      record_device_error(kDevErrBarrierTimeout);
    }
    uint32_t w[36];
    const uint32_t src = ring_a + stage * kTcStageBytes;
#pragma unroll
    for (int j = 0; j < 9; ++j) {
      const uint4 v = lds128(src + 16 * j);
      w[4 * j] = v.x; w[4 * j + 1] = v.y; w[4 * j + 2] = v.z; w[4 * j + 3] = v.w;
    }
    const uint32_t bt = btile_a + stage * kTcBChunkBytes;
    float dcur[8];
#pragma unroll
    for (int pr = 0; pr < 4; ++pr) {
      // Pair t = 4c + pr uses A buffer pr & 1; its previous user was pair t-2,
      // whose completion is the (t/2 - 1)-th commit on that buffer.
      const int t = 4 * c + pr;
      if (t >= 2) wait_mma(pr & 1, ((t >> 1) - 1) & 1);
      if (pr == 0 && warp == 0) {
        // Every MMA issued before pair t-2 has completed, including those of
        // chunk c - S that read this stage's B tile: refill its diagonal.
        tc_fill_btile(bt, xc_a, c, lane);
        fence_proxy_async_smem();
      }
      if (pr == 1 && c > 0) readout(c - 1);  // pair t-2 was chunk c-1's last
#pragma unroll
      for (int bq = 0; bq < 2; ++bq) {
        const int blk = 2 * pr + bq;
        const int o = 18 * blk;
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
        dcur[blk] = __half2float(__ushort_as_half(static_cast<unsigned short>(d16)));
        uint32_t a[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) unpack_nibbles_biased(q[i], &a[4 * i]);
        tmem_st16(lane_tm + kTcACol + (pr & 1) * 32 + bq * 16, a);
      }
      tmem_wait_st();
      tc_fence_before_sync();
      named_barrier_sync(1, kTcThreads);  // all 128 rows of this pair's A are in TMEM
      if (threadIdx.x == 0) {
        tc_fence_after_sync();
        const uint32_t d_tm = tmem + kTcDCol + (c & 1) * 16;
#pragma unroll
        for (int bq = 0; bq < 2; ++bq) {
          const int j = 2 * pr + bq;
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const uint32_t cm = bt + (j * 2 + kk) * 256;
            const uint64_t desc = smem_desc_kmajor(cm, 128, bzero_a - cm);
            tc_mma_f16_ts(d_tm, tmem + kTcACol + (pr & 1) * 32 + bq * 16 + kk * 8, desc, kTcIdesc,
                          (pr | bq | kk) ? 1u : 0u);
          }
        }
        tc_commit(&mma_done[pr & 1]);
        // Every warp read this weight stage before the barrier: refill it.
        if (pr == 3 && issued < nc) issue(issued++);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) dprev[j] = dcur[j];
    if (++stage == S) {
      stage = 0;
      phase ^= 1;
    }
  }
  if (nc > 0) {
    const int t = 4 * nc - 1;  // last pair, buffer 1
    wait_mma(1, (t >> 1) & 1);
    readout(nc - 1);
  }

  // Cluster reduction: rank r's partial row sums go to the leader's slots.
  const int row = row0 + warp * 32 + lane;
  if (cs == 1) {
    if (row < p.N) p.y[row] = __float2half_rn(acc);
  } else {
    st_cluster_f32(map_to_rank(slots + crank * kTcRows + threadIdx.x, 0), acc);
    cluster_sync_all();
    if (crank == 0 && row < p.N) {
      float v = 0.f;
      for (int r = 0; r < cs; ++r) v += slots[r * kTcRows + threadIdx.x];
      p.y[row] = __float2half_rn(v);
    }
  }

  if (!ok) {
    // Wait (bounded) for weight copies that may still be in flight.
    for (int j = 0; j < S; ++j) (void)mbar_wait(&full[j], 0);
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kTcTmemCols);
  }
}

}  // namespace gdsq
