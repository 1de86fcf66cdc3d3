// Fused mixture-of-experts gather over affine-Q4 experts, for decode.
//
// Replaces the per-slot decode loop of moe_mlp_selective
// (gdsllm/runtime/qwen_moe.py:453-474).  The reference, for each of the
// top-k slots, reads the expert id back to the host (`.item()`), runs three
// fused GEMVs (affine_q4_dequant.cu:79-158) and does SiLU, the product and
// the routing-weighted sum as separate torch ops.  Here, for token b and
// slot t with expert e = ids[b][t] (device memory, never read by the host):
//
//   stage 0:  h[b][t] = fp16( silu(fp16(gate_e . x_b)) * fp16(up_e . x_b) )
//   stage 1:  y[b]    = sum_t  w[b][t] * (down_e . h[b][t])      (fp32 sum)
//
// with silu(v) = v / (1 + exp(-v)) evaluated in fp32 on the fp16 value, the
// rounding sequence of F.silu(gate_out) * up_out on fp16 tensors.  Stage 1
// keeps the slot sum in fp32 and rounds once; the reference rounds every
// slot's product and running sum to fp16 (qwen_moe.py:474).
//
// Experts are stacked [E][rows][K/8] uint32 words with [E][rows][K/GS] fp16
// scales and biases (the layer-file layout, convert_qwen_moe.py:205-253).
// Only experts [e_first, e_first + e_count) are resident (expert parallelism:
// each rank holds a contiguous range); slots whose expert lives elsewhere are
// skipped, so stage 1 yields this rank's partial sum.  Optionally the shared
// expert (qwen_moe.py:497-510; separate [1][rows][K/8] tensors) rides along
// as one more slot per token, weighted by sigmoid(x . g) supplied per token,
// so one pair of launches computes the whole MoE MLP.
//
// Schedule (same machinery as the dense fast GEMV in gemv.cuh):
//   * Work item = 32 output lanes.  Stage 0: rows [r0, r0+16) of gate (lanes
//     0..15) and of up (lanes 16..31) for one (token, slot) pair, so the SiLU
//     product is formed in the epilogue of the item that computed both.
//     Stage 1: rows [r0, r0+32) of down for one token, K running over the
//     token's T slots back to back (chunk c belongs to slot c / (K/256)).
//   * K is split across a thread-block cluster (cs CTAs, DSMEM reduction to
//     the leader); each warp streams its 256-column chunks through a private
//     ring fed by 3-D TMA boxes whose z coordinate is the local expert index.
//     Chunks of non-resident experts are never fetched.
//   * Activations (x of the token, or h of the token's slots) are staged in
//     shared memory once per token, as scaled fp32 in the dequantizer's field
//     order; products and sums are fp32 (gemv.cuh, "Exact fp32 products").
#pragma once

#include "gemv.cuh"

namespace gdsq {

constexpr int kMoeMaxSlots = 64;           // top-k limit of one token
constexpr int kMoeChunkBytes = 128;        // one 256-column chunk of one row
constexpr int kMoeStageBytes = 32 * kMoeChunkBytes;
enum : int { kMoeOutF32 = 1, kMoeAccumulate = 2, kMoeClamp = 4 };
constexpr int kMoeShared = -2;             // slot code of the shared expert

struct MoeParams {
  const __half* s0;     // scales of matrix 0 (gate in stage 0, down in stage 1)
  const __half* b0;     // biases of matrix 0
  const __half* s1;     // scales of matrix 1 (up; stage 0 only)
  const __half* b1;
  const __half* x;      // stage 0: tokens [ntok][K]; stage 1: h [ntok][T][K]
  const int* ids;       // [ntok][T] global expert ids
  const __half* route;  // [ntok][T] routing weights (stage 1)
  void* out;            // stage 0: h fp16 [ntok][T][rows]; stage 1: y [ntok][rows]
  int ntok;
  int T;
  int e_first;          // first resident expert
  int e_count;          // resident experts
  int e_total;          // valid ids are 0 .. e_total-1
  int rows;             // rows of one expert matrix
  int K;                // columns of one expert matrix
  int cs;
  int stages;
  int num_items;
  int flags;            // stage 1: kMoeOutF32 | kMoeAccumulate | kMoeClamp
  // Shared expert (has_shared != 0): slot T of every token.
  int has_shared;
  int Ts;               // slots per token in h and in stage 1's K: T + has_shared
  const __half* ss0;    // its scales / biases of matrix 0 [1][rows][K/GS]
  const __half* sb0;
  const __half* ss1;    // matrix 1 (stage 0)
  const __half* sb1;
  const __half* shared_route;  // [ntok] fp16 weight of the shared slot (stage 1)
  // Stage 1, fp16 output: y = residual + fp16(result) in fp16 (the caller's
  // `x + moe(x)`, qwen_moe.py's residual add, in the same two roundings).
  const __half* residual;
  // Generic kernels only: packed words of the matrices (the fast kernels
  // read them through tensor maps).
  const uint32_t* w0;
  const uint32_t* w1;
  const uint32_t* sw0;
  const uint32_t* sw1;
  int group;
};

struct MoeSmemLayout {
  int ring;
  int xs;
  int xsum;
  int sb;
  int sb_stride;
  int red;
  int slots;
  int fin;
  int slot_tab;
  int total;
  int kslice;
};

// `C` = 256-column chunks of one item's K (stage 0: K/256; stage 1: T*K/256).
__host__ __device__ inline MoeSmemLayout moe_smem_layout(int C, int gs, int cs, int stages) {
  MoeSmemLayout L;
  L.kslice = (C + cs - 1) / cs * kChunkCols;
  int off = 1024;  // mbarriers; the ring starts 1024-aligned (128-byte swizzle)
  L.ring = off;
  off += kGemvWarps * stages * kMoeStageBytes;
  L.xs = off;
  off += L.kslice * 4;  // scaled fp32 activations (gemv.cuh, stage_x_affine)
  L.xsum = off;
  const int gsl = L.kslice / gs;
  off += gsl * 4;
  L.sb = off;
  L.sb_stride = gsl | 1;
  off += 32 * L.sb_stride * 4;
  L.red = off;
  off += 2 * kGemvWarps * 32 * 4;
  L.slots = off;
  if (cs > 1) off += 2 * cs * 32 * 4;
  L.fin = off;
  off += 32 * 4;
  L.slot_tab = off;
  off += kMoeMaxSlots * 8;
  L.total = off + 1024;
  return L;
}

// Local index of the expert of (token, slot) pair q, or -1 when it is not
// resident.  Ids outside 0..e_total-1 set kDevErrBadIndex and are skipped.
__device__ __forceinline__ int moe_local_expert(const MoeParams& p, int q) {
  const int e = p.ids[q];
  if (e < 0 || e >= p.e_total) {
    record_device_error(kDevErrBadIndex);
    return -1;
  }
  const int z = e - p.e_first;
  return (z >= 0 && z < p.e_count) ? z : -1;
}

// Local expert of slot t of token tok: >= 0 routed, kMoeShared, or -1.
__device__ __forceinline__ int moe_slot_expert(const MoeParams& p, int tok, int t) {
  if (t >= p.T) return kMoeShared;
  return moe_local_expert(p, tok * p.T + t);
}

__device__ __forceinline__ float moe_finish(float v, int flags) {
  return (flags & kMoeClamp) ? fminf(fmaxf(v, -65504.0f), 65504.0f) : v;
}

template <int STAGE, int GS>
__global__ void __launch_bounds__(kGemvWarps * 32)
    moe_affine_kernel(const MoeParams p, const __grid_constant__ CUtensorMap map0,
                      const __grid_constant__ CUtensorMap map1, const __grid_constant__ CUtensorMap smap0,
                      const __grid_constant__ CUtensorMap smap1) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int cs = p.cs;
  const int S = p.stages;
  const int cpe = p.K / kChunkCols;               // chunks per expert row
  const int C = STAGE == 0 ? cpe : p.Ts * cpe;    // chunks per item
  const int Kx = STAGE == 0 ? p.K : p.Ts * p.K;   // activation columns per token
  const MoeSmemLayout L = moe_smem_layout(C, GS, cs, S);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int crank = cs > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int cluster = blockIdx.x / cs;
  const int nclusters = gridDim.x / cs;
  const int nitems = cluster < p.num_items ? (p.num_items - 1 - cluster) / nclusters + 1 : 0;
  const int rgs = STAGE == 0 ? p.rows / 16 : p.rows / 32;  // items per pair (stage 0) / token

  const int c0 = (C * crank) / cs;
  const int cslice = (C * (crank + 1)) / cs - c0;
  const int per_warp = (cslice + kGemvWarps - 1) / kGemvWarps;
  const int wc0 = min(cslice, warp * per_warp);
  const int mw = min(cslice, wc0 + per_warp) - wc0;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * kMaxStages;
  uint8_t* ring = smem + L.ring + warp * (S * kMoeStageBytes);
  uint8_t* xs = smem + L.xs;
  float* xsum = reinterpret_cast<float*>(smem + L.xsum);
  uint32_t* sb = reinterpret_cast<uint32_t*>(smem + L.sb);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* slots = reinterpret_cast<float*>(smem + L.slots);
  float* fin = reinterpret_cast<float*>(smem + L.fin);
  int* slot_z = reinterpret_cast<int*>(smem + L.slot_tab);
  float* slot_w = reinterpret_cast<float*>(smem + L.slot_tab + kMoeMaxSlots * 4);
  const uint32_t ring_a = smem_addr(ring) + lane * kMoeChunkBytes;
  const uint64_t policy = l2_policy_evict_first();

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    if (warp == 0) {
      prefetch_tensor_map(&map0);
      if (STAGE == 0) prefetch_tensor_map(&map1);
      if (p.has_shared) {
        prefetch_tensor_map(&smap0);
        if (STAGE == 0) prefetch_tensor_map(&smap1);
      }
    }
  }
  __syncwarp();
  if (cs > 1) cluster_arrive_relaxed();  // waited for before the first DSMEM store
  bool peers_waited = false;

  // Expert ids (and, for stage 1, h) come from earlier kernels.
  pdl_wait_primary();

  // Producer cursor over this warp's tasks (item ordinal, warp-local chunk);
  // tasks of non-resident experts are skipped identically by the consumer.
  int p_ii = 0, p_j = 0, p_stage = 0;
  auto seek = [&]() -> int {
    while (p_ii < nitems) {
      if (p_j >= mw) {
        p_j = 0;
        ++p_ii;
        continue;
      }
      const int it = cluster + p_ii * nclusters;
      const int z = STAGE == 0 ? moe_slot_expert(p, (it / rgs) / p.Ts, (it / rgs) % p.Ts)
                               : moe_slot_expert(p, it / rgs, (c0 + wc0 + p_j) / cpe);
      if (z != -1) return z;
      if (STAGE == 0) {
        p_j = 0;
        ++p_ii;
      } else {
        ++p_j;
      }
    }
    return -1;
  };
  auto issue_next = [&]() -> bool {
    const int zs = seek();
    if (zs == -1) return false;
    const bool shared = zs == kMoeShared;
    const int z = shared ? 0 : zs;
    const int it = cluster + p_ii * nclusters;
    const int chunk = c0 + wc0 + p_j;
    if (lane == 0) {
      uint8_t* dst = ring + p_stage * kMoeStageBytes;
      mbar_arrive_expect_tx(&bars[p_stage], kMoeStageBytes);
      if constexpr (STAGE == 0) {
        const int row0 = (it % rgs) * 16;
        tma_load_3d(dst, shared ? &smap0 : &map0, chunk * (kMoeChunkBytes / 8), row0, z, &bars[p_stage], policy);
        tma_load_3d(dst + 16 * kMoeChunkBytes, shared ? &smap1 : &map1, chunk * (kMoeChunkBytes / 8), row0, z,
                    &bars[p_stage], policy);
      } else {
        const int row0 = (it % rgs) * 32;
        tma_load_3d(dst, shared ? &smap0 : &map0, (chunk % cpe) * (kMoeChunkBytes / 8), row0, z, &bars[p_stage],
                    policy);
      }
    }
    ++p_j;
    if (++p_stage == S) p_stage = 0;
    return true;
  };

  int issued = 0;
  for (int t = 0; t < S; ++t) {
    if (!issue_next()) break;
    ++issued;
  }
  pdl_launch_dependents();

  const int gsl = cslice * kChunkCols / GS;   // groups in this CTA's slice
  const int gbase = c0 * (kChunkCols / GS);   // first of them, item-relative
  const int G = p.K / GS;                     // groups per expert row
  const int ld = L.kslice;
  const uint32_t xs_a = smem_addr(xs);
  const uint32_t xsum_a = smem_addr(xsum);
  const uint32_t sb_a = smem_addr(sb) + lane * L.sb_stride * 4;

  bool ok = true;
  int fail_stage = 0, fail_pending = 0;
  uint32_t fail_phase = 0;
  int consumed = 0;
  int stage = 0;
  uint32_t phase = 0;
  int done = 0;
  int staged_tok = -1;

  for (int ii = 0; ii < nitems; ++ii) {
    const int it = cluster + ii * nclusters;
    int tok, row0, pair = 0, zi = 0;
    if constexpr (STAGE == 0) {
      pair = it / rgs;
      tok = pair / p.Ts;
      row0 = (it % rgs) * 16;
      zi = moe_slot_expert(p, tok, pair % p.Ts);
      if (zi == -1) continue;  // uniform over the cluster
    } else {
      tok = it / rgs;
      row0 = (it % rgs) * 32;
    }
    __syncthreads();  // the previous item's readers of xs / sb / slot tables are done
    if (tok != staged_tok) {
      stage_x_affine<GS>(p.x + (size_t)tok * Kx, xs, xsum, 1, 1, Kx, c0 * kChunkCols,
                         cslice * kChunkCols, ld);
      if constexpr (STAGE == 1) {
        for (int t = threadIdx.x; t < p.Ts; t += blockDim.x) {
          slot_z[t] = moe_slot_expert(p, tok, t);
          slot_w[t] = __half2float(t < p.T ? p.route[tok * p.T + t] : p.shared_route[tok]);
        }
      }
      staged_tok = tok;
    }
    if constexpr (STAGE == 1) __syncthreads();  // slot_z is read below
    for (int idx = threadIdx.x; idx < 32 * gsl; idx += blockDim.x) {
      const int r = idx / gsl;
      const int g = idx - r * gsl;
      uint32_t v = 0;
      if constexpr (STAGE == 0) {
        const bool sh = zi == kMoeShared;
        const __half* sc = r < 16 ? (sh ? p.ss0 : p.s0) : (sh ? p.ss1 : p.s1);
        const __half* bi = r < 16 ? (sh ? p.sb0 : p.b0) : (sh ? p.sb1 : p.b1);
        const size_t gi = ((size_t)(sh ? 0 : zi) * p.rows + row0 + (r & 15)) * G + gbase + g;
        v = (uint32_t)__half_as_ushort(sc[gi]) | ((uint32_t)__half_as_ushort(bi[gi]) << 16);
      } else {
        const int gg = gbase + g;          // group index over the token's T*K columns
        const int t = gg / G;
        const int z = slot_z[t];
        if (z != -1) {
          const bool sh = z == kMoeShared;
          const size_t gi = ((size_t)(sh ? 0 : z) * p.rows + row0 + r) * G + (gg - t * G);
          const __half* sc = sh ? p.ss0 : p.s0;
          const __half* bi = sh ? p.sb0 : p.b0;
          v = (uint32_t)__half_as_ushort(sc[gi]) | ((uint32_t)__half_as_ushort(bi[gi]) << 16);
        }
      }
      sb[r * L.sb_stride + g] = v;
    }
    __syncthreads();

    float acc[1] = {0.f};
    for (int j = 0; j < mw; ++j) {
      const int cl = wc0 + j;  // slice-local chunk
      float wt = 1.f;
      if constexpr (STAGE == 1) {
        const int t = (c0 + cl) / cpe;
        if (slot_z[t] == -1) continue;
        wt = slot_w[t];
      }
      if (ok && !mbar_wait(&bars[stage], phase)) {
        ok = false;
        fail_stage = stage;
        fail_phase = phase;
        fail_pending = issued - consumed;
      }
      ++consumed;
      if (ok) {
        const uint32_t src = ring_a + stage * kMoeStageBytes;
        if constexpr (STAGE == 0) {
          chunk_affine<1, GS>(src, lane & 7, xs_a + cl * (kChunkCols * 4), 0, xsum_a, 0, sb_a,
                              cl * (kChunkCols / GS), acc);
        } else {
          float part[1] = {0.f};
          chunk_affine<1, GS>(src, lane & 7, xs_a + cl * (kChunkCols * 4), 0, xsum_a, 0, sb_a,
                              cl * (kChunkCols / GS), part);
          acc[0] = fmaf(wt, part[0], acc[0]);
        }
      }
      __syncwarp();
      if (ok && issue_next()) ++issued;
      if (++stage == S) {
        stage = 0;
        phase ^= 1;
      }
    }

    // Reduce the 4 warps, then the cs CTAs of the cluster, into fin[0..31].
    float* rd = red + (done & 1) * (kGemvWarps * 32);
    rd[warp * 32 + lane] = acc[0] * kUnscale;  // partial sums ran in units of 2^-39
    if (cs > 1 && !peers_waited) {
      cluster_wait();  // every peer is running: DSMEM stores are safe
      peers_waited = true;
    }
    __syncthreads();
    float* sl = slots + (done & 1) * (cs * 32);
    if (threadIdx.x < 32) {
      const int l = threadIdx.x;
      const float v = (rd[l] + rd[32 + l]) + (rd[64 + l] + rd[96 + l]);
      if (cs == 1) fin[l] = v;
      else st_cluster_f32(map_to_rank(sl + crank * 32 + l, 0), v);
    }
    if (cs > 1) cluster_sync_all();
    if (crank == 0) {
      if (cs > 1 && threadIdx.x < 32) {
        float v = 0.f;
        for (int r = 0; r < cs; ++r) v += sl[r * 32 + threadIdx.x];
        fin[threadIdx.x] = v;
      }
      __syncthreads();
      if constexpr (STAGE == 0) {
        if (threadIdx.x < 16) {
          const int l = threadIdx.x;
          const float g = __half2float(__float2half_rn(fin[l]));
          const __half u = __float2half_rn(fin[16 + l]);
          const __half sg = __float2half_rn(g / (1.0f + expf(-g)));
          __half* h = static_cast<__half*>(p.out);
          h[(size_t)pair * p.rows + row0 + l] = __float2half_rn(__half2float(sg) * __half2float(u));
        }
      } else {
        if (threadIdx.x < 32) {
          const size_t o = (size_t)tok * p.rows + row0 + threadIdx.x;
          const float v = fin[threadIdx.x];
          if (p.flags & kMoeOutF32) {
            float* y = static_cast<float*>(p.out);
            y[o] = moe_finish((p.flags & kMoeAccumulate) ? y[o] + v : v, p.flags);
          } else {
            __half* y = static_cast<__half*>(p.out);
            const __half r = __float2half_rn(moe_finish((p.flags & kMoeAccumulate) ? __half2float(y[o]) + v : v,
                                                        p.flags));
            y[o] = p.residual ? __hadd(p.residual[o], r) : r;
          }
        }
      }
    }
    ++done;
  }

  if (cs > 1 && !peers_waited) cluster_wait();  // pairs the early arrive
  if (!ok) {
    if (lane == 0) record_device_error(kDevErrBarrierTimeout);
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
// Generic kernels (any K % group == 0, group % 8 == 0, 4-byte aligned words):
// one warp per output, plain loads.

__device__ __forceinline__ float moe_row_dot(const uint32_t* w, const __half* s, const __half* b,
                                             const __half* x, int K, int group, int lane) {
  float acc = 0.f;
  for (int wd = lane; wd < K / 8; wd += 32) {
    const int g = (wd * 8) / group;
    const float sc = __half2float(s[g]);
    const float bi = __half2float(b[g]);
    const uint32_t packed = w[wd];
#pragma unroll
    for (int n = 0; n < 8; ++n) acc = fmaf(fmaf(float((packed >> (4 * n)) & 15u), sc, bi), __half2float(x[wd * 8 + n]), acc);
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
  return acc;
}

// Stage 0: warp per (pair, row).
__global__ void __launch_bounds__(256) moe_gate_up_generic_kernel(const MoeParams p) {
  const int lane = threadIdx.x & 31;
  const long long gw = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  pdl_launch_dependents();
  pdl_wait_primary();
  if (gw >= (long long)p.ntok * p.Ts * p.rows) return;
  const int pair = static_cast<int>(gw / p.rows);
  const int row = static_cast<int>(gw - (long long)pair * p.rows);
  const int z = moe_slot_expert(p, pair / p.Ts, pair % p.Ts);
  if (z == -1) return;
  const bool sh = z == kMoeShared;
  const int G = p.K / p.group;
  const size_t r = (size_t)(sh ? 0 : z) * p.rows + row;
  const __half* x = p.x + (size_t)(pair / p.Ts) * p.K;
  const float g = moe_row_dot((sh ? p.sw0 : p.w0) + r * (p.K / 8), (sh ? p.ss0 : p.s0) + r * G,
                              (sh ? p.sb0 : p.b0) + r * G, x, p.K, p.group, lane);
  const float u = moe_row_dot((sh ? p.sw1 : p.w1) + r * (p.K / 8), (sh ? p.ss1 : p.s1) + r * G,
                              (sh ? p.sb1 : p.b1) + r * G, x, p.K, p.group, lane);
  if (lane == 0) {
    const float gh = __half2float(__float2half_rn(g));
    const __half sg = __float2half_rn(gh / (1.0f + expf(-gh)));
    static_cast<__half*>(p.out)[(size_t)pair * p.rows + row] =
        __float2half_rn(__half2float(sg) * __half2float(__float2half_rn(u)));
  }
}

// Stage 1: warp per (token, row).
__global__ void __launch_bounds__(256) moe_down_generic_kernel(const MoeParams p) {
  const int lane = threadIdx.x & 31;
  const long long gw = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  pdl_launch_dependents();
  pdl_wait_primary();
  if (gw >= (long long)p.ntok * p.rows) return;
  const int tok = static_cast<int>(gw / p.rows);
  const int row = static_cast<int>(gw - (long long)tok * p.rows);
  const int G = p.K / p.group;
  float acc = 0.f;
  for (int t = 0; t < p.Ts; ++t) {
    const int z = moe_slot_expert(p, tok, t);
    if (z == -1) continue;
    const bool sh = z == kMoeShared;
    const size_t r = (size_t)(sh ? 0 : z) * p.rows + row;
    const float d = moe_row_dot((sh ? p.sw0 : p.w0) + r * (p.K / 8), (sh ? p.ss0 : p.s0) + r * G,
                                (sh ? p.sb0 : p.b0) + r * G, p.x + ((size_t)tok * p.Ts + t) * p.K, p.K, p.group,
                                lane);
    const float wt = __half2float(t < p.T ? p.route[tok * p.T + t] : p.shared_route[tok]);
    acc = fmaf(wt, d, acc);
  }
  if (lane == 0) {
    const size_t o = (size_t)tok * p.rows + row;
    if (p.flags & kMoeOutF32) {
      float* y = static_cast<float*>(p.out);
      y[o] = moe_finish((p.flags & kMoeAccumulate) ? y[o] + acc : acc, p.flags);
    } else {
      __half* y = static_cast<__half*>(p.out);
      const __half r = __float2half_rn(moe_finish((p.flags & kMoeAccumulate) ? __half2float(y[o]) + acc : acc,
                                                  p.flags));
      y[o] = p.residual ? __hadd(p.residual[o], r) : r;
    }
  }
}

// ---------------------------------------------------------------------------
// Routing tail of moe_route (qwen_moe.py:407-413) on the router logits that
// F.linear produced: top-k (largest first; equal logits by lower expert
// index), softmax of the k logits in fp32 cast to fp16; and the shared
// expert's weight sigmoid(fp16(x . g)) (qwen_moe.py:505-509).  One CTA per
// token: warp 0 selects, warp 1 computes the shared gate.  Replaces the
// topk / sort / softmax / cast / linear / sigmoid chain of small torch
// kernels (and their host-visible ids) with one launch.
constexpr int kRouteMaxExperts = 4096;
constexpr int kRouteLaneVals = 16;  // fast selection: up to 32 x 16 = 512 experts, top-k <= 32

// (v, i) ranks before (w, j): the larger logit first, equal logits by the
// lower expert index.
__device__ __forceinline__ bool route_before(float v, int i, float w, int j) {
  return v > w || (v == w && i < j);
}

// Top-k by one warp for E <= 512, K <= 32: every lane sorts its (at most 16)
// strided logits in registers (a bitonic network, no memory traffic), then k
// rounds take the best lane head by a warp arg-max and the winning lane
// pops its head.  Lane r returns the r-th selection.
__device__ __forceinline__ void route_select_sorted(const __half* __restrict__ lg, int E, int K, int lane,
                                                    float* sel_v, int* sel_i) {
  float v[kRouteLaneVals];
  int ix[kRouteLaneVals];
#pragma unroll
  for (int j = 0; j < kRouteLaneVals; ++j) {
    const int i = lane + 32 * j;
    v[j] = i < E ? __half2float(lg[i]) : -INFINITY;
    ix[j] = i < E ? i : 0x7fffffff;
  }
#pragma unroll
  for (int k = 2; k <= kRouteLaneVals; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
#pragma unroll
      for (int i = 0; i < kRouteLaneVals; ++i) {
        const int l = i ^ j;
        if (l > i) {
          const bool first = (i & k) == 0;  // this pair's order: i before l, else l before i
          const bool swap = first ? route_before(v[l], ix[l], v[i], ix[i]) : route_before(v[i], ix[i], v[l], ix[l]);
          if (swap) {
            const float tv = v[i];
            v[i] = v[l];
            v[l] = tv;
            const int ti = ix[i];
            ix[i] = ix[l];
            ix[l] = ti;
          }
        }
      }
    }
  }
  for (int r = 0; r < K; ++r) {
    float bv = v[0];
    int bi = ix[0];
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
      if (route_before(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (r == lane) {
      *sel_v = bv;
      *sel_i = bi;
    }
    if (ix[0] == bi) {  // this lane's head was taken (expert indices are unique)
#pragma unroll
      for (int j = 0; j + 1 < kRouteLaneVals; ++j) {
        v[j] = v[j + 1];
        ix[j] = ix[j + 1];
      }
      v[kRouteLaneVals - 1] = -INFINITY;
      ix[kRouteLaneVals - 1] = 0x7fffffff;
    }
  }
}

// Top-k selection, fp32 softmax of the selected logits and their ids, by
// one warp for one token: lg = the token's E logits, ids_t / w_t its K
// outputs, vals = E + 64 floats of this warp's shared memory.
__device__ __forceinline__ void route_warp(const __half* __restrict__ lg, int E, int K, int lane, int* ids_t,
                                           __half* w_t, float* vals) {
  float sel_v = 0.f;  // lane r keeps the r-th selected logit
  int sel_i = 0;
  if (E <= 32 * kRouteLaneVals && K <= 32) {
    route_select_sorted(lg, E, K, lane, &sel_v, &sel_i);
  } else {
    for (int i = lane; i < E; i += 32) vals[i] = __half2float(lg[i]);
    __syncwarp();
    // Each lane tracks the best of its own strided elements.
    auto lane_best = [&](float* bv, int* bi) {
      *bv = -INFINITY;
      *bi = 0x7fffffff;
      for (int i = lane; i < E; i += 32) {
        const float v = vals[i];
        if (v > *bv) {  // strided order: the first (lowest index) wins ties
          *bv = v;
          *bi = i;
        }
      }
    };
    float bv;
    int bi;
    lane_best(&bv, &bi);
    for (int r = 0; r < K; ++r) {
      float v = bv;
      int i = bi;
#pragma unroll
      for (int m = 16; m > 0; m >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, m);
        const int oi = __shfl_xor_sync(0xffffffffu, i, m);
        if (ov > v || (ov == v && oi < i)) {
          v = ov;
          i = oi;
        }
      }
      if ((r & 31) == lane) {
        sel_v = v;
        sel_i = i;
      }
      if ((i & 31) == lane) {  // the owner removes the winner and rescans
        vals[i] = -INFINITY;
        lane_best(&bv, &bi);
      }
      __syncwarp();
      if (r == 31 && K > 32) {  // lanes now hold selections 0..31: emit them before reuse
        ids_t[lane] = sel_i;
        vals[E + lane] = sel_v;  // park the value for the softmax
      }
    }
  }
  // softmax over the K selected logits (the first is the largest)
  __syncwarp();
  if (K > 32) {
    if (lane < K - 32) {
      ids_t[32 + lane] = sel_i;
      vals[E + 32 + lane] = sel_v;
    }
  } else if (lane < K) {
    ids_t[lane] = sel_i;
    vals[E + lane] = sel_v;
  }
  __syncwarp();
  const float mx = vals[E];
  float e0 = lane < K ? expf(vals[E + lane] - mx) : 0.f;
  float e1 = lane + 32 < K ? expf(vals[E + 32 + lane] - mx) : 0.f;
  float sum = e0 + e1;
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
  if (lane < K) w_t[lane] = __float2half_rn(e0 / sum);
  if (lane + 32 < K) w_t[32 + lane] = __float2half_rn(e1 / sum);
}

__global__ void __launch_bounds__(64) moe_route_kernel(const __half* __restrict__ logits, int E, int K,
                                                       const __half* __restrict__ x,
                                                       const __half* __restrict__ g, int H, int* ids,
                                                       __half* weights, __half* shared_w) {
  extern __shared__ float vals[];  // E logits of this token
  const int tok = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  pdl_launch_dependents();
  pdl_wait_primary();
  if (warp == 0) {
    route_warp(logits + (size_t)tok * E, E, K, lane, ids + (size_t)tok * K, weights + (size_t)tok * K, vals);
  } else if (g != nullptr) {
    float acc = 0.f;
    const __half* xr = x + (size_t)tok * H;
#pragma unroll 8  // independent 16-byte loads in flight, not one round trip per step
    for (int j = lane * 8; j < H; j += 32 * 8) {
      const uint4 xv = *reinterpret_cast<const uint4*>(xr + j);
      const uint4 gv = *reinterpret_cast<const uint4*>(g + j);
      const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
      const uint32_t gs[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 a = __half22float2(u32_as_h2(xs[q]));
        const float2 b = __half22float2(u32_as_h2(gs[q]));
        acc = fmaf(a.x, b.x, fmaf(a.y, b.y, acc));
      }
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    if (lane == 0) {
      const float v = __half2float(__float2half_rn(acc));  // F.linear's fp16 output
      shared_w[tok] = __float2half_rn(1.0f / (1.0f + expf(-v)));
    }
  }
}

// The router's F.linear and the routing in one launch (qwen_moe.py:386-416,
// 505-509).  Every CTA computes rows of logits[t][r] = fp16(x_t . W_r) with
// fp32 sums of the fp16 products (rows 0..E-1 the router, row E the shared
// expert's gate when g is given); then each CTA counts itself done on a
// global counter.  The last one (no CTA waits for another) selects each
// token's top-k with route_warp, writes the softmax weights and
// sigmoid(logits[t][E]), and sets the counter back to 0 for the next call.
// Logits are read through L2 (ld.global.cg): an earlier call's last CTA may
// have left the same addresses in this SM's L1.
constexpr int kRouterWarps = 8;
constexpr int kRouterRowsPerCta = kRouterWarps / 2;  // two warps per row, one half of H each
constexpr int kRouterMaxTokens = 16;

template <int TB>  // token bucket: 1, 4 or 16 (ntok <= TB)
__global__ void __launch_bounds__(kRouterWarps * 32)
    moe_router_kernel(const __half* __restrict__ x, int ntok, int H, const __half* __restrict__ w, int E,
                      const __half* __restrict__ g, int K, __half* logits, int* ids, __half* weights,
                      __half* shared_w, unsigned int* counter) {
  extern __shared__ float scratch[];  // per warp: E + 64 floats, then E + 8 halves of logits
  __shared__ float part[kRouterWarps][TB];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rows = E + (g ? 1 : 0);
  const int ld = E + 1;
  pdl_launch_dependents();
  pdl_wait_primary();
  {
    const int r = blockIdx.x * kRouterRowsPerCta + (warp >> 1);
    const int half = warp & 1;
    float acc[TB];
#pragma unroll
    for (int b = 0; b < TB; ++b) acc[b] = 0.f;
    if (r < rows) {
      const int hh = H / 2;
      const __half* wr = (r < E ? w + (size_t)r * H : g) + half * hh;
      const __half* xr = x + half * hh;
      // all of the warp's weight loads in flight at once for one token
#pragma unroll(TB == 1 ? 8 : (TB == 4 ? 2 : 1))
      for (int j = lane * 8; j < hh; j += 32 * 8) {
        float wf[8];
        const uint4 wv = *reinterpret_cast<const uint4*>(wr + j);
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __half22float2(u32_as_h2(ww[q]));
          wf[2 * q] = f.x;
          wf[2 * q + 1] = f.y;
        }
#pragma unroll
        for (int b = 0; b < TB; ++b) {
          if (b < ntok) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xr + (size_t)b * H + j);
            const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 f = __half22float2(u32_as_h2(xs[q]));
              acc[b] = fmaf(f.x, wf[2 * q], fmaf(f.y, wf[2 * q + 1], acc[b]));
            }
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < TB; ++b) {
      float v = acc[b];
#pragma unroll
      for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
      if (lane == 0) part[warp][b] = v;
    }
    __syncthreads();
    // the two halves of each row, added in a fixed order
    if (threadIdx.x < kRouterRowsPerCta * TB) {
      const int rr = threadIdx.x / TB;
      const int b = threadIdx.x % TB;
      const int row = blockIdx.x * kRouterRowsPerCta + rr;
      if (row < rows && b < ntok)
        logits[(size_t)b * ld + row] = __float2half_rn(part[2 * rr][b] + part[2 * rr + 1][b]);
    }
  }
  __threadfence();  // this thread's logits before the CTA counts itself done
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float* vals = scratch + warp * (E + 64);
  __half* lg = reinterpret_cast<__half*>(scratch + kRouterWarps * (E + 64)) + warp * (E + 8);
  for (int b = warp; b < ntok; b += kRouterWarps) {
    for (int i = lane; i < rows; i += 32) lg[i] = __ldcg(logits + (size_t)b * ld + i);
    __syncwarp();
    route_warp(lg, E, K, lane, ids + (size_t)b * K, weights + (size_t)b * K, vals);
    if (g != nullptr && lane == 0) {
      const float v = __half2float(lg[E]);
      shared_w[b] = __float2half_rn(1.0f / (1.0f + expf(-v)));
    }
    __syncwarp();
  }
  __syncthreads();
  if (threadIdx.x == 0) *counter = 0u;
}

}  // namespace gdsq
