// Decode-step kernels: the work of one LLaMA decode position (batch 1)
// around the fused GEMVs, with the position held in device memory, so that a
// whole token can be captured once as a CUDA graph and replayed
// (gdsllm_b200/decode_step.py).  Each follows the arithmetic order of the
// torch code it replaces in GdsLLM:
//
//   add_rmsnorm_kernel  `x = x + h` (llama.py:285,291) then rms_norm
//                       (llama.py:17-23): fp32 mean of squares, rsqrt,
//                       fp16(x * norm) * weight in fp16
//   rope_kv_kernel      apply_rotary_emb (llama.py:83-105) on q and k, fp32
//                       complex product rounded to fp16, then
//                       KVCache.update (kv_cache.py:44-67) at the position
//   attn_decode_kernel  scores = fp16(q.k) then fp16(scores * (1/sqrt(d)))
//                       (torch divides by a CPU scalar as a multiply by its
//                       fp32 reciprocal), softmax in fp32 rounded to fp16,
//                       fp16(sum p*v) with fp32 sums (llama.py:228-242);
//                       GQA heads share a KV head by index (repeat_kv,
//                       llama.py:167-180)
//   silu_mul_kernel     fp16(silu(gate)) * up in fp16 (llama.py:248-252)
//   argmax_kernel       greedy token (first index of the maximum, as
//                       torch.argmax) and the position advance
//
// Every kernel calls griddepcontrol, so it chains with the GEMVs under
// programmatic dependent launch.  A position outside the cache sets device
// error bit 4 and the kernel writes nothing.
#pragma once

#include "common.cuh"

namespace gdsq {

constexpr int kNormThreads = 512;
constexpr int kNormMaxChunks = 4;  // hidden <= 512 threads * 8 * 4 = 16384
constexpr int kDecodeThreads = 256;
constexpr int kAttnMaxCluster = 16;

// Sum over the block; every thread gets the same value (warps' partials are
// added in warp order).  `red` holds one float per warp; callers separate
// two uses of it with __syncthreads().
template <int kWarps>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) t += red[w];
  return t;
}

template <int kWarps>
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = -INFINITY;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) t = fmaxf(t, red[w]);
  return t;
}

__device__ __forceinline__ void unpack8(const uint4 a, float (&v)[8]) {
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(u32_as_h2(w[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// One CTA per row.  h_out = h_in + delta (delta may be null: h_out is then
// not written); x_out = rms_norm(h_out) * weight.  h_out may alias h_in.
__global__ void __launch_bounds__(kNormThreads)
    add_rmsnorm_kernel(const __half* h_in, const __half* __restrict__ delta, __half* h_out,
                       const __half* __restrict__ weight, __half* __restrict__ x_out, int hidden,
                       float inv_hidden, float eps) {
  __shared__ float red[kNormThreads / 32];
  pdl_launch_dependents();
  pdl_wait_primary();
  const size_t base = (size_t)blockIdx.x * hidden;
  float v[kNormMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const int i = (c * kNormThreads + (int)threadIdx.x) * 8;
    if (i < hidden) {
      uint4 a = *reinterpret_cast<const uint4*>(h_in + base + i);
      if (delta) {
        const uint4 d = *reinterpret_cast<const uint4*>(delta + base + i);
        a.x = h2_as_u32(__hadd2(u32_as_h2(a.x), u32_as_h2(d.x)));
        a.y = h2_as_u32(__hadd2(u32_as_h2(a.y), u32_as_h2(d.y)));
        a.z = h2_as_u32(__hadd2(u32_as_h2(a.z), u32_as_h2(d.z)));
        a.w = h2_as_u32(__hadd2(u32_as_h2(a.w), u32_as_h2(d.w)));
        *reinterpret_cast<uint4*>(h_out + base + i) = a;
      }
      unpack8(a, v[c]);
#pragma unroll
      for (int k = 0; k < 8; ++k) ss = __fadd_rn(ss, __fmul_rn(v[c][k], v[c][k]));
    }
  }
  const float total = block_sum<kNormThreads / 32>(ss, red);
  const float norm = rsqrtf(__fadd_rn(__fmul_rn(total, inv_hidden), eps));
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const int i = (c * kNormThreads + (int)threadIdx.x) * 8;
    if (i < hidden) {
      const uint4 w = *reinterpret_cast<const uint4*>(weight + i);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const __half2 xn = __floats2half2_rn(__fmul_rn(v[c][2 * k], norm), __fmul_rn(v[c][2 * k + 1], norm));
        o[k] = h2_as_u32(__hmul2(xn, u32_as_h2(ww[k])));
      }
      *reinterpret_cast<uint4*>(x_out + base + i) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Grid: num_heads + num_kv_heads CTAs (q heads, then k heads), head_dim/2
// threads, one rotation pair each.  The k-head CTAs also copy v.  The cache
// of one layer is [num_kv_heads][max_seq][head_dim] (batch 1).
__global__ void rope_kv_kernel(const __half* __restrict__ q, const __half* __restrict__ k,
                               const __half* __restrict__ v, __half* __restrict__ q_out,
                               const float2* __restrict__ freqs, const long long* __restrict__ pos_p,
                               __half* __restrict__ k_cache, __half* __restrict__ v_cache, int num_heads,
                               int head_dim, int max_seq) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const long long pos = *pos_p;
  if (pos < 0 || pos >= max_seq) {
    if (blockIdx.x == 0 && threadIdx.x == 0) record_device_error(4);
    return;
  }
  const int i = threadIdx.x;
  const int half_dim = head_dim >> 1;
  const float2 f = freqs[(size_t)pos * half_dim + i];
  const int hb = blockIdx.x;
  const __half2* src;
  __half2* dst;
  if (hb < num_heads) {
    src = reinterpret_cast<const __half2*>(q + (size_t)hb * head_dim);
    dst = reinterpret_cast<__half2*>(q_out + (size_t)hb * head_dim);
  } else {
    const size_t kh = hb - num_heads;
    const size_t row = (kh * max_seq + pos) * head_dim;
    src = reinterpret_cast<const __half2*>(k + kh * head_dim);
    dst = reinterpret_cast<__half2*>(k_cache + row);
    reinterpret_cast<__half2*>(v_cache + row)[i] = reinterpret_cast<const __half2*>(v + kh * head_dim)[i];
  }
  const float2 a = __half22float2(src[i]);
  // (a.x + i a.y)(f.x + i f.y), as c10::complex<float> multiplies
  const float re = a.x * f.x - a.y * f.y;
  const float im = a.x * f.y + a.y * f.x;
  dst[i] = __floats2half2_rn(re, im);
}

// Grid (C, num_heads), cluster (C, 1, 1): the C CTAs of a cluster split the
// positions [0, pos] of one head.  Each computes its scores into shared
// memory, the cluster agrees on the maximum and the sum through distributed
// shared memory, each adds its probability-weighted V rows, and CTA 0 of the
// cluster adds the C partial outputs in rank order.  Shared memory (floats):
// scores [ceil(max_seq / C)] | group partials [256/(HD/8)][HD] |
// cluster partials [C][HD] | maxima [16] | sums [16] | reductions [2][8] |
// (kRope) the new K and V rows [HD] fp16 each.
//
// kRope: q, k_new and v_new are the projections before RoPE (rope_kv_kernel
// folded in).  Every lane rotates its own q elements; the CTA whose
// positions include *pos rotates k_new of its KV head, writes it and v_new
// into the caches at *pos and uses those rows from shared memory (CTAs of
// other query heads of the same KV head write the same values).  Without
// kRope, q is already rotated and row *pos is in the caches.
template <int HD, bool kRope>
__global__ void __launch_bounds__(kDecodeThreads)
    attn_decode_kernel(const __half* __restrict__ q, const __half* __restrict__ k_new,
                       const __half* __restrict__ v_new, const float2* __restrict__ freqs,
                       __half* k_cache, __half* v_cache, const long long* __restrict__ pos_p,
                       __half* __restrict__ out, int num_heads, int num_kv_heads, int max_seq, float scale) {
  constexpr int kPer = HD / 8;            // q / k elements per lane (8 lanes per position)
  constexpr int kVec = kPer / 8;          // 16-byte loads per lane per position
  constexpr int kSlices = HD / 8;         // V: threads per position, 8 dims each
  constexpr int kGroups = kDecodeThreads / kSlices;
  constexpr int kWarps = kDecodeThreads / 32;
  extern __shared__ float sm[];
  const int C = gridDim.x;
  const int c = blockIdx.x;
  const int h = blockIdx.y;
  const int kvh = h / (num_heads / num_kv_heads);
  const int cap = (max_seq + C - 1) / C;
  float* sc = sm;
  float* gacc = sc + ((cap + 3) & ~3);
  float* cacc = gacc + kGroups * HD;
  float* xmax = cacc + C * HD;
  float* xsum = xmax + kAttnMaxCluster;
  float* red = xsum + kAttnMaxCluster;
  __half* krow = reinterpret_cast<__half*>(red + 2 * kWarps);  // 16-byte aligned (offsets are multiples of 4 floats)
  __half* vrow = krow + HD;
  __half* kh_base = k_cache + (size_t)kvh * max_seq * HD;
  __half* vh_base = v_cache + (size_t)kvh * max_seq * HD;

  if (C > 1) cluster_arrive_relaxed();  // waited for before the first DSMEM store
  // Warm L2 with this CTA's K and V rows while the producers finish.  The
  // position read here only sizes the hint; the one used below is read
  // after griddepcontrol.wait.
  if (threadIdx.x == 0) {
    const long long p0 = *(volatile const long long*)pos_p;
    if (p0 >= 0 && p0 < max_seq) {
      const int L0 = (int)p0 + 1;
      const int per0 = (L0 + C - 1) / C;
      const int n0 = min(L0, c * per0 + per0) - c * per0;
      if (n0 > 0) {
        const uint32_t bytes = (uint32_t)n0 * HD * 2;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(kh_base + (size_t)c * per0 * HD),
                     "r"(bytes)
                     : "memory");
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(vh_base + (size_t)c * per0 * HD),
                     "r"(bytes)
                     : "memory");
      }
    }
  }
  pdl_launch_dependents();
  pdl_wait_primary();
  const long long pos = *pos_p;
  if (pos < 0 || pos >= max_seq) {  // every CTA reads the same value and leaves
    if (C > 1) cluster_wait();
    if (c == 0 && h == 0 && threadIdx.x == 0) record_device_error(4);
    return;
  }
  const int L = (int)pos + 1;
  const int per = (L + C - 1) / C;
  const int j0 = c * per;
  const int n = max(0, min(L, j0 + per) - j0);
  const int jnew = (int)pos - j0;  // slice-local index of the new row (valid when < n)
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 3;
  const int s = lane & 7;

  if constexpr (kRope) {
    if (jnew < n && (int)threadIdx.x < HD / 2) {
      const int i = threadIdx.x;
      const float2 f = freqs[(size_t)pos * (HD / 2) + i];
      const float2 a = __half22float2(reinterpret_cast<const __half2*>(k_new + (size_t)kvh * HD)[i]);
      // (a.x + i a.y)(f.x + i f.y), as c10::complex<float> multiplies
      const __half2 kr = __floats2half2_rn(a.x * f.x - a.y * f.y, a.x * f.y + a.y * f.x);
      const __half2 vv = reinterpret_cast<const __half2*>(v_new + (size_t)kvh * HD)[i];
      reinterpret_cast<__half2*>(krow)[i] = kr;
      reinterpret_cast<__half2*>(vrow)[i] = vv;
      reinterpret_cast<__half2*>(kh_base + (size_t)pos * HD)[i] = kr;
      reinterpret_cast<__half2*>(vh_base + (size_t)pos * HD)[i] = vv;
    }
    __syncthreads();
  }

  // Scores: each group of 8 lanes takes one position per pass.
  float qv[kPer];
  {
    const uint4* qp = reinterpret_cast<const uint4*>(q + (size_t)h * HD + s * kPer);
#pragma unroll
    for (int u = 0; u < kVec; ++u) {
      float t[8];
      unpack8(qp[u], t);
#pragma unroll
      for (int e = 0; e < 8; ++e) qv[8 * u + e] = t[e];
    }
    if constexpr (kRope) {
#pragma unroll
      for (int e = 0; e < kPer; e += 2) {
        const float2 f = freqs[(size_t)pos * (HD / 2) + (s * kPer + e) / 2];
        const float a = qv[e], b = qv[e + 1];
        const __half2 r = __floats2half2_rn(a * f.x - b * f.y, a * f.y + b * f.x);
        const float2 rf = __half22float2(r);
        qv[e] = rf.x;
        qv[e + 1] = rf.y;
      }
    }
  }
  const __half* kb = kh_base + (size_t)j0 * HD + s * kPer;
  auto krow_ptr = [&](int jj) -> const __half* {
    if (kRope && jj == jnew) return krow + s * kPer;
    return kb + (size_t)jj * HD;
  };
  // kUnroll positions per lane group per pass, all loads issued first.
  constexpr int kUnroll = 4;
  float lmax = -INFINITY;
  for (int b0 = warp * 4; b0 < n; b0 += kUnroll * kWarps * 4) {
    uint4 kv[kUnroll][kVec];
#pragma unroll
    for (int t = 0; t < kUnroll; ++t) {
      const int jj = b0 + g + t * kWarps * 4;
      const __half* pk = krow_ptr(jj);
#pragma unroll
      for (int u = 0; u < kVec; ++u)
        kv[t][u] = jj < n ? reinterpret_cast<const uint4*>(pk)[u] : make_uint4(0, 0, 0, 0);
    }
    float d[kUnroll];
#pragma unroll
    for (int t = 0; t < kUnroll; ++t) {
      d[t] = 0.f;
#pragma unroll
      for (int u = 0; u < kVec; ++u) {
        float tk[8];
        unpack8(kv[t][u], tk);
#pragma unroll
        for (int e = 0; e < 8; ++e) d[t] = fmaf(tk[e], qv[8 * u + e], d[t]);
      }
    }
#pragma unroll
    for (int m = 4; m > 0; m >>= 1) {
#pragma unroll
      for (int t = 0; t < kUnroll; ++t) d[t] += __shfl_xor_sync(0xffffffffu, d[t], m);
    }
    if (s == 0) {
#pragma unroll
      for (int t = 0; t < kUnroll; ++t) {
        const int jj = b0 + g + t * kWarps * 4;
        if (jj < n) {
          const float x = __half2float(__float2half_rn(__half2float(__float2half_rn(d[t])) * scale));
          sc[jj] = x;
          lmax = fmaxf(lmax, x);
        }
      }
    }
  }
  const float cmax = block_max<kWarps>(lmax, red);
  if (C > 1) {
    cluster_wait();  // every peer is running: DSMEM stores are safe
    if ((int)threadIdx.x < C) st_cluster_f32(map_to_rank(&xmax[c], threadIdx.x), cmax);
    cluster_sync_all();
  } else if (threadIdx.x == 0) {
    xmax[0] = cmax;
  }
  __syncthreads();
  float m = -INFINITY;
  for (int r = 0; r < C; ++r) m = fmaxf(m, xmax[r]);

  float lsum = 0.f;
  for (int j = threadIdx.x; j < n; j += kDecodeThreads) {
    const float e = expf(sc[j] - m);
    sc[j] = e;
    lsum += e;
  }
  const float csum = block_sum<kWarps>(lsum, red + kWarps);
  if (C > 1) {
    if ((int)threadIdx.x < C) st_cluster_f32(map_to_rank(&xsum[c], threadIdx.x), csum);
    cluster_sync_all();
  } else if (threadIdx.x == 0) {
    xsum[0] = csum;
  }
  __syncthreads();
  float total = 0.f;
  for (int r = 0; r < C; ++r) total += xsum[r];
  for (int j = threadIdx.x; j < n; j += kDecodeThreads) sc[j] = __half2float(__float2half_rn(sc[j] / total));
  __syncthreads();

  // Weighted V: thread = (position group, 8 dims).
  const int slice = threadIdx.x % kSlices;
  const int grp = threadIdx.x / kSlices;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  const __half* vb0 = vh_base + (size_t)j0 * HD + slice * 8;
  auto vrow_ptr = [&](int jj) -> const __half* {
    if (kRope && jj == jnew) return vrow + slice * 8;
    return vb0 + (size_t)jj * HD;
  };
  for (int j0g = grp; j0g < n; j0g += kUnroll * kGroups) {
    uint4 vv[kUnroll];
    float pv[kUnroll];
#pragma unroll
    for (int t = 0; t < kUnroll; ++t) {
      const int jj = j0g + t * kGroups;
      vv[t] = jj < n ? *reinterpret_cast<const uint4*>(vrow_ptr(jj)) : make_uint4(0, 0, 0, 0);
      pv[t] = jj < n ? sc[jj] : 0.f;
    }
#pragma unroll
    for (int t = 0; t < kUnroll; ++t) {
      float tv[8];
      unpack8(vv[t], tv);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(pv[t], tv[e], acc[e]);
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) gacc[grp * HD + slice * 8 + e] = acc[e];
  __syncthreads();
  if ((int)threadIdx.x < HD) {
    float part = 0.f;
    for (int r = 0; r < kGroups; ++r) part += gacc[r * HD + threadIdx.x];
    if (C > 1)
      st_cluster_f32(map_to_rank(&cacc[c * HD + threadIdx.x], 0), part);
    else
      out[(size_t)h * HD + threadIdx.x] = __float2half_rn(part);
  }
  if (C > 1) {
    cluster_sync_all();
    if (c == 0 && (int)threadIdx.x < HD) {
      float o = 0.f;
      for (int r = 0; r < C; ++r) o += cacc[r * HD + threadIdx.x];
      out[(size_t)h * HD + threadIdx.x] = __float2half_rn(o);
    }
  }
}

// out = fp16(silu(gate)) * up, 8 elements per thread when the caller
// guarantees n % 8 == 0 and 16-byte alignment (kVec), else one.
template <bool kVec>
__global__ void __launch_bounds__(kDecodeThreads)
    silu_mul_kernel(const __half* __restrict__ gate, const __half* __restrict__ up, __half* __restrict__ out,
                    long long n) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const long long stride = (long long)gridDim.x * blockDim.x;
  auto silu = [](float x) { return __float2half_rn(x / (1.0f + expf(-x))); };
  if constexpr (kVec) {
    for (long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x; u < n / 8; u += stride) {
      const uint4 g = reinterpret_cast<const uint4*>(gate)[u];
      const uint4 p = reinterpret_cast<const uint4*>(up)[u];
      const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
      const uint32_t pw[4] = {p.x, p.y, p.z, p.w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 gf = __half22float2(u32_as_h2(gw[k]));
        o[k] = h2_as_u32(__hmul2(__halves2half2(silu(gf.x), silu(gf.y)), u32_as_h2(pw[k])));
      }
      reinterpret_cast<uint4*>(out)[u] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  } else {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
      out[i] = __hmul(silu(__half2float(gate[i])), up[i]);
  }
}

// One CTA of 1024 threads: token = the first index of the largest logit
// (torch.argmax's tie rule; a NaN is skipped), then *pos += 1 when pos is
// given.  kVec: 8 logits per 16-byte load (n % 8 == 0, 16-byte aligned).
template <bool kVec>
__global__ void __launch_bounds__(1024)
    argmax_kernel(const __half* __restrict__ logits, int n, long long* __restrict__ token, long long* pos) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  pdl_launch_dependents();
  pdl_wait_primary();
  float best = -INFINITY;
  int idx = 0x7fffffff;
  auto take = [&](float v, int i) {  // indices arrive in increasing order per thread
    if (v > best || (idx == 0x7fffffff && v == best)) {
      best = v;
      idx = i;
    }
  };
  if constexpr (kVec) {
    for (int u = threadIdx.x; u < n / 8; u += blockDim.x) {
      float t[8];
      unpack8(reinterpret_cast<const uint4*>(logits)[u], t);
#pragma unroll
      for (int e = 0; e < 8; ++e) take(t[e], 8 * u + e);
    }
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) take(__half2float(logits[i]), i);
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, m);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, m);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    bv[threadIdx.x >> 5] = best;
    bi[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
        best = bv[w];
        idx = bi[w];
      }
    *token = idx == 0x7fffffff ? 0 : idx;
    if (pos) *pos += 1;
  }
}

}  // namespace gdsq
