// One-shot all-reduce (sum) of a small fp16 vector over NVLink peer memory,
// for the tensor-parallel row split (the o and down projections' partial
// outputs, [hidden] fp16 per rank, two per layer).
//
// Every rank owns a data buffer (two slots of `cap` elements) and a flag
// array [kP2PMaxCtas][kP2PMaxRanks] int, both mapped into every peer (CUDA
// IPC); the kernel gets all ranks' pointers.  CTA c handles elements
// [c*per, (c+1)*per):
//   1. copy its slice of this rank's input into its own slot (epoch & 1);
//   2. signal: one thread per peer p does a system-scope release store of the
//      epoch into p's flag [c][rank];
//   3. wait: one thread per peer spins (bounded, %globaltimer) on its own flag
//      [c][p] until it reaches the epoch (acquire);
//   4. sum the slice over all ranks in rank order (fp32, so every rank gets
//      the same bits) with plain peer loads and write the output.
// The epoch is per CTA, kept in the rank's own flag [c][rank] (read at the
// start, written at the end), so CUDA-graph replays advance it on the device.
// Two slots suffice: a rank rewrites slot e & 1 only in call e + 2, after
// every peer signalled call e + 1, which each does only after it finished
// reading call e.
// No multicast, no TMA: plain loads and stores to peer memory.  A wait that
// expires sets device error bit 1, skips the remaining waits and returns.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace gdsq {

constexpr int kP2PMaxRanks = 8;
constexpr int kP2PMaxCtas = 32;
constexpr int kP2PThreads = 128;
constexpr int kP2PElemsPerCta = kP2PThreads * 8;  // one 16-byte load per thread per rank

struct P2PArgs {
  const __half* in;
  __half* out;
  __half* bufs[kP2PMaxRanks];  // each rank's data buffer (2 slots of cap elements)
  int* flags[kP2PMaxRanks];    // each rank's flag array [kP2PMaxCtas][kP2PMaxRanks]
  int n;
  int cap;
  int rank;
  int world;
  unsigned long long wait_ns;  // bound of the wait for the peers
};

__global__ void __launch_bounds__(kP2PThreads) allreduce_oneshot_kernel(const P2PArgs a) {
  __shared__ int s_epoch;
  __shared__ int s_ok;
  const int c = blockIdx.x;
  const int lo = c * kP2PElemsPerCta;
  int* own = a.flags[a.rank] + c * kP2PMaxRanks;
  pdl_launch_dependents();  // the next kernel may prefetch its weights meanwhile
  // The input is the previous kernel's output, and the epoch must be read
  // only after the previous call of this kernel completed: a dependent
  // launch can start while its predecessor still waits on the peers, and
  // an epoch read then would reuse the predecessor's.
  pdl_wait_primary();
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile int*>(own + a.rank) + 1;
    s_ok = 1;
  }
  __syncthreads();
  const int e = s_epoch;
  const size_t slot = (size_t)(e & 1) * a.cap;
  const int i = lo + threadIdx.x * 8;
  const bool active = i < a.n;  // n % 8 == 0
  if (active) {
    const uint4 v = *reinterpret_cast<const uint4*>(a.in + i);
    *reinterpret_cast<uint4*>(a.bufs[a.rank] + slot + i) = v;
  }
  __syncthreads();
  const int p = threadIdx.x;
  if (p < a.world && p != a.rank) st_release_sys(a.flags[p] + c * kP2PMaxRanks + a.rank, e);
  if (p < a.world && p != a.rank) {
    const int* f = own + p;
    if (ld_acquire_sys(f) < e) {
      const unsigned long long t0 = global_timer_ns();
      while (ld_acquire_sys(f) < e) {
        if (global_timer_ns() - t0 > a.wait_ns) {
          record_device_error(kDevErrBarrierTimeout);
          s_ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (active && s_ok) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int r = 0; r < a.world; ++r) {
      const uint4 v = ld_volatile_v4(a.bufs[r] + slot + i);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f2 = __half22float2(u32_as_h2(w[j]));
        acc[2 * j] += f2.x;
        acc[2 * j + 1] += f2.y;
      }
    }
    uint4 o;
    o.x = h2_as_u32(__floats2half2_rn(acc[0], acc[1]));
    o.y = h2_as_u32(__floats2half2_rn(acc[2], acc[3]));
    o.z = h2_as_u32(__floats2half2_rn(acc[4], acc[5]));
    o.w = h2_as_u32(__floats2half2_rn(acc[6], acc[7]));
    *reinterpret_cast<uint4*>(a.out + i) = o;
  }
  __syncthreads();
  if (threadIdx.x == 0) *reinterpret_cast<volatile int*>(own + a.rank) = e;
}

// One-shot all-reduce (sum) with (value, epoch) words: the expert-parallel
// exchange of the fp32 MoE partials ([B, hidden], one per layer), and any
// fp16 / fp32 vector up to kLLMaxCtas * kLLElemsPerCta elements.
//
// Every rank owns a buffer [2 slots][world][cap] of 64-bit words (fp32 bits
// low, epoch high), mapped into every peer, and a local int epoch per CTA.
// CTA c handles elements [c * kLLElemsPerCta, (c + 1) * kLLElemsPerCta):
//   1. epoch e = own epochs[c] + 1 (read after the previous kernel completed);
//   2. store (value, e) for each element into row `rank` of slot e & 1 of
//      every rank's buffer -- one single-copy-atomic 64-bit store each, so
//      no fence or flag is needed;
//   3. poll (bounded) this rank's own buffer until every rank's word of each
//      element carries e, add them in rank order in fp32 (identical bits on
//      every rank), write the output;
//   4. record e in epochs[c].
// Two slots suffice: a rank writes slot e & 1 of a peer again in call e + 2,
// which starts after its call e + 1 saw the peer's words of e + 1, which the
// peer stores only after its call e (the last reader of the slot) completed.
// No rank waits on anything another rank must wait for: each rank's stores
// come before its own waits.
constexpr int kLLThreads = 256;
constexpr int kLLPerThread = 4;
constexpr int kLLElemsPerCta = kLLThreads * kLLPerThread;
constexpr int kLLMaxCtas = 32;

struct LLArgs {
  const void* in;
  void* out;
  unsigned long long* bufs[kP2PMaxRanks];  // each rank's word buffer
  const unsigned long long* own;           // bufs[rank]
  int* epochs;                             // this rank's [kLLMaxCtas] (local only)
  int n;
  int cap;
  int rank;
  int world;
  unsigned long long wait_ns;              // bound of the wait for the peers' words
  const __half* residual;                  // fp32 -> fp16 form: out = residual + fp16(sum) in fp16, or null
};

template <typename T>
__device__ __forceinline__ float ll_load(const T* p) {
  if constexpr (std::is_same<T, float>::value) return *p;
  else return __half2float(*p);
}

template <typename T>
__device__ __forceinline__ void ll_store(T* p, float v) {
  if constexpr (std::is_same<T, float>::value) *p = v;
  else *p = __float2half_rn(v);
}

// TOut = __half with kClamp: the fp32 sum clamped to the fp16 range, then
// rounded (a NaN stays a NaN), as y.clamp(-65504, 65504).half().
template <typename T, typename TOut = T, bool kClamp = false>
__global__ void __launch_bounds__(kLLThreads) allreduce_ll_kernel(const LLArgs a) {
  __shared__ int s_fail;
  const int c = blockIdx.x;
  pdl_launch_dependents();
  pdl_wait_primary();  // the input is the previous kernel's output; the epoch its predecessor's
  if (threadIdx.x == 0) s_fail = 0;
  const int e = *reinterpret_cast<volatile int*>(a.epochs + c) + 1;
  const int base = c * kLLElemsPerCta + threadIdx.x;
  const size_t slot = (size_t)(e & 1) * a.world;
  const unsigned long long tag = (unsigned long long)(unsigned)e << 32;
  const T* in = static_cast<const T*>(a.in);
#pragma unroll
  for (int j = 0; j < kLLPerThread; ++j) {
    const int i = base + j * kLLThreads;
    if (i < a.n) {
      const unsigned long long w = tag | __float_as_uint(ll_load(in + i));
      const size_t off = (slot + a.rank) * a.cap + i;
#pragma unroll
      for (int r = 0; r < kP2PMaxRanks; ++r)
        if (r < a.world) st_volatile_u64(a.bufs[r] + off, w);
    }
  }
  __syncthreads();
  float sum[kLLPerThread];
#pragma unroll
  for (int j = 0; j < kLLPerThread; ++j) sum[j] = 0.f;
  bool ok = true;
  unsigned long long t0 = 0;
  for (int q = 0; q < a.world; ++q) {
    const unsigned long long* src = a.own + (slot + q) * a.cap;
    unsigned long long w[kLLPerThread];
#pragma unroll
    for (int j = 0; j < kLLPerThread; ++j) {
      const int i = base + j * kLLThreads;
      w[j] = i < a.n ? ld_volatile_u64(src + i) : tag;
    }
#pragma unroll
    for (int j = 0; j < kLLPerThread; ++j) {
      while (ok && (w[j] >> 32) != (unsigned long long)(unsigned)e) {
        if (t0 == 0) {
          t0 = global_timer_ns();
        } else if (global_timer_ns() - t0 > a.wait_ns) {
          record_device_error(kDevErrBarrierTimeout);
          ok = false;
          break;
        }
        w[j] = ld_volatile_u64(src + base + j * kLLThreads);
      }
      sum[j] += __uint_as_float((unsigned)w[j]);
    }
  }
  if (!ok) s_fail = 1;
  __syncthreads();
  if (s_fail == 0) {
    TOut* out = static_cast<TOut*>(a.out);
#pragma unroll
    for (int j = 0; j < kLLPerThread; ++j) {
      const int i = base + j * kLLThreads;
      float v = sum[j];
      if constexpr (kClamp) v = v > 65504.f ? 65504.f : (v < -65504.f ? -65504.f : v);
      if constexpr (kClamp) {
        if (i < a.n) {
          const __half r = __float2half_rn(v);
          out[i] = a.residual ? __hadd(a.residual[i], r) : r;
        }
      } else if (i < a.n) {
        ll_store(out + i, v);
      }
    }
  }
  if (threadIdx.x == 0) *reinterpret_cast<volatile int*>(a.epochs + c) = e;
}

}  // namespace gdsq
