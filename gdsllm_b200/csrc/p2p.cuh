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
};

__global__ void __launch_bounds__(kP2PThreads) allreduce_oneshot_kernel(const P2PArgs a) {
  __shared__ int s_epoch;
  __shared__ int s_ok;
  const int c = blockIdx.x;
  const int lo = c * kP2PElemsPerCta;
  int* own = a.flags[a.rank] + c * kP2PMaxRanks;
  pdl_launch_dependents();  // the next kernel may prefetch its weights meanwhile
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile int*>(own + a.rank) + 1;
    s_ok = 1;
  }
  pdl_wait_primary();  // the input is the previous kernel's output
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
        if (global_timer_ns() - t0 > kWaitLimitNs) {
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

}  // namespace gdsq
