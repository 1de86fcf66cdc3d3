// gdsq: C-ABI entry points (include/gdsq.h) and host-side dispatch.
//
// One translation unit holds every kernel so that they can share the
// device-side error word without relocatable device code.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <unordered_map>

#include "gdsq.h"
#include "common.cuh"
#include "dequant.cuh"
#include "gemv.cuh"
#include "gemv_tcb.cuh"
#include "moe.cuh"
#include "p2p.cuh"
#include "decode.cuh"

namespace gdsq {
namespace {

thread_local std::string t_last_error;
int g_pdl_enabled = 0;
std::atomic<unsigned long long> g_peer_wait_ns{kPeerWaitDefaultNs};

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  // Launch-configuration errors are sticky only for the current call.
  return fail(GDSQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct DeviceInfo {
  bool ready = false;
  int ordinal = 0;
  int sms = 0;
  int smem_optin = 0;
};

constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
std::mutex g_device_mutex;

// Cached per-device attributes (the reference queried device 0 on every
// launch, gdsllm/runtime/fused_gemv.cu:117-118).
int device_info(const DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(GDSQ_ERR_UNSUPPORTED, "device %d", dev);
  DeviceInfo& d = g_devices[dev];
  if (!d.ready) {
    std::lock_guard<std::mutex> lock(g_device_mutex);
    if (!d.ready) {
      e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
      e = cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
      if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(smem opt-in)");
      d.ordinal = dev;
      d.ready = true;
    }
  }
  *out = &d;
  return GDSQ_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                   cudaStream_t stream, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Raises a kernel's dynamic shared-memory limit when a launch needs more than
// was last set for that (kernel, device).
std::unordered_map<const void*, int> g_smem_set[kMaxDevices];

template <typename K>
cudaError_t ensure_smem(K kernel, int bytes, int device) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  const void* key = reinterpret_cast<const void*>(kernel);
  std::lock_guard<std::mutex> lock(g_device_mutex);
  auto it = g_smem_set[device].find(key);
  if (it != g_smem_set[device].end() && it->second >= bytes) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) g_smem_set[device][key] = bytes;
  return e;
}

// ---------------------------------------------------------------------------
// Weight tensor maps for the TMA loads of the fast GEMV.  A packed weight
// matrix is described as a 2-D tensor of 8-byte elements: [N rows][row_bytes
// / 8], row pitch row_bytes; one box is 32 rows x one 256-column chunk.
// Encoded maps are cached per (pointer, shape, format, device), so repeated
// calls on resident weights (a decode loop) pay only a hash lookup.

PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;

int get_encoder(PFN_cuTensorMapEncodeTiled_v12000* out) {
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (err == cudaSuccess && q != cudaDriverEntryPointSuccess) err = cudaErrorSymbolNotFound;
    g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (err != cudaSuccess || !g_encode_tiled) return cuda_fail(err, "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
  *out = g_encode_tiled;
  return GDSQ_OK;
}

struct MapKey {
  uintptr_t ptr;
  long long row_bytes;
  int n;
  int fmt;
  int box_rows;
  int depth;  // experts of a 3-D map (1 for a 2-D weight matrix)
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && row_bytes == o.row_bytes && n == o.n && fmt == o.fmt && box_rows == o.box_rows &&
           depth == o.depth;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<uintptr_t>()(k.ptr) ^ (std::hash<long long>()(k.row_bytes) << 1) ^
           ((size_t)k.n << 7) ^ ((size_t)k.fmt << 3) ^ ((size_t)k.box_rows << 40) ^ ((size_t)k.depth << 50);
  }
};
std::mutex g_map_mutex;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps[kMaxDevices];
constexpr size_t kMaxCachedMaps = 16384;

template <int F>
int weight_map(const DeviceInfo& dev, const void* w, int n, long long row_bytes, CUtensorMap* out,
               int box_rows = 32) {
  using T = GemvFormat<F>;
  const MapKey key{reinterpret_cast<uintptr_t>(w), row_bytes, n, F, box_rows, 1};
  {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    auto it = g_maps[dev.ordinal].find(key);
    if (it != g_maps[dev.ordinal].end()) {
      *out = it->second;
      return GDSQ_OK;
    }
  }
  PFN_cuTensorMapEncodeTiled_v12000 encode;
  int st = get_encoder(&encode);
  if (st != GDSQ_OK) return st;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 8), (cuuint64_t)n};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)(T::kChunkBytes / 8), (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(w), dims, strides, box,
                      estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      T::kSwizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(GDSQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for a %d x %lld-byte weight", (int)r, n,
                row_bytes);
  std::lock_guard<std::mutex> lock(g_map_mutex);
  if (g_maps[dev.ordinal].size() >= kMaxCachedMaps) g_maps[dev.ordinal].clear();
  g_maps[dev.ordinal][key] = map;
  *out = map;
  return GDSQ_OK;
}

// Stacked affine-Q4 experts [experts][rows][cols/8 words] as a 3-D tensor of
// 8-byte elements; one box is box_rows rows x one 256-column chunk (128 B,
// 128-byte swizzle) of one expert.
int expert_map(const DeviceInfo& dev, const void* w, int experts, int rows, int cols, int box_rows,
               CUtensorMap* out) {
  const long long row_bytes = cols / 2;
  const MapKey key{reinterpret_cast<uintptr_t>(w), row_bytes, rows, 16, box_rows, experts};
  {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    auto it = g_maps[dev.ordinal].find(key);
    if (it != g_maps[dev.ordinal].end()) {
      *out = it->second;
      return GDSQ_OK;
    }
  }
  PFN_cuTensorMapEncodeTiled_v12000 encode;
  int st = get_encoder(&encode);
  if (st != GDSQ_OK) return st;
  CUtensorMap map;
  const cuuint64_t dims[3] = {(cuuint64_t)(row_bytes / 8), (cuuint64_t)rows, (cuuint64_t)experts};
  const cuuint64_t strides[2] = {(cuuint64_t)row_bytes, (cuuint64_t)row_bytes * rows};
  const cuuint32_t box[3] = {(cuuint32_t)(kMoeChunkBytes / 8), (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(w), dims, strides, box,
                      estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(GDSQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for %d experts of %d x %d", (int)r,
                experts, rows, cols);
  std::lock_guard<std::mutex> lock(g_map_mutex);
  if (g_maps[dev.ordinal].size() >= kMaxCachedMaps) g_maps[dev.ordinal].clear();
  g_maps[dev.ordinal][key] = map;
  *out = map;
  return GDSQ_OK;
}

// ---------------------------------------------------------------------------
// GEMV dispatch

int batch_tile(int nb) {
  if (nb <= 4) return nb;
  if (nb <= 8) return 8;
  return 16;
}

// Launch plan of the fast GEMV kernel for one (format, batch tile, group, N,
// K) on one device.
struct GemvPlan {
  int cs = 1;         // CTAs per cluster (K slices)
  int stages = 1;     // ring stages per warp
  int copy = 1;       // chunks per ring stage
  int nclusters = 1;  // clusters launched (persistent when < row groups)
  int smem = 0;       // dynamic shared memory bytes
};

std::mutex g_plan_mutex;
std::unordered_map<uint64_t, GemvPlan> g_plans[kMaxDevices];

// Optional override "cs:stages[:copy]" for tuning sweeps (GDSQ_GEMV_PLAN).
bool plan_override(int* cs, int* stages, int* copy) {
  const char* e = getenv("GDSQ_GEMV_PLAN");
  if (!e || !*e) return false;
  *copy = 0;
  const int n = sscanf(e, "%d:%d:%d", cs, stages, copy);
  return n >= 2 && *cs >= 1 && *cs <= kMaxCluster && *stages >= 1 && *stages <= kMaxStages;
}

// Picks (cs, stages, copy) by a small cost model: the busiest SM's share of
// 256-column chunk units (plus one unit of fixed cost per CTA work item),
// divided by an issue-efficiency factor that grows with resident warps (16
// warps per SM are taken as enough to hide latency).  Candidates whose
// shared memory does not fit are skipped.
template <int F, int B, int GS, bool TP = false>
int make_plan_model(int N, int K, const DeviceInfo& dev, GemvPlan* out) {
  using T = GemvFormat<F>;
  auto kernel = gemv_fast_kernel<F, B, GS, TP>;
  const int R = (N + 31) / 32;
  const int C = K / kChunkCols;
  int force_cs = 0, force_st = 0, force_cp = 0;
  const bool forced = plan_override(&force_cs, &force_st, &force_cp);
  double best = 1e30;
  bool found = false;
  for (int cs = 1; cs <= kMaxCluster; cs *= 2) {
    if (cs > C) break;
    if (forced && cs != force_cs) continue;
    const int cslice = (C + cs - 1) / cs;
    const int mw = (cslice + kGemvWarps - 1) / kGemvWarps;
    for (int cp = 1; cp <= T::kMaxCopyChunks; ++cp) {
      if (forced && force_cp && cp != force_cp) continue;
      const int nsteps = (mw + cp - 1) / cp;
      for (int st = 1; st <= 4; ++st) {
        if (forced && st != force_st) continue;
        if (!forced && st > 1 && st > nsteps * ((R + 147) / 148)) break;
        const GemvSmemLayout L = gemv_smem_layout<F>(B, K, GS, cs, st, cp);
        if (L.total > dev.smem_optin) continue;
        cudaError_t e = ensure_smem(kernel, L.total, dev.ordinal);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv)");
        int occ = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kGemvWarps * 32, L.total);
        if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        if (occ < 1) continue;
        const long long slots = (long long)dev.sms * occ;
        const long long ctas = (long long)R * cs;
        double load;
        long long resident;
        int nclusters;
        if (ctas <= slots) {
          nclusters = R;
          resident = (ctas + dev.sms - 1) / dev.sms;
          load = (double)resident * (cslice + 1);
        } else {
          nclusters = (int)(slots / cs);
          const int items = (R + nclusters - 1) / nclusters;
          resident = occ;
          load = (double)occ * items * (cslice + 1);
        }
        const double warps = (double)resident * kGemvWarps;
        const double eff = warps >= 16 ? 1.0 : warps / 16.0;
        const double cost = load / eff * (1.0 + 0.02 * cs) / (1.0 + 0.01 * st) * (1.0 + 0.005 * cp);
        if (cost < best) {
          best = cost;
          found = true;
          out->cs = cs;
          out->stages = st;
          out->copy = cp;
          out->nclusters = nclusters;
          out->smem = L.total;
        }
      }
    }
  }
  if (!found) return fail(GDSQ_ERR_UNSUPPORTED, "no GEMV launch plan fits shared memory");
  return GDSQ_OK;
}

// Batch 1 (the decode chain): measured on B200 over the decode shapes in
// dependent launch chains with programmatic dependent launch (4096x4096,
// 12288x4096 and 22016x4096 grouped, 4096x11008), the fastest plans used the
// smallest cluster split giving a few CTAs per SM, at most 4 CTAs per
// cluster, two ring stages and one chunk per stage; wider splits pay a
// cluster reduction per row group, deeper rings only take shared memory
// from co-resident CTAs of the next launch.  Rule: the smallest power of two
// cs <= 4 with R * cs >= 4 * SMs, then fewer stages or a wider split if
// shared memory does not fit.  Batches > 1 keep the cost model above (their
// staged activations make shared memory, hence occupancy, the constraint).
template <int F, int B, int GS, bool TP = false>
int make_plan(int N, int K, const DeviceInfo& dev, GemvPlan* out) {
  if (B > 1) return make_plan_model<F, B, GS, TP>(N, K, dev, out);
  auto kernel = gemv_fast_kernel<F, B, GS, TP>;
  const int R = (N + 31) / 32;
  const int C = K / kChunkCols;
  int force_cs = 0, force_st = 0, force_cp = 0;
  const bool forced = plan_override(&force_cs, &force_st, &force_cp);
  int want_cs = 1;
  while (want_cs < 4 && want_cs * 2 <= C && (long long)R * want_cs < 4LL * dev.sms) want_cs *= 2;
  struct Cand { int cs, st, cp; };
  Cand cands[16];
  int nc = 0;
  if (forced) {
    cands[nc++] = {force_cs, force_st, force_cp ? force_cp : 1};
  } else {
    for (int cs = want_cs; cs <= kMaxCluster && cs <= C; cs *= 2)
      for (int st = 2; st >= 1; --st) cands[nc++] = {cs, st, 1};
  }
  for (int i = 0; i < nc; ++i) {
    const Cand c = cands[i];
    if (c.cs > C || c.cp > GemvFormat<F>::kMaxCopyChunks) continue;
    const GemvSmemLayout L = gemv_smem_layout<F>(B, K, GS, c.cs, c.st, c.cp);
    if (L.total > dev.smem_optin) continue;
    cudaError_t e = ensure_smem(kernel, L.total, dev.ordinal);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv)");
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kGemvWarps * 32, L.total);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (occ < 1) continue;
    if (const char* cap = getenv("GDSQ_GEMV_OCC")) {  // tuning sweeps: CTAs per SM per launch, at most
      const int v = atoi(cap);
      if (v >= 1 && v < occ) occ = v;
    }
    long long slots = (long long)dev.sms * occ;
    int st_pick = c.st;
    int smem_pick = L.total;
    // More than one wave of CTAs, and at least 4 chunks per warp: a one-stage
    // ring that fits every CTA at once streams faster (22016 x 4096, the
    // grouped gate/up: 17.2 vs 20.4 us in a PDL chain; with 1-2 chunks per
    // warp the second stage wins).
    const int mw = ((C + c.cs - 1) / c.cs + kGemvWarps - 1) / kGemvWarps;
    if (!forced && c.st == 2 && (long long)R * c.cs > slots && mw >= 4) {
      const GemvSmemLayout L1 = gemv_smem_layout<F>(B, K, GS, c.cs, 1, c.cp);
      e = ensure_smem(kernel, L1.total, dev.ordinal);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv)");
      int occ1 = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ1, kernel, kGemvWarps * 32, L1.total);
      if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
      if ((long long)R * c.cs <= (long long)dev.sms * occ1) {
        st_pick = 1;
        smem_pick = L1.total;
        slots = (long long)dev.sms * occ1;
      }
    }
    // More than one wave with fewer chunks per warp: a third stage lets a
    // persistent CTA prefetch its next row group's first chunk
    // (11008 x 4096: 10.96 vs 11.51 us; grouped q/k/v 12288 x 4096: 11.93 vs
    // 12.29 us, in PDL chains; single-wave shapes gain nothing).
    if (!forced && c.st == 2 && st_pick == 2 && (long long)R * c.cs > slots && mw < 4 && c.cs <= 2) {
      const GemvSmemLayout L3 = gemv_smem_layout<F>(B, K, GS, c.cs, 3, c.cp);
      if (L3.total <= dev.smem_optin) {
        e = ensure_smem(kernel, L3.total, dev.ordinal);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv)");
        int occ3 = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ3, kernel, kGemvWarps * 32, L3.total);
        if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        if (occ3 >= 1) {
          st_pick = 3;
          smem_pick = L3.total;
          slots = (long long)dev.sms * occ3;
        }
      }
    }
    out->cs = c.cs;
    out->stages = st_pick;
    out->copy = c.cp;
    out->nclusters = (long long)R * c.cs <= slots ? R : (int)(slots / c.cs);
    out->smem = smem_pick;
    if (TP && c.cs > 1) {
      // The finisher CTAs wait for rows of every other cluster, so the whole
      // grid must be resident at once: cap the clusters at what the GPU can
      // hold together (cluster placement can allow fewer than slots / cs).
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(out->nclusters * c.cs);
      cfg.blockDim = dim3(kGemvWarps * 32);
      cfg.dynamicSmemBytes = smem_pick;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = c.cs;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int max_clusters = 0;
      e = cudaOccupancyMaxActiveClusters(&max_clusters, kernel, &cfg);
      if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
      if (max_clusters < 1) continue;
      if (out->nclusters > max_clusters) out->nclusters = max_clusters;
    }
    return GDSQ_OK;
  }
  return fail(GDSQ_ERR_UNSUPPORTED, "no GEMV launch plan fits shared memory");
}

// `wlist` (host array of `p.count` weight pointers) for a grouped launch whose
// rg_start / ys / ns the caller has filled; nullptr for a plain launch.
template <int F, int B, int GS, bool TP = false>
int launch_fast(GemvParams p, const DeviceInfo& dev, cudaStream_t stream, const void* const* wlist = nullptr) {
  if (wlist == nullptr) {
    p.count = 1;
    p.rg_start[0] = 0;
    for (int m = 1; m <= kMaxGroup; ++m) p.rg_start[m] = (p.N + 31) / 32;
    p.ys[0] = p.y;
    p.ns[0] = p.N;
  } else {
    for (int m = p.count + 1; m <= kMaxGroup; ++m) p.rg_start[m] = p.rg_start[p.count];
    p.N = p.rg_start[p.count] * 32;  // the planner sees the concatenated rows
  }
  const uint64_t key = ((uint64_t)TP << 63) | ((uint64_t)F << 60) | ((uint64_t)B << 54) | ((uint64_t)GS << 44) |
                       ((uint64_t)(unsigned)p.N << 22) | (uint64_t)(unsigned)(p.K / 32);
  GemvPlan plan;
  int ocs, ost, ocp;
  const bool forced = plan_override(&ocs, &ost, &ocp);  // tuning runs: plan afresh, do not cache
  bool have = false;
  if (!forced) {
    std::lock_guard<std::mutex> lock(g_plan_mutex);
    auto it = g_plans[dev.ordinal].find(key);
    if (it != g_plans[dev.ordinal].end()) {
      plan = it->second;
      have = true;
    }
  }
  if (!have) {
    int st = make_plan<F, B, GS, TP>(p.N, p.K, dev, &plan);
    if (st != GDSQ_OK) return st;
    if (!forced) {
      std::lock_guard<std::mutex> lock(g_plan_mutex);
      g_plans[dev.ordinal][key] = plan;
    }
  }
  CUtensorMap maps[kMaxGroup];
  for (int m = 0; m < p.count; ++m) {
    const void* wm = wlist ? wlist[m] : p.w;
    int mst = weight_map<F>(dev, wm, p.ns[m], p.row_bytes, &maps[m]);
    if (mst != GDSQ_OK) return mst;
  }
  for (int m = p.count; m < kMaxGroup; ++m) maps[m] = maps[0];
  auto kernel = gemv_fast_kernel<F, B, GS, TP>;
  cudaError_t e = ensure_smem(kernel, plan.smem, dev.ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv)");
  p.cs = plan.cs;
  p.stages = plan.stages;
  p.copy = plan.copy;
  p.num_rg = p.rg_start[p.count];

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.nclusters * plan.cs);
  cfg.blockDim = dim3(kGemvWarps * 32);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (plan.cs > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = plan.cs;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (g_pdl_enabled) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  e = cudaLaunchKernelEx(&cfg, kernel, p, maps[0], maps[1], maps[2], maps[3]);
  if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
  return GDSQ_OK;
}

template <int F>
int launch_fast_group(const GemvParams& p, const DeviceInfo& dev, cudaStream_t stream, const void* const* wl) {
  switch (batch_tile(p.nb)) {
    case 1: return launch_fast<F, 1, 0>(p, dev, stream, wl);
    case 2: return launch_fast<F, 2, 0>(p, dev, stream, wl);
    case 3: return launch_fast<F, 3, 0>(p, dev, stream, wl);
    default: return launch_fast<F, 4, 0>(p, dev, stream, wl);
  }
}

template <int F, int GS>
int launch_fast_batch(const GemvParams& p, const DeviceInfo& dev, cudaStream_t stream) {
  switch (batch_tile(p.nb)) {
    case 1: return launch_fast<F, 1, GS>(p, dev, stream);
    case 2: return launch_fast<F, 2, GS>(p, dev, stream);
    case 3: return launch_fast<F, 3, GS>(p, dev, stream);
    case 4: return launch_fast<F, 4, GS>(p, dev, stream);
    case 8: return launch_fast<F, 8, GS>(p, dev, stream);
    default: return launch_fast<F, 16, GS>(p, dev, stream);
  }
}

// Tensor-core batched GEMV (gemv_tcb.cuh): the default where the CUDA-core
// kernel's multiply-add work (linear in the batch) outgrows the tensor-core
// kernel's fixed dequantization cost (tcb_default); GDSQ_GEMV_TCB=0 turns it
// off, =1 uses it for every batch size.
int tcb_mode() {
  const char* e = getenv("GDSQ_GEMV_TCB");
  if (!e || !*e) return -1;
  return e[0] == '1' ? 1 : 0;
}

// The tensor-core kernel's time is nearly flat in the batch; the CUDA-core
// kernel's grows with it, soonest for long rows and tall matrices.  Measured
// per launch in graph chains with programmatic dependent launch (CUDA cores
// vs tensor cores):
//   K = 11008, batch 3: Q8_0 29.5 vs 23.7 us, Q4_0 and affine-Q4 equal;
//              batch 4: Q4_0 38.9 vs 22.6, Q8_0 40.6 vs 23.8, affine 27.8 vs 23.2 us;
//   N = 32000, batch 4: Q8_0 62.0 vs 53.8, affine 78.7 vs 52.1 us, Q4_0 equal;
//   K = 4096 and N <= 11008, batch 4: within 5 % either way, except
//              affine 4096 x 4096 (9.7 vs 12.3 us), so these stay on CUDA cores.
bool tcb_default(int batch, int out_dim, int in_dim) {
  if (batch >= 5) return true;
  if (batch >= 3 && in_dim >= 8192) return true;
  return batch == 4 && out_dim >= 16384;
}

// One CTA per SM.  Cost = the busiest CTA's chunks (plus two chunks' worth
// of fixed cost per row tile: pipeline fill, epilogue, cluster reduction),
// with a small penalty per cluster doubling.
template <int F, int B, int GS>
int make_tcb_plan(int N, int K, const DeviceInfo& dev, GemvPlan* out) {
  auto kernel = gemv_tcb_kernel<F, B, GS>;
  const int R = (N + kTbRows - 1) / kTbRows;
  const int C = K / kChunkCols;
  int force_cs = 0, force_st = 0, force_cp = 0;
  const bool forced = plan_override(&force_cs, &force_st, &force_cp);
  double best = 1e30;
  bool found = false;
  for (int cs = 1; cs <= kTbMaxCluster; cs *= 2) {
    if (cs > C || cs > dev.sms) break;
    if (forced && cs != force_cs) continue;
    const int cslice = (C + cs - 1) / cs;
    for (int st = 3; st <= kTbMaxStages; ++st) {
      if (forced && st != force_st) continue;
      const TbLayout L = tb_layout<F, B>(cs, st);
      if (L.total > dev.smem_optin) continue;
      const int nclusters = (int)((long long)R * cs <= dev.sms ? R : dev.sms / cs);
      const int items = (R + nclusters - 1) / nclusters;
      const double cost = (double)items * (cslice + 2) * (1.0 + 0.04 * (cs > 1) + 0.02 * (cs > 2) + 0.02 * (cs > 4)) *
                          (1.0 - 0.01 * st);
      if (cost < best) {
        best = cost;
        found = true;
        out->cs = cs;
        out->stages = st;
        out->copy = 1;
        out->nclusters = nclusters;
        out->smem = L.total;
      }
    }
  }
  if (!found) return fail(GDSQ_ERR_UNSUPPORTED, "no tensor-core GEMV plan fits shared memory");
  cudaError_t e = ensure_smem(kernel, out->smem, dev.ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv tcb)");
  return GDSQ_OK;
}

template <int F, int B, int GS>
int launch_tcb(GemvParams p, const DeviceInfo& dev, cudaStream_t stream) {
  const uint64_t key = ((uint64_t)3 << 62) | ((uint64_t)F << 58) | ((uint64_t)B << 52) | ((uint64_t)GS << 42) |
                       ((uint64_t)(unsigned)p.N << 20) | (uint64_t)(unsigned)(p.K / 32);
  GemvPlan plan;
  int ocs, ost, ocp;
  const bool forced = plan_override(&ocs, &ost, &ocp);  // tuning runs: plan afresh, do not cache
  bool have = false;
  if (!forced) {
    std::lock_guard<std::mutex> lock(g_plan_mutex);
    auto it = g_plans[dev.ordinal].find(key);
    if (it != g_plans[dev.ordinal].end()) {
      plan = it->second;
      have = true;
    }
  }
  if (!have) {
    int st = make_tcb_plan<F, B, GS>(p.N, p.K, dev, &plan);
    if (st != GDSQ_OK) return st;
    if (!forced) {
      std::lock_guard<std::mutex> lock(g_plan_mutex);
      g_plans[dev.ordinal][key] = plan;
    }
  }
  CUtensorMap wmap;
  int mst = weight_map<F>(dev, p.w, p.N, p.row_bytes, &wmap, kTbRows);
  if (mst != GDSQ_OK) return mst;
  auto kernel = gemv_tcb_kernel<F, B, GS>;
  cudaError_t e = ensure_smem(kernel, plan.smem, dev.ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv tcb)");
  p.cs = plan.cs;
  p.stages = plan.stages;
  p.copy = 1;
  p.num_rg = (p.N + kTbRows - 1) / kTbRows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.nclusters * plan.cs);
  cfg.blockDim = dim3(kTbThreads);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (plan.cs > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = plan.cs;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (g_pdl_enabled) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  e = cudaLaunchKernelEx(&cfg, kernel, p, wmap);
  if (e != cudaSuccess) return cuda_fail(e, "gemv tcb launch");
  return GDSQ_OK;
}

template <int F, int GS>
int launch_tcb_batch(const GemvParams& p, const DeviceInfo& dev, cudaStream_t stream) {
  switch (batch_tile(p.nb)) {
    case 1: return launch_tcb<F, 1, GS>(p, dev, stream);
    case 2: return launch_tcb<F, 2, GS>(p, dev, stream);
    case 3: return launch_tcb<F, 3, GS>(p, dev, stream);
    case 4: return launch_tcb<F, 4, GS>(p, dev, stream);
    case 8: return launch_tcb<F, 8, GS>(p, dev, stream);
    default: return launch_tcb<F, 16, GS>(p, dev, stream);
  }
}

template <int F>
int launch_generic(const GemvParams& p, cudaStream_t stream) {
  const dim3 grid((p.N + 7) / 8);
  cudaError_t e = launch(gemv_generic_kernel<F>, grid, dim3(256), 0, stream, g_pdl_enabled != 0, p);
  if (e != cudaSuccess) return cuda_fail(e, "gemv (generic) launch");
  return GDSQ_OK;
}

// Smallest shared-memory footprint of the fast kernel (stages = 1, widest
// cluster split): if even this does not fit, use the generic kernel.
template <int F>
int fast_min_smem(int nb, int K, int group) {
  const int C = K / kChunkCols;
  int cs = 1;
  while (cs * 2 <= kMaxCluster && cs * 2 <= C) cs *= 2;
  return gemv_smem_layout<F>(batch_tile(nb), K, group, cs, 1, 1).total;
}

// Tensor-parallel exchange of gdsq_fused_gemv_allreduce (host arrays of the
// ranks' exchange buffers and flags).
struct TpExchange {
  int world;
  int rank;
  int rows;
  const void* const* bufs;
  void* const* flags;
};

int gemv_dispatch(int fmt, const void* w, const void* scales, const void* biases, const void* x,
                  void* y, int out_dim, int in_dim, int group, int batch, void* stream_v,
                  const TpExchange* tp = nullptr) {
  t_last_error.clear();
  const char* name = fmt == kFmtQ4_0 ? "q4_0" : fmt == kFmtQ8_0 ? "q8_0" : "affine_q4";
  if (out_dim < 0 || in_dim < 0)
    return fail(GDSQ_ERR_INVALID_VALUE, "fused %s gemv: negative shape [%d, %d]", name, out_dim,
                in_dim);
  if (batch < 1 || batch > GDSQ_MAX_BATCH)
    return fail(GDSQ_ERR_INVALID_VALUE, "fused %s gemv: batch %d outside 1..%d", name, batch,
                GDSQ_MAX_BATCH);
  if (fmt == kFmtAffineQ4) {
    if (group <= 0 || group % 8 != 0)
      return fail(GDSQ_ERR_INVALID_VALUE, "fused affine_q4 gemv: group_size %d must be a positive multiple of 8", group);
    if (in_dim % group != 0)
      return fail(GDSQ_ERR_INVALID_VALUE, "fused affine_q4 gemv: in_dim %d is not a multiple of group_size %d", in_dim, group);
  } else if (in_dim % 32 != 0) {
    return fail(GDSQ_ERR_INVALID_VALUE, "fused %s gemv: in_dim must be a multiple of 32, got %d",
                name, in_dim);
  }
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (out_dim == 0) return GDSQ_OK;
  if (!y) return fail(GDSQ_ERR_INVALID_VALUE, "fused %s gemv: null output", name);
  if (!aligned(y, 2)) return fail(GDSQ_ERR_MISALIGNED, "fused %s gemv: output not 2-byte aligned", name);
  if (in_dim == 0) {
    cudaError_t e = cudaMemsetAsync(y, 0, (size_t)batch * out_dim * 2, stream);
    return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "cudaMemsetAsync");
  }
  if (!w || !x) return fail(GDSQ_ERR_INVALID_VALUE, "fused %s gemv: null weight or input", name);
  if (fmt == kFmtAffineQ4 && (!scales || !biases))
    return fail(GDSQ_ERR_INVALID_VALUE, "fused affine_q4 gemv: null scales or biases");
  if (!aligned(x, 2)) return fail(GDSQ_ERR_MISALIGNED, "fused %s gemv: input not 2-byte aligned", name);
  if (fmt == kFmtAffineQ4) {
    if (!aligned(w, 4)) return fail(GDSQ_ERR_MISALIGNED, "fused affine_q4 gemv: weight not 4-byte aligned");
    if (!aligned(scales, 2) || !aligned(biases, 2))
      return fail(GDSQ_ERR_MISALIGNED, "fused affine_q4 gemv: scales/biases not 2-byte aligned");
  } else if (!aligned(w, 2)) {
    return fail(GDSQ_ERR_MISALIGNED, "fused %s gemv: weight not 2-byte aligned", name);
  }

  const DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st != GDSQ_OK) return st;

  GemvParams p = {};
  p.w = static_cast<const uint8_t*>(w);
  p.scales = static_cast<const __half*>(scales);
  p.biases = static_cast<const __half*>(biases);
  p.x = static_cast<const __half*>(x);
  p.y = static_cast<__half*>(y);
  p.N = out_dim;
  p.K = in_dim;
  p.nb = batch;
  p.group = group;
  p.row_bytes = fmt == kFmtQ4_0 ? (long long)in_dim / 32 * 18
               : fmt == kFmtQ8_0 ? (long long)in_dim / 32 * 34
                                 : (long long)in_dim / 2;

  const bool shape_ok = in_dim % kChunkCols == 0 && aligned(w, 16) && aligned(x, 16);
  if (tp != nullptr) {
    // The exchange lives in the CUDA-core kernel's epilogue (batch 1).
    if (!shape_ok || batch != 1 || fmt == kFmtAffineQ4)
      return fail(GDSQ_ERR_UNSUPPORTED, "gemv allreduce: needs Q4_0/Q8_0, batch 1, in_dim %% 256 == 0 and 16-byte "
                  "aligned weight and input");
    p.tp_world = tp->world;
    p.tp_rank = tp->rank;
    p.tp_rows = tp->rows;
    for (int r = 0; r < tp->world; ++r) {
      p.tp_bufs[r] = static_cast<unsigned long long*>(const_cast<void*>(tp->bufs[r]));
      p.tp_flags[r] = static_cast<int*>(tp->flags[r]);
    }
    p.tp_own_buf = p.tp_bufs[tp->rank];
    p.tp_own_flags = p.tp_flags[tp->rank];
    p.tp_wait_ns = g_peer_wait_ns.load();
    if (fmt == kFmtQ4_0) return launch_fast<kFmtQ4_0, 1, 0, true>(p, *dev, stream);
    return launch_fast<kFmtQ8_0, 1, 0, true>(p, *dev, stream);
  }
  const int tcb = tcb_mode();
  const bool use_tcb = shape_ok && (tcb == 1 || (tcb == -1 && tcb_default(batch, out_dim, in_dim)));
  if (use_tcb) {
    if (fmt == kFmtQ4_0) return launch_tcb_batch<kFmtQ4_0, 0>(p, *dev, stream);
    if (fmt == kFmtQ8_0) return launch_tcb_batch<kFmtQ8_0, 0>(p, *dev, stream);
    switch (group) {
      case 32: return launch_tcb_batch<kFmtAffineQ4, 32>(p, *dev, stream);
      case 64: return launch_tcb_batch<kFmtAffineQ4, 64>(p, *dev, stream);
      case 128: return launch_tcb_batch<kFmtAffineQ4, 128>(p, *dev, stream);
      case 256: return launch_tcb_batch<kFmtAffineQ4, 256>(p, *dev, stream);
      default: break;  // other group sizes: CUDA-core kernels below
    }
  }
  if (fmt == kFmtQ4_0) {
    if (shape_ok && fast_min_smem<kFmtQ4_0>(batch, in_dim, 0) <= dev->smem_optin)
      return launch_fast_batch<kFmtQ4_0, 0>(p, *dev, stream);
    return launch_generic<kFmtQ4_0>(p, stream);
  }
  if (fmt == kFmtQ8_0) {
    if (shape_ok && fast_min_smem<kFmtQ8_0>(batch, in_dim, 0) <= dev->smem_optin)
      return launch_fast_batch<kFmtQ8_0, 0>(p, *dev, stream);
    return launch_generic<kFmtQ8_0>(p, stream);
  }
  const bool group_ok = group == 32 || group == 64 || group == 128 || group == 256;
  if (shape_ok && group_ok && fast_min_smem<kFmtAffineQ4>(batch, in_dim, group) <= dev->smem_optin) {
    switch (group) {
      case 32: return launch_fast_batch<kFmtAffineQ4, 32>(p, *dev, stream);
      case 64: return launch_fast_batch<kFmtAffineQ4, 64>(p, *dev, stream);
      case 128: return launch_fast_batch<kFmtAffineQ4, 128>(p, *dev, stream);
      default: return launch_fast_batch<kFmtAffineQ4, 256>(p, *dev, stream);
    }
  }
  return launch_generic<kFmtAffineQ4>(p, stream);
}

// ---------------------------------------------------------------------------
// MoE gather dispatch

struct MoePlan {
  int cs = 1;
  int stages = 2;
  int nclusters = 1;
  int smem = 0;
};

// Same cost model as make_plan, over `items` work items of C chunks each.
template <int STAGE, int GS>
int make_moe_plan(int items, int C, const DeviceInfo& dev, MoePlan* out) {
  auto kernel = moe_affine_kernel<STAGE, GS>;
  int force_cs = 0, force_st = 0;
  bool forced = false;
  // Tuning sweeps: "cs:stages" for both stages (GDSQ_MOE_PLAN) or one
  // (GDSQ_MOE_PLAN0 / GDSQ_MOE_PLAN1).
  const char* e_stage = getenv(STAGE == 0 ? "GDSQ_MOE_PLAN0" : "GDSQ_MOE_PLAN1");
  if (const char* e = e_stage ? e_stage : getenv("GDSQ_MOE_PLAN")) {
    forced = sscanf(e, "%d:%d", &force_cs, &force_st) == 2 && force_cs >= 1 && force_cs <= kMaxCluster &&
             force_st >= 1 && force_st <= kMaxStages;
  }
  double best = 1e30;
  bool found = false;
  // Gate/up (K = hidden, 16 + 16 rows per item, many items): measured on
  // B200 over the config-4 decode step, splits above 2 lose (B = 1: 306
  // tok/s at cs = 2 vs 267 at cs = 4), so the model chooses among 1 and 2.
  const int max_cs = STAGE == 0 ? 2 : kMaxCluster;
  for (int cs = 1; cs <= max_cs || (forced && cs <= kMaxCluster); cs *= 2) {
    if (cs > C) break;
    if (forced && cs != force_cs) continue;
    const int cslice = (C + cs - 1) / cs;
    for (int st = forced ? 1 : 2; st <= 4; ++st) {
      if (forced && st != force_st) continue;
      const MoeSmemLayout L = moe_smem_layout(C, GS, cs, st);
      if (L.total > dev.smem_optin) continue;
      cudaError_t e = ensure_smem(kernel, L.total, dev.ordinal);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(moe)");
      int occ = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kGemvWarps * 32, L.total);
      if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
      if (occ < 1) continue;
      const long long slots = (long long)dev.sms * occ;
      const long long ctas = (long long)items * cs;
      // Down stage with more CTAs than one wave holds (batch 8: 1024 items
      // of 44 chunks): a wider split or a deeper ring only adds CTAs or
      // shared memory.  Config 4 at batch 8, cs:stages: 2:2 505 tok/s, 2:4
      // 452, 4:2 430, 4:3 367, 8:2 379.
      if (STAGE == 1 && !forced && ctas > slots && (cs > 2 || st > 2)) continue;
      double load;
      long long resident;
      int nclusters;
      if (ctas <= slots) {
        nclusters = items;
        resident = (ctas + dev.sms - 1) / dev.sms;
        load = (double)resident * (cslice + 1);
      } else {
        nclusters = (int)(slots / cs);
        const int per = (items + nclusters - 1) / nclusters;
        resident = occ;
        load = (double)occ * per * (cslice + 1);
      }
      const double warps = (double)resident * kGemvWarps;
      const double eff = warps >= 16 ? 1.0 : warps / 16.0;
      const double cost = load / eff * (1.0 + 0.02 * cs) / (1.0 + 0.01 * st);
      if (cost < best) {
        best = cost;
        found = true;
        out->cs = cs;
        out->stages = st;
        out->nclusters = nclusters;
        out->smem = L.total;
      }
    }
  }
  if (!found) return fail(GDSQ_ERR_UNSUPPORTED, "no MoE launch plan fits shared memory");
  // As for the plain GEMV: a one-stage ring is faster when it holds every
  // item in one wave of at least 4 CTAs per SM with at least 4 chunks per
  // warp (config 4 gate/up at batch 1: 316.6 vs 303.8 tok/s).  At batch 8
  // no such plan fits, and the down stage at batch 1 (128 items) has too
  // few CTAs; the model's choice stays there.
  if (!forced) {
    cudaError_t e = cudaSuccess;
    {
      for (int cs = 1; cs <= kMaxCluster && cs <= C; cs *= 2) {
        const int mw = ((C + cs - 1) / cs + kGemvWarps - 1) / kGemvWarps;
        if (mw < 4 || (long long)items * cs < 4LL * dev.sms) continue;
        const MoeSmemLayout L1 = moe_smem_layout(C, GS, cs, 1);
        if (L1.total > dev.smem_optin) continue;
        e = ensure_smem(kernel, L1.total, dev.ordinal);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(moe)");
        int occ1 = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ1, kernel, kGemvWarps * 32, L1.total);
        if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        if ((long long)items * cs <= (long long)dev.sms * occ1) {
          out->cs = cs;
          out->stages = 1;
          out->nclusters = items;
          out->smem = L1.total;
          break;
        }
      }
    }
  }
  return GDSQ_OK;
}

template <int STAGE, int GS>
int launch_moe_fast(MoeParams p, const void* w0, const void* w1, const void* sw0, const void* sw1,
                    const DeviceInfo& dev, cudaStream_t stream) {
  const int cpe = p.K / kChunkCols;
  const int C = STAGE == 0 ? cpe : p.Ts * cpe;
  p.num_items = STAGE == 0 ? p.ntok * p.Ts * (p.rows / 16) : p.ntok * (p.rows / 32);
  const uint64_t key = ((uint64_t)1 << 63) | ((uint64_t)STAGE << 61) | ((uint64_t)GS << 50) |
                       ((uint64_t)(unsigned)p.num_items << 16) | (uint64_t)(unsigned)C;
  MoePlan plan;
  bool have = false;
  static std::unordered_map<uint64_t, MoePlan> plans[kMaxDevices];
  {
    std::lock_guard<std::mutex> lock(g_plan_mutex);
    auto it = plans[dev.ordinal].find(key);
    if (it != plans[dev.ordinal].end()) {
      plan = it->second;
      have = true;
    }
  }
  if (!have) {
    int st = make_moe_plan<STAGE, GS>(p.num_items, C, dev, &plan);
    if (st != GDSQ_OK) return st;
    std::lock_guard<std::mutex> lock(g_plan_mutex);
    plans[dev.ordinal][key] = plan;
  }
  CUtensorMap m0, m1, s0, s1;
  const int box_rows = STAGE == 0 ? 16 : 32;
  int st = expert_map(dev, w0, p.e_count, p.rows, p.K, box_rows, &m0);
  if (st != GDSQ_OK) return st;
  m1 = m0;
  if (STAGE == 0) {
    st = expert_map(dev, w1, p.e_count, p.rows, p.K, box_rows, &m1);
    if (st != GDSQ_OK) return st;
  }
  s0 = m0;
  s1 = m1;
  if (p.has_shared) {
    st = expert_map(dev, sw0, 1, p.rows, p.K, box_rows, &s0);
    if (st != GDSQ_OK) return st;
    if (STAGE == 0) {
      st = expert_map(dev, sw1, 1, p.rows, p.K, box_rows, &s1);
      if (st != GDSQ_OK) return st;
    }
  }
  auto kernel = moe_affine_kernel<STAGE, GS>;
  cudaError_t e = ensure_smem(kernel, plan.smem, dev.ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(moe)");
  p.cs = plan.cs;
  p.stages = plan.stages;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.nclusters * plan.cs);
  cfg.blockDim = dim3(kGemvWarps * 32);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (plan.cs > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = plan.cs;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (g_pdl_enabled) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  e = cudaLaunchKernelEx(&cfg, kernel, p, m0, m1, s0, s1);
  if (e != cudaSuccess) return cuda_fail(e, STAGE == 0 ? "moe gate/up launch" : "moe down launch");
  return GDSQ_OK;
}

// Shared argument checks and path choice of both MoE stages.  Matrix 0 is
// gate (stage 0) or down (stage 1); matrix 1 is up (stage 0 only).
int moe_dispatch(int stage, const void* w0, const void* s0, const void* b0, const void* w1,
                 const void* s1, const void* b1, const void* shw0, const void* shs0, const void* shb0,
                 const void* shw1, const void* shs1, const void* shb1, const void* shared_route,
                 const void* x, const int32_t* ids, const void* route, void* out, int ntok, int top_k,
                 int rows, int cols, int group, int e_first, int e_count, int e_total, int flags,
                 void* stream_v, const void* residual = nullptr) {
  t_last_error.clear();
  const char* name = stage == 0 ? "moe gate/up" : "moe down";
  if (residual && (stage != 1 || (flags & (kMoeOutF32 | kMoeAccumulate)) || !aligned(residual, 2)))
    return fail(GDSQ_ERR_INVALID_VALUE, "%s: a residual needs the down stage's fp16 output without "
                "accumulation, 2-byte aligned", name);
  // The shared expert is present when all of its pointers are given.
  const void* sh_ptrs[7] = {shw0, shs0, shb0, shw1, shs1, shb1, shared_route};
  const int n_sh = stage == 0 ? 6 : 3;
  int given = 0;
  for (int i = 0; i < n_sh; ++i) given += sh_ptrs[i] != nullptr;
  if (stage == 1) given += shared_route != nullptr;
  const int n_need = stage == 0 ? 6 : 4;
  if (given != 0 && given != n_need)
    return fail(GDSQ_ERR_INVALID_VALUE, "%s: shared expert pointers must be all given or all null", name);
  const int has_shared = given == n_need ? 1 : 0;
  if (ntok < 0 || top_k < 1 || top_k + has_shared > kMoeMaxSlots)
    return fail(GDSQ_ERR_INVALID_VALUE, "%s: num_tokens %d must be >= 0 and top_k %d in 1..%d", name, ntok,
                top_k, kMoeMaxSlots - has_shared);
  if (rows <= 0 || cols <= 0)
    return fail(GDSQ_ERR_INVALID_VALUE, "%s: expert matrix shape [%d, %d] must be positive", name, rows, cols);
  if (group <= 0 || group % 8 != 0 || cols % group != 0)
    return fail(GDSQ_ERR_INVALID_VALUE, "%s: group_size %d must be a positive multiple of 8 dividing %d", name,
                group, cols);
  if (e_first < 0 || e_count < 1 || e_total < 1 || (long long)e_first + e_count > e_total)
    return fail(GDSQ_ERR_INVALID_VALUE, "%s: resident experts [%d, %d) outside 0..%d", name, e_first,
                e_first + e_count, e_total);
  if (flags & ~(kMoeOutF32 | kMoeAccumulate | kMoeClamp))
    return fail(GDSQ_ERR_INVALID_VALUE, "%s: unknown flags 0x%x", name, flags);
  const long long pairs = (long long)ntok * (top_k + has_shared);
  if (pairs * rows > (1ll << 30))
    return fail(GDSQ_ERR_INVALID_VALUE, "%s: %lld outputs is too many for one call", name, pairs * rows);
  if (ntok == 0) return GDSQ_OK;
  if (!w0 || !s0 || !b0 || !x || !ids || !out || (stage == 0 && (!w1 || !s1 || !b1)) || (stage == 1 && !route))
    return fail(GDSQ_ERR_INVALID_VALUE, "%s: null pointer", name);
  if (!aligned(w0, 4) || (stage == 0 && !aligned(w1, 4)) ||
      (has_shared && (!aligned(shw0, 4) || (stage == 0 && !aligned(shw1, 4)))))
    return fail(GDSQ_ERR_MISALIGNED, "%s: expert weights must be 4-byte aligned", name);
  if (has_shared && (!aligned(shs0, 2) || !aligned(shb0, 2) || (stage == 0 && (!aligned(shs1, 2) || !aligned(shb1, 2))) ||
                     (stage == 1 && !aligned(shared_route, 2))))
    return fail(GDSQ_ERR_MISALIGNED, "%s: shared expert scales, biases and weights need 2-byte alignment", name);
  if (!aligned(s0, 2) || !aligned(b0, 2) || (stage == 0 && (!aligned(s1, 2) || !aligned(b1, 2))) ||
      !aligned(x, 2) || (stage == 1 && !aligned(route, 2)))
    return fail(GDSQ_ERR_MISALIGNED, "%s: scales, biases, activations and weights of the route need 2-byte alignment",
                name);
  if (!aligned(ids, 4)) return fail(GDSQ_ERR_MISALIGNED, "%s: expert ids must be 4-byte aligned", name);
  if (!aligned(out, (stage == 1 && (flags & kMoeOutF32)) ? 4 : 2))
    return fail(GDSQ_ERR_MISALIGNED, "%s: output misaligned", name);

  const DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st != GDSQ_OK) return st;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);

  MoeParams p = {};
  p.s0 = static_cast<const __half*>(s0);
  p.b0 = static_cast<const __half*>(b0);
  p.s1 = static_cast<const __half*>(s1);
  p.b1 = static_cast<const __half*>(b1);
  p.x = static_cast<const __half*>(x);
  p.ids = ids;
  p.route = static_cast<const __half*>(route);
  p.out = out;
  p.ntok = ntok;
  p.T = top_k;
  p.e_first = e_first;
  p.e_count = e_count;
  p.e_total = e_total;
  p.rows = rows;
  p.K = cols;
  p.flags = stage == 1 ? flags : 0;
  p.residual = static_cast<const __half*>(residual);
  p.w0 = static_cast<const uint32_t*>(w0);
  p.w1 = static_cast<const uint32_t*>(w1);
  p.group = group;
  p.has_shared = has_shared;
  p.Ts = top_k + has_shared;
  p.ss0 = static_cast<const __half*>(shs0);
  p.sb0 = static_cast<const __half*>(shb0);
  p.ss1 = static_cast<const __half*>(shs1);
  p.sb1 = static_cast<const __half*>(shb1);
  p.shared_route = static_cast<const __half*>(shared_route);
  p.sw0 = static_cast<const uint32_t*>(shw0);
  p.sw1 = static_cast<const uint32_t*>(shw1);

  const bool fast = cols % kChunkCols == 0 && rows % (stage == 0 ? 16 : 32) == 0 && aligned(w0, 16) &&
                    (stage == 1 || aligned(w1, 16)) && aligned(x, 16) &&
                    (!has_shared || (aligned(shw0, 16) && (stage == 1 || aligned(shw1, 16)))) &&
                    (group == 32 || group == 64 || group == 128 || group == 256) &&
                    moe_smem_layout(stage == 0 ? cols / kChunkCols : p.Ts * cols / kChunkCols, group,
                                    kMaxCluster, 2).total <= dev->smem_optin;
  if (fast) {
    if (stage == 0) {
      switch (group) {
        case 32: return launch_moe_fast<0, 32>(p, w0, w1, shw0, shw1, *dev, stream);
        case 64: return launch_moe_fast<0, 64>(p, w0, w1, shw0, shw1, *dev, stream);
        case 128: return launch_moe_fast<0, 128>(p, w0, w1, shw0, shw1, *dev, stream);
        default: return launch_moe_fast<0, 256>(p, w0, w1, shw0, shw1, *dev, stream);
      }
    }
    switch (group) {
      case 32: return launch_moe_fast<1, 32>(p, w0, w1, shw0, shw1, *dev, stream);
      case 64: return launch_moe_fast<1, 64>(p, w0, w1, shw0, shw1, *dev, stream);
      case 128: return launch_moe_fast<1, 128>(p, w0, w1, shw0, shw1, *dev, stream);
      default: return launch_moe_fast<1, 256>(p, w0, w1, shw0, shw1, *dev, stream);
    }
  }
  const long long warps = stage == 0 ? pairs * rows : (long long)ntok * rows;
  const dim3 grid(static_cast<unsigned>((warps + 7) / 8));
  cudaError_t e = stage == 0 ? launch(moe_gate_up_generic_kernel, grid, dim3(256), 0, stream, g_pdl_enabled != 0, p)
                             : launch(moe_down_generic_kernel, grid, dim3(256), 0, stream, g_pdl_enabled != 0, p);
  if (e != cudaSuccess) return cuda_fail(e, stage == 0 ? "moe gate/up (generic) launch" : "moe down (generic) launch");
  return GDSQ_OK;
}

// ---------------------------------------------------------------------------
// Dequant dispatch

unsigned dequant_grid(uint64_t units, const DeviceInfo& dev) {
  const uint64_t need = (units + 255) / 256;
  const uint64_t cap = (uint64_t)dev.sms * 16;
  return static_cast<unsigned>(need < cap ? need : cap);
}

}  // namespace
}  // namespace gdsq

using namespace gdsq;

extern "C" {

int gdsq_version(void) { return 100; }

const char* gdsq_status_string(int status) {
  switch (status) {
    case GDSQ_OK: return "ok";
    case GDSQ_ERR_INVALID_VALUE: return "invalid value";
    case GDSQ_ERR_MISALIGNED: return "misaligned pointer";
    case GDSQ_ERR_UNSUPPORTED: return "unsupported";
    case GDSQ_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

const char* gdsq_last_error(void) { return t_last_error.c_str(); }

int gdsq_set_pdl(int enable) {
  g_pdl_enabled = enable ? 1 : 0;
  return GDSQ_OK;
}

unsigned long long gdsq_set_peer_wait_limit_ns(unsigned long long ns) {
  return g_peer_wait_ns.exchange(ns == 0 ? kPeerWaitDefaultNs : ns);
}

int gdsq_device_error(int device, int clear, int* out_bits) {
  t_last_error.clear();
  if (!out_bits) return fail(GDSQ_ERR_INVALID_VALUE, "gdsq_device_error: null output");
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  int bits = 0;
  e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&bits, g_device_error, sizeof(int));
  if (e == cudaSuccess && clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  *out_bits = bits;
  return GDSQ_OK;
}

int gdsq_dequant_q4_0(const void* src, void* dst, uint64_t num_blocks, void* stream_v) {
  t_last_error.clear();
  if (num_blocks == 0) return GDSQ_OK;
  if (!src || !dst) return fail(GDSQ_ERR_INVALID_VALUE, "dequant q4_0: null pointer");
  if (!aligned(src, 2) || !aligned(dst, 2))
    return fail(GDSQ_ERR_MISALIGNED, "dequant q4_0: pointers must be 2-byte aligned");
  const DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st != GDSQ_OK) return st;
  const uint64_t units = num_blocks * 4;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  const unsigned grid = dequant_grid(units, *dev);
  const uint8_t* s = static_cast<const uint8_t*>(src);
  __half* d = static_cast<__half*>(dst);
  cudaError_t e = aligned(dst, 16)
                      ? launch(dequant_q4_0_kernel<true>, dim3(grid), dim3(256), 0, stream, false, s, d, units)
                      : launch(dequant_q4_0_kernel<false>, dim3(grid), dim3(256), 0, stream, false, s, d, units);
  return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "dequant q4_0 launch");
}

int gdsq_dequant_q8_0(const void* src, void* dst, uint64_t num_blocks, void* stream_v) {
  t_last_error.clear();
  if (num_blocks == 0) return GDSQ_OK;
  if (!src || !dst) return fail(GDSQ_ERR_INVALID_VALUE, "dequant q8_0: null pointer");
  if (!aligned(src, 2) || !aligned(dst, 2))
    return fail(GDSQ_ERR_MISALIGNED, "dequant q8_0: pointers must be 2-byte aligned");
  const DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st != GDSQ_OK) return st;
  const uint64_t units = num_blocks * 4;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  const unsigned grid = dequant_grid(units, *dev);
  const uint8_t* s = static_cast<const uint8_t*>(src);
  __half* d = static_cast<__half*>(dst);
  cudaError_t e = aligned(dst, 16)
                      ? launch(dequant_q8_0_kernel<true>, dim3(grid), dim3(256), 0, stream, false, s, d, units)
                      : launch(dequant_q8_0_kernel<false>, dim3(grid), dim3(256), 0, stream, false, s, d, units);
  return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "dequant q8_0 launch");
}

int gdsq_dequant_rows_gguf(int gguf_type, const void* table, long long rows, int cols, const long long* ids,
                           long long num_ids, void* dst, void* stream_v) {
  t_last_error.clear();
  if (gguf_type != GDSQ_TYPE_Q4_0 && gguf_type != GDSQ_TYPE_Q8_0)
    return fail(GDSQ_ERR_INVALID_VALUE, "dequant rows: gguf_type %d is neither Q4_0 nor Q8_0", gguf_type);
  if (rows < 0 || cols < 0 || cols % 32 != 0 || num_ids < 0)
    return fail(GDSQ_ERR_INVALID_VALUE, "dequant rows: table [%lld, %d] (cols must be a multiple of 32), %lld ids",
                rows, cols, num_ids);
  if (num_ids == 0 || cols == 0) return GDSQ_OK;
  if (!table || !ids || !dst) return fail(GDSQ_ERR_INVALID_VALUE, "dequant rows: null pointer");
  if (!aligned(table, 2) || !aligned(dst, 2) || !aligned(ids, 8))
    return fail(GDSQ_ERR_MISALIGNED, "dequant rows: table/output must be 2-byte and ids 8-byte aligned");
  const DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st != GDSQ_OK) return st;
  const uint64_t units = (uint64_t)num_ids * (cols / 32) * 4;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  const unsigned grid = dequant_grid(units, *dev);
  const uint8_t* s = static_cast<const uint8_t*>(table);
  __half* d = static_cast<__half*>(dst);
  const int bpr = cols / 32;
  const bool vec = aligned(dst, 16);
  cudaError_t e;
  if (gguf_type == GDSQ_TYPE_Q4_0)
    e = vec ? launch(dequant_rows_kernel<0, true>, dim3(grid), dim3(256), 0, stream, false, s, ids, rows, bpr, d, units)
            : launch(dequant_rows_kernel<0, false>, dim3(grid), dim3(256), 0, stream, false, s, ids, rows, bpr, d,
                     units);
  else
    e = vec ? launch(dequant_rows_kernel<1, true>, dim3(grid), dim3(256), 0, stream, false, s, ids, rows, bpr, d, units)
            : launch(dequant_rows_kernel<1, false>, dim3(grid), dim3(256), 0, stream, false, s, ids, rows, bpr, d,
                     units);
  return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "dequant rows launch");
}

int gdsq_dequant_affine_q4(const void* weight, const void* scales, const void* biases, void* dst,
                           uint64_t num_elements, int in_dim, int group_size, void* stream_v) {
  t_last_error.clear();
  if (group_size <= 0 || group_size % 8 != 0)
    return fail(GDSQ_ERR_INVALID_VALUE, "dequant affine_q4: group_size %d must be a positive multiple of 8", group_size);
  if (in_dim <= 0 || in_dim % group_size != 0)
    return fail(GDSQ_ERR_INVALID_VALUE, "dequant affine_q4: in_dim %d is not a positive multiple of group_size %d", in_dim, group_size);
  if (num_elements % (uint64_t)in_dim != 0)
    return fail(GDSQ_ERR_INVALID_VALUE, "dequant affine_q4: %llu elements is not a whole number of rows of %d",
                (unsigned long long)num_elements, in_dim);
  if (num_elements == 0) return GDSQ_OK;
  if (!weight || !scales || !biases || !dst)
    return fail(GDSQ_ERR_INVALID_VALUE, "dequant affine_q4: null pointer");
  if (!aligned(weight, 4) || !aligned(scales, 2) || !aligned(biases, 2) || !aligned(dst, 2))
    return fail(GDSQ_ERR_MISALIGNED, "dequant affine_q4: weight needs 4-byte, scales/biases/output 2-byte alignment");
  const DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st != GDSQ_OK) return st;
  const uint64_t units = num_elements / 8;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  const unsigned grid = dequant_grid(units, *dev);
  const uint32_t* w = static_cast<const uint32_t*>(weight);
  const __half* s = static_cast<const __half*>(scales);
  const __half* b = static_cast<const __half*>(biases);
  __half* d = static_cast<__half*>(dst);
  cudaError_t e = aligned(dst, 16)
                      ? launch(dequant_affine_q4_kernel<true>, dim3(grid), dim3(256), 0, stream, false, w, s, b, d, units, group_size)
                      : launch(dequant_affine_q4_kernel<false>, dim3(grid), dim3(256), 0, stream, false, w, s, b, d, units, group_size);
  return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "dequant affine_q4 launch");
}

int gdsq_fused_q4_0_gemv(const void* weight, const void* x, void* y, int out_dim, int in_dim,
                         int batch, void* stream) {
  return gemv_dispatch(kFmtQ4_0, weight, nullptr, nullptr, x, y, out_dim, in_dim, 0, batch, stream);
}

int gdsq_fused_q8_0_gemv(const void* weight, const void* x, void* y, int out_dim, int in_dim,
                         int batch, void* stream) {
  return gemv_dispatch(kFmtQ8_0, weight, nullptr, nullptr, x, y, out_dim, in_dim, 0, batch, stream);
}

int gdsq_fused_affine_q4_gemv(const void* weight, const void* scales, const void* biases,
                              const void* x, void* y, int out_dim, int in_dim, int group_size,
                              int batch, void* stream) {
  return gemv_dispatch(kFmtAffineQ4, weight, scales, biases, x, y, out_dim, in_dim, group_size,
                       batch, stream);
}

int gdsq_fused_gemv_allreduce(int gguf_type, const void* weight, const void* x, void* y, int out_dim, int in_dim,
                              const void* const* bufs, void* const* flags, int rows_cap, int rank, int world,
                              void* stream) {
  t_last_error.clear();
  if (gguf_type != GDSQ_TYPE_Q4_0 && gguf_type != GDSQ_TYPE_Q8_0)
    return fail(GDSQ_ERR_INVALID_VALUE, "gemv allreduce: gguf_type %d is neither Q4_0 nor Q8_0", gguf_type);
  if (world < 1 || world > kTpMaxRanks || rank < 0 || rank >= world)
    return fail(GDSQ_ERR_INVALID_VALUE, "gemv allreduce: rank %d of world %d (at most %d ranks)", rank, world,
                kTpMaxRanks);
  const int rgs = (out_dim + 31) / 32;
  if (out_dim < 0 || rgs > kTpMaxRowGroups || rgs * 32 > rows_cap)
    return fail(GDSQ_ERR_INVALID_VALUE, "gemv allreduce: out_dim %d needs %d rows of exchange buffer (have %d, at "
                "most %d)", out_dim, rgs * 32, rows_cap, kTpMaxRowGroups * 32);
  if (!bufs || !flags) return fail(GDSQ_ERR_INVALID_VALUE, "gemv allreduce: null buffer arrays");
  for (int r = 0; r < world; ++r)
    if (!bufs[r] || !flags[r] || !aligned(bufs[r], 8) || !aligned(flags[r], 4))
      return fail(GDSQ_ERR_MISALIGNED, "gemv allreduce: rank %d exchange buffer or flags null or misaligned", r);
  const int fmt = gguf_type == GDSQ_TYPE_Q4_0 ? kFmtQ4_0 : kFmtQ8_0;
  if (world == 1) return gemv_dispatch(fmt, weight, nullptr, nullptr, x, y, out_dim, in_dim, 0, 1, stream);
  TpExchange tp{world, rank, rows_cap, bufs, flags};
  return gemv_dispatch(fmt, weight, nullptr, nullptr, x, y, out_dim, in_dim, 0, 1, stream, &tp);
}

int gdsq_fused_gemv_group(int gguf_type, int count, const void* const* weights, const int* out_dims,
                          void* const* ys, const void* x, int in_dim, int batch, void* stream_v) {
  t_last_error.clear();
  if (gguf_type != GDSQ_TYPE_Q4_0 && gguf_type != GDSQ_TYPE_Q8_0)
    return fail(GDSQ_ERR_INVALID_VALUE, "gemv group: gguf_type %d is neither Q4_0 nor Q8_0", gguf_type);
  if (count < 1 || count > kMaxGroup || !weights || !out_dims || !ys)
    return fail(GDSQ_ERR_INVALID_VALUE, "gemv group: count %d outside 1..%d or null arrays", count, kMaxGroup);
  const int fmt = gguf_type == GDSQ_TYPE_Q4_0 ? kFmtQ4_0 : kFmtQ8_0;
  bool fast = batch >= 1 && batch <= 4 && in_dim > 0 && in_dim % kChunkCols == 0 && x && aligned(x, 16);
  for (int m = 0; m < count; ++m) {
    if (out_dims[m] < 0) return fail(GDSQ_ERR_INVALID_VALUE, "gemv group: negative out_dim %d", out_dims[m]);
    fast = fast && weights[m] && aligned(weights[m], 16) && out_dims[m] > 0 && ys[m] && aligned(ys[m], 2);
    // A matrix that the single GEMV would give to the tensor cores
    fast = fast && !(tcb_mode() == -1 && tcb_default(batch, out_dims[m], in_dim));
  }
  if (count == 1 || !fast || tcb_mode() == 1) {
    // One launch per matrix (every check and path of the single GEMV).
    for (int m = 0; m < count; ++m) {
      const int st = gemv_dispatch(fmt, weights[m], nullptr, nullptr, x, ys[m], out_dims[m], in_dim, 0, batch,
                                   stream_v);
      if (st != GDSQ_OK) return st;
    }
    return GDSQ_OK;
  }
  const DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st != GDSQ_OK) return st;
  GemvParams p = {};
  p.x = static_cast<const __half*>(x);
  p.K = in_dim;
  p.nb = batch;
  p.row_bytes = fmt == kFmtQ4_0 ? (long long)in_dim / 32 * 18 : (long long)in_dim / 32 * 34;
  p.count = count;
  p.rg_start[0] = 0;
  for (int m = 0; m < count; ++m) {
    p.ys[m] = static_cast<__half*>(ys[m]);
    p.ns[m] = out_dims[m];
    p.rg_start[m + 1] = p.rg_start[m] + (out_dims[m] + 31) / 32;
  }
  p.w = static_cast<const uint8_t*>(weights[0]);
  p.y = p.ys[0];
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (fmt == kFmtQ4_0) {
    if (fast_min_smem<kFmtQ4_0>(batch, in_dim, 0) > dev->smem_optin)
      return fail(GDSQ_ERR_UNSUPPORTED, "gemv group: no plan fits shared memory");
    return launch_fast_group<kFmtQ4_0>(p, *dev, stream, weights);
  }
  if (fast_min_smem<kFmtQ8_0>(batch, in_dim, 0) > dev->smem_optin)
    return fail(GDSQ_ERR_UNSUPPORTED, "gemv group: no plan fits shared memory");
  return launch_fast_group<kFmtQ8_0>(p, *dev, stream, weights);
}

int gdsq_moe_affine_q4_gate_up(const void* gate_weight, const void* gate_scales, const void* gate_biases,
                               const void* up_weight, const void* up_scales, const void* up_biases,
                               const void* shared_gate_weight, const void* shared_gate_scales,
                               const void* shared_gate_biases, const void* shared_up_weight,
                               const void* shared_up_scales, const void* shared_up_biases, const void* x,
                               const int32_t* expert_ids, void* h, int num_tokens, int top_k, int inter_dim,
                               int hidden_dim, int group_size, int expert_first, int expert_count,
                               int expert_total, void* stream) {
  return moe_dispatch(0, gate_weight, gate_scales, gate_biases, up_weight, up_scales, up_biases,
                      shared_gate_weight, shared_gate_scales, shared_gate_biases, shared_up_weight,
                      shared_up_scales, shared_up_biases, nullptr, x, expert_ids, nullptr, h, num_tokens, top_k,
                      inter_dim, hidden_dim, group_size, expert_first, expert_count, expert_total, 0, stream);
}

int gdsq_moe_affine_q4_down(const void* down_weight, const void* down_scales, const void* down_biases,
                            const void* shared_down_weight, const void* shared_down_scales,
                            const void* shared_down_biases, const void* h, const int32_t* expert_ids,
                            const void* route_weights, const void* shared_weights, void* y, int num_tokens,
                            int top_k, int hidden_dim, int inter_dim, int group_size, int expert_first,
                            int expert_count, int expert_total, int flags, void* stream) {
  return moe_dispatch(1, down_weight, down_scales, down_biases, nullptr, nullptr, nullptr, shared_down_weight,
                      shared_down_scales, shared_down_biases, nullptr, nullptr, nullptr, shared_weights, h,
                      expert_ids, route_weights, y, num_tokens, top_k, hidden_dim, inter_dim, group_size,
                      expert_first, expert_count, expert_total, flags, stream);
}

int gdsq_moe_affine_q4_down_residual(const void* down_weight, const void* down_scales, const void* down_biases,
                                     const void* shared_down_weight, const void* shared_down_scales,
                                     const void* shared_down_biases, const void* h, const int32_t* expert_ids,
                                     const void* route_weights, const void* shared_weights, void* y,
                                     int num_tokens, int top_k, int hidden_dim, int inter_dim, int group_size,
                                     int expert_first, int expert_count, int expert_total, int flags,
                                     const void* residual, void* stream) {
  if (!residual) {
    t_last_error.clear();
    return fail(GDSQ_ERR_INVALID_VALUE, "moe down: null residual");
  }
  return moe_dispatch(1, down_weight, down_scales, down_biases, nullptr, nullptr, nullptr, shared_down_weight,
                      shared_down_scales, shared_down_biases, nullptr, nullptr, nullptr, shared_weights, h,
                      expert_ids, route_weights, y, num_tokens, top_k, hidden_dim, inter_dim, group_size,
                      expert_first, expert_count, expert_total, flags, stream, residual);
}

}  // extern "C"

namespace gdsq {
namespace {
// Fixed device-side intermediate for gdsq_moe_affine_q4_noalloc: 4 MiB of
// fp16 in the library's own static device memory (one copy per device), so
// that entry point allocates nothing.
constexpr size_t kNoAllocHElems = 2u << 20;
static __device__ __align__(256) __half g_moe_h_scratch[kNoAllocHElems];
void* g_moe_h_addr[kMaxDevices];
bool g_moe_h_ready[kMaxDevices];

// Device address of the array on the current device, looked up once per
// device (with that device current) and cached.  The lookup may not run
// while `stream` is being captured into a CUDA graph, so a first call made
// during a capture is rejected with a message saying so.
int moe_h_scratch(cudaStream_t stream, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(GDSQ_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lock(g_device_mutex);
  if (!g_moe_h_ready[dev]) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(stream, &cap);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
    if (cap != cudaStreamCaptureStatusNone)
      return fail(GDSQ_ERR_INVALID_VALUE,
                  "moe noalloc: the first call on device %d must come before any stream capture (it looks up the "
                  "static scratch's address once); make one uncaptured call first",
                  dev);
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_moe_h_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(MoE scratch)");
    g_moe_h_addr[dev] = addr;
    g_moe_h_ready[dev] = true;
  }
  *out = g_moe_h_addr[dev];
  return GDSQ_OK;
}
}  // namespace
}  // namespace gdsq

extern "C" {

int gdsq_moe_affine_q4_noalloc(const void* gate_weight, const void* gate_scales, const void* gate_biases,
                               const void* up_weight, const void* up_scales, const void* up_biases,
                               const void* down_weight, const void* down_scales, const void* down_biases,
                               const void* shared_gate_weight, const void* shared_gate_scales,
                               const void* shared_gate_biases, const void* shared_up_weight,
                               const void* shared_up_scales, const void* shared_up_biases,
                               const void* shared_down_weight, const void* shared_down_scales,
                               const void* shared_down_biases, const void* x, const int32_t* expert_ids,
                               const void* route_weights, const void* shared_weights, void* y, int num_tokens,
                               int top_k, int hidden_dim, int inter_dim, int group_size, int expert_first,
                               int expert_count, int expert_total, int flags, void* stream) {
  t_last_error.clear();
  const bool shared = shared_gate_weight != nullptr;
  // Both stages must agree on the shared expert: gate/up writes top_k + 1
  // slots per token into the scratch when it is present, and down reads as
  // many.  So its gate, up and down tensors and its weights are all given or
  // all null.
  const void* shared_ptrs[] = {shared_gate_weight, shared_gate_scales, shared_gate_biases, shared_up_weight,
                               shared_up_scales,   shared_up_biases,   shared_down_weight, shared_down_scales,
                               shared_down_biases, shared_weights};
  for (const void* q : shared_ptrs)
    if ((q != nullptr) != shared)
      return fail(GDSQ_ERR_INVALID_VALUE,
                  "moe noalloc: the shared expert's gate, up and down tensors and shared_weights must be all "
                  "given or all null");
  const long long need = (long long)num_tokens * (top_k + (shared ? 1 : 0)) * inter_dim;
  if (num_tokens < 0 || top_k < 1 || inter_dim <= 0)
    return fail(GDSQ_ERR_INVALID_VALUE, "moe noalloc: num_tokens %d, top_k %d, inter_dim %d", num_tokens, top_k,
                inter_dim);
  if (need > (long long)kNoAllocHElems)
    return fail(GDSQ_ERR_INVALID_VALUE,
                "moe noalloc: %d tokens x %d slots x %d intermediate = %lld fp16 exceeds the %zu-element "
                "static scratch; use gdsq_moe_affine_q4_gate_up / _down with a caller buffer",
                num_tokens, top_k + (shared ? 1 : 0), inter_dim, need, kNoAllocHElems);
  if (num_tokens == 0) return GDSQ_OK;
  void* h = nullptr;
  int st = moe_h_scratch(static_cast<cudaStream_t>(stream), &h);
  if (st != GDSQ_OK) return st;
  st = gdsq_moe_affine_q4_gate_up(gate_weight, gate_scales, gate_biases, up_weight, up_scales, up_biases,
                                  shared_gate_weight, shared_gate_scales, shared_gate_biases, shared_up_weight,
                                  shared_up_scales, shared_up_biases, x, expert_ids, h, num_tokens, top_k,
                                  inter_dim, hidden_dim, group_size, expert_first, expert_count, expert_total,
                                  stream);
  if (st != GDSQ_OK) return st;
  return gdsq_moe_affine_q4_down(down_weight, down_scales, down_biases, shared_down_weight, shared_down_scales,
                                 shared_down_biases, h, expert_ids, route_weights, shared_weights, y, num_tokens,
                                 top_k, hidden_dim, inter_dim, group_size, expert_first, expert_count,
                                 expert_total, flags, stream);
}

int gdsq_allreduce_sum_f16(const void* in, void* out, int n, const void* const* bufs, void* const* flags, int cap,
                           int rank, int world, void* stream_v) {
  t_last_error.clear();
  if (world < 1 || world > kP2PMaxRanks || rank < 0 || rank >= world)
    return fail(GDSQ_ERR_INVALID_VALUE, "allreduce: rank %d of world %d (at most %d ranks)", rank, world, kP2PMaxRanks);
  if (n < 0 || n % 8 != 0 || n > cap || (n + kP2PElemsPerCta - 1) / kP2PElemsPerCta > kP2PMaxCtas)
    return fail(GDSQ_ERR_INVALID_VALUE, "allreduce: n %d must be a multiple of 8, <= capacity %d and <= %d", n, cap,
                kP2PMaxCtas * kP2PElemsPerCta);
  if (n == 0) return GDSQ_OK;
  if (!in || !out || !bufs || !flags) return fail(GDSQ_ERR_INVALID_VALUE, "allreduce: null pointer");
  P2PArgs a = {};
  a.in = static_cast<const __half*>(in);
  a.out = static_cast<__half*>(out);
  for (int r = 0; r < world; ++r) {
    if (!bufs[r] || !flags[r] || !aligned(bufs[r], 8) || !aligned(flags[r], 4))
      return fail(GDSQ_ERR_MISALIGNED, "allreduce: rank %d buffer must be 16-byte aligned and non-null", r);
    a.bufs[r] = static_cast<__half*>(const_cast<void*>(bufs[r]));
    a.flags[r] = static_cast<int*>(flags[r]);
  }
  if (!aligned(in, 16) || !aligned(out, 16))
    return fail(GDSQ_ERR_MISALIGNED, "allreduce: input and output must be 16-byte aligned");
  a.n = n;
  a.cap = cap;
  a.rank = rank;
  a.world = world;
  a.wait_ns = g_peer_wait_ns.load();
  const int grid = (n + kP2PElemsPerCta - 1) / kP2PElemsPerCta;
  cudaError_t e = launch(allreduce_oneshot_kernel, dim3(grid), dim3(kP2PThreads), 0,
                         static_cast<cudaStream_t>(stream_v), g_pdl_enabled != 0, a);
  return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "allreduce launch");
}

int gdsq_allreduce_sum_words(int elem_type, const void* in, void* out, int n, const void* const* bufs, void* epochs,
                             int cap, int rank, int world, void* stream_v) {
  return gdsq_allreduce_sum_words_residual(elem_type, in, out, n, bufs, epochs, cap, rank, world, nullptr,
                                           stream_v);
}

int gdsq_allreduce_sum_words_residual(int elem_type, const void* in, void* out, int n, const void* const* bufs,
                                      void* epochs, int cap, int rank, int world, const void* residual,
                                      void* stream_v) {
  t_last_error.clear();
  if (residual && (elem_type != GDSQ_ELEM_F32_TO_F16 || !aligned(residual, 2)))
    return fail(GDSQ_ERR_INVALID_VALUE, "allreduce words: a residual needs GDSQ_ELEM_F32_TO_F16 and 2-byte "
                "alignment");
  if (elem_type != GDSQ_ELEM_F16 && elem_type != GDSQ_ELEM_F32 && elem_type != GDSQ_ELEM_F32_TO_F16)
    return fail(GDSQ_ERR_INVALID_VALUE, "allreduce words: elem_type %d is not fp16, fp32 or fp32 -> fp16",
                elem_type);
  if (world < 1 || world > kP2PMaxRanks || rank < 0 || rank >= world)
    return fail(GDSQ_ERR_INVALID_VALUE, "allreduce words: rank %d of world %d (at most %d ranks)", rank, world,
                kP2PMaxRanks);
  if (n < 0 || n > cap || (n + kLLElemsPerCta - 1) / kLLElemsPerCta > kLLMaxCtas)
    return fail(GDSQ_ERR_INVALID_VALUE, "allreduce words: n %d must be <= capacity %d and <= %d", n, cap,
                kLLMaxCtas * kLLElemsPerCta);
  if (n == 0) return GDSQ_OK;
  if (!in || !out || !bufs || !epochs) return fail(GDSQ_ERR_INVALID_VALUE, "allreduce words: null pointer");
  const int esz = elem_type == GDSQ_ELEM_F16 ? 2 : 4;
  const int osz = elem_type == GDSQ_ELEM_F32 ? 4 : 2;
  if (!aligned(in, esz) || !aligned(out, osz) || !aligned(epochs, 4))
    return fail(GDSQ_ERR_MISALIGNED, "allreduce words: input, output or epochs misaligned");
  LLArgs a = {};
  for (int r = 0; r < world; ++r) {
    if (!bufs[r] || !aligned(bufs[r], 8))
      return fail(GDSQ_ERR_MISALIGNED, "allreduce words: rank %d buffer must be 8-byte aligned and non-null", r);
    a.bufs[r] = static_cast<unsigned long long*>(const_cast<void*>(bufs[r]));
  }
  a.own = a.bufs[rank];
  a.in = in;
  a.out = out;
  a.epochs = static_cast<int*>(epochs);
  a.n = n;
  a.cap = cap;
  a.rank = rank;
  a.world = world;
  a.wait_ns = g_peer_wait_ns.load();
  a.residual = static_cast<const __half*>(residual);
  const int grid = (n + kLLElemsPerCta - 1) / kLLElemsPerCta;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  cudaError_t e;
  if (elem_type == GDSQ_ELEM_F32)
    e = launch(allreduce_ll_kernel<float>, dim3(grid), dim3(kLLThreads), 0, stream, g_pdl_enabled != 0, a);
  else if (elem_type == GDSQ_ELEM_F16)
    e = launch(allreduce_ll_kernel<__half>, dim3(grid), dim3(kLLThreads), 0, stream, g_pdl_enabled != 0, a);
  else
    e = launch(allreduce_ll_kernel<float, __half, true>, dim3(grid), dim3(kLLThreads), 0, stream,
               g_pdl_enabled != 0, a);
  return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "allreduce words launch");
}

int gdsq_moe_router(const void* x, int num_tokens, int hidden_dim, const void* router_weight, int num_experts,
                    const void* shared_gate, int top_k, void* logits, int32_t* expert_ids, void* route_weights,
                    void* shared_weights, unsigned int* counter, void* stream_v) {
  t_last_error.clear();
  if (num_tokens < 0 || num_tokens > kRouterMaxTokens || num_experts < 1 || num_experts > 32 * kRouteLaneVals ||
      top_k < 1 || top_k > 32 || top_k > num_experts || hidden_dim <= 0 || hidden_dim % 512 != 0)
    return fail(GDSQ_ERR_INVALID_VALUE, "moe router: tokens %d (<= %d), experts %d (<= %d), top_k %d (<= 32), "
                "hidden %d (a multiple of 512)", num_tokens, kRouterMaxTokens, num_experts, 32 * kRouteLaneVals,
                top_k, hidden_dim);
  if (num_tokens == 0) return GDSQ_OK;
  if (!x || !router_weight || !logits || !expert_ids || !route_weights || !counter ||
      (shared_gate && !shared_weights))
    return fail(GDSQ_ERR_INVALID_VALUE, "moe router: null pointer");
  if (!aligned(x, 16) || !aligned(router_weight, 16) || (shared_gate && !aligned(shared_gate, 16)) ||
      !aligned(logits, 2) || !aligned(expert_ids, 4) || !aligned(route_weights, 2) || !aligned(counter, 4) ||
      (shared_weights && !aligned(shared_weights, 2)))
    return fail(GDSQ_ERR_MISALIGNED, "moe router: x and the weights 16-byte, ids and counter 4-byte, "
                "fp16 outputs 2-byte alignment");
  const DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st != GDSQ_OK) return st;
  const int rows = num_experts + (shared_gate ? 1 : 0);
  const int grid = (rows + kRouterRowsPerCta - 1) / kRouterRowsPerCta;
  const size_t smem = (size_t)kRouterWarps * (num_experts + 64) * sizeof(float) +
                      (size_t)kRouterWarps * (num_experts + 8) * sizeof(__half);
  auto kernel = num_tokens == 1 ? moe_router_kernel<1> : num_tokens <= 4 ? moe_router_kernel<4>
                                                                          : moe_router_kernel<16>;
  cudaError_t e = ensure_smem(kernel, (int)smem, dev->ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(moe router)");
  e = launch(kernel, dim3(grid), dim3(kRouterWarps * 32), smem, static_cast<cudaStream_t>(stream_v),
             g_pdl_enabled != 0, static_cast<const __half*>(x), num_tokens, hidden_dim,
             static_cast<const __half*>(router_weight), num_experts, static_cast<const __half*>(shared_gate), top_k,
             static_cast<__half*>(logits), expert_ids, static_cast<__half*>(route_weights),
             static_cast<__half*>(shared_weights), counter);
  return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "moe router launch");
}

int gdsq_moe_route(const void* logits, int num_tokens, int num_experts, int top_k, const void* x,
                   const void* shared_gate, int hidden_dim, int32_t* expert_ids, void* route_weights,
                   void* shared_weights, void* stream_v) {
  t_last_error.clear();
  if (num_tokens < 0 || num_experts < 1 || num_experts > kRouteMaxExperts || top_k < 1 || top_k > 64 ||
      top_k > num_experts)
    return fail(GDSQ_ERR_INVALID_VALUE, "moe route: need 0 <= tokens, 1 <= top_k (%d) <= min(64, experts %d), "
                "experts <= %d", top_k, num_experts, kRouteMaxExperts);
  if (num_tokens == 0) return GDSQ_OK;
  if (!logits || !expert_ids || !route_weights) return fail(GDSQ_ERR_INVALID_VALUE, "moe route: null pointer");
  const bool shared = shared_gate != nullptr;
  if (shared && (!x || !shared_weights || hidden_dim <= 0 || hidden_dim % 8 != 0))
    return fail(GDSQ_ERR_INVALID_VALUE, "moe route: the shared gate needs x, an output and hidden_dim %% 8 == 0");
  if (!aligned(logits, 2) || !aligned(expert_ids, 4) || !aligned(route_weights, 2) ||
      (shared && (!aligned(x, 16) || !aligned(shared_gate, 16) || !aligned(shared_weights, 2))))
    return fail(GDSQ_ERR_MISALIGNED, "moe route: logits/weights 2-byte, ids 4-byte, x and the shared gate "
                "16-byte alignment");
  const DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st != GDSQ_OK) return st;
  const size_t smem = (size_t)(num_experts + 64) * sizeof(float);
  cudaError_t e = ensure_smem(moe_route_kernel, (int)smem, dev->ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(moe route)");
  e = launch(moe_route_kernel, dim3(num_tokens), dim3(64), smem, static_cast<cudaStream_t>(stream_v),
             g_pdl_enabled != 0, static_cast<const __half*>(logits), num_experts, top_k,
             static_cast<const __half*>(x), static_cast<const __half*>(shared_gate), hidden_dim, expert_ids,
             static_cast<__half*>(route_weights), static_cast<__half*>(shared_weights));
  return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "moe route launch");
}

// ---------------------------------------------------------------------------
// Decode-step kernels (decode.cuh): the non-GEMV work of one LLaMA decode
// position, position in device memory, for a graph-captured token.

int gdsq_add_rmsnorm_f16(const void* h_in, const void* delta, void* h_out, const void* weight, void* x_out,
                         int rows, int hidden, float eps, void* stream_v) {
  t_last_error.clear();
  if (rows < 0 || hidden <= 0 || hidden % 8 != 0 || hidden > kNormThreads * 8 * kNormMaxChunks)
    return fail(GDSQ_ERR_INVALID_VALUE, "add_rmsnorm: hidden %d must be a positive multiple of 8 up to %d, rows %d",
                hidden, kNormThreads * 8 * kNormMaxChunks, rows);
  if (rows == 0) return GDSQ_OK;
  if (!h_in || !weight || !x_out || (delta && !h_out)) return fail(GDSQ_ERR_INVALID_VALUE, "add_rmsnorm: null pointer");
  if (!aligned(h_in, 16) || !aligned(weight, 16) || !aligned(x_out, 16) ||
      (delta && (!aligned(delta, 16) || !aligned(h_out, 16))))
    return fail(GDSQ_ERR_MISALIGNED, "add_rmsnorm: every pointer must be 16-byte aligned");
  cudaError_t e = launch(add_rmsnorm_kernel, dim3(rows), dim3(kNormThreads), 0, static_cast<cudaStream_t>(stream_v),
                         g_pdl_enabled != 0, static_cast<const __half*>(h_in), static_cast<const __half*>(delta),
                         static_cast<__half*>(h_out), static_cast<const __half*>(weight), static_cast<__half*>(x_out),
                         hidden, 1.0f / static_cast<float>(hidden), eps);
  return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "add_rmsnorm launch");
}

int gdsq_rope_kv_f16(const void* q, const void* k, const void* v, void* q_out, const void* freqs,
                     const long long* pos, void* k_cache, void* v_cache, int num_heads, int num_kv_heads,
                     int head_dim, int max_seq, void* stream_v) {
  t_last_error.clear();
  if (num_heads < 1 || num_kv_heads < 1 || head_dim < 2 || head_dim % 2 != 0 || head_dim > 2048 || max_seq < 1)
    return fail(GDSQ_ERR_INVALID_VALUE, "rope_kv: heads %d / kv heads %d, head_dim %d (even, <= 2048), max_seq %d",
                num_heads, num_kv_heads, head_dim, max_seq);
  if (!q || !k || !v || !q_out || !freqs || !pos || !k_cache || !v_cache)
    return fail(GDSQ_ERR_INVALID_VALUE, "rope_kv: null pointer");
  if (!aligned(q, 4) || !aligned(k, 4) || !aligned(v, 4) || !aligned(q_out, 4) || !aligned(k_cache, 4) ||
      !aligned(v_cache, 4) || !aligned(freqs, 8) || !aligned(pos, 8))
    return fail(GDSQ_ERR_MISALIGNED, "rope_kv: fp16 pointers 4-byte, freqs and pos 8-byte alignment");
  cudaError_t e = launch(rope_kv_kernel, dim3(num_heads + num_kv_heads), dim3(head_dim / 2), 0,
                         static_cast<cudaStream_t>(stream_v), g_pdl_enabled != 0, static_cast<const __half*>(q),
                         static_cast<const __half*>(k), static_cast<const __half*>(v), static_cast<__half*>(q_out),
                         static_cast<const float2*>(freqs), pos, static_cast<__half*>(k_cache),
                         static_cast<__half*>(v_cache), num_heads, head_dim, max_seq);
  return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "rope_kv launch");
}

}  // extern "C"

namespace gdsq {
namespace {
// Shared by the plain and the RoPE-folding attention entry points.
int attention_launch(bool rope, const void* q, const void* k_new, const void* v_new, const void* freqs,
                     const long long* pos, void* k_cache, void* v_cache, void* out, int num_heads, int num_kv_heads,
                     int head_dim, int max_seq, float scale, void* stream_v) {
  if (num_heads < 1 || num_kv_heads < 1 || num_heads % num_kv_heads != 0 || (head_dim != 64 && head_dim != 128) ||
      max_seq < 1)
    return fail(GDSQ_ERR_INVALID_VALUE, "attention: heads %d must be a multiple of kv heads %d, head_dim %d "
                "(64 or 128), max_seq %d", num_heads, num_kv_heads, head_dim, max_seq);
  if (!q || !k_cache || !v_cache || !pos || !out || (rope && (!k_new || !v_new || !freqs)))
    return fail(GDSQ_ERR_INVALID_VALUE, "attention: null pointer");
  if (!aligned(q, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(out, 2) || !aligned(pos, 8) ||
      (rope && (!aligned(k_new, 4) || !aligned(v_new, 4) || !aligned(freqs, 8))))
    return fail(GDSQ_ERR_MISALIGNED, "attention: q and the caches 16-byte, pos and freqs 8-byte, new K/V 4-byte "
                "alignment");
  const DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st != GDSQ_OK) return st;
  // About two CTAs per SM: the cluster (<= 8) splits each head's positions.
  int C = 1;
  while (C < 8 && 2 * C * num_heads <= 2 * dev->sms && 2 * C <= max_seq) C *= 2;
  const int cap = (max_seq + C - 1) / C;
  const int slices = head_dim / 8;
  const int groups = kDecodeThreads / slices;
  const size_t floats = (size_t)((cap + 3) & ~3) + (size_t)groups * head_dim + (size_t)C * head_dim +
                        2 * kAttnMaxCluster + 2 * (kDecodeThreads / 32) + (rope ? head_dim : 0);
  const size_t smem = floats * sizeof(float);
  if (smem > (size_t)dev->smem_optin)
    return fail(GDSQ_ERR_UNSUPPORTED, "attention: max_seq %d needs %zu bytes of shared memory", max_seq, smem);
  auto kernel = rope ? (head_dim == 128 ? attn_decode_kernel<128, true> : attn_decode_kernel<64, true>)
                     : (head_dim == 128 ? attn_decode_kernel<128, false> : attn_decode_kernel<64, false>);
  cudaError_t e = ensure_smem(kernel, (int)smem, dev->ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attention)");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, num_heads);
  cfg.blockDim = dim3(kDecodeThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream_v);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (g_pdl_enabled) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  e = cudaLaunchKernelEx(&cfg, kernel, static_cast<const __half*>(q), static_cast<const __half*>(k_new),
                         static_cast<const __half*>(v_new), static_cast<const float2*>(freqs),
                         static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), pos, static_cast<__half*>(out),
                         num_heads, num_kv_heads, max_seq, scale);
  return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "attention launch");
}
}  // namespace
}  // namespace gdsq

extern "C" {

int gdsq_attention_decode_f16(const void* q, const void* k_cache, const void* v_cache, const long long* pos,
                              void* out, int num_heads, int num_kv_heads, int head_dim, int max_seq, float scale,
                              void* stream_v) {
  t_last_error.clear();
  return attention_launch(false, q, nullptr, nullptr, nullptr, pos, const_cast<void*>(k_cache),
                          const_cast<void*>(v_cache), out, num_heads, num_kv_heads, head_dim, max_seq, scale,
                          stream_v);
}

int gdsq_attention_decode_rope_f16(const void* q, const void* k, const void* v, const void* freqs,
                                   const long long* pos, void* k_cache, void* v_cache, void* out, int num_heads,
                                   int num_kv_heads, int head_dim, int max_seq, float scale, void* stream_v) {
  t_last_error.clear();
  return attention_launch(true, q, k, v, freqs, pos, k_cache, v_cache, out, num_heads, num_kv_heads, head_dim,
                          max_seq, scale, stream_v);
}

int gdsq_silu_mul_f16(const void* gate, const void* up, void* out, long long n, void* stream_v) {
  t_last_error.clear();
  if (n < 0) return fail(GDSQ_ERR_INVALID_VALUE, "silu_mul: negative size");
  if (n == 0) return GDSQ_OK;
  if (!gate || !up || !out) return fail(GDSQ_ERR_INVALID_VALUE, "silu_mul: null pointer");
  if (!aligned(gate, 2) || !aligned(up, 2) || !aligned(out, 2))
    return fail(GDSQ_ERR_MISALIGNED, "silu_mul: fp16 pointers must be 2-byte aligned");
  const DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st != GDSQ_OK) return st;
  const bool vec = n % 8 == 0 && aligned(gate, 16) && aligned(up, 16) && aligned(out, 16);
  const long long units = vec ? n / 8 : n;
  const unsigned grid = (unsigned)std::min<long long>((units + kDecodeThreads - 1) / kDecodeThreads,
                                                      (long long)dev->sms * 8);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  const __half* g = static_cast<const __half*>(gate);
  const __half* u = static_cast<const __half*>(up);
  __half* o = static_cast<__half*>(out);
  cudaError_t e = vec ? launch(silu_mul_kernel<true>, dim3(grid), dim3(kDecodeThreads), 0, stream, g_pdl_enabled != 0,
                               g, u, o, n)
                      : launch(silu_mul_kernel<false>, dim3(grid), dim3(kDecodeThreads), 0, stream,
                               g_pdl_enabled != 0, g, u, o, n);
  return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "silu_mul launch");
}

int gdsq_argmax_f16(const void* logits, int n, long long* token, long long* pos, void* stream_v) {
  t_last_error.clear();
  if (n < 1) return fail(GDSQ_ERR_INVALID_VALUE, "argmax: n %d < 1", n);
  if (!logits || !token) return fail(GDSQ_ERR_INVALID_VALUE, "argmax: null pointer");
  if (!aligned(logits, 2) || !aligned(token, 8) || (pos && !aligned(pos, 8)))
    return fail(GDSQ_ERR_MISALIGNED, "argmax: logits 2-byte, token and pos 8-byte alignment");
  const bool vec = n % 8 == 0 && aligned(logits, 16);
  cudaError_t e = launch(vec ? argmax_kernel<true> : argmax_kernel<false>, dim3(1), dim3(1024), 0,
                         static_cast<cudaStream_t>(stream_v), g_pdl_enabled != 0,
                         static_cast<const __half*>(logits), n, token, pos);
  return e == cudaSuccess ? GDSQ_OK : cuda_fail(e, "argmax launch");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// The reference's C++ launcher ABI (include/gdsq_reference_abi.h).

#include "gdsq_reference_abi.h"

namespace {
void report(int status, const char* what) {
  if (status != GDSQ_OK)
    fprintf(stderr, "%s: %s (%s)\n", what, gdsq_status_string(status), gdsq_last_error());
}
}  // namespace

void launch_fused_q4_0_gemv(const void* weight, const __half* x, __half* y, int out_dim, int in_dim,
                            cudaStream_t stream) {
  report(gdsq_fused_q4_0_gemv(weight, x, y, out_dim, in_dim, 1, stream), "fused_q4_0_gemv");
}

void launch_fused_q8_0_gemv(const void* weight, const __half* x, __half* y, int out_dim, int in_dim,
                            cudaStream_t stream) {
  report(gdsq_fused_q8_0_gemv(weight, x, y, out_dim, in_dim, 1, stream), "fused_q8_0_gemv");
}

void launch_dequant_q8_0(const void* src, __half* dst, size_t num_blocks, cudaStream_t stream) {
  report(gdsq_dequant_q8_0(src, dst, num_blocks, stream), "dequant_q8_0");
}

void launch_dequant_q4_0(const void* src, __half* dst, size_t num_blocks, cudaStream_t stream) {
  report(gdsq_dequant_q4_0(src, dst, num_blocks, stream), "dequant_q4_0");
}

void launch_dequant_affine_q4(const uint32_t* weight, const __half* scales, const __half* biases,
                              __half* dst, size_t num_elements, int in_dim, int group_size,
                              cudaStream_t stream) {
  report(gdsq_dequant_affine_q4(weight, scales, biases, dst, num_elements, in_dim, group_size, stream),
         "dequant_affine_q4");
}

void launch_fused_affine_q4_gemv(const uint32_t* weight, const __half* scales, const __half* biases,
                                 const __half* x, __half* y, int out_dim, int in_dim, int group_size,
                                 cudaStream_t stream) {
  report(gdsq_fused_affine_q4_gemv(weight, scales, biases, x, y, out_dim, in_dim, group_size, 1, stream),
         "fused_affine_q4_gemv");
}
