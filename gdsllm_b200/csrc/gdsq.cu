// gdsq: C-ABI entry points (include/gdsq.h) and host-side dispatch.
//
// One translation unit holds every kernel so that they can share the
// device-side error word without relocatable device code.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "gdsq.h"
#include "common.cuh"
#include "dequant.cuh"
#include "gemv.cuh"

namespace gdsq {
namespace {

thread_local std::string t_last_error;
int g_pdl_enabled = 0;

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

// Raises a kernel's dynamic shared memory limit once per (kernel, device).
// The cache is one array per kernel instantiation (a function-local static of
// this template), indexed by device.
template <typename K>
cudaError_t ensure_smem(K kernel, int bytes, int device) {
  static int set_bytes[kMaxDevices] = {};
  if (bytes <= 48 * 1024 || set_bytes[device] >= bytes) return cudaSuccess;
  std::lock_guard<std::mutex> lock(g_device_mutex);
  if (set_bytes[device] >= bytes) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) set_bytes[device] = bytes;
  return e;
}

// ---------------------------------------------------------------------------
// GEMV dispatch

int batch_tile(int nb) {
  if (nb <= 4) return nb;
  if (nb <= 8) return 8;
  return 16;
}

template <int F, int B, int GS>
int launch_fast(const GemvParams& p, const DeviceInfo& dev, cudaStream_t stream, int device) {
  const GemvSmemLayout L = gemv_smem_layout<F>(B, p.K, GS);
  auto kernel = gemv_fast_kernel<F, B, GS>;
  cudaError_t e = ensure_smem(kernel, L.total, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv)");
  const dim3 grid((p.N + 31) / 32);
  e = launch(kernel, grid, dim3(kGemvWarps * 32), L.total, stream, g_pdl_enabled != 0, p);
  if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
  (void)dev;
  return GDSQ_OK;
}

template <int F, int GS>
int launch_fast_batch(const GemvParams& p, const DeviceInfo& dev, cudaStream_t stream,
                      int device) {
  switch (batch_tile(p.nb)) {
    case 1: return launch_fast<F, 1, GS>(p, dev, stream, device);
    case 2: return launch_fast<F, 2, GS>(p, dev, stream, device);
    case 3: return launch_fast<F, 3, GS>(p, dev, stream, device);
    case 4: return launch_fast<F, 4, GS>(p, dev, stream, device);
    case 8: return launch_fast<F, 8, GS>(p, dev, stream, device);
    default: return launch_fast<F, 16, GS>(p, dev, stream, device);
  }
}

template <int F>
int launch_generic(const GemvParams& p, cudaStream_t stream) {
  const dim3 grid((p.N + 7) / 8);
  cudaError_t e = launch(gemv_generic_kernel<F>, grid, dim3(256), 0, stream, g_pdl_enabled != 0, p);
  if (e != cudaSuccess) return cuda_fail(e, "gemv (generic) launch");
  return GDSQ_OK;
}

template <int F>
int fast_smem_bytes(int nb, int K, int group) {
  return gemv_smem_layout<F>(batch_tile(nb), K, group).total;
}

int gemv_dispatch(int fmt, const void* w, const void* scales, const void* biases, const void* x,
                  void* y, int out_dim, int in_dim, int group, int batch, void* stream_v) {
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
  int device = 0;
  cudaGetDevice(&device);

  GemvParams p;
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
  if (fmt == kFmtQ4_0) {
    if (shape_ok && fast_smem_bytes<kFmtQ4_0>(batch, in_dim, 0) <= dev->smem_optin)
      return launch_fast_batch<kFmtQ4_0, 0>(p, *dev, stream, device);
    return launch_generic<kFmtQ4_0>(p, stream);
  }
  if (fmt == kFmtQ8_0) {
    if (shape_ok && fast_smem_bytes<kFmtQ8_0>(batch, in_dim, 0) <= dev->smem_optin)
      return launch_fast_batch<kFmtQ8_0, 0>(p, *dev, stream, device);
    return launch_generic<kFmtQ8_0>(p, stream);
  }
  const bool group_ok = group == 32 || group == 64 || group == 128 || group == 256;
  if (shape_ok && group_ok &&
      fast_smem_bytes<kFmtAffineQ4>(batch, in_dim, group) <= dev->smem_optin) {
    switch (group) {
      case 32: return launch_fast_batch<kFmtAffineQ4, 32>(p, *dev, stream, device);
      case 64: return launch_fast_batch<kFmtAffineQ4, 64>(p, *dev, stream, device);
      case 128: return launch_fast_batch<kFmtAffineQ4, 128>(p, *dev, stream, device);
      default: return launch_fast_batch<kFmtAffineQ4, 256>(p, *dev, stream, device);
    }
  }
  return launch_generic<kFmtAffineQ4>(p, stream);
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

}  // extern "C"
