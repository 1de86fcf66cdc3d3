// gds_io_ext: the Python op boundary of GdsLLM's decode path, rebuilt on the
// gdsq C ABI (include/gdsq.h).
//
// Mirrors the reference module gdsllm/runtime/gds_bindings.cpp:516-615: the
// same op names, argument names, defaults, return shapes and RuntimeError
// conditions, so gdsllm/runtime/llama.py:106-166, qwen_moe.py:20-73 and the
// schedulers run unchanged when this module is imported in its place.
//
// Differences, all additive:
//   * x may hold B <= 16 rows of K (any shape with numel == B*K); the fused
//     GEMVs then return [B, N].  B == 1 returns [1, N] as before.
//   * every op takes a device guard on the handle's device (the reference
//     launched on whatever device was current).
//   * kernel launch failures raise instead of printing to stderr.
//   * bounds of offsets against the handle size and the dtype/device of x and
//     of the output buffer are checked before launch.
//   * handle_from_tensor() wraps an existing CUDA tensor as a handle (tests,
//     synthetic weights); set_pdl() / device_error() expose library controls.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cuda_runtime.h>
#include <cufile.h>
#include <dlfcn.h>
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "gdsq.h"

namespace py = pybind11;

namespace {

// ---------------------------------------------------------------------------
// cuFile, resolved at run time so that the module imports on hosts without a
// GPUDirect Storage stack (reads then go through pread + cudaMemcpy, which is
// what cuFile's compatibility mode does as well).

struct CuFileApi {
  bool resolved = false;
  bool available = false;
  bool initialized = false;
  bool driver_open = false;
  CUfileError_t (*driver_open_fn)() = nullptr;
  CUfileError_t (*driver_close_fn)() = nullptr;
  CUfileError_t (*buf_register)(const void*, size_t, int) = nullptr;
  CUfileError_t (*buf_deregister)(const void*) = nullptr;
  CUfileError_t (*handle_register)(CUfileHandle_t*, CUfileDescr_t*) = nullptr;
  void (*handle_deregister)(CUfileHandle_t) = nullptr;
  ssize_t (*read)(CUfileHandle_t, void*, size_t, off_t, off_t) = nullptr;
};

CuFileApi g_cufile;
std::mutex g_cufile_mutex;

void resolve_cufile() {
  if (g_cufile.resolved) return;
  g_cufile.resolved = true;
  void* lib = dlopen("libcufile.so.0", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) lib = dlopen("libcufile.so", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) return;
  auto sym = [&](const char* n) { return dlsym(lib, n); };
  g_cufile.driver_open_fn = reinterpret_cast<CUfileError_t (*)()>(sym("cuFileDriverOpen"));
  void* close_fn = sym("cuFileDriverClose_v2");
  if (!close_fn) close_fn = sym("cuFileDriverClose");
  g_cufile.driver_close_fn = reinterpret_cast<CUfileError_t (*)()>(close_fn);
  g_cufile.buf_register =
      reinterpret_cast<CUfileError_t (*)(const void*, size_t, int)>(sym("cuFileBufRegister"));
  g_cufile.buf_deregister = reinterpret_cast<CUfileError_t (*)(const void*)>(sym("cuFileBufDeregister"));
  g_cufile.handle_register =
      reinterpret_cast<CUfileError_t (*)(CUfileHandle_t*, CUfileDescr_t*)>(sym("cuFileHandleRegister"));
  g_cufile.handle_deregister = reinterpret_cast<void (*)(CUfileHandle_t)>(sym("cuFileHandleDeregister"));
  g_cufile.read = reinterpret_cast<ssize_t (*)(CUfileHandle_t, void*, size_t, off_t, off_t)>(sym("cuFileRead"));
  g_cufile.available = g_cufile.driver_open_fn && g_cufile.driver_close_fn && g_cufile.buf_register &&
                       g_cufile.buf_deregister && g_cufile.handle_register &&
                       g_cufile.handle_deregister && g_cufile.read;
}

// gdsllm/runtime/gds_io.cu:53-69: open the driver once; failure is not fatal.
// cuFile is used only when GDSLLM_USE_CUFILE=1 is set: opening the cuFile
// driver can block for minutes on hosts without the nvidia-fs stack, and
// without it cuFile's compatibility mode is the same pread + copy that the
// fallback below performs.
void gds_init() {
  std::lock_guard<std::mutex> lock(g_cufile_mutex);
  if (g_cufile.initialized) return;
  const char* want = getenv("GDSLLM_USE_CUFILE");
  if (want && want[0] == '1') resolve_cufile();
  if (g_cufile.available) {
    CUfileError_t st = g_cufile.driver_open_fn();
    g_cufile.driver_open = st.err == CU_FILE_SUCCESS;
    if (!g_cufile.driver_open)
      fprintf(stderr, "gds_io_ext: cuFileDriverOpen returned %d; reads use the compatibility path\n",
              static_cast<int>(st.err));
  }
  g_cufile.initialized = true;
}

// gdsllm/runtime/gds_io.cu:71-78
void gds_shutdown() {
  std::lock_guard<std::mutex> lock(g_cufile_mutex);
  if (!g_cufile.initialized) return;
  if (g_cufile.driver_open) g_cufile.driver_close_fn();
  g_cufile.driver_open = false;
  g_cufile.initialized = false;
}

bool gds_is_driver_open() { return g_cufile.driver_open; }

void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------

// A device buffer that weights live in.  Either owned (cudaMalloc, 4 KB
// rounded, optionally registered with cuFile: gdsllm/runtime/gds_io.cu:93-131)
// or a view of a torch tensor that it keeps alive.
class GdsBufferHandle {
 public:
  static std::shared_ptr<GdsBufferHandle> allocate(size_t size, int device_id) {
    auto h = std::shared_ptr<GdsBufferHandle>(new GdsBufferHandle());
    h->device_id_ = device_id;
    h->size_ = ((size + 4095) / 4096) * 4096;
    if (h->size_ == 0) h->size_ = 4096;
    c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device_id));
    check_cuda(cudaMalloc(&h->ptr_, h->size_), "gds_alloc: cudaMalloc");
    h->owned_ = true;
    if (g_cufile.driver_open) {
      CUfileError_t st = g_cufile.buf_register(h->ptr_, h->size_, 0);
      h->registered_ = st.err == CU_FILE_SUCCESS;
    }
    return h;
  }

  static std::shared_ptr<GdsBufferHandle> wrap(const torch::Tensor& t) {
    if (!t.is_cuda()) throw std::runtime_error("handle_from_tensor: tensor must be on a CUDA device");
    if (!t.is_contiguous()) throw std::runtime_error("handle_from_tensor: tensor must be contiguous");
    auto h = std::shared_ptr<GdsBufferHandle>(new GdsBufferHandle());
    h->tensor_ = t;
    h->ptr_ = t.data_ptr();
    h->size_ = static_cast<size_t>(t.numel()) * t.element_size();
    h->device_id_ = t.get_device();
    return h;
  }

  ~GdsBufferHandle() {
    if (owned_ && ptr_) {
      if (registered_ && g_cufile.available) g_cufile.buf_deregister(ptr_);
      int prev = 0;
      cudaGetDevice(&prev);
      cudaSetDevice(device_id_);
      cudaFree(ptr_);
      cudaSetDevice(prev);
    }
  }

  GdsBufferHandle(const GdsBufferHandle&) = delete;
  GdsBufferHandle& operator=(const GdsBufferHandle&) = delete;

  void* dev_ptr() const { return ptr_; }
  size_t size() const { return size_; }
  int device_id() const { return device_id_; }
  bool registered() const { return registered_; }

 private:
  GdsBufferHandle() = default;
  void* ptr_ = nullptr;
  size_t size_ = 0;
  int device_id_ = 0;
  bool registered_ = false;
  bool owned_ = false;
  torch::Tensor tensor_;
};

using Handle = std::shared_ptr<GdsBufferHandle>;

// Reads `size` bytes at `file_offset` into the buffer at `buf_offset`
// (gdsllm/runtime/gds_io.cu:135-191).  cuFile first; if the file cannot be
// registered or the read fails, a pread + cudaMemcpy loop.
ssize_t gds_read(GdsBufferHandle& buf, const std::string& path, size_t size, off_t file_offset,
                 off_t buf_offset) {
  if (!buf.dev_ptr()) throw std::runtime_error("gds_read: invalid buffer");
  if (static_cast<size_t>(buf_offset) + size > buf.size())
    throw std::runtime_error("gds_read: read would exceed buffer size");
  if (size == 0) return 0;
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(buf.device_id()));
  if (g_cufile.available && g_cufile.initialized && g_cufile.driver_open) {
    int fd = open(path.c_str(), O_RDONLY | O_DIRECT);
    if (fd < 0) fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("gds_read: cannot open file '" + path + "': " + strerror(errno));
    CUfileDescr_t descr;
    memset(&descr, 0, sizeof(descr));
    descr.handle.fd = fd;
    descr.type = CU_FILE_HANDLE_TYPE_OPAQUE_FD;
    CUfileHandle_t fh;
    CUfileError_t st = g_cufile.handle_register(&fh, &descr);
    if (st.err == CU_FILE_SUCCESS) {
      ssize_t n = g_cufile.read(fh, buf.dev_ptr(), size, file_offset, buf_offset);
      g_cufile.handle_deregister(fh);
      close(fd);
      if (n >= 0) return n;
    } else {
      close(fd);
    }
  }
  int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) throw std::runtime_error("gds_read: cannot open file '" + path + "': " + strerror(errno));
  const size_t kChunk = 16u << 20;
  void* staging = nullptr;
  cudaError_t e = cudaMallocHost(&staging, std::min(size, kChunk));
  if (e != cudaSuccess) {
    close(fd);
    check_cuda(e, "gds_read: cudaMallocHost");
  }
  size_t done = 0;
  while (done < size) {
    const size_t want = std::min(kChunk, size - done);
    ssize_t n = pread(fd, staging, want, file_offset + static_cast<off_t>(done));
    if (n <= 0) break;
    e = cudaMemcpy(static_cast<char*>(buf.dev_ptr()) + buf_offset + done, staging, n, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) break;
    done += static_cast<size_t>(n);
  }
  cudaFreeHost(staging);
  close(fd);
  check_cuda(e, "gds_read: cudaMemcpy");
  return static_cast<ssize_t>(done);
}

// ---------------------------------------------------------------------------
// Asynchronous, double-buffered loading (additive).  The reference reads a
// layer synchronously before its compute (gdsllm/runtime/gds_io.cu:135-191,
// called from torch_bridge.py:148-177), so the GPU idles while a layer that
// is not resident is read.  load_file_async() returns at once with a
// PendingLoad.  One worker thread per process reads the file in chunks into
// two pinned staging buffers in turn and copies each chunk to the device
// with one cudaMemcpyAsync on its own stream: the read of chunk i + 1
// overlaps the copy of chunk i, and both overlap whatever the caller's
// streams run meanwhile.  PendingLoad.wait() returns the buffer handle once
// the reads are done and makes the caller's current stream wait, on the
// device, for the copies, so work queued after it sees the data.

constexpr size_t kAsyncChunk = size_t(8) << 20;

struct LoadJob {
  Handle h;
  std::string path;
  size_t size = 0;
  off_t file_offset = 0;
  std::mutex m;
  std::condition_variable cv;
  bool done = false;
  std::string error;
  cudaEvent_t copied = nullptr;  // recorded on the loader's stream after the last copy
  ~LoadJob() {
    if (copied) cudaEventDestroy(copied);  // a load nobody waited for
  }
};

class AsyncLoader {
 public:
  static AsyncLoader& get() {
    static AsyncLoader* loader = new AsyncLoader();  // never destroyed: the worker runs until exit
    return *loader;
  }

  std::shared_ptr<LoadJob> submit(Handle h, const std::string& path, size_t size, off_t file_offset) {
    auto job = std::make_shared<LoadJob>();
    job->h = std::move(h);
    job->path = path;
    job->size = size;
    job->file_offset = file_offset;
    {
      std::lock_guard<std::mutex> lock(m_);
      queue_.push_back(job);
    }
    cv_.notify_one();
    return job;
  }

 private:
  AsyncLoader() { std::thread([this] { loop(); }).detach(); }

  void loop() {
    for (;;) {
      std::shared_ptr<LoadJob> job;
      {
        std::unique_lock<std::mutex> lock(m_);
        cv_.wait(lock, [this] { return !queue_.empty(); });
        job = queue_.front();
        queue_.erase(queue_.begin());
      }
      std::string err;
      try {
        run(*job);
      } catch (const std::exception& ex) {
        err = ex.what();
      }
      {
        std::lock_guard<std::mutex> lock(job->m);
        job->error = err;
        job->done = true;
      }
      job->cv.notify_all();
    }
  }

  // Per device: the copy stream and the two pinned staging buffers, each
  // with an event recorded after the copy that last read it.
  struct DeviceState {
    cudaStream_t stream = nullptr;
    void* staging[2] = {nullptr, nullptr};
    cudaEvent_t free[2] = {nullptr, nullptr};
  };

  DeviceState& state(int dev) {
    DeviceState& d = devices_[dev];
    if (!d.stream) {
      check_cuda(cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking), "load_file_async: stream");
      for (int i = 0; i < 2; ++i) {
        check_cuda(cudaHostAlloc(&d.staging[i], kAsyncChunk, cudaHostAllocPortable), "load_file_async: cudaHostAlloc");
        check_cuda(cudaEventCreateWithFlags(&d.free[i], cudaEventDisableTiming | cudaEventBlockingSync),
                   "load_file_async: cudaEventCreate");
        check_cuda(cudaEventRecord(d.free[i], d.stream), "load_file_async: cudaEventRecord");
      }
    }
    return d;
  }

  void run(LoadJob& job) {
    const int dev = job.h->device_id();
    check_cuda(cudaSetDevice(dev), "load_file_async: cudaSetDevice");
    DeviceState& d = state(dev);
    int fd = open(job.path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("load_file_async: cannot open file '" + job.path + "': " + strerror(errno));
    size_t done = 0;
    int b = 0;
    cudaError_t e = cudaSuccess;
    while (done < job.size) {
      // the copy that last read this staging buffer must be finished
      e = cudaEventSynchronize(d.free[b]);
      if (e != cudaSuccess) break;
      const size_t want = std::min(kAsyncChunk, job.size - done);
      const ssize_t n = pread(fd, d.staging[b], want, job.file_offset + static_cast<off_t>(done));
      if (n <= 0) break;
      e = cudaMemcpyAsync(static_cast<char*>(job.h->dev_ptr()) + done, d.staging[b], static_cast<size_t>(n),
                          cudaMemcpyHostToDevice, d.stream);
      if (e == cudaSuccess) e = cudaEventRecord(d.free[b], d.stream);
      if (e != cudaSuccess) break;
      done += static_cast<size_t>(n);
      b ^= 1;
    }
    close(fd);
    if (e != cudaSuccess || done < job.size) cudaStreamSynchronize(d.stream);  // no copy outlives a failed load
    check_cuda(e, "load_file_async: copy");
    if (done < job.size)
      throw std::runtime_error("load_file_async: expected " + std::to_string(job.size) + " bytes, got " +
                               std::to_string(done));
    check_cuda(cudaEventCreateWithFlags(&job.copied, cudaEventDisableTiming), "load_file_async: cudaEventCreate");
    check_cuda(cudaEventRecord(job.copied, d.stream), "load_file_async: cudaEventRecord");
  }

  std::mutex m_;
  std::condition_variable cv_;
  std::vector<std::shared_ptr<LoadJob>> queue_;
  std::unordered_map<int, DeviceState> devices_;  // touched by the worker thread only
};

// The Python-side handle of one asynchronous load.
class PendingLoad {
 public:
  explicit PendingLoad(std::shared_ptr<LoadJob> job) : job_(std::move(job)) {}

  bool ready() {
    std::lock_guard<std::mutex> lock(job_->m);
    return job_->done;
  }

  // Blocks (without the GIL) until the file is read, then orders the copies
  // before later work on the current stream of the buffer's device.
  Handle wait() {
    {
      py::gil_scoped_release release;
      std::unique_lock<std::mutex> lock(job_->m);
      job_->cv.wait(lock, [this] { return job_->done; });
    }
    if (!job_->error.empty()) throw std::runtime_error(job_->error);
    if (job_->copied) {
      const int dev = job_->h->device_id();
      c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(dev));
      cudaStream_t s = c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(dev)).stream();
      check_cuda(cudaStreamWaitEvent(s, job_->copied, 0), "PendingLoad.wait: cudaStreamWaitEvent");
      cudaEventDestroy(job_->copied);
      job_->copied = nullptr;
    }
    return job_->h;
  }

 private:
  std::shared_ptr<LoadJob> job_;
};

// load_file / load_file_region without blocking: the buffer is allocated
// now (on device_id), the read and the copies run on the loader's thread.
PendingLoad py_load_file_async(const std::string& filepath, int64_t size_bytes, int64_t file_offset, int device_id) {
  if (size_bytes < 0 || file_offset < 0)
    throw std::runtime_error("load_file_async: negative size or offset");
  auto h = GdsBufferHandle::allocate(static_cast<size_t>(size_bytes), device_id);
  return PendingLoad(AsyncLoader::get().submit(h, filepath, static_cast<size_t>(size_bytes),
                                               static_cast<off_t>(file_offset)));
}

torch::Dtype parse_dtype(const std::string& s) {
  if (s == "float16" || s == "half") return torch::kFloat16;
  if (s == "float32" || s == "float") return torch::kFloat32;
  if (s == "bfloat16") return torch::kBFloat16;
  if (s == "int8") return torch::kInt8;
  if (s == "int32" || s == "int") return torch::kInt32;
  throw std::runtime_error("Unsupported dtype: " + s);
}

void raise_status(int status, const char* op) {
  if (status == GDSQ_OK) return;
  std::string msg = std::string(op) + ": " + gdsq_status_string(status);
  const char* detail = gdsq_last_error();
  if (detail && *detail) msg += std::string(" (") + detail + ")";
  throw std::runtime_error(msg);
}

void require_handle(const Handle& h, const char* op) {
  if (!h || !h->dev_ptr()) throw std::runtime_error(std::string(op) + ": invalid buffer handle");
}

void require_range(const Handle& h, int64_t offset, int64_t bytes, const char* op, const char* what) {
  if (offset < 0 || bytes < 0 || static_cast<uint64_t>(offset) + static_cast<uint64_t>(bytes) > h->size())
    throw std::runtime_error(std::string(op) + ": " + what + " [" + std::to_string(offset) + ", +" +
                             std::to_string(bytes) + ") exceeds buffer size " + std::to_string(h->size()));
}

const char* at_offset(const Handle& h, int64_t offset) {
  return static_cast<const char*>(h->dev_ptr()) + offset;
}

// Activation checks shared by both fused GEMVs.  Returns the batch count.
int check_activation(const torch::Tensor& x, int64_t in_dim, const Handle& h, const char* op) {
  if (!x.is_cuda() || x.get_device() != h->device_id())
    throw std::runtime_error(std::string(op) + ": x must be a CUDA tensor on device " +
                             std::to_string(h->device_id()));
  if (x.scalar_type() != torch::kFloat16)
    throw std::runtime_error(std::string(op) + ": x must be float16");
  const int64_t n = x.numel();
  if (in_dim == 0 || n == in_dim) return 1;
  if (n % in_dim != 0 || n / in_dim > GDSQ_MAX_BATCH)
    throw std::runtime_error(std::string(op) + ": input size " + std::to_string(n) + " != in_dim " +
                             std::to_string(in_dim));
  return static_cast<int>(n / in_dim);
}

torch::Tensor prepare_output(c10::optional<torch::Tensor> out, const std::vector<int64_t>& shape,
                             int64_t numel, const Handle& h, const char* op) {
  if (out.has_value()) {
    torch::Tensor o = out.value();
    if (o.numel() < numel)
      throw std::runtime_error(std::string(op) + ": scratch buffer too small (" + std::to_string(o.numel()) +
                               " < " + std::to_string(numel) + ")");
    if (!o.is_cuda() || o.get_device() != h->device_id() || o.scalar_type() != torch::kFloat16 ||
        !o.is_contiguous())
      throw std::runtime_error(std::string(op) + ": scratch must be a contiguous float16 CUDA tensor on device " +
                               std::to_string(h->device_id()));
    return o.flatten().slice(0, 0, numel).view(shape);
  }
  auto opts = torch::TensorOptions().dtype(torch::kFloat16).device(torch::kCUDA, h->device_id());
  return torch::empty(shape, opts);
}

void* current_stream(const Handle& h) {
  return static_cast<void*>(
      at::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(h->device_id())).stream());
}

// ---------------------------------------------------------------------------
// Load / view ops (gdsllm/runtime/gds_bindings.cpp:95-247)

// Prefetches started with prefetch_file(), picked up by the next load_file /
// load_file_region of the same (path, size, offset, device): a caller that
// prefetches layer i + 1 before computing layer i gets the read and the
// copies overlapped with that compute, and the reference's unchanged
// ModelWeights.load_layer (gdsllm/runtime/torch_bridge.py:148-177) receives
// the prefetched buffer.
using PrefetchKey = std::tuple<std::string, int64_t, int64_t, int>;
struct PrefetchKeyHash {
  size_t operator()(const PrefetchKey& k) const {
    return std::hash<std::string>()(std::get<0>(k)) ^ (std::hash<int64_t>()(std::get<1>(k)) * 31) ^
           (std::hash<int64_t>()(std::get<2>(k)) * 131) ^ std::hash<int>()(std::get<3>(k));
  }
};
std::mutex g_prefetch_mutex;
std::unordered_map<PrefetchKey, std::shared_ptr<PendingLoad>, PrefetchKeyHash> g_prefetched;

void py_prefetch_file(const std::string& path, int64_t size_bytes, int64_t file_offset, int device_id) {
  auto pending = std::make_shared<PendingLoad>(py_load_file_async(path, size_bytes, file_offset, device_id));
  std::lock_guard<std::mutex> lock(g_prefetch_mutex);
  g_prefetched[PrefetchKey(path, size_bytes, file_offset, device_id)] = std::move(pending);
}

// The prefetched buffer of this exact region, if any (waited for), else null.
Handle take_prefetched(const std::string& path, int64_t size_bytes, int64_t file_offset, int device_id) {
  std::shared_ptr<PendingLoad> pending;
  {
    std::lock_guard<std::mutex> lock(g_prefetch_mutex);
    auto it = g_prefetched.find(PrefetchKey(path, size_bytes, file_offset, device_id));
    if (it == g_prefetched.end()) return nullptr;
    pending = it->second;
    g_prefetched.erase(it);
  }
  return pending->wait();
}

Handle py_load_file(const std::string& path, int64_t size_bytes, int device_id) {
  if (Handle pre = take_prefetched(path, size_bytes, 0, device_id)) return pre;
  auto h = GdsBufferHandle::allocate(size_bytes, device_id);
  ssize_t n = gds_read(*h, path, size_bytes, 0, 0);
  if (n < size_bytes)
    throw std::runtime_error("py_load_file: expected " + std::to_string(size_bytes) + " bytes, got " +
                             std::to_string(n));
  return h;
}

Handle py_load_file_region(const std::string& path, int64_t size_bytes, int64_t file_offset,
                           int device_id) {
  if (Handle pre = take_prefetched(path, size_bytes, file_offset, device_id)) return pre;
  auto h = GdsBufferHandle::allocate(size_bytes, device_id);
  ssize_t n = gds_read(*h, path, size_bytes, file_offset, 0);
  if (n < size_bytes)
    throw std::runtime_error("py_load_file_region: expected " + std::to_string(size_bytes) +
                             " bytes, got " + std::to_string(n));
  return h;
}

py::tuple py_load_expert(const std::string& path, int64_t w_off, int64_t w_size, int64_t s_off,
                         int64_t s_size, int64_t b_off, int64_t b_size, int device_id) {
  auto h = GdsBufferHandle::allocate(w_size + s_size + b_size, device_id);
  if (gds_read(*h, path, w_size, w_off, 0) < w_size)
    throw std::runtime_error("py_load_expert: short read on weight");
  if (gds_read(*h, path, s_size, s_off, w_size) < s_size)
    throw std::runtime_error("py_load_expert: short read on scale");
  if (gds_read(*h, path, b_size, b_off, w_size + s_size) < b_size)
    throw std::runtime_error("py_load_expert: short read on bias");
  return py::make_tuple(h, static_cast<int64_t>(0), w_size, w_size + s_size);
}

torch::Tensor view_of(const Handle& h, std::vector<int64_t> shape, const std::string& dtype,
                      int64_t offset) {
  auto opts = torch::TensorOptions().dtype(parse_dtype(dtype)).device(torch::kCUDA, h->device_id());
  void* ptr = static_cast<char*>(h->dev_ptr()) + offset;
  Handle keep = h;
  return torch::from_blob(ptr, shape, [keep](void*) {}, opts);
}

torch::Tensor py_view_tensor(Handle h, std::vector<int64_t> shape, const std::string& dtype,
                             int64_t offset) {
  require_handle(h, "py_view_tensor");
  // The view must lie inside the buffer: offset + numel * element size.
  int64_t numel = 1;
  for (int64_t d : shape) {
    if (d < 0) throw std::runtime_error("py_view_tensor: negative dimension " + std::to_string(d));
    numel *= d;
  }
  const int64_t elem = static_cast<int64_t>(c10::elementSize(parse_dtype(dtype)));
  require_range(h, offset, numel * elem, "py_view_tensor", "view");
  return view_of(h, std::move(shape), dtype, offset);
}

torch::Tensor py_load_tensor(const std::string& path, std::vector<int64_t> shape, const std::string& dtype,
                             int64_t file_offset, int64_t size_bytes, int device_id) {
  auto h = GdsBufferHandle::allocate(size_bytes, device_id);
  ssize_t n = gds_read(*h, path, size_bytes, file_offset, 0);
  if (n < size_bytes)
    throw std::runtime_error("py_load_tensor: expected " + std::to_string(size_bytes) + " bytes, got " +
                             std::to_string(n));
  return view_of(h, std::move(shape), dtype, 0);
}

// ---------------------------------------------------------------------------
// Compute ops

// gdsllm/runtime/gds_bindings.cpp:255-314
torch::Tensor py_dequant_gguf(Handle h, std::vector<int64_t> shape, const std::string& gguf_type,
                              int64_t offset, c10::optional<torch::Tensor> output) {
  const char* op = "py_dequant_gguf";
  require_handle(h, op);
  int64_t numel = 1;
  for (auto s : shape) numel *= s;
  if (numel % 32 != 0)
    throw std::runtime_error(
        "py_dequant_gguf: total elements must be a multiple of 32 (block size), got " + std::to_string(numel));
  const int64_t blocks = numel / 32;
  int64_t block_bytes;
  if (gguf_type == "q4_0") block_bytes = 18;
  else if (gguf_type == "q8_0") block_bytes = 34;
  else throw std::runtime_error("py_dequant_gguf: unsupported type '" + gguf_type + "'");
  require_range(h, offset, blocks * block_bytes, op, "weight bytes");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(h->device_id()));
  torch::Tensor out = prepare_output(output, shape, numel, h, op);
  const int st = gguf_type == "q4_0"
                     ? gdsq_dequant_q4_0(at_offset(h, offset), out.data_ptr(), blocks, current_stream(h))
                     : gdsq_dequant_q8_0(at_offset(h, offset), out.data_ptr(), blocks, current_stream(h));
  raise_status(st, op);
  return out;
}

// Additive: F.embedding over a GGUF table without dequantizing the whole
// table (the reference's _embed_tokens does, gdsllm/runtime/scheduler.py:
// 22-45).  token_ids: int64 CUDA tensor of any shape; returns fp16
// [*token_ids.shape, cols], bit-identical to dequant_gguf + F.embedding.
torch::Tensor py_embedding_gguf(Handle h, torch::Tensor token_ids, std::vector<int64_t> shape,
                                const std::string& gguf_type, int64_t offset) {
  const char* op = "py_embedding_gguf";
  require_handle(h, op);
  if (shape.size() != 2) throw std::runtime_error("py_embedding_gguf: shape must be [rows, cols]");
  const int64_t rows = shape[0], cols = shape[1];
  if (cols % 32 != 0)
    throw std::runtime_error("py_embedding_gguf: cols must be a multiple of 32, got " + std::to_string(cols));
  int64_t block_bytes;
  if (gguf_type == "q4_0") block_bytes = 18;
  else if (gguf_type == "q8_0") block_bytes = 34;
  else throw std::runtime_error("py_embedding_gguf: unsupported type '" + gguf_type + "'");
  if (!token_ids.is_cuda() || token_ids.get_device() != h->device_id() || token_ids.scalar_type() != torch::kLong)
    throw std::runtime_error("py_embedding_gguf: token_ids must be an int64 tensor on the buffer's device");
  require_range(h, offset, rows * (cols / 32) * block_bytes, op, "table bytes");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(h->device_id()));
  torch::Tensor ids = token_ids.contiguous();
  std::vector<int64_t> out_shape(ids.sizes().begin(), ids.sizes().end());
  out_shape.push_back(cols);
  auto opts = torch::TensorOptions().dtype(torch::kFloat16).device(torch::kCUDA, h->device_id());
  torch::Tensor out = torch::empty(out_shape, opts);
  const int st = gdsq_dequant_rows_gguf(gguf_type == "q4_0" ? GDSQ_TYPE_Q4_0 : GDSQ_TYPE_Q8_0, at_offset(h, offset),
                                        rows, static_cast<int>(cols), reinterpret_cast<const long long*>(ids.data_ptr()),
                                        ids.numel(), out.data_ptr(), current_stream(h));
  raise_status(st, op);
  return out;
}

// gdsllm/runtime/gds_bindings.cpp:333-387
torch::Tensor py_fused_dequant_gemv(Handle h, torch::Tensor x, std::vector<int64_t> weight_shape,
                                    const std::string& gguf_type, int64_t offset) {
  const char* op = "py_fused_dequant_gemv";
  require_handle(h, op);
  if (weight_shape.size() != 2)
    throw std::runtime_error("py_fused_dequant_gemv: weight_shape must be [out_dim, in_dim]");
  const int64_t out_dim = weight_shape[0];
  const int64_t in_dim = weight_shape[1];
  if (in_dim % 32 != 0)
    throw std::runtime_error("py_fused_dequant_gemv: in_dim must be a multiple of 32, got " +
                             std::to_string(in_dim));
  int64_t block_bytes;
  if (gguf_type == "q4_0") block_bytes = 18;
  else if (gguf_type == "q8_0") block_bytes = 34;
  else throw std::runtime_error("py_fused_dequant_gemv: unsupported type '" + gguf_type + "'");
  const int batch = check_activation(x, in_dim, h, op);
  require_range(h, offset, out_dim * (in_dim / 32) * block_bytes, op, "weight bytes");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(h->device_id()));
  torch::Tensor xc = x.contiguous();
  auto opts = torch::TensorOptions().dtype(torch::kFloat16).device(torch::kCUDA, h->device_id());
  torch::Tensor out = torch::empty({batch, out_dim}, opts);
  const int st = gguf_type == "q4_0"
                     ? gdsq_fused_q4_0_gemv(at_offset(h, offset), xc.data_ptr(), out.data_ptr(),
                                            static_cast<int>(out_dim), static_cast<int>(in_dim), batch,
                                            current_stream(h))
                     : gdsq_fused_q8_0_gemv(at_offset(h, offset), xc.data_ptr(), out.data_ptr(),
                                            static_cast<int>(out_dim), static_cast<int>(in_dim), batch,
                                            current_stream(h));
  raise_status(st, op);
  return out;
}

// gdsllm/runtime/gds_bindings.cpp:404-457
torch::Tensor py_dequant_affine_q4(Handle h, std::vector<int64_t> weight_shape, int64_t weight_offset,
                                   int64_t scale_offset, int64_t bias_offset, int group_size,
                                   c10::optional<torch::Tensor> output) {
  const char* op = "py_dequant_affine_q4";
  require_handle(h, op);
  if (weight_shape.size() < 2)
    throw std::runtime_error("py_dequant_affine_q4: weight_shape must have >= 2 dims");
  int64_t numel = 1;
  for (auto s : weight_shape) numel *= s;
  const int64_t in_dim = weight_shape.back();
  if (group_size <= 0 || in_dim % group_size != 0 || group_size % 8 != 0)
    throw std::runtime_error("py_dequant_affine_q4: in_dim " + std::to_string(in_dim) +
                             " must be a multiple of group_size " + std::to_string(group_size) +
                             " (itself a multiple of 8)");
  require_range(h, weight_offset, numel / 2, op, "packed weights");
  require_range(h, scale_offset, numel / group_size * 2, op, "scales");
  require_range(h, bias_offset, numel / group_size * 2, op, "biases");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(h->device_id()));
  torch::Tensor out = prepare_output(output, weight_shape, numel, h, op);
  const int st = gdsq_dequant_affine_q4(at_offset(h, weight_offset), at_offset(h, scale_offset),
                                        at_offset(h, bias_offset), out.data_ptr(), numel,
                                        static_cast<int>(in_dim), group_size, current_stream(h));
  raise_status(st, op);
  return out;
}

// gdsllm/runtime/gds_bindings.cpp:466-512
torch::Tensor py_fused_affine_q4_gemv(Handle h, torch::Tensor x, std::vector<int64_t> weight_shape,
                                      int64_t weight_offset, int64_t scale_offset, int64_t bias_offset,
                                      int group_size) {
  const char* op = "py_fused_affine_q4_gemv";
  require_handle(h, op);
  if (weight_shape.size() != 2)
    throw std::runtime_error("py_fused_affine_q4_gemv: weight_shape must be [out_dim, in_dim]");
  const int64_t out_dim = weight_shape[0];
  const int64_t in_dim = weight_shape[1];
  if (group_size <= 0 || in_dim % group_size != 0 || group_size % 8 != 0)
    throw std::runtime_error("py_fused_affine_q4_gemv: in_dim " + std::to_string(in_dim) +
                             " must be a multiple of group_size " + std::to_string(group_size) +
                             " (itself a multiple of 8)");
  const int batch = check_activation(x, in_dim, h, op);
  require_range(h, weight_offset, out_dim * in_dim / 2, op, "packed weights");
  require_range(h, scale_offset, out_dim * (in_dim / group_size) * 2, op, "scales");
  require_range(h, bias_offset, out_dim * (in_dim / group_size) * 2, op, "biases");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(h->device_id()));
  torch::Tensor xc = x.contiguous();
  auto opts = torch::TensorOptions().dtype(torch::kFloat16).device(torch::kCUDA, h->device_id());
  torch::Tensor out = torch::empty({batch, out_dim}, opts);
  const int st = gdsq_fused_affine_q4_gemv(at_offset(h, weight_offset), at_offset(h, scale_offset),
                                           at_offset(h, bias_offset), xc.data_ptr(), out.data_ptr(),
                                           static_cast<int>(out_dim), static_cast<int>(in_dim), group_size,
                                           batch, current_stream(h));
  raise_status(st, op);
  return out;
}

// Additive op (no reference counterpart as one call): the routed-expert part
// of moe_mlp_selective's decode branch, gdsllm/runtime/qwen_moe.py:453-474,
// with expert ids and routing weights left in device memory.
// gate/up/down = (words int32 [E, rows, cols/8], scales fp16 [E, rows,
// cols/group], biases fp16), experts expert_first .. expert_first+E-1 of
// expert_total.  Returns y with x's shape (fp16, or fp32 with out_fp32).
using ExpertStack = std::tuple<torch::Tensor, torch::Tensor, torch::Tensor>;

void check_stack(const ExpertStack& m, const char* what, int64_t rows, int64_t cols, int group,
                 int64_t experts, const torch::Device& dev) {
  const auto& w = std::get<0>(m);
  const auto& sc = std::get<1>(m);
  const auto& bi = std::get<2>(m);
  const std::string op = std::string("fused_moe_affine_q4: ") + what;
  for (const torch::Tensor* t : {&w, &sc, &bi}) {
    if (!t->is_cuda() || t->device() != dev) throw std::runtime_error(op + " tensors must be on " + dev.str());
    if (!t->is_contiguous()) throw std::runtime_error(op + " tensors must be contiguous");
    if (t->dim() != 3) throw std::runtime_error(op + " tensors must be 3-D [experts, rows, ...]");
  }
  if (w.scalar_type() != torch::kInt32 && w.scalar_type() != torch::kUInt32)
    throw std::runtime_error(op + " weight must be int32/uint32 packed words");
  if (sc.scalar_type() != torch::kFloat16 || bi.scalar_type() != torch::kFloat16)
    throw std::runtime_error(op + " scales and biases must be float16");
  if (w.size(0) != experts || w.size(1) != rows || w.size(2) != cols / 8)
    throw std::runtime_error(op + " weight shape must be [" + std::to_string(experts) + ", " + std::to_string(rows) +
                             ", " + std::to_string(cols / 8) + "]");
  const std::vector<int64_t> gshape = {experts, rows, cols / group};
  if (sc.sizes().vec() != gshape || bi.sizes().vec() != gshape)
    throw std::runtime_error(op + " scales/biases shape must be [" + std::to_string(experts) + ", " +
                             std::to_string(rows) + ", " + std::to_string(cols / group) + "]");
}

torch::Tensor py_fused_moe_affine_q4(torch::Tensor x, torch::Tensor expert_ids, torch::Tensor route_weights,
                                     ExpertStack gate, ExpertStack up, ExpertStack down, int group_size,
                                     int64_t expert_first, int64_t expert_total,
                                     c10::optional<torch::Tensor> out, bool accumulate, bool out_fp32,
                                     c10::optional<torch::Tensor> h, c10::optional<std::vector<torch::Tensor>> shared,
                                     c10::optional<torch::Tensor> shared_weights, bool clamp,
                                     c10::optional<torch::Tensor> residual) {
  const char* op = "fused_moe_affine_q4";
  if (!x.is_cuda() || x.scalar_type() != torch::kFloat16)
    throw std::runtime_error("fused_moe_affine_q4: x must be a CUDA float16 tensor");
  const torch::Device dev = x.device();
  if (!expert_ids.is_cuda() || expert_ids.device() != dev || expert_ids.dim() < 1)
    throw std::runtime_error("fused_moe_affine_q4: expert_ids must be a CUDA tensor [..., top_k] on x's device");
  if (expert_ids.scalar_type() != torch::kInt32 && expert_ids.scalar_type() != torch::kInt64)
    throw std::runtime_error("fused_moe_affine_q4: expert_ids must be int32 or int64");
  const int64_t top_k = expert_ids.size(-1);
  const int64_t ntok = top_k > 0 ? expert_ids.numel() / top_k : 0;
  const auto& gw = std::get<0>(gate);
  if (gw.dim() != 3) throw std::runtime_error("fused_moe_affine_q4: gate weight must be 3-D");
  const int64_t experts = gw.size(0);
  const int64_t inter = gw.size(1);
  const int64_t hidden = gw.size(2) * 8;
  if (group_size <= 0 || group_size % 8 != 0 || hidden % group_size != 0 || inter % group_size != 0)
    throw std::runtime_error("fused_moe_affine_q4: group_size " + std::to_string(group_size) +
                             " must be a multiple of 8 dividing hidden " + std::to_string(hidden) +
                             " and intermediate " + std::to_string(inter));
  check_stack(gate, "gate", inter, hidden, group_size, experts, dev);
  check_stack(up, "up", inter, hidden, group_size, experts, dev);
  check_stack(down, "down", hidden, inter, group_size, experts, dev);
  if (x.numel() != ntok * hidden)
    throw std::runtime_error("fused_moe_affine_q4: x has " + std::to_string(x.numel()) + " elements, expected " +
                             std::to_string(ntok) + " tokens x " + std::to_string(hidden));
  if (route_weights.numel() != ntok * top_k || !route_weights.is_cuda() || route_weights.device() != dev)
    throw std::runtime_error("fused_moe_affine_q4: route_weights must be a CUDA tensor with one weight per id");
  if (expert_total < 0) expert_total = expert_first + experts;
  // shared expert: [gate w, s, b, up w, s, b, down w, s, b] with one expert each
  const bool has_shared = shared.has_value();
  const void* sh[9] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  torch::Tensor sw;
  if (has_shared) {
    const auto& v = *shared;
    if (v.size() != 9)
      throw std::runtime_error("fused_moe_affine_q4: shared must hold 9 tensors (gate, up, down: words, scales, biases)");
    check_stack({v[0], v[1], v[2]}, "shared gate", inter, hidden, group_size, 1, dev);
    check_stack({v[3], v[4], v[5]}, "shared up", inter, hidden, group_size, 1, dev);
    check_stack({v[6], v[7], v[8]}, "shared down", hidden, inter, group_size, 1, dev);
    for (int i = 0; i < 9; ++i) sh[i] = v[i].data_ptr();
    if (!shared_weights.has_value() || shared_weights->numel() != ntok || !shared_weights->is_cuda() ||
        shared_weights->device() != dev)
      throw std::runtime_error("fused_moe_affine_q4: shared needs shared_weights, one weight per token");
    sw = shared_weights->to(torch::kFloat16).contiguous();
  }
  const int64_t slots = top_k + (has_shared ? 1 : 0);
  c10::cuda::CUDAGuard guard(dev);
  void* stream = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
  torch::Tensor ids = expert_ids.to(torch::kInt32).contiguous();
  torch::Tensor rw = route_weights.to(torch::kFloat16).contiguous();
  torch::Tensor xc = x.contiguous();
  const auto out_dtype = out_fp32 ? torch::kFloat32 : torch::kFloat16;
  torch::Tensor y;
  if (out.has_value()) {
    y = *out;
    if (!y.is_cuda() || y.device() != dev || y.scalar_type() != out_dtype || !y.is_contiguous() ||
        y.numel() != ntok * hidden)
      throw std::runtime_error(std::string("fused_moe_affine_q4: out must be a contiguous ") +
                               (out_fp32 ? "float32" : "float16") + " CUDA tensor of " +
                               std::to_string(ntok * hidden) + " elements");
  } else {
    if (accumulate) throw std::runtime_error("fused_moe_affine_q4: accumulate=True needs out");
    y = torch::empty(x.sizes(), x.options().dtype(out_dtype));
  }
  torch::Tensor hb;
  if (h.has_value()) {
    hb = *h;
    if (!hb.is_cuda() || hb.device() != dev || hb.scalar_type() != torch::kFloat16 || !hb.is_contiguous() ||
        hb.numel() < ntok * slots * inter)
      throw std::runtime_error("fused_moe_affine_q4: h must be a contiguous float16 CUDA tensor of at least " +
                               std::to_string(ntok * slots * inter) + " elements");
  } else {
    hb = torch::empty({ntok, slots, inter}, x.options());
  }
  int st = gdsq_moe_affine_q4_gate_up(
      gw.data_ptr(), std::get<1>(gate).data_ptr(), std::get<2>(gate).data_ptr(), std::get<0>(up).data_ptr(),
      std::get<1>(up).data_ptr(), std::get<2>(up).data_ptr(), sh[0], sh[1], sh[2], sh[3], sh[4], sh[5],
      xc.data_ptr(), ids.data_ptr<int32_t>(),
      hb.data_ptr(), static_cast<int>(ntok), static_cast<int>(top_k), static_cast<int>(inter),
      static_cast<int>(hidden), group_size, static_cast<int>(expert_first), static_cast<int>(experts),
      static_cast<int>(expert_total), stream);
  raise_status(st, op);
  const int flags = (out_fp32 ? GDSQ_MOE_OUT_F32 : 0) | (accumulate ? GDSQ_MOE_ACCUMULATE : 0) |
                    (clamp ? GDSQ_MOE_CLAMP : 0);
  if (residual.has_value()) {
    const torch::Tensor& r = *residual;
    if (out_fp32 || accumulate || !r.is_cuda() || r.device() != dev || r.scalar_type() != torch::kFloat16 ||
        !r.is_contiguous() || r.numel() != ntok * hidden)
      throw std::runtime_error("fused_moe_affine_q4: residual must be a contiguous float16 CUDA tensor shaped like "
                               "x, with an fp16 output that does not accumulate");
    st = gdsq_moe_affine_q4_down_residual(
        std::get<0>(down).data_ptr(), std::get<1>(down).data_ptr(), std::get<2>(down).data_ptr(), sh[6], sh[7],
        sh[8], hb.data_ptr(), ids.data_ptr<int32_t>(), rw.data_ptr(), has_shared ? sw.data_ptr() : nullptr,
        y.data_ptr(), static_cast<int>(ntok), static_cast<int>(top_k), static_cast<int>(hidden),
        static_cast<int>(inter), group_size, static_cast<int>(expert_first), static_cast<int>(experts),
        static_cast<int>(expert_total), flags, r.data_ptr(), stream);
    raise_status(st, op);
    return y;
  }
  st = gdsq_moe_affine_q4_down(std::get<0>(down).data_ptr(), std::get<1>(down).data_ptr(),
                               std::get<2>(down).data_ptr(), sh[6], sh[7], sh[8], hb.data_ptr(),
                               ids.data_ptr<int32_t>(), rw.data_ptr(), has_shared ? sw.data_ptr() : nullptr,
                               y.data_ptr(), static_cast<int>(ntok), static_cast<int>(top_k),
                               static_cast<int>(hidden), static_cast<int>(inter), group_size,
                               static_cast<int>(expert_first), static_cast<int>(experts),
                               static_cast<int>(expert_total), flags, stream);
  raise_status(st, op);
  return y;
}

// Additive op: the routing tail of moe_route (qwen_moe.py:407-413) on router
// logits [..., E] fp16 in one launch, plus sigmoid(x . shared_gate).
// Returns (ids int32 [..., k], weights fp16 [..., k], shared weight fp16 [...] or None).
py::tuple py_moe_route(torch::Tensor logits, int top_k, c10::optional<torch::Tensor> x,
                       c10::optional<torch::Tensor> shared_gate) {
  if (!logits.is_cuda() || logits.scalar_type() != torch::kFloat16 || logits.dim() < 1)
    throw std::runtime_error("moe_route: logits must be a CUDA float16 tensor [..., num_experts]");
  const torch::Device dev = logits.device();
  const int64_t e = logits.size(-1);
  const int64_t ntok = e > 0 ? logits.numel() / e : 0;
  c10::cuda::CUDAGuard guard(dev);
  torch::Tensor lc = logits.contiguous();
  auto lead = logits.sizes().vec();
  lead.pop_back();
  auto ids_shape = lead;
  ids_shape.push_back(top_k);
  torch::Tensor ids = torch::empty(ids_shape, logits.options().dtype(torch::kInt32));
  torch::Tensor w = torch::empty(ids_shape, logits.options());
  torch::Tensor xc, gc, sw;
  int hidden = 0;
  if (shared_gate.has_value()) {
    if (!x.has_value()) throw std::runtime_error("moe_route: shared_gate needs x");
    xc = x->contiguous();
    gc = shared_gate->contiguous();
    hidden = static_cast<int>(gc.numel());
    if (!xc.is_cuda() || xc.device() != dev || xc.scalar_type() != torch::kFloat16 || xc.numel() != ntok * hidden ||
        !gc.is_cuda() || gc.device() != dev || gc.scalar_type() != torch::kFloat16)
      throw std::runtime_error("moe_route: x [tokens, hidden] and shared_gate [hidden] must be CUDA float16");
    sw = torch::empty(lead, logits.options());
  }
  void* stream = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
  raise_status(gdsq_moe_route(lc.data_ptr(), static_cast<int>(ntok), static_cast<int>(e), top_k,
                              shared_gate.has_value() ? xc.data_ptr() : nullptr,
                              shared_gate.has_value() ? gc.data_ptr() : nullptr, hidden, ids.data_ptr<int32_t>(),
                              w.data_ptr(), shared_gate.has_value() ? sw.data_ptr() : nullptr, stream),
               "moe_route");
  if (shared_gate.has_value()) return py::make_tuple(ids, w, sw);
  return py::make_tuple(ids, w, py::none());
}

int py_device_error(int device, bool clear) {
  int bits = 0;
  raise_status(gdsq_device_error(device, clear ? 1 : 0, &bits), "device_error");
  return bits;
}

}  // namespace

PYBIND11_MODULE(gds_io_ext, m) {
  m.doc() = "GdsLLM decode-path op boundary on the gdsq sm_100a kernels (B200)";
  m.attr("backend") = "gdsq-sm100a";
  m.attr("gdsq_version") = gdsq_version();

  m.def("init", &gds_init, "Initialize the cuFile driver. Call once at startup.");
  m.def("shutdown", &gds_shutdown, "Shut down the cuFile driver. Call once at exit.");
  m.def("is_driver_open", &gds_is_driver_open, "Returns True if cuFile driver opened successfully.");

  py::class_<GdsBufferHandle, Handle>(m, "GdsBufferHandle", "Handle to a CUDA buffer holding weights.")
      .def_property_readonly("size", &GdsBufferHandle::size)
      .def_property_readonly("device_id", &GdsBufferHandle::device_id)
      .def_property_readonly("registered", &GdsBufferHandle::registered)
      .def_property_readonly("data_ptr", [](const GdsBufferHandle& h) {
        return reinterpret_cast<uintptr_t>(h.dev_ptr());
      });

  m.def("load_file", &py_load_file, "Load an entire file into a CUDA buffer.", py::arg("filepath"),
        py::arg("size_bytes"), py::arg("device_id") = 0);
  m.def("load_file_region", &py_load_file_region, "Load a contiguous file region into a CUDA buffer.",
        py::arg("filepath"), py::arg("size_bytes"), py::arg("file_offset"), py::arg("device_id") = 0);
  m.def("load_expert", &py_load_expert, "Load one expert's weight+scale+bias into one CUDA buffer.",
        py::arg("filepath"), py::arg("w_file_offset"), py::arg("w_size"), py::arg("s_file_offset"),
        py::arg("s_size"), py::arg("b_file_offset"), py::arg("b_size"), py::arg("device_id") = 0);
  m.def("view_tensor", &py_view_tensor, "A torch.Tensor view into a GdsBufferHandle at an offset.",
        py::arg("handle"), py::arg("shape"), py::arg("dtype"), py::arg("offset"));
  m.def("load_tensor", &py_load_tensor, "Load a file region directly as a CUDA tensor.", py::arg("filepath"),
        py::arg("shape"), py::arg("dtype") = "float16", py::arg("file_offset") = 0, py::arg("size_bytes") = 0,
        py::arg("device_id") = 0);

  m.def("dequant_gguf", &py_dequant_gguf, "Dequantize GGUF Q4_0/Q8_0 blocks from a buffer to fp16.",
        py::arg("handle"), py::arg("shape"), py::arg("gguf_type"), py::arg("offset"),
        py::arg("output") = py::none());
  m.def("fused_dequant_gemv", &py_fused_dequant_gemv, "Fused dequant + GEMV for Q4_0/Q8_0 (decode).",
        py::arg("handle"), py::arg("x"), py::arg("weight_shape"), py::arg("gguf_type"), py::arg("offset"));
  py::class_<PendingLoad>(m, "PendingLoad", "An asynchronous file load started by load_file_async.")
      .def_property_readonly("ready", &PendingLoad::ready, "True once the file has been read.")
      .def("wait", &PendingLoad::wait,
           "Waits for the read, orders the copies before later work on the current stream and returns the "
           "GdsBufferHandle.");
  m.def("load_file_async", &py_load_file_async,
        "Start loading a file region into a new CUDA buffer without blocking: double-buffered pinned staging, "
        "one cudaMemcpyAsync per chunk on a loader stream.",
        py::arg("filepath"), py::arg("size_bytes"), py::arg("file_offset") = 0, py::arg("device_id") = 0);
  m.def("prefetch_file", &py_prefetch_file,
        "load_file_async whose buffer the next load_file / load_file_region of the same region returns.",
        py::arg("filepath"), py::arg("size_bytes"), py::arg("file_offset") = 0, py::arg("device_id") = 0);
  m.def("embedding_gguf", &py_embedding_gguf,
        "Embedding lookup over a GGUF Q4_0/Q8_0 table: dequantizes only the looked-up rows.", py::arg("handle"),
        py::arg("token_ids"), py::arg("shape"), py::arg("gguf_type"), py::arg("offset"));
  m.def("dequant_affine_q4", &py_dequant_affine_q4, "Dequantize affine Q4 (uint32 + scales + biases) to fp16.",
        py::arg("handle"), py::arg("weight_shape"), py::arg("weight_offset"), py::arg("scale_offset"),
        py::arg("bias_offset"), py::arg("group_size"), py::arg("output") = py::none());
  m.def("fused_affine_q4_gemv", &py_fused_affine_q4_gemv, "Fused affine Q4 dequant + GEMV (decode).",
        py::arg("handle"), py::arg("x"), py::arg("weight_shape"), py::arg("weight_offset"),
        py::arg("scale_offset"), py::arg("bias_offset"), py::arg("group_size"));

  m.def("fused_moe_affine_q4", &py_fused_moe_affine_q4,
        "Routed-expert MLP of a MoE layer (decode): gate/up + SiLU*mul, then down with the routing-weighted "
        "sum, expert ids read on the device.",
        py::arg("x"), py::arg("expert_ids"), py::arg("route_weights"), py::arg("gate"), py::arg("up"),
        py::arg("down"), py::arg("group_size") = 128, py::arg("expert_first") = 0, py::arg("expert_total") = -1,
        py::arg("out") = py::none(), py::arg("accumulate") = false, py::arg("out_fp32") = false,
        py::arg("h") = py::none(), py::arg("shared") = py::none(), py::arg("shared_weights") = py::none(),
        py::arg("clamp") = false, py::arg("residual") = py::none());
  m.def("moe_route", &py_moe_route,
        "Top-k expert ids, softmax weights and the shared expert's sigmoid gate from router logits (one launch).",
        py::arg("logits"), py::arg("top_k"), py::arg("x") = py::none(), py::arg("shared_gate") = py::none());
  m.def("handle_from_tensor", &GdsBufferHandle::wrap,
        "Wrap a contiguous CUDA tensor as a GdsBufferHandle (the tensor stays alive with the handle).",
        py::arg("tensor"));
  m.def("set_pdl", [](bool on) { gdsq_set_pdl(on ? 1 : 0); },
        "Enable programmatic dependent launch for the GEMV kernels.", py::arg("enable"));
  m.def("device_error", &py_device_error, "Read (and optionally clear) the kernel-side error word.",
        py::arg("device") = 0, py::arg("clear") = true);
}
