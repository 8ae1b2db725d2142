// libad_b200: the C-ABI runtime under the Python CUDA device.
//
// Replaces the reference's per-backend helpers
//   autodiff/device/opencl/cl_helper.py:151-170  (init_buffer)
//   autodiff/device/opencl/cl_helper.py:262-332  (read_buffers / write_buffer)
//   autodiff/device/opencl/cl_helper.py:357-455  (build_kernel: compile + bind + enqueue)
//   autodiff/device/cuda/cuda_helper.py:80-222   (cuMemAlloc, HtoD/DtoH, NVRTC, cuLaunchKernel)
// with one native library: device context, device memory, pinned host memory,
// streams and events, NVRTC compilation straight to an sm_100a cubin, kernel
// launch, CUDA-graph capture/replay of loop bodies, TMA descriptor encoding,
// and NCCL communicators for data-parallel gradient all-reduce.
//
// Every entry point returns 0 on success and a non-zero status otherwise; the
// message is available from ad_last_error() (thread-local).  No entry point
// takes torch or numpy types: only plain pointers, sizes and opaque handles.
//
// The CUDA driver API is reached through cudaGetDriverEntryPoint so the
// library does not link libcuda (it loads on machines without a GPU driver);
// NCCL is dlopen'ed on first use.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_profiler_api.h>
#include <nvrtc.h>
#include <nccl.h>
#include <dlfcn.h>

#include <chrono>
#include <condition_variable>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/ad_b200.h"

namespace {

thread_local std::string g_err;

int fail(const char* fmt, ...) {
  char buf[2048];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return 1;
}

#define CK(call)                                                                        \
  do {                                                                                  \
    cudaError_t e_ = (call);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return fail("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
  } while (0)

// ---------------------------------------------------------------- driver API
typedef CUresult (*PFN_ModuleLoadData)(CUmodule*, const void*);
typedef CUresult (*PFN_ModuleUnload)(CUmodule);
typedef CUresult (*PFN_ModuleGetFunction)(CUfunction*, CUmodule, const char*);
typedef CUresult (*PFN_LaunchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned,
                                      unsigned, unsigned, CUstream, void**, void**);
typedef CUresult (*PFN_LaunchKernelEx)(const CUlaunchConfig*, CUfunction, void**, void**);
typedef CUresult (*PFN_FuncSetAttribute)(CUfunction, CUfunction_attribute, int);
typedef CUresult (*PFN_FuncGetAttribute)(int*, CUfunction_attribute, CUfunction);
typedef CUresult (*PFN_GetErrorString)(CUresult, const char**);
typedef CUresult (*PFN_TensorMapEncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                              const cuuint32_t*, CUtensorMapInterleave,
                                              CUtensorMapSwizzle, CUtensorMapL2promotion,
                                              CUtensorMapFloatOOBfill);

struct Driver {
  bool ok = false;
  PFN_ModuleLoadData moduleLoadData = nullptr;
  PFN_ModuleUnload moduleUnload = nullptr;
  PFN_ModuleGetFunction moduleGetFunction = nullptr;
  PFN_LaunchKernel launchKernel = nullptr;
  PFN_LaunchKernelEx launchKernelEx = nullptr;
  PFN_FuncSetAttribute funcSetAttribute = nullptr;
  PFN_FuncGetAttribute funcGetAttribute = nullptr;
  PFN_GetErrorString getErrorString = nullptr;
  PFN_TensorMapEncodeTiled tensorMapEncodeTiled = nullptr;
};
Driver g_drv;
std::mutex g_drv_mu;

template <typename T>
int get_entry(const char* name, T* out) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr)
    return fail("driver entry point %s unavailable (%s)", name, cudaGetErrorString(e));
  *out = reinterpret_cast<T>(p);
  return 0;
}

int driver() {
  std::lock_guard<std::mutex> lk(g_drv_mu);
  if (g_drv.ok) return 0;
  if (get_entry("cuModuleLoadData", &g_drv.moduleLoadData)) return 1;
  if (get_entry("cuModuleUnload", &g_drv.moduleUnload)) return 1;
  if (get_entry("cuModuleGetFunction", &g_drv.moduleGetFunction)) return 1;
  if (get_entry("cuLaunchKernel", &g_drv.launchKernel)) return 1;
  if (get_entry("cuLaunchKernelEx", &g_drv.launchKernelEx)) return 1;
  if (get_entry("cuFuncSetAttribute", &g_drv.funcSetAttribute)) return 1;
  if (get_entry("cuFuncGetAttribute", &g_drv.funcGetAttribute)) return 1;
  if (get_entry("cuGetErrorString", &g_drv.getErrorString)) return 1;
  if (get_entry("cuTensorMapEncodeTiled", &g_drv.tensorMapEncodeTiled)) return 1;
  g_drv.ok = true;
  return 0;
}

int cu_fail(CUresult r, const char* what) {
  const char* s = "?";
  if (g_drv.getErrorString) g_drv.getErrorString(r, &s);
  return fail("%s failed: %s (%d)", what, s, (int)r);
}

// ---------------------------------------------------------------- NCCL (dlopen)
struct Nccl {
  bool ok = false;
  void* h = nullptr;
  ncclResult_t (*getUniqueId)(ncclUniqueId*);
  ncclResult_t (*commInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t);
  ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*commAbort)(ncclComm_t);
  ncclResult_t (*commDestroy)(ncclComm_t);
  ncclResult_t (*groupStart)();
  ncclResult_t (*groupEnd)();
  ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  const char* (*getErrorString)(ncclResult_t);
};
Nccl g_nccl;
std::mutex g_nccl_mu;

int nccl() {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (g_nccl.ok) return 0;
  const char* names[] = {getenv("AD_NCCL_LIB"), "libnccl.so.2", "libnccl.so"};
  for (const char* n : names) {
    if (!n) continue;
    g_nccl.h = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
    if (g_nccl.h) break;
  }
  if (!g_nccl.h) return fail("cannot dlopen libnccl.so.2: %s", dlerror());
#define SYM(field, name)                                                       \
  g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(g_nccl.h, name)); \
  if (!g_nccl.field) return fail("NCCL symbol %s missing", name);
  SYM(getUniqueId, "ncclGetUniqueId");
  SYM(commInitRankConfig, "ncclCommInitRankConfig");
  SYM(allReduce, "ncclAllReduce");
  SYM(commGetAsyncError, "ncclCommGetAsyncError");
  SYM(commAbort, "ncclCommAbort");
  SYM(commDestroy, "ncclCommDestroy");
  SYM(groupStart, "ncclGroupStart");
  SYM(groupEnd, "ncclGroupEnd");
  SYM(allGather, "ncclAllGather");
  SYM(getErrorString, "ncclGetErrorString");
#undef SYM
  g_nccl.ok = true;
  return 0;
}

}  // namespace

namespace ad_b200_internal {
void set_error(const char* msg) { g_err = msg; }
}  // namespace ad_b200_internal

// ---------------------------------------------------------------- objects
struct ad_ctx {
  int device = 0;
  std::vector<cudaStream_t> streams;  // 0 = compute, 1 = copy-in, 2 = copy-out, 3 = comm
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  double nccl_timeout_s = 300.0;
  std::vector<char> last_log;
  // pinned staging ring for copies from / to pageable host memory
  std::vector<void*> stage;
  std::vector<cudaEvent_t> stage_ev;
  std::vector<bool> stage_busy;
  // peer-memory all-reduce (ad_peer_*): this rank's registered region, the
  // peers' mappings of theirs, barrier flags and the device-side table
  uint64_t peer_base = 0;
  size_t peer_bytes = 0;
  std::vector<void*> peer_maps;       // opened IPC mappings (to close)
  void* peer_flags = nullptr;         // this rank's flag area (cudaMalloc)
  void* peer_tab = nullptr;           // device copy of PeerTab
};

struct ad_kernel {
  CUmodule mod = nullptr;
  CUfunction fn = nullptr;
  std::string name;
};

struct ad_graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

static int stream_of(ad_ctx* c, int s, cudaStream_t* out) {
  if (!c) return fail("null context");
  if (s < 0 || s >= (int)c->streams.size()) return fail("bad stream index %d", s);
  *out = c->streams[s];
  return 0;
}

static int set_dev(ad_ctx* c) {
  CK(cudaSetDevice(c->device));
  return 0;
}

// ---------------------------------------------------------------- host copy pool
// Copies between pageable and pinned host memory run on a few persistent
// threads: one thread moves ~5-10 GB/s, the PCIe link ~50 GB/s per direction.
class CopyPool {
 public:
  static CopyPool& get() {
    static CopyPool pool;
    return pool;
  }
  // dst[0, n) = src[0, n), split over the workers and the calling thread
  void copy(void* dst, const void* src, size_t n) {
    const size_t min_piece = 1 << 20;
    size_t parts = n / min_piece;
    if (parts > workers_.size() + 1) parts = workers_.size() + 1;
    if (parts <= 1) {
      memcpy(dst, src, n);
      return;
    }
    size_t piece = ((n + parts - 1) / parts + 4095) & ~size_t(4095);
    std::lock_guard<std::mutex> one_caller(call_m_);
    std::unique_lock<std::mutex> lk(m_);
    dst_ = static_cast<char*>(dst);
    src_ = static_cast<const char*>(src);
    n_ = n;
    piece_ = piece;
    next_ = 1;  // piece 0 is the caller's
    pending_ = 0;
    for (size_t i = 1; i < parts && i * piece < n; ++i) ++pending_;
    ++gen_;
    lk.unlock();
    cv_.notify_all();
    memcpy(dst, src, piece < n ? piece : n);
    lk.lock();
    done_cv_.wait(lk, [&] { return pending_ == 0; });
  }

 private:
  CopyPool() {
    unsigned hw = std::thread::hardware_concurrency();
    unsigned want = hw > 2 ? (hw / 2 < 8 ? hw / 2 : 8) : 1;
    if (const char* e = getenv("AD_COPY_THREADS")) {  // threads incl. the caller
      int v = atoi(e);
      if (v >= 1 && v <= 64) want = (unsigned)v;
    }
    unsigned nw = want - 1;
    for (unsigned i = 0; i < nw; ++i) workers_.emplace_back([this] { run(); });
  }
  ~CopyPool() {
    {
      std::lock_guard<std::mutex> lk(m_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  void run() {
    uint64_t seen = 0;
    std::unique_lock<std::mutex> lk(m_);
    for (;;) {
      cv_.wait(lk, [&] { return stop_ || (gen_ != seen && next_ * piece_ < n_ && pending_ > 0); });
      if (stop_) return;
      size_t i = next_++;
      if (i * piece_ >= n_) {
        seen = gen_;
        continue;
      }
      char* d = dst_ + i * piece_;
      const char* s = src_ + i * piece_;
      size_t len = n_ - i * piece_ < piece_ ? n_ - i * piece_ : piece_;
      lk.unlock();
      memcpy(d, s, len);
      lk.lock();
      if (--pending_ == 0) {
        seen = gen_;
        done_cv_.notify_all();
      }
    }
  }
  std::vector<std::thread> workers_;
  std::mutex call_m_, m_;
  std::condition_variable cv_, done_cv_;
  char* dst_ = nullptr;
  const char* src_ = nullptr;
  size_t n_ = 0, piece_ = 1, next_ = 0, pending_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

constexpr size_t kStageChunk = 8u << 20;  // bytes per staging slot
constexpr int kStageSlots = 4;

int ensure_stage(ad_ctx* c) {
  if (!c->stage.empty()) return 0;
  for (int i = 0; i < kStageSlots; ++i) {
    void* p = nullptr;
    cudaEvent_t e;
    CK(cudaHostAlloc(&p, kStageChunk, cudaHostAllocPortable));
    CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    c->stage.push_back(p);
    c->stage_ev.push_back(e);
    c->stage_busy.push_back(false);
  }
  return 0;
}

extern "C" {

int ad_version(void) { return AD_B200_ABI_VERSION; }

const char* ad_last_error(void) { return g_err.c_str(); }

int ad_device_count(int* n) {
  int k = 0;
  cudaError_t e = cudaGetDeviceCount(&k);
  if (e != cudaSuccess) {
    *n = 0;
    return fail("cudaGetDeviceCount: %s", cudaGetErrorString(e));
  }
  *n = k;
  return 0;
}

int ad_init(int device, int n_streams, ad_ctx** out) {
  if (!out) return fail("null out");
  *out = nullptr;
  if (driver()) return 1;
  CK(cudaSetDevice(device));
  CK(cudaFree(nullptr));  // create the primary context
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail("device %d is sm_%d%d; this library is built for sm_100a (B200)", device, prop.major,
                prop.minor);
  ad_ctx* c = new ad_ctx();
  c->device = device;
  if (n_streams < 1) n_streams = 4;
  for (int i = 0; i < n_streams; ++i) {
    cudaStream_t s;
    cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      delete c;
      return fail("cudaStreamCreate: %s", cudaGetErrorString(e));
    }
    c->streams.push_back(s);
  }
  *out = c;
  return 0;
}

int ad_destroy(ad_ctx* c) {
  if (!c) return 0;
  cudaSetDevice(c->device);
  for (auto s : c->streams) cudaStreamSynchronize(s);
  ad_peer_close(c);
  if (c->comm && g_nccl.ok) g_nccl.commDestroy(c->comm);
  for (auto e : c->stage_ev) cudaEventDestroy(e);
  for (auto p : c->stage) cudaFreeHost(p);
  for (auto s : c->streams) cudaStreamDestroy(s);
  delete c;
  return 0;
}

int ad_device_info(ad_ctx* c, int* sm_count, int* smem_optin, size_t* free_b, size_t* total_b) {
  if (set_dev(c)) return 1;
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, c->device));
  if (sm_count) *sm_count = prop.multiProcessorCount;
  if (smem_optin) *smem_optin = (int)prop.sharedMemPerBlockOptin;
  size_t f = 0, t = 0;
  CK(cudaMemGetInfo(&f, &t));
  if (free_b) *free_b = f;
  if (total_b) *total_b = t;
  return 0;
}

// ---- device memory (the arena is one allocation; sub-allocation is host-side)
int ad_malloc(ad_ctx* c, size_t bytes, uint64_t* dptr) {
  if (set_dev(c)) return 1;
  void* p = nullptr;
  CK(cudaMalloc(&p, bytes ? bytes : 256));
  *dptr = reinterpret_cast<uint64_t>(p);
  return 0;
}

int ad_free(ad_ctx* c, uint64_t dptr) {
  if (set_dev(c)) return 1;
  CK(cudaFree(reinterpret_cast<void*>(dptr)));
  return 0;
}

int ad_memset(ad_ctx* c, uint64_t dptr, int value, size_t bytes, int stream) {
  cudaStream_t s;
  if (stream_of(c, stream, &s)) return 1;
  CK(cudaMemsetAsync(reinterpret_cast<void*>(dptr), value, bytes, s));
  return 0;
}

int ad_pinned_alloc(size_t bytes, void** p) {
  CK(cudaHostAlloc(p, bytes ? bytes : 64, cudaHostAllocPortable));
  return 0;
}

int ad_pinned_free(void* p) {
  CK(cudaFreeHost(p));
  return 0;
}

int ad_h2d(ad_ctx* c, uint64_t dst, const void* src, size_t bytes, int stream) {
  cudaStream_t s;
  if (stream_of(c, stream, &s)) return 1;
  CK(cudaMemcpyAsync(reinterpret_cast<void*>(dst), src, bytes, cudaMemcpyHostToDevice, s));
  return 0;
}

int ad_d2h(ad_ctx* c, void* dst, uint64_t src, size_t bytes, int stream) {
  cudaStream_t s;
  if (stream_of(c, stream, &s)) return 1;
  CK(cudaMemcpyAsync(dst, reinterpret_cast<const void*>(src), bytes, cudaMemcpyDeviceToHost, s));
  return 0;
}

int ad_d2d(ad_ctx* c, uint64_t dst, uint64_t src, size_t bytes, int stream) {
  cudaStream_t s;
  if (stream_of(c, stream, &s)) return 1;
  CK(cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), bytes,
                     cudaMemcpyDeviceToDevice, s));
  return 0;
}

int ad_host_copy(void* dst, const void* src, size_t bytes) {
  if (!bytes) return 0;
  if (!dst || !src) return fail("ad_host_copy: null pointer");
  CopyPool::get().copy(dst, src, bytes);
  return 0;
}

int ad_h2d_pageable(ad_ctx* c, uint64_t dst, const void* src, size_t bytes, int stream) {
  cudaStream_t s;
  if (stream_of(c, stream, &s) || set_dev(c) || ensure_stage(c)) return 1;
  const char* from = static_cast<const char*>(src);
  for (size_t off = 0, i = 0; off < bytes; off += kStageChunk, ++i) {
    int k = int(i % kStageSlots);
    size_t len = bytes - off < kStageChunk ? bytes - off : kStageChunk;
    if (c->stage_busy[k]) CK(cudaEventSynchronize(c->stage_ev[k]));  // its last copy has been read
    CopyPool::get().copy(c->stage[k], from + off, len);
    CK(cudaMemcpyAsync(reinterpret_cast<void*>(dst + off), c->stage[k], len, cudaMemcpyHostToDevice, s));
    CK(cudaEventRecord(c->stage_ev[k], s));
    c->stage_busy[k] = true;
  }
  return 0;
}

int ad_d2h_pageable(ad_ctx* c, void* dst, uint64_t src, size_t bytes, int stream) {
  cudaStream_t s;
  if (stream_of(c, stream, &s) || set_dev(c) || ensure_stage(c)) return 1;
  char* to = static_cast<char*>(dst);
  size_t n = (bytes + kStageChunk - 1) / kStageChunk;
  auto issue = [&](size_t i) -> int {
    int k = int(i % kStageSlots);
    size_t off = i * kStageChunk, len = bytes - off < kStageChunk ? bytes - off : kStageChunk;
    if (c->stage_busy[k]) CK(cudaEventSynchronize(c->stage_ev[k]));
    CK(cudaMemcpyAsync(c->stage[k], reinterpret_cast<const void*>(src + off), len, cudaMemcpyDeviceToHost, s));
    CK(cudaEventRecord(c->stage_ev[k], s));
    c->stage_busy[k] = true;
    return 0;
  };
  for (size_t i = 0; i < n && i < (size_t)kStageSlots; ++i)
    if (issue(i)) return 1;
  for (size_t i = 0; i < n; ++i) {
    int k = int(i % kStageSlots);
    size_t off = i * kStageChunk, len = bytes - off < kStageChunk ? bytes - off : kStageChunk;
    CK(cudaEventSynchronize(c->stage_ev[k]));
    c->stage_busy[k] = false;
    CopyPool::get().copy(to + off, c->stage[k], len);
    if (i + kStageSlots < n && issue(i + kStageSlots)) return 1;
  }
  return 0;
}

int ad_stream_sync(ad_ctx* c, int stream) {
  cudaStream_t s;
  if (stream_of(c, stream, &s)) return 1;
  CK(cudaStreamSynchronize(s));
  return 0;
}

int ad_sync(ad_ctx* c) {
  if (set_dev(c)) return 1;
  CK(cudaDeviceSynchronize());
  return 0;
}

// ---- events
int ad_event_create(ad_ctx* c, int timing, void** ev) {
  if (set_dev(c)) return 1;
  cudaEvent_t e;
  CK(cudaEventCreateWithFlags(&e, timing ? cudaEventDefault : cudaEventDisableTiming));
  *ev = e;
  return 0;
}

int ad_event_destroy(void* ev) {
  CK(cudaEventDestroy(static_cast<cudaEvent_t>(ev)));
  return 0;
}

int ad_event_record(ad_ctx* c, void* ev, int stream) {
  cudaStream_t s;
  if (stream_of(c, stream, &s)) return 1;
  CK(cudaEventRecord(static_cast<cudaEvent_t>(ev), s));
  return 0;
}

int ad_stream_wait_event(ad_ctx* c, int stream, void* ev) {
  cudaStream_t s;
  if (stream_of(c, stream, &s)) return 1;
  CK(cudaStreamWaitEvent(s, static_cast<cudaEvent_t>(ev), 0));
  return 0;
}

int ad_event_sync(void* ev) {
  CK(cudaEventSynchronize(static_cast<cudaEvent_t>(ev)));
  return 0;
}

int ad_event_elapsed_ms(void* start, void* end, float* ms) {
  CK(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(end)));
  return 0;
}

// ---- NVRTC: source -> sm_100a cubin -> module -> function
int ad_compile_cubin(const char* src, const char* name, const char* const* opts, int n_opts,
                     void** cubin, size_t* cubin_size, char* log, size_t log_len) {
  nvrtcProgram prog;
  nvrtcResult r = nvrtcCreateProgram(&prog, src, name, 0, nullptr, nullptr);
  if (r != NVRTC_SUCCESS) return fail("nvrtcCreateProgram: %s", nvrtcGetErrorString(r));
  std::vector<const char*> o;
  bool has_arch = false;
  for (int i = 0; i < n_opts; ++i) {
    o.push_back(opts[i]);
    if (strstr(opts[i], "-arch") || strstr(opts[i], "--gpu-architecture")) has_arch = true;
  }
  if (!has_arch) o.push_back("--gpu-architecture=sm_100a");
  r = nvrtcCompileProgram(prog, (int)o.size(), o.data());
  size_t ls = 0;
  nvrtcGetProgramLogSize(prog, &ls);
  std::string lg(ls, '\0');
  if (ls) nvrtcGetProgramLog(prog, &lg[0]);
  if (log && log_len) {
    size_t n = std::min(log_len - 1, lg.size());
    memcpy(log, lg.data(), n);
    log[n] = 0;
  }
  if (r != NVRTC_SUCCESS) {
    nvrtcDestroyProgram(&prog);
    return fail("NVRTC compile of %s failed: %s\n%s", name, nvrtcGetErrorString(r),
                lg.substr(0, 1800).c_str());
  }
  size_t n = 0;
  r = nvrtcGetCUBINSize(prog, &n);
  if (r != NVRTC_SUCCESS || n == 0) {
    nvrtcDestroyProgram(&prog);
    return fail("nvrtcGetCUBINSize: %s", nvrtcGetErrorString(r));
  }
  void* buf = malloc(n);
  nvrtcGetCUBIN(prog, static_cast<char*>(buf));
  nvrtcDestroyProgram(&prog);
  *cubin = buf;
  *cubin_size = n;
  return 0;
}

void ad_free_host(void* p) { free(p); }

int ad_load_kernel(ad_ctx* c, const void* cubin, const char* fn_name, ad_kernel** out) {
  if (driver()) return 1;
  if (set_dev(c)) return 1;
  ad_kernel* k = new ad_kernel();
  CUresult r = g_drv.moduleLoadData(&k->mod, cubin);
  if (r != CUDA_SUCCESS) {
    delete k;
    return cu_fail(r, "cuModuleLoadData");
  }
  r = g_drv.moduleGetFunction(&k->fn, k->mod, fn_name);
  if (r != CUDA_SUCCESS) {
    g_drv.moduleUnload(k->mod);
    delete k;
    return cu_fail(r, "cuModuleGetFunction");
  }
  k->name = fn_name;
  *out = k;
  return 0;
}

int ad_kernel_free(ad_kernel* k) {
  if (!k) return 0;
  if (k->mod && g_drv.ok) g_drv.moduleUnload(k->mod);
  delete k;
  return 0;
}

int ad_kernel_set_smem(ad_kernel* k, int bytes) {
  if (driver()) return 1;
  CUresult r =
      g_drv.funcSetAttribute(k->fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, bytes);
  if (r != CUDA_SUCCESS) return cu_fail(r, "cuFuncSetAttribute(MAX_DYNAMIC_SHARED)");
  return 0;
}

int ad_kernel_attr(ad_kernel* k, int* regs, int* static_smem, int* max_threads) {
  if (driver()) return 1;
  int v = 0;
  if (regs) {
    g_drv.funcGetAttribute(&v, CU_FUNC_ATTRIBUTE_NUM_REGS, k->fn);
    *regs = v;
  }
  if (static_smem) {
    g_drv.funcGetAttribute(&v, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, k->fn);
    *static_smem = v;
  }
  if (max_threads) {
    g_drv.funcGetAttribute(&v, CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, k->fn);
    *max_threads = v;
  }
  return 0;
}

int ad_launch(ad_ctx* c, ad_kernel* k, unsigned gx, unsigned gy, unsigned gz, unsigned bx,
              unsigned by, unsigned bz, unsigned smem, void** args, int stream) {
  cudaStream_t s;
  if (stream_of(c, stream, &s)) return 1;
  if (!k) return fail("null kernel");
  CUresult r = g_drv.launchKernel(k->fn, gx, gy, gz, bx, by, bz, smem, (CUstream)s, args, nullptr);
  if (r != CUDA_SUCCESS) {
    char what[256];
    snprintf(what, sizeof(what), "cuLaunchKernel(%s grid=%u,%u,%u block=%u,%u,%u smem=%u)",
             k->name.c_str(), gx, gy, gz, bx, by, bz, smem);
    return cu_fail(r, what);
  }
  return 0;
}

int ad_check(ad_ctx* c) {
  if (set_dev(c)) return 1;
  CK(cudaGetLastError());
  return 0;
}

// ---- TMA descriptors (2-D, row-major, fp32 or other 4-byte types)
int ad_tmap_2d(uint64_t base, uint64_t rows, uint64_t cols, uint64_t row_stride_bytes,
               uint32_t box_rows, uint32_t box_cols, int elem_bytes, int swizzle_bytes,
               void* out128) {
  if (driver()) return 1;
  CUtensorMapDataType dt;
  if (elem_bytes == 4) dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  else if (elem_bytes == 2) dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  else return fail("unsupported TMA element size %d", elem_bytes);
  CUtensorMapSwizzle sw;
  switch (swizzle_bytes) {
    case 0: sw = CU_TENSOR_MAP_SWIZZLE_NONE; break;
    case 32: sw = CU_TENSOR_MAP_SWIZZLE_32B; break;
    case 64: sw = CU_TENSOR_MAP_SWIZZLE_64B; break;
    case 128: sw = CU_TENSOR_MAP_SWIZZLE_128B; break;
    default: return fail("bad swizzle %d", swizzle_bytes);
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_drv.tensorMapEncodeTiled(
      reinterpret_cast<CUtensorMap*>(out128), dt, 2, reinterpret_cast<void*>(base), dims, strides,
      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cu_fail(r, "cuTensorMapEncodeTiled");
  return 0;
}

// ---- CUDA graphs: capture everything launched on `stream` between begin/end
int ad_graph_begin(ad_ctx* c, int stream) {
  cudaStream_t s;
  if (stream_of(c, stream, &s)) return 1;
  CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  return 0;
}

int ad_graph_end(ad_ctx* c, int stream, ad_graph** out) {
  cudaStream_t s;
  if (stream_of(c, stream, &s)) return 1;
  ad_graph* g = new ad_graph();
  cudaError_t e = cudaStreamEndCapture(s, &g->graph);
  if (e != cudaSuccess) {
    delete g;
    return fail("cudaStreamEndCapture: %s", cudaGetErrorString(e));
  }
  e = cudaGraphInstantiate(&g->exec, g->graph, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g->graph);
    delete g;
    return fail("cudaGraphInstantiate: %s", cudaGetErrorString(e));
  }
  *out = g;
  return 0;
}

int ad_graph_launch(ad_ctx* c, ad_graph* g, int stream) {
  cudaStream_t s;
  if (stream_of(c, stream, &s)) return 1;
  CK(cudaGraphLaunch(g->exec, s));
  return 0;
}

int ad_graph_destroy(ad_graph* g) {
  if (!g) return 0;
  if (g->exec) cudaGraphExecDestroy(g->exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  delete g;
  return 0;
}

// ---- NCCL
int ad_nccl_unique_id(void* out128) {
  if (nccl()) return 1;
  ncclUniqueId id;
  ncclResult_t r = g_nccl.getUniqueId(&id);
  if (r != ncclSuccess) return fail("ncclGetUniqueId: %s", g_nccl.getErrorString(r));
  memcpy(out128, &id, sizeof(id));
  return 0;
}

static int nccl_wait(ad_ctx* c, const char* what) {
  auto t0 = std::chrono::steady_clock::now();
  while (true) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = g_nccl.commGetAsyncError(c->comm, &st);
    if (r != ncclSuccess) return fail("%s: ncclCommGetAsyncError: %s", what, g_nccl.getErrorString(r));
    if (st == ncclSuccess) return 0;
    if (st != ncclInProgress) {
      g_nccl.commAbort(c->comm);
      c->comm = nullptr;
      return fail("%s: %s", what, g_nccl.getErrorString(st));
    }
    double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > c->nccl_timeout_s) {
      g_nccl.commAbort(c->comm);
      c->comm = nullptr;
      return fail("%s: timed out after %.1f s (communicator aborted)", what, el);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

int ad_nccl_init(ad_ctx* c, int rank, int world, const void* uid128, double timeout_s) {
  if (nccl()) return 1;
  if (set_dev(c)) return 1;
  ncclUniqueId id;
  memcpy(&id, uid128, sizeof(id));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  c->nccl_timeout_s = timeout_s > 0 ? timeout_s : 300.0;
  ncclResult_t r = g_nccl.commInitRankConfig(&c->comm, world, id, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    c->comm = nullptr;
    return fail("ncclCommInitRankConfig: %s", g_nccl.getErrorString(r));
  }
  if (nccl_wait(c, "ncclCommInitRankConfig")) return 1;
  c->rank = rank;
  c->world = world;
  return 0;
}

int ad_allreduce_f32(ad_ctx* c, uint64_t send, uint64_t recv, size_t count, int op_max,
                     int stream) {
  if (!c || !c->comm) return fail("NCCL communicator not initialised");
  cudaStream_t s;
  if (stream_of(c, stream, &s)) return 1;
  ncclResult_t r = g_nccl.allReduce(reinterpret_cast<const void*>(send), reinterpret_cast<void*>(recv),
                                    count, ncclFloat32, op_max ? ncclMax : ncclSum, c->comm, s);
  if (r != ncclSuccess && r != ncclInProgress) return fail("ncclAllReduce: %s", g_nccl.getErrorString(r));
  return nccl_wait(c, "ncclAllReduce");
}

int ad_nccl_abort(ad_ctx* c) {
  if (c && c->comm && g_nccl.ok) g_nccl.commAbort(c->comm);
  if (c) c->comm = nullptr;
  return 0;
}

}  // extern "C"

// ---------------------------------------------------------------- peer-memory all-reduce
// Gradient sums over the GPUs of one node without NCCL: every rank maps every
// other rank's arena (CUDA IPC over NVLink) and one kernel sums in two shots --
// rank r adds up shard r of the range from all ranks' copies (in rank order, so
// every rank gets bit-identical sums) and stores the result into every rank's
// copy.  Ranks meet at a flag barrier before reading (all gradients written:
// a rank's kernel runs only after its earlier kernels finished) and after
// storing (all shards complete before anyone reads its copy, and nobody
// overwrites a range a slower rank is still reading).  Each block of the kernel
// meets the same block of the other ranks, so blocks never wait for each other.
// Every wait is bounded (2 s of %globaltimer): on expiry the kernel records
// error 7 in the device's error word and returns.
namespace {
constexpr int kPeerMaxRanks = 8, kPeerMaxOps = 64, kPeerBlocks = 128, kPeerThreads = 512, kPeerUnroll = 4;
constexpr size_t kPeerFlagWords = 2ull * kPeerMaxOps * kPeerBlocks * kPeerMaxRanks;
constexpr size_t kPeerFlagBytes = (kPeerFlagWords + (size_t)kPeerMaxOps * kPeerBlocks) * 4;

struct PeerTab {
  float* data[kPeerMaxRanks];      // each rank's registered region, as mapped here
  unsigned* flags[kPeerMaxRanks];  // each rank's flag words, as mapped here
  unsigned* counters;              // this rank's per-(op, block) epochs
  int rank, world;
};

__device__ __forceinline__ void peer_st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned peer_ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long peer_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// thread 0 only: publish `epoch` for (phase, op, block) to every rank, then wait
// until every rank has published it here
__device__ bool peer_barrier(const PeerTab& t, int phase, int op, int b, unsigned epoch) {
  const size_t base = ((size_t)(phase * kPeerMaxOps + op) * kPeerBlocks + b) * kPeerMaxRanks;
  for (int j = 0; j < t.world; ++j) peer_st_release(t.flags[j] + base + t.rank, epoch);
  const unsigned* mine = t.flags[t.rank] + base;
  const unsigned long long t0 = peer_now();
  for (int j = 0; j < t.world; ++j)
    while ((int)(peer_ld_acquire(mine + j) - epoch) < 0)
      if (peer_now() - t0 > 2000000000ull) return false;
  return true;
}

__global__ void __launch_bounds__(kPeerThreads) peer_allreduce_kernel(const PeerTab* __restrict__ tp,
                                                                     size_t off, size_t count, int op,
                                                                     int* err) {
  __shared__ PeerTab t;
  __shared__ unsigned epoch;
  __shared__ int ok;
  const int b = blockIdx.x;
  if (threadIdx.x == 0) {
    t = *tp;
    unsigned* ctr = t.counters + op * kPeerBlocks + b;
    epoch = *ctr + 1;
    *ctr = epoch;
    ok = peer_barrier(t, 0, op, b, epoch);
    if (!ok) atomicExch(err, 7);
  }
  __syncthreads();
  if (ok) {
    const size_t per = ((count + t.world - 1) / t.world + 3) / 4 * 4;
    const size_t s0 = min(count, (size_t)t.rank * per), s1 = min(count, s0 + per);
    const size_t chunk = ((s1 - s0 + gridDim.x - 1) / gridDim.x + 3) / 4 * 4;
    const size_t c0 = min(s1, s0 + (size_t)b * chunk), c1 = min(s1, c0 + chunk);
    // kPeerUnroll float4 per thread per sweep, loads of every rank issued before the adds,
    // so each thread keeps several NVLink reads in flight
    const size_t step = 4 * (size_t)blockDim.x;
    for (size_t e0 = c0 + 4 * (size_t)threadIdx.x; e0 < c1; e0 += step * kPeerUnroll) {
      float4 acc[kPeerUnroll];
#pragma unroll
      for (int u = 0; u < kPeerUnroll; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < kPeerMaxRanks; ++j) {
        if (j >= t.world) break;
        float4 v[kPeerUnroll] = {};
#pragma unroll
        for (int u = 0; u < kPeerUnroll; ++u) {
          const size_t e = e0 + u * step;
          if (e < c1) v[u] = __ldcg(reinterpret_cast<const float4*>(t.data[j] + off + e));  // L2, not a stale L1 line
        }
#pragma unroll
        for (int u = 0; u < kPeerUnroll; ++u) {   // rank order: the same sums on every rank
          acc[u].x += v[u].x;
          acc[u].y += v[u].y;
          acc[u].z += v[u].z;
          acc[u].w += v[u].w;
        }
      }
#pragma unroll
      for (int j = 0; j < kPeerMaxRanks; ++j) {
        if (j >= t.world) break;
#pragma unroll
        for (int u = 0; u < kPeerUnroll; ++u) {
          const size_t e = e0 + u * step;
          if (e < c1) __stcg(reinterpret_cast<float4*>(t.data[j] + off + e), acc[u]);
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && ok) {
    __threadfence_system();
    if (!peer_barrier(t, 1, op, b, epoch)) atomicExch(err, 7);
  }
}
}  // namespace

extern "C" {

int ad_peer_init(ad_ctx* c, uint64_t base, size_t bytes) {
  if (!c || !c->comm) return fail("ad_peer_init: NCCL communicator not initialised");
  if (c->world > kPeerMaxRanks) return fail("ad_peer_init: at most %d ranks", kPeerMaxRanks);
  if (set_dev(c)) return 1;
  cudaStream_t s = c->streams[0];
  CK(cudaMalloc(&c->peer_flags, kPeerFlagBytes));
  CK(cudaMemset(c->peer_flags, 0, kPeerFlagBytes));
  // exchange (arena handle, flags handle) of every rank with one NCCL all-gather
  cudaIpcMemHandle_t mine[2];
  CK(cudaIpcGetMemHandle(&mine[0], reinterpret_cast<void*>(base)));
  CK(cudaIpcGetMemHandle(&mine[1], c->peer_flags));
  const size_t hb = sizeof(mine);
  void* dbuf = nullptr;
  CK(cudaMalloc(&dbuf, hb * (c->world + 1)));
  char* send = static_cast<char*>(dbuf) + hb * c->world;
  CK(cudaMemcpy(send, mine, hb, cudaMemcpyHostToDevice));
  ncclResult_t r = g_nccl.allGather(send, dbuf, hb, ncclChar, c->comm, s);
  if (r != ncclSuccess && r != ncclInProgress) {
    cudaFree(dbuf);
    return fail("ncclAllGather: %s", g_nccl.getErrorString(r));
  }
  if (nccl_wait(c, "ncclAllGather")) { cudaFree(dbuf); return 1; }
  std::vector<cudaIpcMemHandle_t> all(2 * c->world);
  CK(cudaStreamSynchronize(s));
  CK(cudaMemcpy(all.data(), dbuf, hb * c->world, cudaMemcpyDeviceToHost));
  CK(cudaFree(dbuf));
  PeerTab tab{};
  for (int j = 0; j < c->world; ++j) {
    if (j == c->rank) {
      tab.data[j] = reinterpret_cast<float*>(base);
      tab.flags[j] = static_cast<unsigned*>(c->peer_flags);
      continue;
    }
    void* pd = nullptr;
    void* pf = nullptr;
    CK(cudaIpcOpenMemHandle(&pd, all[2 * j], cudaIpcMemLazyEnablePeerAccess));
    c->peer_maps.push_back(pd);
    CK(cudaIpcOpenMemHandle(&pf, all[2 * j + 1], cudaIpcMemLazyEnablePeerAccess));
    c->peer_maps.push_back(pf);
    tab.data[j] = static_cast<float*>(pd);
    tab.flags[j] = static_cast<unsigned*>(pf);
  }
  tab.counters = static_cast<unsigned*>(c->peer_flags) + kPeerFlagWords;
  tab.rank = c->rank;
  tab.world = c->world;
  CK(cudaMalloc(&c->peer_tab, sizeof(PeerTab)));
  CK(cudaMemcpy(c->peer_tab, &tab, sizeof(PeerTab), cudaMemcpyHostToDevice));
  c->peer_base = base;
  c->peer_bytes = bytes;
  return 0;
}

int ad_peer_allreduce_f32(ad_ctx* c, uint64_t ptr, size_t count, int op, int stream, uint64_t err) {
  cudaStream_t s;
  if (stream_of(c, stream, &s)) return 1;
  if (!c->peer_tab) return fail("ad_peer_allreduce_f32: ad_peer_init was not called");
  if (op < 0 || op >= kPeerMaxOps) return fail("ad_peer_allreduce_f32: op slot %d outside [0, %d)", op, kPeerMaxOps);
  if (ptr < c->peer_base || ptr + 4 * count > c->peer_base + c->peer_bytes)
    return fail("ad_peer_allreduce_f32: range outside the registered region");
  if ((ptr - c->peer_base) % 16 || count % 4) return fail("ad_peer_allreduce_f32: range must be 16-byte aligned");
  peer_allreduce_kernel<<<kPeerBlocks, kPeerThreads, 0, s>>>(static_cast<const PeerTab*>(c->peer_tab),
                                                           (ptr - c->peer_base) / 4, count, op,
                                                           reinterpret_cast<int*>(err));
  CK(cudaGetLastError());
  return 0;
}

int ad_peer_close(ad_ctx* c) {
  if (!c) return 0;
  cudaSetDevice(c->device);
  for (void* p : c->peer_maps) cudaIpcCloseMemHandle(p);
  c->peer_maps.clear();
  if (c->peer_tab) cudaFree(c->peer_tab);
  if (c->peer_flags) cudaFree(c->peer_flags);
  c->peer_tab = c->peer_flags = nullptr;
  c->peer_base = 0;
  c->peer_bytes = 0;
  return 0;
}
int ad_profiler_range(int on) {
  CK(on ? cudaProfilerStart() : cudaProfilerStop());
  return 0;
}

}  // extern "C"
