// runtime.cpp — the C-ABI of libojx: device/context, caching allocator, copies,
// streams/events, error reporting and the GEMM route selection.
//
// Replaces torchcl/runtime/context.py (device + queue singletons),
// torchcl/runtime/memory.py (CLBufferPool), torchcl/runtime/stream.py and the
// kernel choice of torchcl/ops/engine.py:156-255.
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>
#include "internal.h"

namespace ojx {

static thread_local std::string t_last_error;
static thread_local int t_last_code = OJX_OK;
static thread_local int t_last_route = OJX_ROUTE_NONE;
std::atomic<uint64_t> g_launches{0};
std::atomic<uint64_t> g_wait_budget{4000000000ull};  // about 2 s at B200 clocks
std::atomic<int> g_silence_producer_once{0};
std::atomic<int> g_silence_contributors_once{0};

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  t_last_code = code;
  return code;
}

int last_error_code() { return t_last_code; }

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return OJX_OK;
  const int code = e == cudaErrorMemoryAllocation ? OJX_ERR_OOM : OJX_ERR_CUDA;
  set_error(code, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  if (e == cudaErrorMemoryAllocation) (void)cudaGetLastError();  // not sticky; clear it
  return code;
}

void set_last_route(int route) { t_last_route = route; }

int ensure_smem_attr(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int>* done = new std::map<std::pair<const void*, int>, int>();
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  auto key = std::make_pair(kernel, dev);
  auto it = done->find(key);
  if (it != done->end() && it->second >= bytes) return OJX_OK;
  int st = cuda_status(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
                       "cudaFuncSetAttribute");
  // Whole shared-memory carveout, so kernels sized for two CTAs per SM get both.
  if (!st)
    st = cuda_status(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                          cudaSharedmemCarveoutMaxShared),
                     "cudaFuncSetAttribute(carveout)");
  if (!st) (*done)[key] = bytes;
  return st;
}

const DeviceProps& current_props() {
  static std::mutex mu;
  static DeviceProps props[128];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 128) dev = 0;
  std::lock_guard<std::mutex> g(mu);
  DeviceProps& p = props[dev];
  if (p.device != dev) {
    cudaDeviceGetAttribute(&p.sm_count, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&p.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&p.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&p.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
    p.device = dev;
  }
  return p;
}

// ── caching allocator ───────────────────────────────────────────────────────
// Bins: 512 B minimum, powers of two up to 64 MiB (the slab policy of
// torchcl/runtime/memory.py:20-24, with a floor that keeps every block 256-byte
// aligned for TMA), and 2 MiB multiples above that so very large tensors do not
// waste up to half their size.  A freed block goes back to its bin; an OOM frees
// every cached block and retries once (memory.py:109-115).  Reuse is ordered on
// the device only through the stream the caller uses for the block: like the
// reference's single in-order queue, callers that hand a freed buffer to another
// stream must synchronise first.
class Pool {
 public:
  static size_t bin_size(size_t n) {
    if (n <= 512) return 512;
    if (n <= (size_t(64) << 20)) {
      size_t b = 512;
      while (b < n) b <<= 1;
      return b;
    }
    const size_t g = size_t(2) << 20;
    return (n + g - 1) / g * g;
  }

  int malloc(size_t n, void** out, size_t* cap) {
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t c = bin_size(n);
    std::lock_guard<std::mutex> g(mu_);
    auto& bin = bins_[{dev, c}];
    void* p = nullptr;
    if (!bin.empty()) {
      p = bin.back();
      bin.pop_back();
      st_.reuse_count++;
      st_.cached_bytes -= static_cast<int64_t>(c);
    } else {
      cudaError_t e = raw_malloc(&p, c);
      if (e == cudaErrorMemoryAllocation) {
        (void)cudaGetLastError();
        release_cached_locked();
        st_.evictions++;
        e = raw_malloc(&p, c);
      }
      if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return set_error(e == cudaErrorMemoryAllocation ? OJX_ERR_OOM : OJX_ERR_CUDA,
                         "ojx_malloc(%zu): %s after evicting the cache", n, cudaGetErrorString(e));
      }
      st_.alloc_count++;
      st_.total_allocated_bytes += static_cast<int64_t>(c);
    }
    active_[p] = {dev, c};
    st_.active_bytes += static_cast<int64_t>(c);
    st_.active_buffers = static_cast<int64_t>(active_.size());
    st_.peak_bytes = std::max(st_.peak_bytes, st_.active_bytes);
    *out = p;
    if (cap) *cap = c;
    return OJX_OK;
  }

  int free(void* p) {
    if (!p) return OJX_OK;
    std::lock_guard<std::mutex> g(mu_);
    auto it = active_.find(p);
    if (it == active_.end()) return set_error(OJX_ERR_INVALID, "ojx_free(%p): not a live pool block", p);
    const Block b = it->second;
    active_.erase(it);
    bins_[{b.dev, b.cap}].push_back(p);
    st_.free_count++;
    st_.active_bytes -= static_cast<int64_t>(b.cap);
    st_.cached_bytes += static_cast<int64_t>(b.cap);
    st_.active_buffers = static_cast<int64_t>(active_.size());
    return OJX_OK;
  }

  int empty_cache() {
    std::lock_guard<std::mutex> g(mu_);
    return release_cached_locked();
  }

  void stats(ojx_pool_stats* out) {
    std::lock_guard<std::mutex> g(mu_);
    *out = st_;
  }

  void fail_next(int64_t n) {
    std::lock_guard<std::mutex> g(mu_);
    fail_next_ = n;
  }

 private:
  struct Block {
    int dev;
    size_t cap;
  };
  cudaError_t raw_malloc(void** p, size_t n) {
    if (fail_next_ > 0) {
      --fail_next_;
      return cudaErrorMemoryAllocation;
    }
    return cudaMalloc(p, n);
  }
  int release_cached_locked() {
    int cur = 0;
    cudaGetDevice(&cur);
    int st = OJX_OK;
    for (auto& kv : bins_) {
      if (kv.second.empty()) continue;
      cudaSetDevice(kv.first.first);
      for (void* p : kv.second) {
        const cudaError_t e = cudaFree(p);
        if (e != cudaSuccess && st == OJX_OK) st = cuda_status(e, "cudaFree(cached block)");
      }
      kv.second.clear();
    }
    bins_.clear();
    st_.cached_bytes = 0;
    cudaSetDevice(cur);
    return st;
  }

  std::mutex mu_;
  std::map<std::pair<int, size_t>, std::vector<void*>> bins_;
  std::unordered_map<void*, Block> active_;
  ojx_pool_stats st_{};
  int64_t fail_next_ = 0;
};

static Pool& pool() {
  static Pool* p = new Pool();  // never destroyed: blocks may outlive static teardown
  return *p;
}

// ── per-stream workspaces ───────────────────────────────────────────────────
struct WsKey {
  int dev;
  cudaStream_t s;
  int slot;
  bool operator<(const WsKey& o) const {
    if (dev != o.dev) return dev < o.dev;
    if (s != o.s) return s < o.s;
    return slot < o.slot;
  }
};
struct WsBuf {
  void* p = nullptr;
  size_t bytes = 0;
};

static thread_local int t_ws_error = OJX_OK;
int workspace_error() { return t_ws_error == OJX_OK ? OJX_ERR_OOM : t_ws_error; }

static void* stream_workspace_impl(cudaStream_t s, size_t bytes, int slot, bool zero) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (s && cudaStreamIsCapturing(s, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
    return capture_workspace(s, bytes, zero);
  static std::mutex mu;
  static std::map<WsKey, WsBuf>* bufs = new std::map<WsKey, WsBuf>();
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  WsBuf& w = (*bufs)[{dev, s, slot}];
  if (w.bytes >= bytes && w.p) return w.p;
  if (w.p) {
    // Growing: earlier launches on this stream may still read the old buffer.
    if (cuda_status(cudaStreamSynchronize(s), "workspace grow: stream sync")) return nullptr;
    cudaFree(w.p);
    w = WsBuf{};
  }
  const size_t g2 = size_t(2) << 20;
  const size_t nb = (std::max<size_t>(bytes, 1) + g2 - 1) / g2 * g2;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, nb);
  if (e == cudaErrorMemoryAllocation) {
    (void)cudaGetLastError();
    pool().empty_cache();
    e = cudaMalloc(&p, nb);
  }
  if (e != cudaSuccess) {
    cuda_status(e, "workspace cudaMalloc");
    return nullptr;
  }
  if (zero && cuda_status(cudaMemsetAsync(p, 0, nb, s), "workspace clear")) {
    cudaFree(p);
    return nullptr;
  }
  w.p = p;
  w.bytes = nb;
  return p;
}

void* stream_workspace(cudaStream_t s, size_t bytes, int slot, bool zero) {
  void* p = stream_workspace_impl(s, bytes, slot, zero);
  if (!p) {
    // set_error has recorded the message; keep its code for the caller.
    t_ws_error = last_error_code();
  }
  return p;
}

static bool valid_dtype(int dt) { return dt == OJX_F32 || dt == OJX_BF16 || dt == OJX_F16; }
static bool valid_unary(int op) { return op >= OJX_UN_RELU && op <= OJX_UN_SQUARE; }
static bool valid_binary(int op) { return op >= OJX_BIN_ADD && op <= OJX_BIN_DIV; }

}  // namespace ojx

using namespace ojx;

extern "C" {

int ojx_abi_version(void) { return OJX_ABI_VERSION; }

int ojx_device_count(int* count) {
  if (!count) return set_error(OJX_ERR_INVALID, "count is NULL");
  int n = 0;
  const cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    *count = 0;
    return cuda_status(e, "cudaGetDeviceCount");
  }
  *count = n;
  return OJX_OK;
}

int ojx_init(int device, ojx_device_info* info) {
  int n = 0;
  int st = ojx_device_count(&n);
  if (st) return st;
  if (device < 0 || device >= n)
    return set_error(OJX_ERR_INVALID, "device %d out of range (%d CUDA device(s))", device, n);
  if ((st = cuda_status(cudaSetDevice(device), "cudaSetDevice"))) return st;
  if ((st = cuda_status(cudaFree(nullptr), "context init"))) return st;
  const DeviceProps& p = current_props();
  if (p.cc_major < 10)
    return set_error(OJX_ERR_UNSUPPORTED, "device %d is sm_%d%d; libojx is built for sm_100a", device,
                     p.cc_major, p.cc_minor);
  if (info) {
    cudaDeviceProp prop;
    if ((st = cuda_status(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties")))
      return st;
    std::memset(info, 0, sizeof(*info));
    std::snprintf(info->name, sizeof(info->name), "%s", prop.name);
    info->device = device;
    info->cc_major = prop.major;
    info->cc_minor = prop.minor;
    info->sm_count = prop.multiProcessorCount;
    info->total_mem_bytes = static_cast<int64_t>(prop.totalGlobalMem);
    info->l2_bytes = prop.l2CacheSize;
    info->max_smem_per_block = static_cast<int32_t>(prop.sharedMemPerBlockOptin);
    int clk = 0;
    cudaDeviceGetAttribute(&clk, cudaDevAttrClockRate, device);
    info->clock_khz = clk;
  }
  return OJX_OK;
}

int ojx_current_device(int* device) {
  if (!device) return set_error(OJX_ERR_INVALID, "device is NULL");
  return cuda_status(cudaGetDevice(device), "cudaGetDevice");
}

int ojx_synchronize(void) { return cuda_status(cudaDeviceSynchronize(), "cudaDeviceSynchronize"); }

const char* ojx_last_error(void) { return t_last_error.c_str(); }

int ojx_poll_device_error(void) {
  unsigned int w = 0;
  int st = read_and_clear_device_error(&w);
  if (st) return st;
  if (w & 2u) {  // bit 1: a debug-build bounds check failed (sm100.cuh, OJX_DEVERR_BOUNDS)
    long long info[4] = {0, 0, 0, 0};
    if ((st = read_bounds_info(info))) return st;
    return set_error(OJX_ERR_BOUNDS,
                     "device-side bounds check failed at site %lld (coordinates %lld, %lld; "
                     "extent %lld); the access was skipped",
                     info[0], info[1], info[2], info[3]);
  }
  if (w & 1u)  // bit 0: a bounded wait expired (sm100.cuh, OJX_DEVERR_TIMEOUT)
    return set_error(OJX_ERR_TIMEOUT,
                     "a device-side wait exceeded its budget; the kernel returned early and its "
                     "output is incomplete");
  return OJX_OK;
}

int ojx_debug_bounds_enabled(void) { return debug_bounds_build() ? 1 : 0; }

int ojx_set_wait_budget(uint64_t cycles) {
  if (cycles == 0) return set_error(OJX_ERR_INVALID, "wait budget must be positive");
  g_wait_budget.store(cycles);
  return OJX_OK;
}

uint64_t ojx_kernel_launch_count(void) { return g_launches.load(); }

int ojx_last_route(void) { return t_last_route; }

int ojx_malloc(size_t nbytes, void** dptr, size_t* capacity) {
  if (!dptr) return set_error(OJX_ERR_INVALID, "dptr is NULL");
  return pool().malloc(nbytes, dptr, capacity);
}

int ojx_free(void* dptr) { return pool().free(dptr); }

int ojx_empty_cache(void) { return pool().empty_cache(); }

int ojx_pool_stats_get(ojx_pool_stats* out) {
  if (!out) return set_error(OJX_ERR_INVALID, "out is NULL");
  pool().stats(out);
  return OJX_OK;
}

int ojx_pool_bin_size(size_t nbytes, size_t* capacity) {
  if (!capacity) return set_error(OJX_ERR_INVALID, "capacity is NULL");
  *capacity = Pool::bin_size(nbytes);
  return OJX_OK;
}

int ojx_pool_debug_fail_next(int64_t n_allocs) {
  pool().fail_next(n_allocs);
  return OJX_OK;
}

static int copy(void* dst, const void* src, size_t n, ojx_stream s, const char* what) {
  if (n == 0) return OJX_OK;
  if (!dst || !src) return set_error(OJX_ERR_INVALID, "%s: NULL pointer", what);
  return cuda_status(cudaMemcpyAsync(dst, src, n, cudaMemcpyDefault, static_cast<cudaStream_t>(s)),
                     what);
}

int ojx_memcpy_h2d(void* dst, const void* src, size_t n, ojx_stream s) {
  return copy(dst, src, n, s, "ojx_memcpy_h2d");
}
int ojx_memcpy_d2h(void* dst, const void* src, size_t n, ojx_stream s) {
  return copy(dst, src, n, s, "ojx_memcpy_d2h");
}
int ojx_memcpy_d2d(void* dst, const void* src, size_t n, ojx_stream s) {
  return copy(dst, src, n, s, "ojx_memcpy_d2d");
}
int ojx_memset(void* dst, int value, size_t n, ojx_stream s) {
  if (n == 0) return OJX_OK;
  if (!dst) return set_error(OJX_ERR_INVALID, "ojx_memset: NULL pointer");
  return cuda_status(cudaMemsetAsync(dst, value, n, static_cast<cudaStream_t>(s)), "ojx_memset");
}
int ojx_host_alloc(size_t n, void** p) {
  if (!p) return set_error(OJX_ERR_INVALID, "host_ptr is NULL");
  return cuda_status(cudaHostAlloc(p, std::max<size_t>(n, 1), cudaHostAllocDefault), "cudaHostAlloc");
}
int ojx_host_free(void* p) { return cuda_status(cudaFreeHost(p), "cudaFreeHost"); }

int ojx_stream_create(ojx_stream* s) {
  if (!s) return set_error(OJX_ERR_INVALID, "s is NULL");
  cudaStream_t cs;
  int st = cuda_status(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "cudaStreamCreate");
  if (!st) *s = cs;
  return st;
}
int ojx_stream_destroy(ojx_stream s) {
  return cuda_status(cudaStreamDestroy(static_cast<cudaStream_t>(s)), "cudaStreamDestroy");
}
int ojx_stream_synchronize(ojx_stream s) {
  return cuda_status(cudaStreamSynchronize(static_cast<cudaStream_t>(s)), "cudaStreamSynchronize");
}
int ojx_stream_wait_event(ojx_stream s, ojx_event e) {
  return cuda_status(
      cudaStreamWaitEvent(static_cast<cudaStream_t>(s), static_cast<cudaEvent_t>(e), 0),
      "cudaStreamWaitEvent");
}
int ojx_event_create(ojx_event* e, int enable_timing) {
  if (!e) return set_error(OJX_ERR_INVALID, "e is NULL");
  cudaEvent_t ev;
  int st = cuda_status(
      cudaEventCreateWithFlags(&ev, enable_timing ? cudaEventDefault : cudaEventDisableTiming),
      "cudaEventCreate");
  if (!st) *e = ev;
  return st;
}
int ojx_event_destroy(ojx_event e) {
  return cuda_status(cudaEventDestroy(static_cast<cudaEvent_t>(e)), "cudaEventDestroy");
}
int ojx_event_record(ojx_event e, ojx_stream s) {
  return cuda_status(cudaEventRecord(static_cast<cudaEvent_t>(e), static_cast<cudaStream_t>(s)),
                     "cudaEventRecord");
}
int ojx_event_query(ojx_event e, int* done) {
  if (!done) return set_error(OJX_ERR_INVALID, "done is NULL");
  const cudaError_t r = cudaEventQuery(static_cast<cudaEvent_t>(e));
  if (r == cudaErrorNotReady) {
    (void)cudaGetLastError();
    *done = 0;
    return OJX_OK;
  }
  *done = r == cudaSuccess;
  return cuda_status(r, "cudaEventQuery");
}
int ojx_event_synchronize(ojx_event e) {
  return cuda_status(cudaEventSynchronize(static_cast<cudaEvent_t>(e)), "cudaEventSynchronize");
}
int ojx_event_elapsed_ms(ojx_event a, ojx_event b, float* ms) {
  if (!ms) return set_error(OJX_ERR_INVALID, "ms is NULL");
  return cuda_status(
      cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(a), static_cast<cudaEvent_t>(b)),
      "cudaEventElapsedTime");
}

}  // extern "C"

namespace ojx {
constexpr int kEmptyProblem = -1;

// Checks a descriptor and fills in dense leading dimensions.  Returns OJX_OK,
// kEmptyProblem (nothing to compute) or an error code.
static int prepare_desc(const ojx_gemm_desc* in, ojx_gemm_desc* out, const char* who) {
  if (!in) return set_error(OJX_ERR_INVALID, "%s: desc is NULL", who);
  ojx_gemm_desc d = *in;
  if (d.M < 0 || d.N < 0 || d.K < 0)
    return set_error(OJX_ERR_INVALID, "%s: negative dimension (%lld, %lld, %lld)", who,
                     (long long)d.M, (long long)d.N, (long long)d.K);
  if (!valid_dtype(d.dtype_a) || !valid_dtype(d.dtype_b) || !valid_dtype(d.dtype_c))
    return set_error(OJX_ERR_INVALID, "%s: unknown dtype", who);
  if (d.n_unary < 0 || d.n_unary > OJX_MAX_UNARY)
    return set_error(OJX_ERR_INVALID, "%s: n_unary %d out of range", who, d.n_unary);
  for (int i = 0; i < d.n_unary; ++i)
    if (!valid_unary(d.unary[i]))
      return set_error(OJX_ERR_INVALID, "%s: unknown unary op %d", who, d.unary[i]);
  if (d.operand_kind != OJX_OPERAND_NONE) {
    if (d.operand_kind != OJX_OPERAND_ROW && d.operand_kind != OJX_OPERAND_FULL)
      return set_error(OJX_ERR_INVALID, "%s: unknown operand kind %d", who, d.operand_kind);
    if (!d.operand) return set_error(OJX_ERR_INVALID, "%s: operand pointer is NULL", who);
    if (!valid_binary(d.binary_op))
      return set_error(OJX_ERR_INVALID, "%s: unknown binary op %d", who, d.binary_op);
    if (!valid_dtype(d.dtype_operand))
      return set_error(OJX_ERR_INVALID, "%s: unknown operand dtype", who);
  }
  if (d.M == 0 || d.N == 0) return kEmptyProblem;
  if (!d.c || (d.K > 0 && (!d.a || !d.b)))
    return set_error(OJX_ERR_INVALID, "%s: NULL matrix pointer", who);
  if (d.lda == 0) d.lda = d.trans_a ? d.M : d.K;
  if (d.ldb == 0) d.ldb = d.trans_b ? d.K : d.N;
  if (d.ldc == 0) d.ldc = d.N;
  if (d.ld_operand == 0) d.ld_operand = d.N;
  if (d.lda < (d.trans_a ? d.M : d.K) || d.ldb < (d.trans_b ? d.K : d.N) || d.ldc < d.N ||
      (d.operand_kind == OJX_OPERAND_FULL && d.ld_operand < d.N))
    return set_error(OJX_ERR_INVALID, "%s: leading dimension smaller than the row length", who);
  if (current_props().cc_major < 10)
    return set_error(OJX_ERR_NOT_INITIALIZED, "%s: current device is not sm_100 (call ojx_init)", who);
  *out = d;
  return OJX_OK;
}

static int gemm_one(const ojx_gemm_desc& d, cudaStream_t s) {
  const bool f16 = d.dtype_a == d.dtype_b && (d.dtype_a == OJX_BF16 || d.dtype_a == OJX_F16);
  const bool f32 = d.dtype_a == OJX_F32 && d.dtype_b == OJX_F32;
  int route = OJX_ROUTE_SIMT;
  if (!(d.flags & OJX_GEMM_FLAG_FORCE_SIMT) && d.K > 0) {
    if (f16) {
      const bool skinny_ok = !(d.flags & OJX_GEMM_FLAG_NO_SKINNY) && skinny_supported(d);
      if (skinny_ok && (d.M <= 16 || (d.flags & OJX_GEMM_FLAG_FORCE_SKINNY)))
        route = OJX_ROUTE_SKINNY;
      else if (tc_gemm_supported(d))
        route = OJX_ROUTE_TC_F16;
    } else if (f32 && d.fp32_mode != OJX_FP32_FFMA && d.M <= INT32_MAX && d.N <= INT32_MAX &&
               d.K <= INT32_MAX) {
      if (d.fp32_mode == OJX_FP32_3XTF32 || d.M > 16) route = OJX_ROUTE_TC_3XTF32;
    }
  }
  int st;
  switch (route) {
    case OJX_ROUTE_SKINNY: {
      NvtxRange r("ojx_gemm skinny");
      st = launch_skinny_gemm(d, s);
      break;
    }
    case OJX_ROUTE_TC_F16: {
      NvtxRange r("ojx_gemm tc_f16");
      st = launch_tc_gemm(d, s);
      break;
    }
    case OJX_ROUTE_TC_3XTF32: {
      NvtxRange r("ojx_gemm tc_3xtf32");
      st = launch_tc_gemm_3xtf32(d, s);
      break;
    }
    default: {
      NvtxRange r("ojx_gemm simt");
      st = launch_simt_gemm(d, s);
      break;
    }
  }
  if (st == OJX_OK) set_last_route(route);
  return st;
}
}  // namespace ojx

extern "C" {

int ojx_gemm(const ojx_gemm_desc* in, ojx_stream stream) {
  set_last_route(OJX_ROUTE_NONE);
  ojx_gemm_desc d;
  const int st = prepare_desc(in, &d, "ojx_gemm");
  if (st == kEmptyProblem) return OJX_OK;
  if (st) return st;
  return gemm_one(d, static_cast<cudaStream_t>(stream));
}

int ojx_gemm_batched(const ojx_gemm_desc* in, int64_t batch, int64_t stride_a, int64_t stride_b,
                     int64_t stride_c, int64_t stride_operand, ojx_stream stream) {
  NvtxRange nvtx("ojx_gemm_batched");
  set_last_route(OJX_ROUTE_NONE);
  if (batch < 0 || stride_a < 0 || stride_b < 0 || stride_c < 0 || stride_operand < 0)
    return set_error(OJX_ERR_INVALID, "ojx_gemm_batched: negative batch or stride");
  if (batch == 0) return OJX_OK;
  ojx_gemm_desc d;
  int st = prepare_desc(in, &d, "ojx_gemm_batched");
  if (st == kEmptyProblem) return OJX_OK;
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (batch == 1) return gemm_one(d, s);
  if (stride_c < (d.M - 1) * d.ldc + d.N)
    return set_error(OJX_ERR_INVALID,
                     "ojx_gemm_batched: stride_c %lld makes the problems' outputs overlap",
                     (long long)stride_c);
  const bool f16 = d.dtype_a == d.dtype_b && (d.dtype_a == OJX_BF16 || d.dtype_a == OJX_F16);
  const bool f32 = d.dtype_a == OJX_F32 && d.dtype_b == OJX_F32;
  const int64_t tiles = ((d.M + 127) / 128) * ((d.N + 127) / 128) * batch;
  const bool one_launch = !(d.flags & OJX_GEMM_FLAG_FORCE_SIMT) && d.K > 0 && tiles <= INT32_MAX &&
                          batch <= 65535;
  BatchInfo bi{batch, stride_a, stride_b, stride_c, stride_operand};
  // The f16 kernel reads A and B through rank-3 TMA maps: their batch strides must
  // be 16-byte multiples.  The 3xTF32 path copies its operands into its own
  // aligned layout first, so any stride works there.
  if (one_launch && f16 && tc_gemm_supported(d) && (stride_a * 2) % 16 == 0 &&
      (stride_b * 2) % 16 == 0) {
    st = launch_tc_gemm(d, s, nullptr, &bi);
    if (st == OJX_OK) {
      set_last_route(OJX_ROUTE_TC_F16);
      return OJX_OK;
    }
    if (st != OJX_ERR_UNSUPPORTED) return st;
  } else if (one_launch && f32 && d.fp32_mode != OJX_FP32_FFMA && d.M <= INT32_MAX &&
             d.N <= INT32_MAX && d.K <= INT32_MAX && (d.fp32_mode == OJX_FP32_3XTF32 || d.M > 16)) {
    st = launch_tc_gemm_3xtf32(d, s, &bi);
    if (st == OJX_OK) {
      set_last_route(OJX_ROUTE_TC_3XTF32);
      return OJX_OK;
    }
    if (st != OJX_ERR_UNSUPPORTED) return st;
  }
  // Any other case: one launch per problem on the stream, in order.
  const int ea = dtype_size(d.dtype_a), eb = dtype_size(d.dtype_b), ec = dtype_size(d.dtype_c);
  const int eo = dtype_size(d.dtype_operand);
  for (int64_t b = 0; b < batch; ++b) {
    ojx_gemm_desc db = d;
    db.a = static_cast<const char*>(d.a) + b * stride_a * ea;
    db.b = static_cast<const char*>(d.b) + b * stride_b * eb;
    db.c = static_cast<char*>(d.c) + b * stride_c * ec;
    if (d.operand) db.operand = static_cast<const char*>(d.operand) + b * stride_operand * eo;
    if ((st = gemm_one(db, s))) return st;
  }
  return OJX_OK;
}

}  // extern "C"

namespace ojx {
namespace {
// Streams and events of ojx_gemm_host_io, one set per device.
struct IoStreams {
  cudaStream_t h2d = nullptr, comp = nullptr, d2h = nullptr;
  std::vector<cudaEvent_t> ev;
  std::mutex mu;  // one call at a time issues on these streams
};
IoStreams* io_streams(int dev) {
  static std::mutex mu;
  static std::map<int, IoStreams*>* m = new std::map<int, IoStreams*>();
  std::lock_guard<std::mutex> g(mu);
  IoStreams*& io = (*m)[dev];
  if (!io) {
    auto* n = new IoStreams();
    if (cudaStreamCreateWithFlags(&n->h2d, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&n->comp, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&n->d2h, cudaStreamNonBlocking) != cudaSuccess) {
      (void)cudaGetLastError();
      delete n;
      return nullptr;
    }
    io = n;
  }
  return io;
}
int io_events(IoStreams* io, size_t n) {
  while (io->ev.size() < n) {
    cudaEvent_t e;
    if (int st = cuda_status(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate"))
      return st;
    io->ev.push_back(e);
  }
  return OJX_OK;
}
}  // namespace
}  // namespace ojx

extern "C" {

int ojx_gemm_host_io(const ojx_gemm_desc* in, void* dev_a, void* dev_c, int64_t chunk_rows,
                     ojx_stream stream) {
  NvtxRange nvtx("ojx_gemm_host_io");
  set_last_route(OJX_ROUTE_NONE);
  ojx_gemm_desc d;
  int st = prepare_desc(in, &d, "ojx_gemm_host_io");
  if (st == kEmptyProblem) return OJX_OK;
  if (st) return st;
  if (!dev_a || !dev_c) return set_error(OJX_ERR_INVALID, "ojx_gemm_host_io: NULL staging buffer");
  if (d.trans_a || d.lda != d.K || d.ldc != d.N)
    return set_error(OJX_ERR_INVALID,
                     "ojx_gemm_host_io: A must be row-major [M,K] and C [M,N], both dense");
  int dev = 0;
  if ((st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice"))) return st;
  IoStreams* io = io_streams(dev);
  if (!io) return set_error(OJX_ERR_CUDA, "ojx_gemm_host_io: cannot create its streams");
  std::lock_guard<std::mutex> g(io->mu);
  const int64_t M = d.M;
  // Chunks of whole 128-row tile blocks: about 8 of them, so the first upload and
  // the last download (the parts not hidden behind a GEMM) stay small.
  int64_t rows = chunk_rows > 0 ? chunk_rows : ((M + 7) / 8 + 127) / 128 * 128;
  if (rows >= M || M <= 256) rows = M;
  const int64_t n_chunks = (M + rows - 1) / rows;
  if ((st = io_events(io, static_cast<size_t>(2 * n_chunks + 2)))) return st;
  cudaEvent_t* ev = io->ev.data();
  const size_t ea = dtype_size(d.dtype_a), ec = dtype_size(d.dtype_c), eo = dtype_size(d.dtype_operand);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // everything after the work already queued on the caller's stream
  if ((st = cuda_status(cudaEventRecord(ev[0], s), "event record"))) return st;
  for (cudaStream_t x : {io->h2d, io->comp, io->d2h})
    if ((st = cuda_status(cudaStreamWaitEvent(x, ev[0], 0), "stream wait"))) return st;
  int route = OJX_ROUTE_NONE;
  for (int64_t c = 0; c < n_chunks; ++c) {
    const int64_t r0 = c * rows, nr = std::min(rows, M - r0);
    char* da = static_cast<char*>(dev_a) + static_cast<size_t>(r0 * d.K) * ea;
    char* dc = static_cast<char*>(dev_c) + static_cast<size_t>(r0 * d.N) * ec;
    const char* ha = static_cast<const char*>(d.a) + static_cast<size_t>(r0 * d.K) * ea;
    char* hc = static_cast<char*>(d.c) + static_cast<size_t>(r0 * d.N) * ec;
    cudaEvent_t up = ev[2 + 2 * c], done = ev[3 + 2 * c];
    if ((st = cuda_status(cudaMemcpyAsync(da, ha, static_cast<size_t>(nr * d.K) * ea,
                                          cudaMemcpyHostToDevice, io->h2d), "chunk upload")) ||
        (st = cuda_status(cudaEventRecord(up, io->h2d), "event record")) ||
        (st = cuda_status(cudaStreamWaitEvent(io->comp, up, 0), "stream wait")))
      return st;
    ojx_gemm_desc dd = d;
    dd.M = nr;
    dd.a = da;
    dd.c = dc;
    if (d.operand_kind == OJX_OPERAND_FULL)
      dd.operand = static_cast<const char*>(d.operand) + static_cast<size_t>(r0 * d.ld_operand) * eo;
    if ((st = gemm_one(dd, io->comp))) return st;
    route = t_last_route;
    if ((st = cuda_status(cudaEventRecord(done, io->comp), "event record")) ||
        (st = cuda_status(cudaStreamWaitEvent(io->d2h, done, 0), "stream wait")) ||
        (st = cuda_status(cudaMemcpyAsync(hc, dc, static_cast<size_t>(nr * d.N) * ec,
                                          cudaMemcpyDeviceToHost, io->d2h), "chunk download")))
      return st;
  }
  // the caller's stream continues once C is in host memory
  if ((st = cuda_status(cudaEventRecord(ev[1], io->d2h), "event record")) ||
      (st = cuda_status(cudaStreamWaitEvent(s, ev[1], 0), "stream wait")))
    return st;
  set_last_route(route);
  return OJX_OK;
}

int ojx_elementwise(void* out, int32_t dtype_out, const void* a, int32_t dtype_a, const void* b,
                    int32_t dtype_b, int32_t binary_op, const int32_t* unary, int32_t n_unary,
                    int64_t n, ojx_stream s) {
  if (n < 0) return set_error(OJX_ERR_INVALID, "ojx_elementwise: negative length");
  if (n == 0) return OJX_OK;
  if (!out || !a) return set_error(OJX_ERR_INVALID, "ojx_elementwise: NULL pointer");
  if (!valid_dtype(dtype_out) || !valid_dtype(dtype_a) || (b && !valid_dtype(dtype_b)))
    return set_error(OJX_ERR_INVALID, "ojx_elementwise: unknown dtype");
  if (b && !valid_binary(binary_op))
    return set_error(OJX_ERR_INVALID, "ojx_elementwise: unknown binary op %d", binary_op);
  if (n_unary < 0 || n_unary > OJX_MAX_UNARY || (n_unary > 0 && !unary))
    return set_error(OJX_ERR_INVALID, "ojx_elementwise: bad unary chain");
  for (int i = 0; i < n_unary; ++i)
    if (!valid_unary(unary[i]))
      return set_error(OJX_ERR_INVALID, "ojx_elementwise: unknown unary op %d", unary[i]);
  return launch_elementwise(out, dtype_out, a, dtype_a, b, dtype_b, binary_op, unary, n_unary, n,
                            static_cast<cudaStream_t>(s));
}

int ojx_transpose(void* out, const void* in, int64_t rows, int64_t cols, int32_t dtype,
                  ojx_stream s) {
  if (rows < 0 || cols < 0) return set_error(OJX_ERR_INVALID, "ojx_transpose: negative shape");
  if (rows * cols == 0) return OJX_OK;
  if (!out || !in) return set_error(OJX_ERR_INVALID, "ojx_transpose: NULL pointer");
  if (!valid_dtype(dtype)) return set_error(OJX_ERR_INVALID, "ojx_transpose: unknown dtype");
  return launch_transpose(out, in, rows, cols, dtype, static_cast<cudaStream_t>(s));
}

int ojx_fill(void* out, double value, int64_t n, int32_t dtype, ojx_stream s) {
  if (n < 0) return set_error(OJX_ERR_INVALID, "ojx_fill: negative length");
  if (n == 0) return OJX_OK;
  if (!out) return set_error(OJX_ERR_INVALID, "ojx_fill: NULL pointer");
  if (!valid_dtype(dtype)) return set_error(OJX_ERR_INVALID, "ojx_fill: unknown dtype");
  return launch_fill(out, value, n, dtype, static_cast<cudaStream_t>(s));
}

int ojx_cast(void* out, int32_t dtype_out, const void* in, int32_t dtype_in, int64_t n,
             ojx_stream s) {
  if (n < 0) return set_error(OJX_ERR_INVALID, "ojx_cast: negative length");
  if (n == 0) return OJX_OK;
  if (!out || !in) return set_error(OJX_ERR_INVALID, "ojx_cast: NULL pointer");
  if (!valid_dtype(dtype_out) || !valid_dtype(dtype_in))
    return set_error(OJX_ERR_INVALID, "ojx_cast: unknown dtype");
  return launch_cast(out, dtype_out, in, dtype_in, n, static_cast<cudaStream_t>(s));
}

int ojx_attention(void* out, const void* q, const void* k, const void* v, int32_t dtype,
                  int64_t batch, int64_t heads, int64_t M, int64_t N, int64_t D, float scale,
                  int32_t causal, int64_t max_keys, int32_t flags, ojx_stream stream) {
  set_last_route(OJX_ROUTE_NONE);
  NvtxRange nvtx("ojx_attention");
  if (batch < 0 || heads < 0 || M < 0 || N < 0 || D < 0)
    return set_error(OJX_ERR_INVALID, "ojx_attention: negative size");
  if (!valid_dtype(dtype)) return set_error(OJX_ERR_INVALID, "ojx_attention: unknown dtype");
  const int64_t BH = batch * heads;
  if (BH == 0 || M == 0 || D == 0) return OJX_OK;
  if (!out || !q || (N > 0 && (!k || !v)))
    return set_error(OJX_ERR_INVALID, "ojx_attention: NULL pointer");
  if (M > INT32_MAX || N > INT32_MAX) return set_error(OJX_ERR_INVALID, "ojx_attention: too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t nk = max_keys > 0 && N > max_keys ? max_keys : N;
  const int es = dtype_size(dtype);
  if (nk == 0) {  // no keys: every output is an empty sum
    return cuda_status(cudaMemsetAsync(out, 0, static_cast<size_t>(BH * M * D) * es, s),
                       "attention memset");
  }
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!(flags & OJX_ATTN_FLAG_COMPOSED) && flash_attn_supported(dtype, D) && al16(q) && al16(k) &&
      al16(v) && al16(out)) {
    // Two query tiles per CTA (ping-pong) measured faster than one on every shape
    // tried (1024-8192 queries, D 64/128, causal or not), wave quantisation included;
    // OJX_ATTN_FLAG_ONE_QTILE still selects the one-tile kernel.
    const bool two = !(flags & OJX_ATTN_FLAG_ONE_QTILE);
    const int st = two ? launch_flash_attn2(q, k, v, out, dtype, BH, M, N, nk, D, scale, causal ? 1 : 0, s)
                       : launch_flash_attn(q, k, v, out, dtype, BH, M, N, nk, D, scale, causal ? 1 : 0, s);
    if (st == OJX_OK) set_last_route(OJX_ROUTE_FLASH_ATTN);
    return st;
  }
  const int64_t ld = (nk + 7) / 8 * 8;  // 16-byte rows for fp32 and 16-bit elements
  const int dtype_p = dtype;            // P in the input's precision (fp32 stays fp32)
  float* S = static_cast<float*>(
      stream_workspace(s, static_cast<size_t>(BH * M * ld) * sizeof(float), 4, false));
  if (!S) return workspace_error();
  void* P = stream_workspace(s, static_cast<size_t>(BH * M * ld) * es, 5, false);
  if (!P) return workspace_error();
  // S = Q K^T (keys beyond nk are not read)
  ojx_gemm_desc g{};
  g.M = M, g.N = nk, g.K = D;
  g.dtype_a = g.dtype_b = dtype, g.dtype_c = OJX_F32;
  g.trans_b = 1;
  g.lda = D, g.ldb = D, g.ldc = ld;
  g.a = q, g.b = k, g.c = S;
  int st = ojx_gemm_batched(&g, BH, M * D, N * D, M * ld, 0, stream);
  if (st) return st;
  const int route1 = t_last_route;
  if ((st = launch_attn_softmax(S, ld, BH * M, static_cast<int>(M), static_cast<int>(nk), scale,
                                causal ? 1 : 0, P, dtype_p, s)))
    return st;
  // O = P V
  ojx_gemm_desc h{};
  h.M = M, h.N = D, h.K = nk;
  h.dtype_a = dtype_p, h.dtype_b = dtype, h.dtype_c = dtype;
  h.lda = ld, h.ldb = D, h.ldc = D;
  h.a = P, h.b = v, h.c = out;
  st = ojx_gemm_batched(&h, BH, M * ld, N * D, M * D, 0, stream);
  if (st == OJX_OK && route1 != t_last_route) set_last_route(OJX_ROUTE_NONE);
  return st;
}

int ojx_sum_columns(void* out, int32_t dtype_out, const void* in, int32_t dtype_in, int64_t rows,
                    int64_t cols, int64_t ld, ojx_stream s) {
  NvtxRange nvtx("ojx_sum_columns");
  if (rows < 0 || cols < 0) return set_error(OJX_ERR_INVALID, "ojx_sum_columns: negative size");
  if (cols == 0) return OJX_OK;
  if (!out || (rows > 0 && !in)) return set_error(OJX_ERR_INVALID, "ojx_sum_columns: NULL pointer");
  if (!valid_dtype(dtype_out) || !valid_dtype(dtype_in))
    return set_error(OJX_ERR_INVALID, "ojx_sum_columns: unknown dtype");
  if (ld == 0) ld = cols;
  if (ld < cols) return set_error(OJX_ERR_INVALID, "ojx_sum_columns: ld %lld < cols %lld",
                                  static_cast<long long>(ld), static_cast<long long>(cols));
  return launch_sum_columns(out, dtype_out, in, dtype_in, rows, cols, ld, static_cast<cudaStream_t>(s));
}

int ojx_ipc_get_handle(void* dptr, void* handle_out) {
  if (!dptr || !handle_out) return set_error(OJX_ERR_INVALID, "ojx_ipc_get_handle: NULL pointer");
  static_assert(sizeof(cudaIpcMemHandle_t) == OJX_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  int st = cuda_status(cudaIpcGetMemHandle(&h, dptr), "cudaIpcGetMemHandle");
  if (!st) std::memcpy(handle_out, &h, sizeof(h));
  return st;
}

int ojx_ipc_open_handle(const void* handle, void** dptr) {
  if (!handle || !dptr) return set_error(OJX_ERR_INVALID, "ojx_ipc_open_handle: NULL pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess),
                     "cudaIpcOpenMemHandle");
}

int ojx_ipc_close_handle(void* dptr) {
  return cuda_status(cudaIpcCloseMemHandle(dptr), "cudaIpcCloseMemHandle");
}

int ojx_gemm_allgather(const ojx_gemm_desc* in, void* const* c_peers, int32_t n_peers,
                       int64_t col_offset, ojx_stream stream) {
  set_last_route(OJX_ROUTE_NONE);
  NvtxRange nvtx("ojx_gemm_allgather");
  if (!in || !c_peers) return set_error(OJX_ERR_INVALID, "ojx_gemm_allgather: NULL argument");
  if (n_peers < 1 || n_peers > OJX_MAX_PEERS)
    return set_error(OJX_ERR_INVALID, "ojx_gemm_allgather: %d peers (1..%d)", n_peers, OJX_MAX_PEERS);
  if (col_offset < 0) return set_error(OJX_ERR_INVALID, "ojx_gemm_allgather: negative column offset");
  ojx_gemm_desc d = *in;
  for (int i = 0; i < n_peers; ++i)
    if (!c_peers[i]) return set_error(OJX_ERR_INVALID, "ojx_gemm_allgather: peer %d is NULL", i);
  if (d.M <= 0 || d.N <= 0 || d.K <= 0)
    return set_error(OJX_ERR_INVALID, "ojx_gemm_allgather: empty problem");
  if (d.ldc == 0) return set_error(OJX_ERR_INVALID, "ojx_gemm_allgather: ldc (the full row length) is required");
  if (d.ldc < col_offset + d.N)
    return set_error(OJX_ERR_INVALID, "ojx_gemm_allgather: column block exceeds ldc");
  if (d.lda == 0) d.lda = d.trans_a ? d.M : d.K;
  if (d.ldb == 0) d.ldb = d.trans_b ? d.K : d.N;
  if (d.ld_operand == 0) d.ld_operand = d.N;
  if (d.n_unary < 0 || d.n_unary > OJX_MAX_UNARY) return set_error(OJX_ERR_INVALID, "bad n_unary");
  for (int i = 0; i < d.n_unary; ++i)
    if (!valid_unary(d.unary[i])) return set_error(OJX_ERR_INVALID, "unknown unary op %d", d.unary[i]);
  if (d.operand_kind != OJX_OPERAND_NONE &&
      (!d.operand || !valid_binary(d.binary_op) || !valid_dtype(d.dtype_operand)))
    return set_error(OJX_ERR_INVALID, "ojx_gemm_allgather: bad epilogue operand");
  if (current_props().cc_major < 10)
    return set_error(OJX_ERR_NOT_INITIALIZED, "ojx_gemm_allgather: current device is not sm_100");
  d.c = c_peers[0];
  Dests dests{};
  dests.n = n_peers;
  dests.col_offset = col_offset;
  for (int i = 0; i < n_peers; ++i) dests.p[i] = c_peers[i];
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st;
  if (!(d.flags & OJX_GEMM_FLAG_NO_SKINNY) && d.M <= 16 && skinny_supported(d)) {
    st = launch_skinny_gemm(d, s, &dests);
    if (!st) set_last_route(OJX_ROUTE_SKINNY);
  } else if (tc_gemm_supported(d)) {
    st = launch_tc_gemm(d, s, &dests);
    if (!st) set_last_route(OJX_ROUTE_TC_F16);
  } else {
    st = set_error(OJX_ERR_UNSUPPORTED,
                   "ojx_gemm_allgather: needs bf16/fp16 operands with 16-byte aligned rows");
  }
  return st;
}

int ojx_debug_silence_producer_once(void) {
  g_silence_producer_once.store(1);
  return OJX_OK;
}

int ojx_debug_silence_skinny_contributors_once(void) {
  g_silence_contributors_once.store(1);
  return OJX_OK;
}

}  // extern "C"
