// ojx_kernels.cu — the single CUDA translation unit of libojx.  All kernel
// sources are included here so they share one device error word (g_dev_error)
// without relocatable device code.
#include "kernels_simt.cuh"
#include "gemm_tc.cuh"
#include "gemm_skinny.cuh"
#include "attention.cuh"
#include "flash_attn.cuh"
#include "flash_attn2.cuh"
#include <mutex>

// ── decode GEMM for callers that cannot allocate device memory ───────────────
//
// Some callers must not have this library allocate GPU memory behind their
// back: a serving engine that reserves nearly all HBM at start-up (for its KV
// cache and weights) and treats any later cudaMalloc as a failure, or a
// latency-critical decode loop in which a cudaMalloc/cudaFree could synchronise
// the device and stall the other streams.  ojx_gemm's skinny route takes its
// split-K scratch (partial sums and per-group arrival counters) from a per-stream
// workspace that it grows with cudaMalloc.  ojx_gemm_skinny_noalloc runs the same
// kernel with that scratch in the fixed array below instead, and calls no
// allocating routine.
//
// Limits and sharing:
//  * the array holds kNoAllocScratchBytes (8 MiB) on every GPU that loads the
//    library, for the life of the process;
//  * problems whose scratch does not fit are rejected with OJX_ERR_INVALID;
//  * every call shares the one array and leaves its contents behind.  The arrival
//    counters carry a per-launch epoch, so whatever an earlier call left there is
//    ignored; the partial slots are always written before they are read.  Two
//    calls that run at the same time on the GPU (different streams, no ordering)
//    race on the array: order them on one stream or synchronise;
//  * the first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) and sets the kernel's shared-memory limit; make that
//    first call before capturing a stream.
namespace ojx {

constexpr size_t kNoAllocCounterBytes = 64 * 1024;  // up to 8192 column groups
constexpr size_t kNoAllocScratchBytes = 8u << 20;    // counters + partial slots

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device (the host-side name is only a
// stand-in and must never be handed to a kernel).
static void* g_noalloc_ptr[128];
static std::mutex g_noalloc_mu;

static int noalloc_setup(void** out) {
  int dev = 0;
  int st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
  if (st) return st;
  if (dev < 0 || dev >= 128) return set_error(OJX_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    // No clearing is needed (or issued: a cudaMemset here would run on the legacy
    // stream, unordered with a caller's non-blocking stream): a __device__ array
    // starts zeroed, and the arrival counters are tagged with a launch epoch, so
    // counts an earlier call left behind never match a new launch's epoch.
    if ((st = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress")))
      return st;
    const void* kernels[4] = {reinterpret_cast<const void*>(skinny_gemm_kernel<1, 1>),
                              reinterpret_cast<const void*>(skinny_gemm_kernel<1, 0>),
                              reinterpret_cast<const void*>(skinny_gemm_kernel<0, 1>),
                              reinterpret_cast<const void*>(skinny_gemm_kernel<0, 0>)};
    for (const void* k : kernels) {
      if ((st = cuda_status(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM),
                            "cudaFuncSetAttribute")))
        return st;
      if ((st = cuda_status(cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                                                 cudaSharedmemCarveoutMaxShared),
                            "cudaFuncSetAttribute(carveout)")))
        return st;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return OJX_OK;
}

}  // namespace ojx

extern "C" int ojx_gemm_skinny_noalloc(const ojx_gemm_desc* in, ojx_stream stream) {
  using namespace ojx;
  NvtxRange nvtx("ojx_gemm_skinny_noalloc");
  if (!in) return set_error(OJX_ERR_INVALID, "ojx_gemm_skinny_noalloc: desc is NULL");
  ojx_gemm_desc d = *in;
  if (d.dtype_a != d.dtype_b || (d.dtype_a != OJX_BF16 && d.dtype_a != OJX_F16))
    return set_error(OJX_ERR_INVALID, "ojx_gemm_skinny_noalloc: A and B must both be bf16 or both fp16");
  if (d.dtype_c != OJX_F32 && d.dtype_c != OJX_BF16 && d.dtype_c != OJX_F16)
    return set_error(OJX_ERR_INVALID, "ojx_gemm_skinny_noalloc: unknown output dtype");
  if (d.M < 1 || d.M > SK_MN || d.N < 1 || d.K < 1 || d.N > INT32_MAX || d.K > INT32_MAX)
    return set_error(OJX_ERR_INVALID, "ojx_gemm_skinny_noalloc: needs 1 <= M <= %d and N, K >= 1", SK_MN);
  if (d.trans_a) return set_error(OJX_ERR_INVALID, "ojx_gemm_skinny_noalloc: A must be row-major [M, K]");
  if (!d.a || !d.b || !d.c) return set_error(OJX_ERR_INVALID, "ojx_gemm_skinny_noalloc: NULL matrix pointer");
  if (d.lda == 0) d.lda = d.K;
  if (d.ldb == 0) d.ldb = d.trans_b ? d.K : d.N;
  if (d.ldc == 0) d.ldc = d.N;
  if (d.ld_operand == 0) d.ld_operand = d.N;
  if (d.lda < d.K || d.ldb < (d.trans_b ? d.K : d.N) || d.ldc < d.N)
    return set_error(OJX_ERR_INVALID, "ojx_gemm_skinny_noalloc: leading dimension smaller than a row");
  if (reinterpret_cast<uintptr_t>(d.a) % 16 || reinterpret_cast<uintptr_t>(d.b) % 16 ||
      (d.lda * 2) % 16 || (d.ldb * 2) % 16)
    return set_error(OJX_ERR_INVALID, "ojx_gemm_skinny_noalloc: A and B need 16-byte aligned rows");
  if (d.n_unary < 0 || d.n_unary > OJX_MAX_UNARY)
    return set_error(OJX_ERR_INVALID, "ojx_gemm_skinny_noalloc: n_unary out of range");
  for (int i = 0; i < d.n_unary; ++i)
    if (d.unary[i] < OJX_UN_RELU || d.unary[i] > OJX_UN_SQUARE)
      return set_error(OJX_ERR_INVALID, "ojx_gemm_skinny_noalloc: unknown unary op %d", d.unary[i]);
  if (d.operand_kind != OJX_OPERAND_NONE &&
      ((d.operand_kind != OJX_OPERAND_ROW && d.operand_kind != OJX_OPERAND_FULL) || !d.operand ||
       d.binary_op < OJX_BIN_ADD || d.binary_op > OJX_BIN_DIV ||
       (d.dtype_operand != OJX_F32 && d.dtype_operand != OJX_BF16 && d.dtype_operand != OJX_F16)))
    return set_error(OJX_ERR_INVALID, "ojx_gemm_skinny_noalloc: bad epilogue operand");
  const DeviceProps& dp = current_props();
  if (dp.cc_major < 10)
    return set_error(OJX_ERR_NOT_INITIALIZED, "ojx_gemm_skinny_noalloc: current device is not sm_100");

  SkinnyParams p{};
  p.M = static_cast<int>(d.M);
  p.N = static_cast<int>(d.N);
  p.K = static_cast<int>(d.K);
  p.n_groups = (p.N + SK_TPU * SK_BN - 1) / (SK_TPU * SK_BN);
  p.KB = (p.K + SK_BK - 1) / SK_BK;
  p.U = static_cast<long long>(p.n_groups) * p.KB;
  p.G = skinny_grid(p.n_groups, p.KB, p.U, dp.sm_count);  // the same grid as ojx_gemm's skinny route
  p.maxc = skinny_max_contrib(p.n_groups, p.KB, p.U, p.G);
  const size_t counter_bytes = static_cast<size_t>(p.n_groups) * 8;
  const size_t part_bytes = static_cast<size_t>(p.n_groups) * p.maxc * SK_SLOT * 4;
  if (counter_bytes > kNoAllocCounterBytes || part_bytes > kNoAllocScratchBytes - kNoAllocCounterBytes)
    return set_error(OJX_ERR_INVALID,
                     "ojx_gemm_skinny_noalloc: N=%d K=%d needs %zu bytes of scratch; the fixed "
                     "array holds %zu (use ojx_gemm for larger problems)",
                     p.N, p.K, counter_bytes + part_bytes, kNoAllocScratchBytes);
  void* scratch = nullptr;
  int st = noalloc_setup(&scratch);
  if (st) return st;
  p.counters = static_cast<unsigned long long*>(scratch);
  p.partials = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + kNoAllocCounterBytes);
  p.epoch = g_skinny_epoch.fetch_add(1);
  if (p.epoch == 0) p.epoch = g_skinny_epoch.fetch_add(1);
  p.budget = g_wait_budget.load();
  p.silence_producer = 0;
  // This launch must stay a plain one that never lets the next kernel in early:
  // it does not publish the ranges it writes to the per-stream record the skinny
  // route consults before loading W ahead of its dependency wait, so a following
  // eager skinny launch may only overlap a grid that has completed.
  p.trigger_early = 0;
  p.early_w = 0;

  const CUtensorMapDataType tdt =
      d.dtype_a == OJX_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tw, tx;
  const bool w_mn = !d.trans_b;
  if (w_mn)
    st = make_tmap_2d_sw128_uncached(&tw, tdt, 2, d.b, p.N, p.K, d.ldb * 2, 64, 64);
  else
    st = make_tmap_2d_sw128_uncached(&tw, tdt, 2, d.b, p.K, p.N, d.ldb * 2, 64, SK_BN);
  if (st) return st;
  if ((st = make_tmap_2d_sw128_uncached(&tx, tdt, 2, d.a, p.K, p.M, d.lda * 2, 64, SK_MN))) return st;
  const EpiParams ep = make_epi(d);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf = d.dtype_a == OJX_BF16;
  if (bf && w_mn) skinny_gemm_kernel<1, 1><<<p.G, SK_THREADS, SK_SMEM, s>>>(tw, tx, ep, p);
  else if (bf) skinny_gemm_kernel<1, 0><<<p.G, SK_THREADS, SK_SMEM, s>>>(tw, tx, ep, p);
  else if (w_mn) skinny_gemm_kernel<0, 1><<<p.G, SK_THREADS, SK_SMEM, s>>>(tw, tx, ep, p);
  else skinny_gemm_kernel<0, 0><<<p.G, SK_THREADS, SK_SMEM, s>>>(tw, tx, ep, p);
  g_launches.fetch_add(1);
  return cuda_status(cudaGetLastError(), "skinny_gemm_noalloc launch");
}
