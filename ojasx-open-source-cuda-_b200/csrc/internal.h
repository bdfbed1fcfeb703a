// internal.h — shared host-side declarations of libojx (not part of the C-ABI).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>
#include <atomic>
#include <nvtx3/nvToolsExt.h>
#include "../../include/ojx.h"

namespace ojx {

// Thread-local error message; returns `code` so call sites can `return set_error(...)`.
int set_error(int code, const char* fmt, ...);
// Code passed to this thread's last set_error.
int last_error_code();
// OJX_OK if e == cudaSuccess, else records the CUDA error string and returns OJX_ERR_CUDA
// (OJX_ERR_OOM for cudaErrorMemoryAllocation).
int cuda_status(cudaError_t e, const char* what);

extern std::atomic<uint64_t> g_launches;   // kernels launched by this library
extern std::atomic<uint64_t> g_wait_budget;  // SM cycles a device-side wait may spin
extern std::atomic<int> g_silence_producer_once;
// Next tagged skinny launch: contributors publish nothing (ojx_debug_silence_skinny_contributors_once).
extern std::atomic<int> g_silence_contributors_once;
void set_last_route(int route);

struct DeviceProps {
  int device = -1;
  int sm_count = 0;
  int max_smem_optin = 0;
  int cc_major = 0, cc_minor = 0;
};
// Properties of the current device (cached per device).
const DeviceProps& current_props();

// Per-stream scratch buffers, grown on demand and kept for the life of the
// process.  slot selects one of several independent buffers per stream.  With
// `zero`, a freshly (re)allocated buffer is cleared on the stream.  Returns
// nullptr and sets the error on failure.
// While `s` is being captured into a graph (ojx_graph_capture_begin), every call
// returns a fresh buffer owned by that capture instead (capture_workspace).
void* stream_workspace(cudaStream_t s, size_t bytes, int slot, bool zero);
void* capture_workspace(cudaStream_t s, size_t bytes, bool zero);
// Status code of this thread's last failed stream_workspace call.
int workspace_error();

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device).
int ensure_smem_attr(const void* kernel, int bytes);

// Output destinations of an all-gathering GEMM (every rank's C buffer).
struct Dests {
  int n;
  int64_t col_offset;
  void* p[OJX_MAX_PEERS];
};

// A batch of GEMMs sharing one descriptor: problem b reads A at a + b*stride_a
// elements (0: every problem reads the same A), likewise B, and writes C at
// c + b*stride_c with its epilogue operand at operand + b*stride_op.
struct BatchInfo {
  int64_t batch;
  int64_t stride_a, stride_b, stride_c, stride_op;
};

// Kernel families (implemented in the .cu files).  `dests` (optional) replaces
// the single output d.c by several buffers written with the same values.
int launch_tc_gemm(const ojx_gemm_desc& d, cudaStream_t s, const Dests* dests = nullptr,
                   const BatchInfo* bi = nullptr);
int launch_tc_gemm_3xtf32(const ojx_gemm_desc& d, cudaStream_t s, const BatchInfo* bi = nullptr);
int launch_skinny_gemm(const ojx_gemm_desc& d, cudaStream_t s, const Dests* dests = nullptr);
int launch_simt_gemm(const ojx_gemm_desc& d, cudaStream_t s);
bool tc_gemm_supported(const ojx_gemm_desc& d);
bool skinny_supported(const ojx_gemm_desc& d);

int launch_elementwise(void* out, int dt_out, const void* a, int dt_a, const void* b, int dt_b,
                       int bin, const int32_t* un, int n_un, int64_t n, cudaStream_t s);
int launch_transpose(void* out, const void* in, int64_t rows, int64_t cols, int dtype,
                     cudaStream_t s);
int launch_fill(void* out, double v, int64_t n, int dtype, cudaStream_t s);
int launch_cast(void* out, int dt_out, const void* in, int dt_in, int64_t n, cudaStream_t s);
bool flash_attn_supported(int dtype, int64_t D);
int launch_flash_attn(const void* q, const void* k, const void* v, void* out, int dtype, int64_t BH,
                      int64_t M, int64_t N, int64_t nk, int64_t D, float scale, int causal,
                      cudaStream_t s);
int launch_flash_attn2(const void* q, const void* k, const void* v, void* out, int dtype, int64_t BH,
                      int64_t M, int64_t N, int64_t nk, int64_t D, float scale, int causal,
                      cudaStream_t s);
int launch_attn_softmax(const float* S, int64_t ld, int64_t rows, int M, int nk, float scale,
                        int causal, void* P, int dtype_p, cudaStream_t s);
int launch_sum_columns(void* out, int dt_out, const void* in, int dt_in, int64_t rows, int64_t cols,
                       int64_t ld, cudaStream_t s);
int read_and_clear_device_error(unsigned int* word);
// The first failed device-side bounds check (site, coordinate, coordinate, extent)
// of the OJX_DEBUG_BOUNDS build; debug_bounds_build() says whether this is that build.
int read_bounds_info(long long info[4]);
bool debug_bounds_build();

inline int dtype_size(int dt) { return dt == OJX_F32 ? 4 : 2; }

// NVTX range around the enqueue of one GEMM / attention (a profiler such as Nsight
// Systems or `ncu --nvtx --nvtx-include` sees which library call launched which
// kernels; with no tool attached the push and pop return at once).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

}  // namespace ojx
