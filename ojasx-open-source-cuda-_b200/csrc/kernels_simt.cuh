// kernels_simt.cu — the non-tensor-core kernels of libojx:
//   * simt_gemm_kernel: any dtype mix, any strides, any shape; fp32 FMA with k
//     ascending per output element (the accumulation order of the reference's
//     matmul.cl kernels, with each multiply-add fused).  Used for fp32_mode FFMA,
//     for fp32 problems with M <= 16, and whenever a tcgen05 route cannot describe
//     the operands (unaligned strides/pointers, mixed dtypes, K == 0).
//   * elementwise_kernel: fused binary + unary chain over a flat range
//     (torchcl/jit/compiler.py:64-133).
//   * transpose / fill / cast.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <algorithm>
#include "sm100.cuh"
#include "epilogue.cuh"
#include "internal.h"

namespace ojx {

constexpr int SG_BM = 64, SG_BN = 64, SG_BK = 16;

template <int DTA, int DTB>
__global__ void __launch_bounds__(256)
    simt_gemm_kernel(const void* __restrict__ A, int64_t sam, int64_t sak,
                     const void* __restrict__ B, int64_t sbk, int64_t sbn, const EpiParams ep,
                     int M, int N, int K) {
  __shared__ float As[SG_BK][SG_BM + 4];
  __shared__ float Bs[SG_BK][SG_BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * SG_BM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * SG_BN;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  const bool a_kfast = sak == 1;  // consecutive threads walk k (row-major A)
  const bool b_nfast = sbn == 1;  // consecutive threads walk n (row-major B)
  for (int k0 = 0; k0 < K; k0 += SG_BK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + i * 256;
      const int mm = a_kfast ? idx / SG_BK : idx % SG_BM;
      const int kk = a_kfast ? idx % SG_BK : idx / SG_BM;
      const int64_t gm = m0 + mm;
      const int gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < K) ? load_elem(A, gm * sam + gk * sak, DTA) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + i * 256;
      const int nn = b_nfast ? idx % SG_BN : idx / SG_BK;
      const int kk = b_nfast ? idx / SG_BN : idx % SG_BK;
      const int64_t gn = n0 + nn;
      const int gk = k0 + kk;
      Bs[kk][nn] = (gn < N && gk < K) ? load_elem(B, gk * sbk + gn * sbn, DTB) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SG_BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = m0 + ty * 4 + i;
    if (row >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t col = n0 + tx * 4 + j;
      if (col < N && epi_store_ok(ep, SITE_SIMT_STORE, row, col, 1))
        store_elem(ep.c, row * ep.ldc + col, ep.dtype_c, epilogue_value(ep, acc[i][j], row, col));
    }
  }
}

int launch_simt_gemm(const ojx_gemm_desc& d, cudaStream_t s) {
  if (d.M > INT32_MAX || d.N > INT32_MAX || d.K > INT32_MAX)
    return set_error(OJX_ERR_UNSUPPORTED, "SIMT GEMM dimensions must fit in 32 bits");
  const int64_t sam = d.trans_a ? 1 : d.lda, sak = d.trans_a ? d.lda : 1;
  const int64_t sbk = d.trans_b ? 1 : d.ldb, sbn = d.trans_b ? d.ldb : 1;
  const EpiParams ep = make_epi(d);
  dim3 grid(static_cast<unsigned>((d.N + SG_BN - 1) / SG_BN),
            static_cast<unsigned>((d.M + SG_BM - 1) / SG_BM));
  if (grid.y > 65535) return set_error(OJX_ERR_UNSUPPORTED, "SIMT GEMM: M too large");
  const int M = static_cast<int>(d.M), N = static_cast<int>(d.N), K = static_cast<int>(d.K);
#define OJX_SIMT(DA, DB)                                                                 \
  if (d.dtype_a == DA && d.dtype_b == DB) {                                              \
    simt_gemm_kernel<DA, DB><<<grid, 256, 0, s>>>(d.a, sam, sak, d.b, sbk, sbn, ep, M, N, K); \
    g_launches.fetch_add(1);                                                             \
    return cuda_status(cudaGetLastError(), "simt_gemm launch");                          \
  }
  OJX_SIMT(OJX_F32, OJX_F32) OJX_SIMT(OJX_BF16, OJX_BF16) OJX_SIMT(OJX_F16, OJX_F16)
  OJX_SIMT(OJX_F32, OJX_BF16) OJX_SIMT(OJX_BF16, OJX_F32) OJX_SIMT(OJX_F32, OJX_F16)
  OJX_SIMT(OJX_F16, OJX_F32) OJX_SIMT(OJX_BF16, OJX_F16) OJX_SIMT(OJX_F16, OJX_BF16)
#undef OJX_SIMT
  return set_error(OJX_ERR_INVALID, "unsupported dtype pair %d/%d", d.dtype_a, d.dtype_b);
}

// ── elementwise ─────────────────────────────────────────────────────────────
struct EwParams {
  int32_t bin;
  int32_t n_un;
  uint32_t un_packed;  // 4 bits per unary op
};

__global__ void __launch_bounds__(256)
    elementwise_kernel(void* __restrict__ out, int dt_out, const void* __restrict__ a, int dt_a,
                       const void* __restrict__ b, int dt_b, const EwParams p, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    float v = load_elem(a, i, dt_a);
    if (b) v = apply_binary(p.bin, v, load_elem(b, i, dt_b));
    for (int k = 0; k < p.n_un; ++k) v = apply_unary(unary_at(p.un_packed, k), v);
    store_elem(out, i, dt_out, v);
  }
}

static int grid_for(int64_t n) {
  const DeviceProps& p = current_props();
  const int64_t blocks = (n + 255) / 256;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, int64_t(p.sm_count) * 16)));
}

int launch_elementwise(void* out, int dt_out, const void* a, int dt_a, const void* b, int dt_b,
                       int bin, const int32_t* un, int n_un, int64_t n, cudaStream_t s) {
  if (n <= 0) return OJX_OK;
  EwParams p{};
  p.bin = bin;
  p.n_un = n_un;
  for (int i = 0; i < n_un; ++i) p.un_packed |= (static_cast<uint32_t>(un[i]) & 15u) << (4 * i);
  elementwise_kernel<<<grid_for(n), 256, 0, s>>>(out, dt_out, a, dt_a, b, dt_b, p, n);
  g_launches.fetch_add(1);
  return cuda_status(cudaGetLastError(), "elementwise launch");
}

// ── transpose: out[c][r] = in[r][c], 32x32 tiles through shared memory ─────────
template <typename T>
__global__ void __launch_bounds__(256)
    transpose_kernel(T* __restrict__ out, const T* __restrict__ in, int64_t rows, int64_t cols) {
  __shared__ T tile[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * 32, r0 = static_cast<int64_t>(blockIdx.y) * 32;
  for (int i = ty; i < 32; i += 8) {
    const int64_t r = r0 + i, c = c0 + tx;
    if (r < rows && c < cols) tile[i][tx] = in[r * cols + c];
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int64_t c = c0 + i, r = r0 + tx;
    if (r < rows && c < cols) out[c * rows + r] = tile[tx][i];
  }
}

int launch_transpose(void* out, const void* in, int64_t rows, int64_t cols, int dtype,
                     cudaStream_t s) {
  if (rows <= 0 || cols <= 0) return OJX_OK;
  if ((rows + 31) / 32 > 65535) return set_error(OJX_ERR_UNSUPPORTED, "transpose: too many rows");
  dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((rows + 31) / 32));
  if (dtype == OJX_F32)
    transpose_kernel<float><<<grid, 256, 0, s>>>(static_cast<float*>(out),
                                                 static_cast<const float*>(in), rows, cols);
  else
    transpose_kernel<unsigned short><<<grid, 256, 0, s>>>(
        static_cast<unsigned short*>(out), static_cast<const unsigned short*>(in), rows, cols);
  g_launches.fetch_add(1);
  return cuda_status(cudaGetLastError(), "transpose launch");
}

__global__ void __launch_bounds__(256) fill_kernel(void* out, int dtype, float v, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    store_elem(out, i, dtype, v);
}

int launch_fill(void* out, double v, int64_t n, int dtype, cudaStream_t s) {
  if (n <= 0) return OJX_OK;
  fill_kernel<<<grid_for(n), 256, 0, s>>>(out, dtype, static_cast<float>(v), n);
  g_launches.fetch_add(1);
  return cuda_status(cudaGetLastError(), "fill launch");
}

__global__ void __launch_bounds__(256)
    cast_kernel(void* __restrict__ out, int dt_out, const void* __restrict__ in, int dt_in, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    store_elem(out, i, dt_out, load_elem(in, i, dt_in));
}

int launch_cast(void* out, int dt_out, const void* in, int dt_in, int64_t n, cudaStream_t s) {
  if (n <= 0) return OJX_OK;
  cast_kernel<<<grid_for(n), 256, 0, s>>>(out, dt_out, in, dt_in, n);
  g_launches.fetch_add(1);
  return cuda_status(cudaGetLastError(), "cast launch");
}

// ── column sums (bias gradient) ─────────────────────────────────────────────
// out[c] = sum over r of in[r * ld + c] in fp32.  Rows are split into blocks of
// CS_ROWS: pass 1 gives every (block, column) pair one thread that sums its rows in
// ascending order from 0 (8 loads in flight, added in row order), pass 2 adds the
// block sums of a column in ascending block order.  The order is fixed, so the
// result is deterministic; a warp reads 32 consecutive columns of a row per load.
constexpr int CS_ROWS = 64;

template <int DT>
__device__ __forceinline__ float cs_load(const void* p, int64_t i) {
  if (DT == OJX_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  if (DT == OJX_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return static_cast<const float*>(p)[i];
}

template <int DT>
__global__ void __launch_bounds__(256) colsum_block_kernel(const void* __restrict__ in, int64_t rows,
                                                           int64_t cols, int64_t ld,
                                                           float* __restrict__ part) {
  const int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * CS_ROWS;
  const int64_t r1 = min(rows, r0 + CS_ROWS);
  float s = 0.0f;
  int64_t r = r0;
  for (; r + 8 <= r1; r += 8) {
    float x[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] = cs_load<DT>(in, (r + k) * ld + c);
#pragma unroll
    for (int k = 0; k < 8; ++k) s = __fadd_rn(s, x[k]);
  }
  for (; r < r1; ++r) s = __fadd_rn(s, cs_load<DT>(in, r * ld + c));
  part[static_cast<int64_t>(blockIdx.y) * cols + c] = s;
}

// The same sums with 8 consecutive columns per thread and 16-byte loads (used when
// rows and the base are 16-byte aligned and cols % 8 == 0); per column the rows are
// added in exactly the order of colsum_block_kernel, so the results are identical.
template <int DT>
__global__ void __launch_bounds__(256) colsum_block8_kernel(const void* __restrict__ in, int64_t rows,
                                                            int64_t cols, int64_t ld,
                                                            float* __restrict__ part) {
  const int64_t c0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (c0 >= cols) return;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * CS_ROWS;
  const int64_t r1 = min(rows, r0 + CS_ROWS);
  constexpr int ESZ = DT == OJX_F32 ? 4 : 2;
  const char* base = static_cast<const char*>(in) + c0 * ESZ;
  float s[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) s[k] = 0.0f;
  // one row's 8 values (16 or 32 bytes) added to the 8 column sums
  auto add_row = [&](const uint4 (&v)[2]) {
    if (DT == OJX_F32) {
      const float x[8] = {__uint_as_float(v[0].x), __uint_as_float(v[0].y), __uint_as_float(v[0].z),
                          __uint_as_float(v[0].w), __uint_as_float(v[1].x), __uint_as_float(v[1].y),
                          __uint_as_float(v[1].z), __uint_as_float(v[1].w)};
#pragma unroll
      for (int k = 0; k < 8; ++k) s[k] = __fadd_rn(s[k], x[k]);
    } else {
      const uint32_t w[4] = {v[0].x, v[0].y, v[0].z, v[0].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float lo, hi;
        if (DT == OJX_BF16) {
          const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[k]);
          lo = __low2float(h);
          hi = __high2float(h);
        } else {
          const __half2 h = *reinterpret_cast<const __half2*>(&w[k]);
          lo = __low2float(h);
          hi = __high2float(h);
        }
        s[2 * k] = __fadd_rn(s[2 * k], lo);
        s[2 * k + 1] = __fadd_rn(s[2 * k + 1], hi);
      }
    }
  };
  auto load_row = [&](int64_t rr, uint4 (&v)[2]) {
    const uint4* src = reinterpret_cast<const uint4*>(base + rr * ld * ESZ);
    v[0] = __ldg(src);
    v[1] = ESZ == 4 ? __ldg(src + 1) : make_uint4(0, 0, 0, 0);
  };
  int64_t r = r0;
  for (; r + 4 <= r1; r += 4) {  // four rows' loads in flight, added in row order
    uint4 buf[4][2];
#pragma unroll
    for (int q = 0; q < 4; ++q) load_row(r + q, buf[q]);
#pragma unroll
    for (int q = 0; q < 4; ++q) add_row(buf[q]);
  }
  for (; r < r1; ++r) {
    uint4 v[2];
    load_row(r, v);
    add_row(v);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) part[static_cast<int64_t>(blockIdx.y) * cols + c0 + k] = s[k];
}

__global__ void __launch_bounds__(256) colsum_final_kernel(const float* __restrict__ part,
                                                           int64_t n_blocks, int64_t cols,
                                                           void* __restrict__ out, int dt_out) {
  const int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.0f;
  for (int64_t b = 0; b < n_blocks; ++b) s = __fadd_rn(s, part[b * cols + c]);
  store_elem(out, c, dt_out, s);
}

int launch_sum_columns(void* out, int dt_out, const void* in, int dt_in, int64_t rows, int64_t cols,
                       int64_t ld, cudaStream_t s) {
  if (cols <= 0) return OJX_OK;
  const int64_t n_blocks = (rows + CS_ROWS - 1) / CS_ROWS;
  const dim3 grid_c(static_cast<unsigned>((cols + 255) / 256));
  if (n_blocks == 0) return launch_fill(out, 0.0, cols, dt_out, s);
  if (n_blocks > 65535 || grid_c.x > 2147483647u)
    return set_error(OJX_ERR_INVALID, "ojx_sum_columns: %lld rows x %lld columns is too large",
                     static_cast<long long>(rows), static_cast<long long>(cols));
  float* part = static_cast<float*>(
      stream_workspace(s, static_cast<size_t>(n_blocks * cols) * sizeof(float), 3, false));
  if (!part) return workspace_error();
  const int esz = dtype_size(dt_in);
  const bool vec = cols % 8 == 0 && (ld * esz) % 16 == 0 && (reinterpret_cast<uintptr_t>(in) & 15) == 0;
  if (vec) {
    const dim3 grid8(static_cast<unsigned>((cols / 8 + 255) / 256), static_cast<unsigned>(n_blocks));
    switch (dt_in) {
      case OJX_BF16: colsum_block8_kernel<OJX_BF16><<<grid8, 256, 0, s>>>(in, rows, cols, ld, part); break;
      case OJX_F16: colsum_block8_kernel<OJX_F16><<<grid8, 256, 0, s>>>(in, rows, cols, ld, part); break;
      default: colsum_block8_kernel<OJX_F32><<<grid8, 256, 0, s>>>(in, rows, cols, ld, part); break;
    }
  } else {
    const dim3 grid1(grid_c.x, static_cast<unsigned>(n_blocks));
    switch (dt_in) {
      case OJX_BF16: colsum_block_kernel<OJX_BF16><<<grid1, 256, 0, s>>>(in, rows, cols, ld, part); break;
      case OJX_F16: colsum_block_kernel<OJX_F16><<<grid1, 256, 0, s>>>(in, rows, cols, ld, part); break;
      default: colsum_block_kernel<OJX_F32><<<grid1, 256, 0, s>>>(in, rows, cols, ld, part); break;
    }
  }
  g_launches.fetch_add(1);
  if (int st = cuda_status(cudaGetLastError(), "sum_columns launch")) return st;
  colsum_final_kernel<<<grid_c, 256, 0, s>>>(part, n_blocks, cols, out, dt_out);
  g_launches.fetch_add(1);
  return cuda_status(cudaGetLastError(), "sum_columns launch");
}

int read_bounds_info(long long info[4]) {
  return cuda_status(cudaMemcpyFromSymbol(info, g_bounds_info, 4 * sizeof(long long)),
                     "read bounds record");
}

bool debug_bounds_build() { return kDebugBounds; }

int read_and_clear_device_error(unsigned int* word) {
  unsigned int zero = 0;
  int st = cuda_status(cudaMemcpyFromSymbol(word, g_dev_error, sizeof(unsigned int)),
                       "read device error word");
  if (st) return st;
  return cuda_status(cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(unsigned int)),
                     "clear device error word");
}

}  // namespace ojx
