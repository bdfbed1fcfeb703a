// attention.cuh — scaled dot-product attention from the batched GEMM and a
// row-softmax kernel (the reference's fused_attention, torchcl/api.py:667-695 and
// flash_attention.cl:8-187, which runs one 256-work-item group per query row).
//
//   S_bh = Q_bh @ K_bh^T              batched tcgen05 GEMM (K read transposed), fp32
//   P_bh = softmax(scale * S_bh)      attn_softmax_kernel (causal mask, reference's
//                                     1e-6 in the denominator), fp32 or 16-bit
//   O_bh = P_bh @ V_bh                batched tcgen05 GEMM, output in the input dtype
//
// S and P live in per-stream workspaces with a row stride padded to 8 elements
// (16-byte rows for the tensor maps).
#include <cuda_runtime.h>
#include "epilogue.cuh"
#include "internal.h"

namespace ojx {

constexpr int ATT_THREADS = 256;

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, w) : __fadd_rn(v, w);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red[] may still be read by the previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = is_max ? -INFINITY : 0.0f;
  for (int w = 0; w < ATT_THREADS / 32; ++w) r = is_max ? fmaxf(r, red[w]) : __fadd_rn(r, red[w]);
  return r;
}

// One block per query row r (problem r / M, query index r % M).  Keys j < nk
// take part (causal: j <= query index); p = exp(s - max) / (sum + 1e-6) with
// s = scale * S; masked keys get p = 0.
template <int DTP>
__global__ void __launch_bounds__(ATT_THREADS) attn_softmax_kernel(const float* __restrict__ S,
                                                                   int64_t ld, int M, int nk,
                                                                   float scale, int causal,
                                                                   void* __restrict__ P) {
  __shared__ float red[ATT_THREADS / 32];
  const int64_t r = blockIdx.x;
  const int qi = static_cast<int>(r % M);
  const int n_valid = causal ? min(nk, qi + 1) : nk;
  const float* s = S + r * ld;
  float mx = -1e20f;  // the reference's initial maximum
  for (int j = threadIdx.x; j < n_valid; j += ATT_THREADS) mx = fmaxf(mx, s[j] * scale);
  mx = block_reduce(mx, true, red);
  float sum = 0.0f;
  for (int j = threadIdx.x; j < n_valid; j += ATT_THREADS) sum = __fadd_rn(sum, expf(s[j] * scale - mx));
  sum = block_reduce(sum, false, red);
  const float inv = __fadd_rn(sum, 1e-6f);
  for (int j = threadIdx.x; j < nk; j += ATT_THREADS) {
    const float p = j < n_valid ? __fdiv_rn(expf(s[j] * scale - mx), inv) : 0.0f;
    store_elem(P, r * ld + j, DTP, p);
  }
}

int launch_attn_softmax(const float* S, int64_t ld, int64_t rows, int M, int nk, float scale,
                        int causal, void* P, int dtype_p, cudaStream_t s) {
  if (rows <= 0) return OJX_OK;
  if (rows > 2147483647LL) return set_error(OJX_ERR_INVALID, "attention: too many query rows");
  const unsigned grid = static_cast<unsigned>(rows);
  switch (dtype_p) {
    case OJX_BF16:
      attn_softmax_kernel<OJX_BF16><<<grid, ATT_THREADS, 0, s>>>(S, ld, M, nk, scale, causal, P);
      break;
    case OJX_F16:
      attn_softmax_kernel<OJX_F16><<<grid, ATT_THREADS, 0, s>>>(S, ld, M, nk, scale, causal, P);
      break;
    default:
      attn_softmax_kernel<OJX_F32><<<grid, ATT_THREADS, 0, s>>>(S, ld, M, nk, scale, causal, P);
      break;
  }
  g_launches.fetch_add(1);
  return cuda_status(cudaGetLastError(), "attention softmax launch");
}

}  // namespace ojx
