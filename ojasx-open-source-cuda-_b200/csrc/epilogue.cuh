// epilogue.cuh — the fused elementwise epilogue shared by every GEMM kernel and
// by the standalone elementwise kernel.
//
// Semantics follow the OjasX JIT templates (torchcl/jit/compiler.py:33-52):
//   relu    fmax(v, 0)
//   sigmoid 1 / (1 + exp(-v))
//   tanh    tanh(v)
//   neg/abs/exp/log/sqrt/square
//   silu    v / (1 + exp(-v))
//   gelu    v * 0.5 * (1 + tanh(0.7978845608 * (v + 0.044715 * v * v * v)))
// and the binary ops add/sub/mul/div.  Arithmetic is written with explicit
// round-to-nearest intrinsics so that nvcc does not contract it into FMAs: each
// operation rounds once, as the expression reads.  exp/tanh/log/sqrt are CUDA's
// own functions (not the fast-math intrinsics).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "../../include/ojx.h"

namespace ojx {

__device__ __forceinline__ float apply_unary(int op, float v) {
  switch (op) {
    case OJX_UN_RELU: return fmaxf(v, 0.0f);
    case OJX_UN_SIGMOID: return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
    case OJX_UN_TANH: return tanhf(v);
    case OJX_UN_NEG: return -v;
    case OJX_UN_ABS: return fabsf(v);
    case OJX_UN_EXP: return expf(v);
    case OJX_UN_LOG: return logf(v);
    case OJX_UN_SQRT: return __fsqrt_rn(v);
    case OJX_UN_SILU: return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
    case OJX_UN_GELU: {
      const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
      const float inner = __fmul_rn(0.7978845608f, __fadd_rn(v, cube));
      return __fmul_rn(__fmul_rn(v, 0.5f), __fadd_rn(1.0f, tanhf(inner)));
    }
    case OJX_UN_SQUARE: return __fmul_rn(v, v);
    default: return v;
  }
}

__device__ __forceinline__ float apply_binary(int op, float a, float b) {
  switch (op) {
    case OJX_BIN_ADD: return __fadd_rn(a, b);
    case OJX_BIN_SUB: return __fsub_rn(a, b);
    case OJX_BIN_MUL: return __fmul_rn(a, b);
    case OJX_BIN_DIV: return __fdiv_rn(a, b);
    default: return a;
  }
}

__device__ __forceinline__ float load_elem(const void* p, int64_t i, int dtype) {
  switch (dtype) {
    case OJX_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    case OJX_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    default: return reinterpret_cast<const float*>(p)[i];
  }
}

__device__ __forceinline__ void store_elem(void* p, int64_t i, int dtype, float v) {
  switch (dtype) {
    case OJX_BF16: reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    case OJX_F16: reinterpret_cast<__half*>(p)[i] = __float2half_rn(v); break;
    default: reinterpret_cast<float*>(p)[i] = v; break;
  }
}

// Everything a GEMM epilogue needs, passed by value as a kernel parameter.
struct EpiParams {
  void* c;
  int64_t ldc;
  const void* operand;
  int64_t ld_operand;
  int32_t dtype_c;
  int32_t dtype_operand;
  int32_t operand_kind;  // OJX_OPERAND_*
  int32_t binary_op;
  int32_t operand_is_lhs;
  int32_t n_unary;
  int32_t unary[OJX_MAX_UNARY];
};

// Host: copy the epilogue fields of a GEMM descriptor.
EpiParams make_epi(const ojx_gemm_desc& d);

// v = epilogue(acc) for output element (row, col); the caller checks bounds.
__device__ __forceinline__ float epilogue_value(const EpiParams& ep, float acc, int64_t row,
                                                int64_t col) {
  float v = acc;
  if (ep.operand_kind != OJX_OPERAND_NONE) {
    const int64_t idx = ep.operand_kind == OJX_OPERAND_ROW ? col : row * ep.ld_operand + col;
    const float x = load_elem(ep.operand, idx, ep.dtype_operand);
    v = ep.operand_is_lhs ? apply_binary(ep.binary_op, x, v) : apply_binary(ep.binary_op, v, x);
  }
  for (int i = 0; i < ep.n_unary; ++i) v = apply_unary(ep.unary[i], v);
  return v;
}

}  // namespace ojx
