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
#include "sm100.cuh"

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

// Everything a GEMM epilogue needs, passed by value as a kernel parameter.  The
// unary chain is packed 4 bits per op (op i in bits 4i..4i+3) so that reading it
// never goes through local memory.
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
  uint32_t unary_packed;
  // Output destinations: dst[0..n_dst) all receive the same values at
  // (row * ldc + col_offset + col).  One destination (c, offset 0) for a plain
  // GEMM; every rank's C buffer for an all-gathering sharded GEMM.
  int32_t n_dst;
  int64_t col_offset;
  void* dst[OJX_MAX_PEERS];
  // Logical output extent [m_rows, n_cols] (stores land at row < m_rows, col <
  // n_cols); read only by the debug build's bounds checks.
  int64_t m_rows;
  int64_t n_cols;
};

// Debug build: a store of n values at (row, col .. col+n-1) lies inside the output.
__device__ __forceinline__ bool epi_store_ok(const EpiParams& ep, int site, int64_t row,
                                             int64_t col, int n) {
  if (!kDebugBounds) return true;
  const bool ok = row >= 0 && col >= 0 && row < ep.m_rows && col + n <= ep.n_cols;
  return bounds_check(ok, site, row, col, row < ep.m_rows ? ep.n_cols : ep.m_rows);
}

struct Dests;
// Host: copy the epilogue fields of a GEMM descriptor (and the destinations of an
// all-gathering GEMM, when given).
EpiParams make_epi(const ojx_gemm_desc& d, const Dests* dests = nullptr);

__device__ __forceinline__ int unary_at(uint32_t packed, int i) {
  return static_cast<int>((packed >> (4 * i)) & 15u);
}

// v = epilogue(acc) for one output element (row, col); the caller checks bounds.
__device__ __forceinline__ float epilogue_value(const EpiParams& ep, float acc, int64_t row,
                                                int64_t col) {
  float v = acc;
  if (ep.operand_kind != OJX_OPERAND_NONE) {
    const int64_t idx = ep.operand_kind == OJX_OPERAND_ROW ? col : row * ep.ld_operand + col;
    const float x = load_elem(ep.operand, idx, ep.dtype_operand);
    v = ep.operand_is_lhs ? apply_binary(ep.binary_op, x, v) : apply_binary(ep.binary_op, v, x);
  }
  for (int i = 0; i < ep.n_unary; ++i) v = apply_unary(unary_at(ep.unary_packed, i), v);
  return v;
}

// ── 8-wide row pieces with 16-byte accesses ────────────────────────────────

// x[0..7] = p[i0 .. i0+7]; only the first `valid` are read (the rest are 0).
// 16-byte vector loads when the whole piece is inside and aligned.
__device__ __forceinline__ void load8(const void* p, int dtype, int64_t i0, int valid,
                                      float (&x)[8]) {
  const int esz = dtype == OJX_F32 ? 4 : 2;
  const char* src = static_cast<const char*>(p) + i0 * esz;
  if (valid >= 8 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    if (dtype == OJX_F32) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(src));
      const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
      x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
      x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (dtype == OJX_BF16) {
          const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[k]);
          x[2 * k] = __low2float(h);
          x[2 * k + 1] = __high2float(h);
        } else {
          const __half2 h = *reinterpret_cast<const __half2*>(&w[k]);
          x[2 * k] = __low2float(h);
          x[2 * k + 1] = __high2float(h);
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = j < valid ? load_elem(p, i0 + j, dtype) : 0.0f;
  }
}

// p[i0 .. i0+7] = v (only the first `valid`): one 16-byte store for 16-bit
// types (two for fp32) when the whole piece is inside and aligned.
__device__ __forceinline__ void store8(void* p, int dtype, int64_t i0, int valid,
                                       const float (&v)[8]) {
  const int esz = dtype == OJX_F32 ? 4 : 2;
  char* dst = static_cast<char*>(p) + i0 * esz;
  if (valid >= 8 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    if (dtype == OJX_F32) {
      reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (dtype == OJX_BF16) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
          w[k] = *reinterpret_cast<const uint32_t*>(&h);
        } else {
          const __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
          w[k] = *reinterpret_cast<const uint32_t*>(&h);
        }
      }
      *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < valid) store_elem(p, i0 + j, dtype, v[j]);
  }
}

// ── 16-wide variants: one dispatch per 16 consecutive columns of a row ─────────

// x[0..15] = p[i0 .. i0+15] (only the first `valid` when the row ends early).
__device__ __forceinline__ void load16(const void* p, int dtype, int64_t i0, int valid,
                                       float (&x)[16]) {
  const int esz = dtype == OJX_F32 ? 4 : 2;
  const char* src = static_cast<const char*>(p) + i0 * esz;
  if (valid == 16 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    if (dtype == OJX_F32) {
      const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 f = __ldg(s4 + j);
        x[4 * j] = f.x; x[4 * j + 1] = f.y; x[4 * j + 2] = f.z; x[4 * j + 3] = f.w;
      }
    } else {
      const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint4 u = __ldg(s4 + j);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (dtype == OJX_BF16) {
            const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[k]);
            x[8 * j + 2 * k] = __low2float(h);
            x[8 * j + 2 * k + 1] = __high2float(h);
          } else {
            const __half2 h = *reinterpret_cast<const __half2*>(&w[k]);
            x[8 * j + 2 * k] = __low2float(h);
            x[8 * j + 2 * k + 1] = __high2float(h);
          }
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = j < valid ? load_elem(p, i0 + j, dtype) : 0.0f;
  }
}

// v[j] = op(v[j]) for N values: one dispatch for the whole vector.
template <int N>
__device__ __forceinline__ void unary_n(int op, float (&v)[N]) {
#define OJX_UN(EXPR)                                          \
  _Pragma("unroll") for (int j = 0; j < N; ++j) {             \
    const float x = v[j];                                     \
    v[j] = (EXPR);                                            \
  }                                                           \
  break;
  switch (op) {
    case OJX_UN_RELU: OJX_UN(fmaxf(x, 0.0f))
    case OJX_UN_SIGMOID: OJX_UN(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))))
    case OJX_UN_TANH: OJX_UN(tanhf(x))
    case OJX_UN_NEG: OJX_UN(-x)
    case OJX_UN_ABS: OJX_UN(fabsf(x))
    case OJX_UN_EXP: OJX_UN(expf(x))
    case OJX_UN_LOG: OJX_UN(logf(x))
    case OJX_UN_SQRT: OJX_UN(__fsqrt_rn(x))
    case OJX_UN_SILU: OJX_UN(__fdiv_rn(x, __fadd_rn(1.0f, expf(-x))))
    case OJX_UN_GELU: OJX_UN(apply_unary(OJX_UN_GELU, x))
    case OJX_UN_SQUARE: OJX_UN(__fmul_rn(x, x))
    default: break;
  }
#undef OJX_UN
}

__device__ __forceinline__ void unary16(int op, float (&v)[16]) { unary_n<16>(op, v); }

// unary_n for results that are rounded to bf16/fp16 afterwards: the logistic
// ops divide with __fdividef and exponentiate with __expf (errors of a few fp32
// ulp, far below 16-bit precision) instead of the correctly rounded division,
// which costs several hundred cycles per value.  Every other op is unary_n's.
template <int N>
__device__ __forceinline__ void unary_n_half(int op, float (&v)[N]) {
  if (op == OJX_UN_SILU) {
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = __fdividef(v[j], 1.0f + __expf(-v[j]));
  } else if (op == OJX_UN_SIGMOID) {
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = __fdividef(1.0f, 1.0f + __expf(-v[j]));
  } else {
    unary_n<N>(op, v);
  }
}

// v[j] = v[j] op x[j] (x[j] op v[j] when lhs) for N values.
template <int N>
__device__ __forceinline__ void binary_n(int op, bool lhs, float (&v)[N], const float (&x)[N]) {
#define OJX_BN(EXPR)                                          \
  _Pragma("unroll") for (int j = 0; j < N; ++j) {             \
    const float a = lhs ? x[j] : v[j], b = lhs ? v[j] : x[j]; \
    v[j] = (EXPR);                                            \
  }                                                           \
  break;
  switch (op) {
    case OJX_BIN_ADD: OJX_BN(__fadd_rn(a, b))
    case OJX_BIN_SUB: OJX_BN(__fsub_rn(a, b))
    case OJX_BIN_MUL: OJX_BN(__fmul_rn(a, b))
    case OJX_BIN_DIV: OJX_BN(__fdiv_rn(a, b))
    default: break;
  }
#undef OJX_BN
}

__device__ __forceinline__ void binary16(int op, bool lhs, float (&v)[16], const float (&x)[16]) {
  binary_n<16>(op, lhs, v, x);
}

// Epilogue of 16 consecutive columns col0.. of one row (valid = columns < N).
__device__ __forceinline__ void epilogue16(const EpiParams& ep, float (&v)[16], int64_t row,
                                           int64_t col0, int valid) {
  if (ep.operand_kind != OJX_OPERAND_NONE) {
    float x[16];
    const int64_t i0 = ep.operand_kind == OJX_OPERAND_ROW ? col0 : row * ep.ld_operand + col0;
    load16(ep.operand, ep.dtype_operand, i0, valid, x);
    binary16(ep.binary_op, ep.operand_is_lhs != 0, v, x);
  }
  for (int i = 0; i < ep.n_unary; ++i) unary16(unary_at(ep.unary_packed, i), v);
}

}  // namespace ojx
