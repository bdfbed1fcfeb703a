// ojx_oracle.cpp — CPU restatement of the OjasX GEMM + fused-epilogue path.
//
// TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's
// CPU-baseline leg load this library, and only as the checker / the timed CPU
// baseline.  The product path (libojx.so) never calls it.
//
// What it restates (paths inside the OjasX project):
//  * torchcl/kernels/matmul.cl:19-120  matmul_reg_tiled_f32, :123-224 (+bias),
//    :227-268 matmul_tiled_f32, :297-343 linear_forward_tiled_f32,
//    :346-385 naive/bias, :422-463 matmul_tiled_fp16.  Every one of them computes,
//    per output element, `sum = 0; for k ascending: sum += A[m,k] * B[k,n]` in fp32
//    (tiles only change which work-item loads what; zero-padded tail tiles add
//    0 * 0).  The fp16 kernels convert operands to float first and round the
//    result to half once.  The bias kernels add bias[col] after the sum
//    (matmul.cl:218-219).
//  * torchcl/jit/compiler.py:33-52 (op strings) and :137-196 (kernel templates):
//    out = u_n(...u_1(a op b)) in fp32 with libm exp/tanh/log/sqrt.
//  * reduction.cl:170-181 sum_columns_f32 (oracle_sum_columns) and
//    flash_attention.cl:8-187 (oracle_attention), see each function.
// OpenCL leaves FMA contraction of `sum += a*b` to the implementation, so the
// GEMM comes in two variants: fused == 0 rounds the product and the sum
// separately (this file is compiled with -ffp-contract=off), fused == 1 uses one
// fma per step.  bf16 is an extension (the reference has no bf16 route): bf16
// operands are widened to fp32 and the same loop runs.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#include <omp.h>

namespace {

enum { F32 = 0, BF16 = 1, F16 = 2 };
enum { UN_RELU = 1, UN_SIGMOID, UN_TANH, UN_NEG, UN_ABS, UN_EXP, UN_LOG, UN_SQRT, UN_SILU, UN_GELU, UN_SQUARE };
enum { BIN_ADD = 1, BIN_SUB, BIN_MUL, BIN_DIV };
enum { OPND_NONE = 0, OPND_ROW = 1, OPND_FULL = 2 };

inline float bf16_to_f32(uint16_t h) {
  uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline uint16_t f32_to_bf16(float f) {  // round to nearest even, NaN kept quiet
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}
inline float f16_to_f32(uint16_t h) {
  _Float16 x;
  std::memcpy(&x, &h, 2);
  return static_cast<float>(x);
}
inline uint16_t f32_to_f16(float f) {
  _Float16 x = static_cast<_Float16>(f);
  uint16_t h;
  std::memcpy(&h, &x, 2);
  return h;
}
inline float load(const void* p, int64_t i, int dt) {
  switch (dt) {
    case BF16: return bf16_to_f32(static_cast<const uint16_t*>(p)[i]);
    case F16: return f16_to_f32(static_cast<const uint16_t*>(p)[i]);
    default: return static_cast<const float*>(p)[i];
  }
}
inline void store(void* p, int64_t i, int dt, float v) {
  switch (dt) {
    case BF16: static_cast<uint16_t*>(p)[i] = f32_to_bf16(v); break;
    case F16: static_cast<uint16_t*>(p)[i] = f32_to_f16(v); break;
    default: static_cast<float*>(p)[i] = v; break;
  }
}

// torchcl/jit/compiler.py:33-45, evaluated as written (one rounding per operation).
inline float unary(int op, float x) {
  switch (op) {
    case UN_RELU: return std::fmax(x, 0.0f);
    case UN_SIGMOID: return (1.0f / (1.0f + std::exp(-(x))));
    case UN_TANH: return std::tanh(x);
    case UN_NEG: return (-(x));
    case UN_ABS: return std::fabs(x);
    case UN_EXP: return std::exp(x);
    case UN_LOG: return std::log(x);
    case UN_SQRT: return std::sqrt(x);
    case UN_SILU: return ((x) / (1.0f + std::exp(-(x))));
    case UN_GELU:
      return ((x) * 0.5f * (1.0f + std::tanh(0.7978845608f * ((x) + 0.044715f * (x) * (x) * (x)))));
    case UN_SQUARE: return ((x) * (x));
    default: return x;
  }
}
// torchcl/jit/compiler.py:47-52
inline float binary(int op, float a, float b) {
  switch (op) {
    case BIN_ADD: return (a + b);
    case BIN_SUB: return (a - b);
    case BIN_MUL: return (a * b);
    case BIN_DIV: return (a / b);
    default: return a;
  }
}

struct Epi {
  const void* operand;
  int kind, dtype, binop, lhs;
  int64_t ld;
  const int* un;
  int n_un;
  float apply(float acc, int64_t row, int64_t col) const {
    float v = acc;
    if (kind != OPND_NONE) {
      const float x = load(operand, kind == OPND_ROW ? col : row * ld + col, dtype);
      v = lhs ? binary(binop, x, v) : binary(binop, v, x);
    }
    for (int i = 0; i < n_un; ++i) v = unary(un[i], v);
    return v;
  }
};

// Per output row: acc[n] accumulates A[m,k]*B[k,n] for k = 0, 1, ..., K-1, each
// column independently (the i-k-j loop keeps every element's own k order).
template <bool FUSED>
void gemm_row(const float* arow, const float* Bf, int64_t K, int64_t N, float* acc) {
  for (int64_t n = 0; n < N; ++n) acc[n] = 0.0f;
  for (int64_t k = 0; k < K; ++k) {
    const float a = arow[k];
    const float* brow = Bf + k * N;
    if (FUSED) {
      for (int64_t n = 0; n < N; ++n) acc[n] = __builtin_fmaf(a, brow[n], acc[n]);
    } else {
      for (int64_t n = 0; n < N; ++n) acc[n] = acc[n] + a * brow[n];
    }
  }
}

}  // namespace

extern "C" {

int oracle_version(void) { return 1; }

// C = epilogue(op(A) op(B)); see the header comment.  rows/n_rows (optional)
// restrict the computation to the listed output rows (the other rows of C are
// left untouched).  threads <= 0 uses every OpenMP thread.
int oracle_gemm(int64_t M, int64_t N, int64_t K, int dtype_a, int dtype_b, int dtype_c, int trans_a,
                int trans_b, const void* a, int64_t lda, const void* b, int64_t ldb, void* c,
                int64_t ldc, const void* operand, int operand_kind, int operand_dtype,
                int64_t ld_operand, int binary_op, int operand_is_lhs, const int* un, int n_un,
                int fused, int threads, const int64_t* rows, int64_t n_rows) {
  if (M < 0 || N < 0 || K < 0) return 1;
  if (lda == 0) lda = trans_a ? M : K;
  if (ldb == 0) ldb = trans_b ? K : N;
  if (ldc == 0) ldc = N;
  if (ld_operand == 0) ld_operand = N;
  // Widen B once to a dense fp32 [K, N] (row-major, k-major rows).
  std::vector<float> Bf(static_cast<size_t>(K) * N);
  for (int64_t k = 0; k < K; ++k)
    for (int64_t n = 0; n < N; ++n)
      Bf[k * N + n] = load(b, trans_b ? n * ldb + k : k * ldb + n, dtype_b);
  const Epi ep{operand, operand_kind, operand_dtype, binary_op, operand_is_lhs, ld_operand, un, n_un};
  const int64_t R = rows ? n_rows : M;
  const int nt = threads > 0 ? threads : omp_get_max_threads();
#pragma omp parallel num_threads(nt)
  {
    std::vector<float> arow(K), acc(N);
#pragma omp for schedule(dynamic, 1)
    for (int64_t r = 0; r < R; ++r) {
      const int64_t m = rows ? rows[r] : r;
      for (int64_t k = 0; k < K; ++k) arow[k] = load(a, trans_a ? k * lda + m : m * lda + k, dtype_a);
      if (fused)
        gemm_row<true>(arow.data(), Bf.data(), K, N, acc.data());
      else
        gemm_row<false>(arow.data(), Bf.data(), K, N, acc.data());
      for (int64_t n = 0; n < N; ++n) store(c, m * ldc + n, dtype_c, ep.apply(acc[n], m, n));
    }
  }
  return 0;
}

// Same computation for the listed output columns only: out[m, j] for j < n_cols
// (out is [M, n_cols] row-major).  Each element is one ascending-k dot product.
int oracle_gemm_cols(int64_t M, int64_t N, int64_t K, int dtype_a, int dtype_b, int dtype_c,
                     int trans_a, int trans_b, const void* a, int64_t lda, const void* b,
                     int64_t ldb, void* out, const void* operand, int operand_kind,
                     int operand_dtype, int64_t ld_operand, int binary_op, int operand_is_lhs,
                     const int* un, int n_un, int fused, int threads, const int64_t* cols,
                     int64_t n_cols) {
  if (M < 0 || N < 0 || K < 0) return 1;
  if (lda == 0) lda = trans_a ? M : K;
  if (ldb == 0) ldb = trans_b ? K : N;
  if (ld_operand == 0) ld_operand = N;
  const Epi ep{operand, operand_kind, operand_dtype, binary_op, operand_is_lhs, ld_operand, un, n_un};
  const int nt = threads > 0 ? threads : omp_get_max_threads();
  std::vector<float> Bc(static_cast<size_t>(n_cols) * K);
  for (int64_t j = 0; j < n_cols; ++j)
    for (int64_t k = 0; k < K; ++k)
      Bc[j * K + k] = load(b, trans_b ? cols[j] * ldb + k : k * ldb + cols[j], dtype_b);
#pragma omp parallel num_threads(nt)
  {
    std::vector<float> arow(K);
#pragma omp for schedule(dynamic, 4)
    for (int64_t m = 0; m < M; ++m) {
      for (int64_t k = 0; k < K; ++k) arow[k] = load(a, trans_a ? k * lda + m : m * lda + k, dtype_a);
      for (int64_t j = 0; j < n_cols; ++j) {
        const float* bc = Bc.data() + j * K;
        float s = 0.0f;
        if (fused)
          for (int64_t k = 0; k < K; ++k) s = __builtin_fmaf(arow[k], bc[k], s);
        else
          for (int64_t k = 0; k < K; ++k) s = s + arow[k] * bc[k];
        store(out, m * n_cols + j, dtype_c, ep.apply(s, m, cols[j]));
      }
    }
  }
  return 0;
}

// out[i] = u_n(...u_1(a[i] op b[i])) (b == NULL: unary chain only);
// torchcl/jit/compiler.py:64-133 and the generated kernels at :150-196.
int oracle_elementwise(void* out, int dt_out, const void* a, int dt_a, const void* b, int dt_b,
                       int binary_op, const int* un, int n_un, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float v = load(a, i, dt_a);
    if (b) v = binary(binary_op, v, load(b, i, dt_b));
    for (int k = 0; k < n_un; ++k) v = unary(un[k], v);
    store(out, i, dt_out, v);
  }
  return 0;
}

// dtype conversion with the rounding the GPU path uses (RNE).
int oracle_cast(void* out, int dt_out, const void* in, int dt_in, int64_t n) {
  for (int64_t i = 0; i < n; ++i) store(out, i, dt_out, load(in, i, dt_in));
  return 0;
}

// out[c] = sum of in[r * ld + c] over r, in fp32 (the bias gradient: column sums).
// block == 0: reduction.cl:170-181 sum_columns_f32 exactly (one accumulator from
// 0.0f, rows in ascending order).  block > 0: the order of the GPU kernel (rows in
// blocks of `block`, each block summed in ascending order from 0.0f, then the
// block sums added in ascending order from 0.0f).
int oracle_sum_columns(float* out, const void* in, int dt_in, int64_t rows, int64_t cols,
                       int64_t ld, int64_t block) {
  for (int64_t c = 0; c < cols; ++c) {
    if (block <= 0) {
      float s = 0.0f;
      for (int64_t r = 0; r < rows; ++r) s = s + load(in, r * ld + c, dt_in);
      out[c] = s;
      continue;
    }
    float total = 0.0f;
    for (int64_t r0 = 0; r0 < rows; r0 += block) {
      float s = 0.0f;
      const int64_t r1 = r0 + block < rows ? r0 + block : rows;
      for (int64_t r = r0; r < r1; ++r) s = s + load(in, r * ld + c, dt_in);
      total = total + s;
    }
    out[c] = total;
  }
  return 0;
}

// Attention, as torchcl/kernels/flash_attention.cl:8-97 (flash_attention_f32) and
// :100-187 (flash_attention_causal_f32) compute it, launched by engine.py:755-773
// with one 256-work-item group per query row.  Per row: score[j] = (sum over k
// ascending of q[k]*k_j[k]) * scale; (causal: only j <= row index within M; other
// scores count as masked); max over the scores; e[j] = exp(score[j] - max); the
// group sums e in two steps (work-item t adds e[t], e[t+256], ... in order, then
// work-item 0 adds the 256 partial sums in order); p[j] = e[j] / (sum + 1e-6);
// out[d] = sum over j ascending of p[j] * v_j[d].  Only keys j < 2048 take part
// (the reference's score buffer holds 2048 entries, flash_attention.cl:6).
// Q, K, V, out: [B*H][rows][D] fp32 (or 16-bit patterns, widened first).
// max_keys <= 0 keeps every key instead of the reference's 2048.
int oracle_attention(float* out, const void* q, const void* k, const void* v, int dt,
                     int64_t BH, int64_t M, int64_t N, int64_t D, float scale, int causal,
                     int64_t max_keys) {
  const int64_t NK = max_keys > 0 && N > max_keys ? max_keys : N;
#pragma omp parallel for schedule(static)
  for (int64_t row = 0; row < BH * M; ++row) {
    const int64_t bh = row / M, qi = row % M;
    const int64_t nk = causal ? (qi + 1 < NK ? qi + 1 : NK) : NK;
    std::vector<float> sc(static_cast<size_t>(nk));
    for (int64_t j = 0; j < nk; ++j) {
      float acc = 0.0f;
      for (int64_t d = 0; d < D; ++d)
        acc = acc + load(q, row * D + d, dt) * load(k, (bh * N + j) * D + d, dt);
      sc[j] = acc * scale;
    }
    float mx = -1e20f;
    for (int64_t j = 0; j < nk; ++j) mx = sc[j] > mx ? sc[j] : mx;
    float part[256] = {0.0f};
    for (int64_t j = 0; j < nk; ++j) {
      sc[j] = std::exp(sc[j] - mx);
      part[j % 256] = part[j % 256] + sc[j];
    }
    float sum = 0.0f;
    for (int t = 0; t < 256; ++t) sum = sum + part[t];
    for (int64_t j = 0; j < nk; ++j) sc[j] = sc[j] / (sum + 1e-6f);
    for (int64_t d = 0; d < D; ++d) {
      float acc = 0.0f;
      for (int64_t j = 0; j < nk; ++j) acc = acc + sc[j] * load(v, (bh * N + j) * D + d, dt);
      out[row * D + d] = acc;
    }
  }
  return 0;
}

}  // extern "C"
