// ref_kernels.cpp — builds the OjasX reference's own OpenCL C kernels
// (torchcl/kernels/matmul.cl, activation.cl, elementwise.cl, precision.cl,
// reduction.cl, winograd_gemm.cl and flash_attention.cl, read from the reference tree at build time; the paths are passed
// as -D macros by oracle/build_oracle.py) for the host through clshim.h, and launches each with the
// NDRange geometry torchcl/ops/engine.py gives it.
// TEST INFRASTRUCTURE ONLY: output goes to oracle/_ref/ and is used to pin the
// oracle restatement (ojx_oracle.cpp); nothing of the reference is copied here.
#include <cstring>
#include "fiber.h"

namespace cl_matmul {
#include REF_MATMUL_CL
}
namespace cl_activation {
#include REF_ACTIVATION_CL
}
namespace cl_elementwise {
#include REF_ELEMENTWISE_CL
}
namespace cl_precision {
#include REF_PRECISION_CL
}
// reduction.cl takes __local pointers as kernel arguments, which the shim's
// per-thread-static __local cannot express; inside this namespace __local is
// empty.  Only sum_columns_f32 (no local memory) is launched from here.
#undef __local
#define __local
namespace cl_reduction {
#include REF_REDUCTION_CL
}
#undef __local
#define __local static thread_local
namespace cl_winograd {
#include REF_WINOGRAD_GEMM_CL
}
namespace cl_attention {
#include REF_FLASH_ATTENTION_CL
}

namespace {
size_t up(size_t n, size_t m) { return (n + m - 1) / m * m; }
void run2(size_t g0, size_t g1, size_t l0, size_t l1, const std::function<void()>& f) {
  const size_t g[2] = {g0, g1}, l[2] = {l0, l1};
  clshim::run_ndrange(g, l, f);
}
// engine.py _compute_global_size(n) with the 256 work-group of the 1-D launchers.
void run1(size_t n, const std::function<void()>& f) { run2(up(n ? n : 1, 256), 1, 256, 1, f); }
}  // namespace

extern "C" {

// engine.py:166-171 (reg-tiled: (ceil(N/64)*16, ceil(M/64)*16) x (16,16))
int ref_matmul_reg_tiled_f32(const float* A, const float* B, float* C, int M, int N, int K) {
  run2(size_t((N + 63) / 64) * 16, size_t((M + 63) / 64) * 16, 16, 16,
       [&] { cl_matmul::matmul_reg_tiled_f32(A, B, C, M, N, K); });
  return 0;
}
// engine.py:197-202
int ref_matmul_reg_tiled_bias_f32(const float* A, const float* B, const float* bias, float* C, int M,
                                  int N, int K) {
  run2(size_t((N + 63) / 64) * 16, size_t((M + 63) / 64) * 16, 16, 16,
       [&] { cl_matmul::matmul_reg_tiled_bias_f32(A, B, bias, C, M, N, K); });
  return 0;
}
// engine.py:173-179 ((ceil16(M), ceil16(N)) x (16,16))
int ref_matmul_naive_f32(const float* A, const float* B, float* C, int M, int N, int K) {
  run2(up(M, 16), up(N, 16), 16, 16, [&] { cl_matmul::matmul_naive_f32(A, B, C, M, N, K); });
  return 0;
}
// engine.py:204-209
int ref_matmul_bias_f32(const float* A, const float* B, const float* bias, float* C, int M, int N,
                        int K) {
  run2(up(M, 16), up(N, 16), 16, 16, [&] { cl_matmul::matmul_bias_f32(A, B, bias, C, M, N, K); });
  return 0;
}
// matmul.cl:227-268 with TILE_SIZE 16
int ref_matmul_tiled_f32(const float* A, const float* B, float* C, int M, int N, int K) {
  run2(up(M, 16), up(N, 16), 16, 16, [&] { cl_matmul::matmul_tiled_f32(A, B, C, M, N, K); });
  return 0;
}
// engine.py:365-378 (TILE_SIZE 16)
int ref_linear_forward_tiled_f32(const float* A, const float* B, const float* bias, float* C, int M,
                                 int N, int K, int has_bias) {
  run2(up(M, 16), up(N, 16), 16, 16,
       [&] { cl_matmul::linear_forward_tiled_f32(A, B, bias, C, M, N, K, has_bias); });
  return 0;
}
// engine.py:332-349
int ref_transpose_f32(const float* A, float* B, int M, int N) {
  run2(up(M, 16), up(N, 16), 16, 16, [&] { cl_matmul::transpose_f32(A, B, M, N); });
  return 0;
}
// engine.py:228-244 (TILE_SIZE 16); operands and result are IEEE half bit patterns
int ref_matmul_tiled_fp16(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K) {
  const half* a = reinterpret_cast<const half*>(A);
  const half* b = reinterpret_cast<const half*>(B);
  half* c = reinterpret_cast<half*>(C);
  run2(up(M, 16), up(N, 16), 16, 16, [&] { cl_matmul::matmul_tiled_fp16(a, b, c, M, N, K); });
  return 0;
}

// activation.cl unary kernels by name: relu, sigmoid, tanh, gelu, silu.
int ref_activation(const char* name, const float* a, float* c, int n) {
  if (!std::strcmp(name, "relu")) run1(n, [&] { cl_activation::relu_f32(a, c, n); });
  else if (!std::strcmp(name, "sigmoid")) run1(n, [&] { cl_activation::sigmoid_f32(a, c, n); });
  else if (!std::strcmp(name, "tanh")) run1(n, [&] { cl_activation::tanh_f32(a, c, n); });
  else if (!std::strcmp(name, "gelu")) run1(n, [&] { cl_activation::gelu_f32(a, c, n); });
  else if (!std::strcmp(name, "silu")) run1(n, [&] { cl_activation::silu_f32(a, c, n); });
  else return 1;
  return 0;
}
// elementwise.cl binary kernels by name: add, sub, mul, div.
int ref_binary(const char* name, const float* a, const float* b, float* c, int n) {
  if (!std::strcmp(name, "add")) run1(n, [&] { cl_elementwise::add_f32(a, b, c, n); });
  else if (!std::strcmp(name, "sub")) run1(n, [&] { cl_elementwise::sub_f32(a, b, c, n); });
  else if (!std::strcmp(name, "mul")) run1(n, [&] { cl_elementwise::mul_f32(a, b, c, n); });
  else if (!std::strcmp(name, "div")) run1(n, [&] { cl_elementwise::div_f32(a, b, c, n); });
  else return 1;
  return 0;
}
// elementwise.cl unary kernels by name: neg, abs, exp, log, sqrt.
int ref_unary(const char* name, const float* a, float* c, int n) {
  if (!std::strcmp(name, "neg")) run1(n, [&] { cl_elementwise::neg_f32(a, c, n); });
  else if (!std::strcmp(name, "abs")) run1(n, [&] { cl_elementwise::abs_f32(a, c, n); });
  else if (!std::strcmp(name, "exp")) run1(n, [&] { cl_elementwise::exp_f32(a, c, n); });
  else if (!std::strcmp(name, "log")) run1(n, [&] { cl_elementwise::log_f32(a, c, n); });
  else if (!std::strcmp(name, "sqrt")) run1(n, [&] { cl_elementwise::sqrt_f32(a, c, n); });
  else return 1;
  return 0;
}
// reduction.cl:170-181 sum_columns_f32 over cols rounded up to 256 work-items
// (engine.py:807-822); the kernel uses no local memory, so the group size does
// not change its result.
int ref_sum_columns_f32(const float* in, float* out, int rows, int cols) {
  run1(size_t(cols), [&] { cl_reduction::sum_columns_f32(in, out, rows, cols); });
  return 0;
}
// winograd_gemm.cl:91-119 matmul_batched_strided_f32 with blas.bmm's geometry
// (global (N, M, B), local chosen by the runtime: one work-item per group here).
int ref_matmul_batched_strided_f32(const float* A, const float* B, float* C, int batch, int M,
                                   int N, int K) {
  const size_t g[3] = {size_t(N), size_t(M), size_t(batch)}, l[3] = {1, 1, 1};
  clshim::run_ndrange3(g, l, [&] {
    cl_winograd::matmul_batched_strided_f32(A, B, C, batch, M, N, K, M * K, K * N, M * N);
  });
  return 0;
}
// flash_attention.cl:8-187 with engine.py:755-773's geometry: one group of 256
// work-items per query row.
int ref_flash_attention_f32(const float* Q, const float* K, const float* V, float* O, int B, int H,
                            int M, int N, int D, float scale, int causal) {
  run2(size_t(B) * H * M * 256, 1, 256, 1, [&] {
    if (causal)
      cl_attention::flash_attention_causal_f32(Q, K, V, O, B, H, M, N, D, scale);
    else
      cl_attention::flash_attention_f32(Q, K, V, O, B, H, M, N, D, scale);
  });
  return 0;
}
// precision.cl
int ref_pack_fp32_to_fp16(const float* in, uint16_t* out, int n) {
  half* o = reinterpret_cast<half*>(out);
  run1(n, [&] { cl_precision::pack_fp32_to_fp16(in, o, n); });
  return 0;
}
int ref_unpack_fp16_to_fp32(const uint16_t* in, float* out, int n) {
  const half* i = reinterpret_cast<const half*>(in);
  run1(n, [&] { cl_precision::unpack_fp16_to_fp32(i, out, n); });
  return 0;
}

}  // extern "C"
