// ojx_kernels.cu — the single CUDA translation unit of libojx.  All kernel
// sources are included here so they share one device error word (g_dev_error)
// without relocatable device code.
#include "kernels_simt.cuh"
#include "gemm_tc.cuh"
#include "gemm_skinny.cuh"
