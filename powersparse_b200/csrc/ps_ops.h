// Launchers of the fused operator kernels (ps_ops.cu).
#pragma once

#include <cuda_runtime.h>

#include "ps_matrix.h"

namespace psb {

// C[rows x N] (+)= A * B[cols x N]; N a positive multiple of 32.
void spmm_launch(const Matrix& m, int N, const float* B, float* C, cudaStream_t stream);

// out[s][e] (+)= A_e * <lhs[row(e)], rhs[col(e)]>; N is 32 or 128.
void sddmm_launch(const Matrix& m, int N, const float* lhs, const float* rhs, float* const* out,
                  cudaStream_t stream);

}  // namespace psb
