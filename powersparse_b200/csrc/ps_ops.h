// Launchers of the fused operator kernels (ps_ops.cu).
#pragma once

#include <cuda_runtime.h>

#include "ps_matrix.h"

namespace psb {

// C[rows x N] (+)= A * B[cols x N]; N a positive multiple of 32.
void spmm_launch(const Matrix& m, int N, const float* B, float* C, cudaStream_t stream);

// C[rows x N] (+)= A' * B, A' with A's sparsity and the per-call values
// `values[p]` (device, CSR order of the constructor's input) in place of sp_data.
void spmm_values_launch(const Matrix& m, int N, const float* values, const float* B, float* C,
                        cudaStream_t stream);

// spmm_launch whose finished rows are also stored to `n_peers` peer replicas (device
// pointers, possibly on other GPUs, each at this panel's first row): a row is stored
// by the lane group that makes its last add into C, by the wide-row fold, or (rows
// without elements) by a copy kernel.  N is 32, 64 or 128.  The first call at a
// residue cut builds the per-row add counts (allocates, synchronous).
void spmm_push_launch(const Matrix& m, int N, const float* B, float* C, float* const* peers, int n_peers,
                      cudaStream_t stream);

// In place, for every row r: values[p] = softmax over p in [row_ptr[r], row_ptr[r+1])
// (values: device, CSR order, MatrixNNZ() floats).
void edge_softmax_launch(const Matrix& m, float* values, cudaStream_t stream);

// spmm_launch with the wide-row scratch in a fixed device array instead of the
// matrix's cudaMalloc'd buffer; allocates nothing.  Throws std::invalid_argument
// when wide_rows * N exceeds kNoAllocScratchDoubles.  Calls that overlap on the
// GPU share the array and race.
constexpr long long kNoAllocScratchDoubles = 1LL << 21;  // 16 MiB
void spmm_launch_noalloc(const Matrix& m, int N, const float* B, float* C, cudaStream_t stream);
// Resolves the fixed array's address on `device` (the current device).  The first
// resolution loads this library's operator code onto the device, which allocates
// (the array among it); matrices call this when they are created or loaded, so
// spmm_launch_noalloc itself never does.
void noalloc_prepare(int device);

// out[s][e] (+)= A_e * <lhs[row(e)], rhs[col(e)]>; N is 32 or 128.
void sddmm_launch(const Matrix& m, int N, const float* lhs, const float* rhs, float* const* out,
                  cudaStream_t stream);

// out[p] = A_p * <lhs[row(p)], rhs[col(p)]> for every CSR position p of the
// constructor's input (one store per element, no zeroing needed); N is 32 or 128.
void sddmm_csr_launch(const Matrix& m, int N, const float* lhs, const float* rhs, float* out,
                      cudaStream_t stream);

}  // namespace psb
