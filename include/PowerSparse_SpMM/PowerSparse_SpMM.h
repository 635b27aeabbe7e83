// PowerSparse C++ API: SpMM.  Drop-in for PowerSparse_SpMM/PowerSparse_SpMM.h of
// ParCIS/PowerSparse (same declaration and contract).
#ifndef POWERSPARSE_SPMM_H
#define POWERSPARSE_SPMM_H

#include "../utils/matrix_utils.h"

namespace PowerSparse {

// FP32 C = A * B, with row-major B and C. Zero C before each independent call.
// Supply GroupTypeNum() blocking streams (nullptr is allowed for a single workset).
// Multiple worksets synchronize the device; a single workset uses the default stream.
// One fused kernel covers every workset; it starts after the work already queued
// on all the given streams.
void SpMM(const PowerSparseMatrixGPU& ps_matrix_gpu, int N, const float* B_gpu, float* C_gpu,
          int ps_stream_num, const cudaStream_t* ps_stream);

}  // namespace PowerSparse

#endif  // POWERSPARSE_SPMM_H
