// PowerSparse C++ API: SDDMM.  Drop-in for PowerSparse_SDDMM/PowerSparse_SDDMM.h of
// ParCIS/PowerSparse (same declaration and contract).
#ifndef POWERSPARSE_SDDMM_H
#define POWERSPARSE_SDDMM_H

#include "../utils/matrix_utils.h"

namespace PowerSparse {

// FP32 sampled (lhs * rhs^T) times sparse values; N is 32 or 128.
// Dense inputs are row-major. Output is in workset order, not original CSR order.
// Zero every output workset before each independent call. Streams follow SpMM.
void SDDMM(const PowerSparseMatrixGPU& ps_matrix_gpu, int N, const float* lhs_gpu, const float* rhs_gpu,
           float** sddmm_output_gpu, int ps_stream_num, const cudaStream_t* ps_stream);

}  // namespace PowerSparse

#endif  // POWERSPARSE_SDDMM_H
