// PowerSparse C++ operator API over the C ABI (libpowersparse.so).
//
// PowerSparseMatrixGPU (utils/matrix_utils.cu:470-663 of the reference), SpMM
// (PowerSparse_SpMM/spmm_solution.cu:7-34) and SDDMM
// (PowerSparse_SDDMM/sddmm_solution.cu:7-50): same argument checks, messages,
// exception types, stream contract and synchronization.  The kernels behind
// them are the fused B200 kernels of libpowersparse_b200.so.
#include "PowerSparse_SDDMM/PowerSparse_SDDMM.h"
#include "PowerSparse_SpMM/PowerSparse_SpMM.h"
#include "utils/cuda_utils.h"

#include <stdexcept>
#include <string>
#include <vector>

namespace PowerSparse {

void ThrowStatus(int status) {
  if (status == PS_OK) return;
  const std::string msg = ps_last_error();
  if (status == PS_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
  throw std::runtime_error(msg);
}

PowerSparseMatrixGPU::PowerSparseMatrixGPU(int row_num, int col_num, int nnz_num, const int* row_ptr,
                                           const int* col_ind, const float* sp_data) {
  ThrowStatus(ps_matrix_create(row_num, col_num, nnz_num, row_ptr, col_ind, sp_data, &_handle));
}

namespace {

// The fused launch goes on one stream; it first waits for the work already
// queued on every stream the caller handed over (the reference queued workset s
// on stream s).
cudaStream_t JoinStreams(int count, const cudaStream_t* streams) {
  if (count <= 1) return nullptr;
  for (int s = 1; s < count; ++s) {
    cudaEvent_t ev;
    CUDA_CALL(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    CUDA_CALL(cudaEventRecord(ev, streams[s]));
    CUDA_CALL(cudaStreamWaitEvent(streams[0], ev, 0));
    CUDA_CALL(cudaEventDestroy(ev));
  }
  return streams[0];
}

}  // namespace

void SpMM(const PowerSparseMatrixGPU& matrix, int N, const float* B, float* C, int stream_count,
          const cudaStream_t* streams) {
  if (N <= 0 || N % 32 != 0 || N / 32 > 65535)
    throw std::invalid_argument("SpMM requires N to be a positive multiple of 32, with N/32 <= 65535");
  if (!B || !C || stream_count != matrix.GroupTypeNum() || (stream_count > 1 && !streams))
    throw std::invalid_argument("Invalid SpMM buffers or stream count");
  const cudaStream_t stream = JoinStreams(stream_count, streams);
  ThrowStatus(ps_spmm(matrix.Handle(), N, B, C, stream));
  // Preserve the synchronization behavior of the original multi-workset API.
  if (stream_count > 1) CUDA_CALL(cudaDeviceSynchronize());
}

void SDDMM(const PowerSparseMatrixGPU& matrix, int N, const float* lhs, const float* rhs, float** output,
           int stream_count, const cudaStream_t* streams) {
  if (N != 32 && N != 128)
    throw std::invalid_argument("SDDMM dispatcher expects a benchmark width of N=32 or N=128");
  if (!lhs || !rhs || !output || stream_count != matrix.GroupTypeNum() || (stream_count > 1 && !streams))
    throw std::invalid_argument("Invalid SDDMM buffers or stream count");
  for (int s = 0; s < stream_count; ++s) {
    if (matrix.GroupNum()[s] == 0) continue;
    if (!output[s]) throw std::invalid_argument("Missing SDDMM output workset");
  }
  const cudaStream_t stream = JoinStreams(stream_count, streams);
  ThrowStatus(ps_sddmm(matrix.Handle(), N, lhs, rhs, output, stream));
  if (stream_count > 1) CUDA_CALL(cudaDeviceSynchronize());
}

}  // namespace PowerSparse
