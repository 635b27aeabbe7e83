// PowerSparse C++ API: the preprocessed block/residue matrix.
//
// Drop-in for utils/matrix_utils.h of ParCIS/PowerSparse (same namespace, class,
// constructor, accessors, macros and exceptions).  The object owns a handle of
// the C ABI in powersparse_b200.h; preprocessing runs on the GPU and yields the
// reference's layout bit for bit.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <limits>
#include <stdexcept>

#include "powersparse_b200.h"

#define GROUP_SIZE(I) (32 * (1 << ((I) - 1)))
#define CEIL(X, Y) ((X) / (Y) + ((X) % (Y) != 0))
#define FLOOR(X, Y) ((X) / (Y))

namespace PowerSparse {

enum SigBitMode { PPL = 0, FFC = 1 };
enum FreqSort { FreqNoSort = 0, FreqDoSort = 1 };
enum GroupSort { GroupNoSort = 0, GroupDoSort = 1 };

// Throws the exception the reference throws for a failed C ABI call.
void ThrowStatus(int status);

// Owns the GPU worksets built from host CSR arrays. Construct and destroy on
// the same CUDA device; complete outstanding operator calls before destruction.
class PowerSparseMatrixGPU {
 public:
  PowerSparseMatrixGPU(int row_num, int col_num, int nnz_num, const int* row_ptr, const int* col_ind,
                       const float* sp_data);
  ~PowerSparseMatrixGPU() { ps_matrix_destroy(_handle); }
  PowerSparseMatrixGPU(const PowerSparseMatrixGPU&) = delete;
  PowerSparseMatrixGPU& operator=(const PowerSparseMatrixGPU&) = delete;
  PowerSparseMatrixGPU(PowerSparseMatrixGPU&&) = delete;
  PowerSparseMatrixGPU& operator=(PowerSparseMatrixGPU&&) = delete;

  int MatrixRow() const { return ps_matrix_row(_handle); }
  int MatrixCol() const { return ps_matrix_col(_handle); }
  int MatrixNNZ() const { return ps_matrix_nnz(_handle); }
  int GroupTypeNum() const { return ps_matrix_group_type_num(_handle); }
  int GroupFineSize() const { return ps_matrix_group_fine_size(_handle); }
  const int* GroupNum() const { return ps_matrix_group_num(_handle); }
  const int* const* WorksetColInd() const { return ps_matrix_workset_col_ind(_handle); }
  const float* const* WorksetSpData() const { return ps_matrix_workset_sp_data(_handle); }
  const int* const* GroupDestination() const { return ps_matrix_group_destination(_handle); }
  const int* ResidueOffset() const { return ps_matrix_residue_offset(_handle); }
  const bool* ResidueAtomic() const { return ps_matrix_residue_atomic(_handle); }

  // The C ABI handle (for callers that mix the two interfaces).
  const ps_matrix* Handle() const { return _handle; }

 private:
  ps_matrix* _handle = nullptr;
};

// The reference kernels use signed 32-bit dense element offsets and reject larger
// shapes with this check.  The B200 kernels use 64-bit offsets, so SpMM and SDDMM
// here do not call it; it is kept for callers that do.
inline void ValidateDenseShape(int rows, int cols, int n) {
  if (n <= 0 || int64_t(rows) * n > std::numeric_limits<int>::max() ||
      int64_t(cols) * n > std::numeric_limits<int>::max())
    throw std::invalid_argument("Dense dimensions exceed the 32-bit kernel indexing range");
}

}  // namespace PowerSparse
