// Sparse matrix input of the drop-in CLI: MatrixMarket text (the reference's
// format, benchmarks/matrix_market.{h,cpp}) or this package's binary CSR.
#pragma once

#include <string>
#include <vector>

struct CsrMatrix {
  int rows = 0, cols = 0;
  std::vector<int> row_ptr, col_ind;
  std::vector<float> values;
  int nnz() const { return static_cast<int>(values.size()); }
};

// MatrixMarket coordinate pattern/real/integer, general/symmetric -> CSR.  Two
// passes (count, fill); entries keep file order within a row and a symmetric
// off-diagonal entry (i, j) also yields (j, i) right after it, as the
// reference's reader does (benchmarks/matrix_market.cpp:97-134).  Files that
// start with the binary CSR magic "PSCSR001" are read directly.
CsrMatrix ReadMatrixMarket(const std::string& path);
