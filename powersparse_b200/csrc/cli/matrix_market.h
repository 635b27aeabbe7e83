// Sparse matrix input of the drop-in CLI: MatrixMarket text (the reference's
// format, benchmarks/matrix_market.{h,cpp}) or this package's binary CSR.
#pragma once

#include <memory>
#include <string>
#include <utility>
#include <vector>

// std::vector allocator whose resize leaves new elements uninitialized (no zero
// fill): the reader's threads write every element, touching the pages in parallel.
template <typename T>
struct UninitAllocator : std::allocator<T> {
  template <typename U>
  struct rebind {
    using other = UninitAllocator<U>;
  };
  UninitAllocator() = default;
  template <typename U>
  UninitAllocator(const UninitAllocator<U>&) noexcept {}
  template <typename U>
  void construct(U* p) noexcept {
    ::new (static_cast<void*>(p)) U;
  }
  template <typename U, typename... Args>
  void construct(U* p, Args&&... args) {
    ::new (static_cast<void*>(p)) U(std::forward<Args>(args)...);
  }
};

struct CsrMatrix {
  int rows = 0, cols = 0;
  std::vector<int, UninitAllocator<int>> row_ptr, col_ind;
  std::vector<float, UninitAllocator<float>> values;
  int nnz() const { return static_cast<int>(values.size()); }
};

// Reads `path` into CSR.  Files that start with "PSCSR001" are this package's
// binary CSR (little-endian: magic, int64 rows, cols, nnz, int32 row_ptr[rows+1],
// int32 col_ind[nnz], float32 values[nnz]).  Anything else is MatrixMarket
// coordinate text with the subset and meaning of the reference's reader
// (benchmarks/matrix_market.cpp:97-134): field pattern/real/integer, symmetry
// general/symmetric; entries keep their file order within a row, and a symmetric
// off-diagonal entry (i, j) also yields (j, i) right after it.  The same inputs
// are accepted and the same CSR is produced; malformed input raises
// std::runtime_error with the reference's messages (the first problem in file
// order is the one reported).
//
// The text is parsed in parallel: the file is mapped, cut into one chunk of lines
// per thread, every thread parses its chunk once into entries bucketed by block
// of rows, and a second parallel step places each block's entries (a row's
// entries from chunk t follow those from chunks before t, so file order is
// kept).  `threads` <= 0 uses the hardware concurrency.
CsrMatrix ReadMatrixMarket(const std::string& path, int threads = 0);

// ReadMatrixMarket with the smallest chunk of text a thread takes given explicitly
// (ReadMatrixMarket uses 4 MiB); small values exercise the chunk boundaries.
CsrMatrix ReadMatrixMarketChunked(const std::string& path, int threads, long long min_chunk_bytes);
