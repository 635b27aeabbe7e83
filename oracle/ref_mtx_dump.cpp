// Harness around the reference's MatrixMarket reader (TEST INFRASTRUCTURE ONLY).
//
//   ref_mtx_dump IN.mtx OUT.csr
//
// Links benchmarks/matrix_market.cpp of the reference (built from its sources by
// oracle/Makefile) and writes the CSR it produces in the binary format of
// powersparse_b200.synth.write_csr_bin, so tests can compare the CLI's reader with
// it byte for byte.  Prints one JSON line with the read time.  A reader error is
// printed as the reference's CLI prints it ("Error: <message>") with exit code 1.
#include "benchmarks/matrix_market.h"

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <fstream>
#include <iostream>
#include <stdexcept>

int main(int argc, char** argv) {
  if (argc != 3) {
    std::cerr << "usage: ref_mtx_dump IN.mtx OUT.csr\n";
    return 2;
  }
  try {
    const auto t0 = std::chrono::steady_clock::now();
    const CsrMatrix m = ReadMatrixMarket(argv[1]);
    const double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    std::ofstream out(argv[2], std::ios::binary);
    const int64_t dims[3] = {m.rows, m.cols, (int64_t)m.values.size()};
    out.write("PSCSR001", 8);
    out.write(reinterpret_cast<const char*>(dims), sizeof(dims));
    out.write(reinterpret_cast<const char*>(m.row_ptr.data()), std::streamsize(4 * m.row_ptr.size()));
    out.write(reinterpret_cast<const char*>(m.col_ind.data()), std::streamsize(4 * m.col_ind.size()));
    out.write(reinterpret_cast<const char*>(m.values.data()), std::streamsize(4 * m.values.size()));
    if (!out) throw std::runtime_error("cannot write output");
    std::printf("{\"rows\":%d,\"cols\":%d,\"nnz\":%lld,\"read_s\":%.6f}\n", m.rows, m.cols,
                (long long)m.values.size(), s);
    return 0;
  } catch (const std::exception& e) {
    std::cerr << "Error: " << e.what() << '\n';
    return 1;
  }
}
