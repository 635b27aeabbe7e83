// powersparse_mtx2csr IN.mtx OUT.csr [THREADS [MIN_CHUNK_BYTES]]
//
// Converts a MatrixMarket file to the package's binary CSR (the format the CLI,
// powersparse_b200.synth.read_csr_bin and the layout tools read), with the CLI's
// own reader: a billion-entry text file is parsed once, and later runs load the
// binary file at disk speed.  Prints one JSON line with the shape and the read
// time.  Exit codes: 0 ok, 1 read or write error (message on stderr, as the CLI
// prints it), 2 usage.
#include "matrix_market.h"

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <fstream>
#include <iostream>
#include <stdexcept>
#include <string>

int main(int argc, char** argv) {
  if (argc < 3 || argc > 5) {
    std::cerr << "Usage: " << argv[0] << " IN.mtx OUT.csr [THREADS [MIN_CHUNK_BYTES]]\n";
    return 2;
  }
  try {
    const int threads = argc > 3 ? std::stoi(argv[3]) : 0;
    const long long chunk = argc > 4 ? std::stoll(argv[4]) : (4LL << 20);
    const auto t0 = std::chrono::steady_clock::now();
    const CsrMatrix m = ReadMatrixMarketChunked(argv[1], threads, chunk);
    const double read_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    std::ofstream out(argv[2], std::ios::binary);
    const int64_t dims[3] = {m.rows, m.cols, (int64_t)m.values.size()};
    out.write("PSCSR001", 8);
    out.write(reinterpret_cast<const char*>(dims), sizeof(dims));
    out.write(reinterpret_cast<const char*>(m.row_ptr.data()), std::streamsize(4 * m.row_ptr.size()));
    out.write(reinterpret_cast<const char*>(m.col_ind.data()), std::streamsize(4 * m.col_ind.size()));
    out.write(reinterpret_cast<const char*>(m.values.data()), std::streamsize(4 * m.values.size()));
    if (!out) throw std::runtime_error(std::string("Cannot write ") + argv[2]);
    std::printf("{\"rows\":%d,\"cols\":%d,\"nnz\":%lld,\"read_s\":%.6f}\n", m.rows, m.cols,
                (long long)m.values.size(), read_s);
    return 0;
  } catch (const std::exception& e) {
    std::cerr << "Error: " << e.what() << '\n';
    return 1;
  }
}
