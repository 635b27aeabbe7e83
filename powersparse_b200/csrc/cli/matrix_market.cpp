// MatrixMarket / binary CSR reader of the drop-in CLI.
//
// Accepts what the reference's reader accepts (benchmarks/matrix_market.cpp):
// "%%MatrixMarket matrix coordinate {pattern|real|integer} {general|symmetric}",
// 1-based indices inside the declared shape, finite FP32 values, the declared
// entry count, a 32-bit CSR capacity limit, and rejects anything else with a
// std::runtime_error.  Parsing uses strtoll/strtod on whole lines.
#include "matrix_market.h"

#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <limits>
#include <sstream>
#include <stdexcept>

namespace {

constexpr long long kMaxIndex = std::numeric_limits<int>::max() - 32;

inline bool is_space(char c) { return c == ' ' || c == '\t' || c == '\r' || c == '\n' || c == '\f' || c == '\v'; }

const char* skip(const char* p) {
  while (is_space(*p)) ++p;
  return p;
}

// Next line that is not blank and not a comment.
bool next_record(std::istream& in, std::string& line) {
  while (std::getline(in, line)) {
    const char* p = skip(line.c_str());
    if (*p && *p != '%') return true;
  }
  if (in.bad()) throw std::runtime_error("Error reading MatrixMarket input");
  return false;
}

long long parse_integer(const char*& p) {
  p = skip(p);
  errno = 0;
  char* end = nullptr;
  const long long v = std::strtoll(p, &end, 10);
  if (end == p || errno == ERANGE || (*end && !is_space(*end)))
    throw std::runtime_error("Invalid integer in MatrixMarket input");
  p = end;
  return v;
}

void expect_end(const char* p) {
  if (*skip(p)) throw std::runtime_error("Unexpected extra fields in MatrixMarket record");
}

struct Banner {
  int rows = 0, cols = 0, entries = 0;
  bool pattern = false, integer = false, symmetric = false;
};

Banner read_banner(std::istream& in) {
  std::string line;
  if (!std::getline(in, line)) throw std::runtime_error("Empty MatrixMarket file");
  std::istringstream words(line);
  std::string magic, object, format, field, symmetry, extra;
  if (!(words >> magic >> object >> format >> field >> symmetry) || (words >> extra) ||
      magic != "%%MatrixMarket" || object != "matrix" || format != "coordinate" ||
      (field != "pattern" && field != "real" && field != "integer") ||
      (symmetry != "general" && symmetry != "symmetric"))
    throw std::runtime_error("Expected MatrixMarket coordinate pattern/real/integer general/symmetric");
  if (!next_record(in, line)) throw std::runtime_error("Missing MatrixMarket dimensions");
  const char* p = line.c_str();
  const long long r = parse_integer(p), c = parse_integer(p), e = parse_integer(p);
  expect_end(p);
  if (r <= 0 || c <= 0 || e <= 0 || r > kMaxIndex || c > kMaxIndex || e > kMaxIndex ||
      (symmetry == "symmetric" && r != c))
    throw std::runtime_error("Matrix must be nonempty and fit 32-bit CSR indices");
  Banner b;
  b.rows = int(r);
  b.cols = int(c);
  b.entries = int(e);
  b.pattern = field == "pattern";
  b.integer = field == "integer";
  b.symmetric = symmetry == "symmetric";
  return b;
}

template <typename Sink>
void for_each_entry(std::istream& in, const Banner& b, Sink&& sink) {
  std::string line;
  for (int k = 0; k < b.entries; ++k) {
    if (!next_record(in, line)) throw std::runtime_error("Truncated MatrixMarket input");
    const char* p = line.c_str();
    const long long i = parse_integer(p), j = parse_integer(p);
    if (i < 1 || i > b.rows || j < 1 || j > b.cols)
      throw std::runtime_error("MatrixMarket index outside the declared dimensions");
    float v = 1.0f;
    if (b.integer) {
      v = static_cast<float>(parse_integer(p));
    } else if (!b.pattern) {
      p = skip(p);
      char* end = nullptr;
      const double x = std::strtod(p, &end);
      if (end == p || (*end && !is_space(*end)) || !std::isfinite(x) ||
          std::abs(x) > std::numeric_limits<float>::max())
        throw std::runtime_error("Invalid finite FP32 value in MatrixMarket input");
      v = static_cast<float>(x);
      p = end;
    }
    expect_end(p);
    sink(int(i - 1), int(j - 1), v);
    if (b.symmetric && i != j) sink(int(j - 1), int(i - 1), v);
  }
  if (next_record(in, line)) throw std::runtime_error("More entries than declared in MatrixMarket input");
}

CsrMatrix read_binary(std::ifstream& in) {
  int64_t dims[3];
  in.read(reinterpret_cast<char*>(dims), sizeof(dims));
  if (!in || dims[0] <= 0 || dims[1] <= 0 || dims[2] <= 0 || dims[0] > kMaxIndex || dims[1] > kMaxIndex ||
      dims[2] > kMaxIndex)
    throw std::runtime_error("Invalid binary CSR header");
  CsrMatrix m;
  m.rows = int(dims[0]);
  m.cols = int(dims[1]);
  m.row_ptr.resize(size_t(m.rows) + 1);
  m.col_ind.resize(size_t(dims[2]));
  m.values.resize(size_t(dims[2]));
  in.read(reinterpret_cast<char*>(m.row_ptr.data()), sizeof(int) * m.row_ptr.size());
  in.read(reinterpret_cast<char*>(m.col_ind.data()), sizeof(int) * m.col_ind.size());
  in.read(reinterpret_cast<char*>(m.values.data()), sizeof(float) * m.values.size());
  if (!in) throw std::runtime_error("Truncated binary CSR input");
  return m;
}

}  // namespace

CsrMatrix ReadMatrixMarket(const std::string& path) {
  std::ifstream in(path, std::ios::binary);
  if (!in) throw std::runtime_error("Cannot open matrix: " + path);
  char magic[8] = {};
  in.read(magic, 8);
  if (in.gcount() == 8 && std::memcmp(magic, "PSCSR001", 8) == 0) return read_binary(in);
  in.clear();
  in.seekg(0);

  const Banner b = read_banner(in);
  CsrMatrix m;
  m.rows = b.rows;
  m.cols = b.cols;
  m.row_ptr.assign(size_t(b.rows) + 1, 0);
  long long total = 0;
  for_each_entry(in, b, [&](int r, int, float) {
    if (++total > kMaxIndex) throw std::runtime_error("Expanded matrix exceeds 32-bit CSR capacity");
    ++m.row_ptr[size_t(r) + 1];
  });
  for (int r = 0; r < b.rows; ++r) m.row_ptr[size_t(r) + 1] += m.row_ptr[r];
  m.col_ind.resize(size_t(total));
  m.values.resize(size_t(total));
  std::vector<int> fill(m.row_ptr.begin(), m.row_ptr.end() - 1);

  in.clear();
  in.seekg(0);
  if (!in) throw std::runtime_error("Matrix input must be a seekable regular file");
  const Banner again = read_banner(in);
  if (again.rows != b.rows || again.cols != b.cols || again.entries != b.entries ||
      again.pattern != b.pattern || again.integer != b.integer || again.symmetric != b.symmetric)
    throw std::runtime_error("Matrix header changed between reader passes");
  for_each_entry(in, b, [&](int r, int c, float v) {
    const int at = fill[r]++;
    if (at >= m.row_ptr[size_t(r) + 1]) throw std::runtime_error("Matrix row counts changed between reader passes");
    m.col_ind[at] = c;
    m.values[at] = v;
  });
  for (int r = 0; r < b.rows; ++r)
    if (fill[r] != m.row_ptr[size_t(r) + 1])
      throw std::runtime_error("Matrix row counts changed between reader passes");
  return m;
}
