// Drop-in benchmark CLI: powersparse_{spmm,sddmm} MATRIX.mtx N DEVICE CHECK REPEATS
//
// Same command line, exit codes, stderr messages and CSV columns as the
// reference's benchmarks/benchmark.cu (compiled twice; POWERSPARSE_BENCH_SDDMM
// selects the operator, as in its CMakeLists.txt:45):
//   --header                   print the CSV header
//   N                          32 or 128 (checked before anything else, exit 2)
//   CHECK=1                    verify the layout is a permutation of the CSR and
//                              compare the operator with a serial FP64 CPU loop
//   REPEATS                    timed back-to-back calls after 30 warm-up calls
// Dense inputs come from std::mt19937(1): values (rng() % 3) / 10, lhs first.
// MATRIX may also be a binary CSR file (see matrix_market.h).
#include "PowerSparse_SDDMM/PowerSparse_SDDMM.h"
#include "PowerSparse_SpMM/PowerSparse_SpMM.h"
#include "matrix_market.h"
#include "utils/cuda_utils.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <iomanip>
#include <iostream>
#include <limits>
#include <random>
#include <string>
#include <tuple>
#include <vector>

#ifdef POWERSPARSE_BENCH_SDDMM
constexpr bool kSddmm = true;
#else
constexpr bool kSddmm = false;
#endif
constexpr int kWarmup = 30;
constexpr unsigned kSeed = 1;
constexpr const char* kOperator = kSddmm ? "SDDMM" : "SpMM";

namespace {

using Matrix = PowerSparse::PowerSparseMatrixGPU;

template <typename T>
class DeviceVector {
 public:
  explicit DeviceVector(size_t n = 0) : n_(n) {
    if (n) CUDA_CALL(cudaMalloc(reinterpret_cast<void**>(&p_), n * sizeof(T)));
  }
  ~DeviceVector() { cudaFree(p_); }
  DeviceVector(const DeviceVector&) = delete;
  DeviceVector& operator=(const DeviceVector&) = delete;
  DeviceVector(DeviceVector&& o) noexcept : p_(o.p_), n_(o.n_) { o.p_ = nullptr; o.n_ = 0; }
  T* data() const { return p_; }
  size_t size() const { return n_; }
  void zero() { if (n_) CUDA_CALL(cudaMemset(p_, 0, n_ * sizeof(T))); }
  void upload(const std::vector<T>& h) {
    if (h.size() != n_) throw std::invalid_argument("Upload size mismatch");
    if (n_) CUDA_CALL(cudaMemcpy(p_, h.data(), n_ * sizeof(T), cudaMemcpyHostToDevice));
  }

 private:
  T* p_ = nullptr;
  size_t n_ = 0;
};

template <typename T>
std::vector<T> download(const T* d, size_t n) {
  std::vector<T> h(n);
  if (n) CUDA_CALL(cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost));
  return h;
}

int parse_int(const char* text, const char* name) {
  const std::string s(text);
  size_t used = 0;
  int v = 0;
  try {
    v = std::stoi(s, &used);
  } catch (...) {
    throw std::invalid_argument(std::string("Invalid ") + name + ": " + s);
  }
  if (used != s.size()) throw std::invalid_argument(std::string("Invalid ") + name);
  return v;
}

std::vector<float> dense_input(size_t n, std::mt19937& rng) {
  std::vector<float> v(n);
  for (auto& x : v) x = static_cast<float>(rng() % 3) / 10.0f;
  return v;
}

bool close(float actual, double expected) {
  return std::isfinite(actual) && std::isfinite(expected) &&
         std::abs(double(actual) - expected) <= 1e-3 + 1e-3 * std::abs(expected);
}

std::string csv_quote(const std::string& s) {
  std::string out = "\"";
  for (char c : s) {
    if (c == '"') out += '"';
    out += c;
  }
  return out + '"';
}

struct Workset {
  std::vector<int> rows, offsets, cols;
  std::vector<float> values;
};

Workset read_workset(const Matrix& m, int s, const std::vector<int>& residue) {
  Workset w;
  const int groups = m.GroupNum()[s];
  w.rows = download(m.GroupDestination()[s], size_t(groups));
  if (s == 0) {
    w.offsets = residue;
  } else {
    w.offsets.resize(size_t(groups) + 1);
    for (int g = 0; g <= groups; ++g) w.offsets[g] = g * GROUP_SIZE(s);
  }
  w.cols = download(m.WorksetColInd()[s], size_t(w.offsets.back()));
  w.values = download(m.WorksetSpData()[s], size_t(w.offsets.back()));
  return w;
}

// The layout holds exactly the CSR's (row, column, value) multiset.
void check_layout(const CsrMatrix& csr, const Matrix& m, const std::vector<int>& residue) {
  using Entry = std::tuple<int, int, float>;
  std::vector<Entry> want, have;
  want.reserve(csr.values.size());
  have.reserve(csr.values.size());
  for (int r = 0; r < csr.rows; ++r)
    for (int p = csr.row_ptr[r]; p < csr.row_ptr[r + 1]; ++p) want.emplace_back(r, csr.col_ind[p], csr.values[p]);
  for (int s = 0; s < m.GroupTypeNum(); ++s) {
    const Workset w = read_workset(m, s, residue);
    for (size_t g = 0; g < w.rows.size(); ++g)
      for (int p = w.offsets[g]; p < w.offsets[g + 1]; ++p) have.emplace_back(w.rows[g], w.cols[p], w.values[p]);
  }
  std::sort(want.begin(), want.end());
  std::sort(have.begin(), have.end());
  if (want != have) throw std::runtime_error("Preprocessing changed the sparse matrix");
}

void check_spmm(const CsrMatrix& csr, int n, const std::vector<float>& b, const float* d_out) {
  const std::vector<float> got = download(d_out, size_t(csr.rows) * n);
  std::vector<double> row(n);
  for (int r = 0; r < csr.rows; ++r) {
    std::fill(row.begin(), row.end(), 0.0);
    for (int p = csr.row_ptr[r]; p < csr.row_ptr[r + 1]; ++p)
      for (int j = 0; j < n; ++j) row[j] += double(csr.values[p]) * b[size_t(csr.col_ind[p]) * n + j];
    for (int j = 0; j < n; ++j)
      if (!close(got[size_t(r) * n + j], row[j]))
        throw std::runtime_error("SpMM mismatch at row " + std::to_string(r) + ", feature " + std::to_string(j));
  }
}

void check_sddmm(const Matrix& m, const std::vector<int>& residue, int n, const std::vector<float>& lhs,
                 const std::vector<float>& rhs, const std::vector<float*>& out) {
  for (int s = 0; s < m.GroupTypeNum(); ++s) {
    const Workset w = read_workset(m, s, residue);
    const std::vector<float> got = download(out[s], w.values.size());
    for (size_t g = 0; g < w.rows.size(); ++g)
      for (int p = w.offsets[g]; p < w.offsets[g + 1]; ++p) {
        double e = 0;
        for (int j = 0; j < n; ++j) e += double(lhs[size_t(w.rows[g]) * n + j]) * rhs[size_t(w.cols[p]) * n + j];
        e *= w.values[p];
        if (!close(got[p], e))
          throw std::runtime_error("SDDMM mismatch in workset " + std::to_string(s) + ", position " +
                                   std::to_string(p));
      }
  }
}

void print_header() {
  std::cout << "algorithm,operator,matrix,rows,cols,nnz,N,device,gpu,compute_capability,"
               "cuda_runtime,cuda_driver,warmup,repeats,seed,check,preprocess_ms,ms,gflops\n";
}

int run(int argc, char** argv) {
  if (argc == 2 && std::string(argv[1]) == "--header") {
    print_header();
    return 0;
  }
  if (argc != 6) {
    std::cerr << "Usage: " << argv[0] << " MATRIX.mtx N DEVICE CHECK REPEATS\n"
              << "CHECK: 0=skip, 1=verify preprocessing and compare with a CPU reference\n"
              << "SpMM and SDDMM benchmark widths are set to N=32 or 128 in main.\n";
    return 2;
  }
  const std::string path = argv[1];
  const int n = parse_int(argv[2], "N"), device = parse_int(argv[3], "DEVICE");
  const int check = parse_int(argv[4], "CHECK"), repeats = parse_int(argv[5], "REPEATS");
  if (device < 0 || (check != 0 && check != 1) || repeats <= 0)
    throw std::invalid_argument("DEVICE must be nonnegative, CHECK 0 or 1, and REPEATS positive");
  CUDA_CALL(cudaSetDevice(device));
  CUDA_CALL(cudaFree(nullptr));
  cudaDeviceProp prop{};
  CUDA_CALL(cudaGetDeviceProperties(&prop, device));
  if (prop.major < 10) throw std::runtime_error("These kernels require an sm_100 (Blackwell B200) GPU");
  int runtime = 0, driver = 0;
  CUDA_CALL(cudaRuntimeGetVersion(&runtime));
  CUDA_CALL(cudaDriverGetVersion(&driver));
  std::cerr << kOperator << ": " << path << ", N=" << n << ", GPU=" << prop.name << '\n';
  const CsrMatrix csr = ReadMatrixMarket(path);

  CUDA_CALL(cudaDeviceSynchronize());
  const auto t0 = std::chrono::steady_clock::now();
  const Matrix matrix(csr.rows, csr.cols, csr.nnz(), csr.row_ptr.data(), csr.col_ind.data(), csr.values.data());
  CUDA_CALL(cudaDeviceSynchronize());
  const double preprocess_ms =
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  const std::vector<int> residue = download(matrix.ResidueOffset(), size_t(matrix.GroupNum()[0]) + 1);

  std::mt19937 rng(kSeed);
  std::vector<float> lhs;
  if (kSddmm) lhs = dense_input(size_t(csr.rows) * n, rng);
  const std::vector<float> rhs = dense_input(size_t(csr.cols) * n, rng);
  DeviceVector<float> d_lhs(lhs.size()), d_rhs(rhs.size());
  d_lhs.upload(lhs);
  d_rhs.upload(rhs);
  DeviceVector<float> dense_out(kSddmm ? 0 : size_t(csr.rows) * n);
  std::vector<DeviceVector<float>> sparse_out;
  std::vector<float*> out_ptrs;
  if (kSddmm) {
    sparse_out.reserve(matrix.GroupTypeNum());
    for (int s = 0; s < matrix.GroupTypeNum(); ++s) {
      const size_t count = s == 0 ? size_t(residue.back()) : size_t(matrix.GroupNum()[s]) * GROUP_SIZE(s);
      sparse_out.emplace_back(count);
      out_ptrs.push_back(sparse_out.back().data());
    }
  }
  const int S = matrix.GroupTypeNum();
  std::vector<cudaStream_t> streams(S, nullptr);
  if (S > 1)
    for (auto& st : streams) CUDA_CALL(cudaStreamCreate(&st));
  struct StreamGuard {
    std::vector<cudaStream_t>& v;
    ~StreamGuard() { for (auto s : v) if (s) cudaStreamDestroy(s); }
  } guard{streams};

  auto reset = [&] {
    dense_out.zero();
    for (auto& o : sparse_out) o.zero();
    CUDA_CALL(cudaDeviceSynchronize());
  };
  auto invoke = [&] {
    if (kSddmm)
      PowerSparse::SDDMM(matrix, n, d_lhs.data(), d_rhs.data(), out_ptrs.data(), S, streams.data());
    else
      PowerSparse::SpMM(matrix, n, d_rhs.data(), dense_out.data(), S, streams.data());
  };
  reset();
  if (check) {
    check_layout(csr, matrix, residue);
    invoke();
    CUDA_CALL(cudaDeviceSynchronize());
    if (kSddmm) check_sddmm(matrix, residue, n, lhs, rhs, out_ptrs);
    else check_spmm(csr, n, rhs, dense_out.data());
    std::cerr << "Preprocessing and CPU reference checks passed (atol=rtol=1e-3).\n";
    reset();
  }
  for (int i = 0; i < kWarmup; ++i) invoke();
  CUDA_CALL(cudaDeviceSynchronize());
  reset();
  cudaEvent_t start, stop;
  CUDA_CALL(cudaEventCreate(&start));
  CUDA_CALL(cudaEventCreate(&stop));
  CUDA_CALL(cudaEventRecord(start));
  // As in the reference harness, outputs are not cleared between timed calls.
  for (int i = 0; i < repeats; ++i) invoke();
  CUDA_CALL(cudaEventRecord(stop));
  CUDA_CALL(cudaEventSynchronize(stop));
  float total_ms = 0;
  CUDA_CALL(cudaEventElapsedTime(&total_ms, start, stop));
  cudaEventDestroy(start);
  cudaEventDestroy(stop);
  const double ms = double(total_ms) / repeats;
  if (!std::isfinite(ms) || ms <= 0) throw std::runtime_error("Invalid measured latency");
  const double gflops = 2.0 * csr.nnz() * n / (ms * 1e6);
  std::cout << std::setprecision(10) << "PowerSparse," << kOperator << ',' << csv_quote(path) << ',' << csr.rows
            << ',' << csr.cols << ',' << csr.nnz() << ',' << n << ',' << device << ',' << csv_quote(prop.name)
            << ',' << prop.major << '.' << prop.minor << ',' << runtime << ',' << driver << ',' << kWarmup << ','
            << repeats << ',' << kSeed << ',' << (check ? "passed" : "skipped") << ',' << preprocess_ms << ','
            << ms << ',' << gflops << '\n';
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    if (argc == 6) {
      const int n = parse_int(argv[2], "N");
      if (n != 32 && n != 128) {
        std::cerr << kOperator << " benchmark: N=" << n << " was not selected in main; please use N=32 or N=128.\n";
        return 2;
      }
    }
    return run(argc, argv);
  } catch (const std::exception& e) {
    std::cerr << "Error: " << e.what() << '\n';
    return 1;
  }
}
