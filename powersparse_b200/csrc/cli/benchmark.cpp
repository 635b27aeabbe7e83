// Drop-in benchmark CLI: powersparse_{spmm,sddmm} MATRIX.mtx N DEVICE CHECK REPEATS
//
// The command line, exit codes (0 ok, 1 error, 2 usage), stderr messages, dense
// inputs and CSV row are those of the reference's benchmarks/benchmark.cu, so
// scripts and result files written for it keep working; the program itself is
// organised differently.  One source, compiled twice: POWERSPARSE_BENCH_SDDMM
// selects the operator (as the reference's CMakeLists.txt:45 does).
//   --header    the CSV header
//   N           32 or 128, checked before anything else (exit 2)
//   CHECK=1     the layout must hold exactly the input's (row, column, value)
//               entries, and the operator must match an FP64 host product within
//               atol = rtol = 1e-3 (the reference's tolerance)
//   REPEATS     timed calls, back to back after 30 warm-up calls, outputs not
//               cleared in between; GFLOPS = 2 nnz N / time
// Dense inputs: std::mt19937 seeded with 1, each value (draw % 3) / 10, the SDDMM
// lhs drawn before the rhs.  MATRIX may also be a binary CSR (matrix_market.h).
#include "PowerSparse_SDDMM/PowerSparse_SDDMM.h"
#include "PowerSparse_SpMM/PowerSparse_SpMM.h"
#include "matrix_market.h"
#include "utils/cuda_utils.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <iomanip>
#include <iostream>
#include <memory>
#include <random>
#include <sstream>
#include <string>
#include <utility>
#include <vector>

namespace {

#ifdef POWERSPARSE_BENCH_SDDMM
constexpr bool kIsSddmm = true;
#else
constexpr bool kIsSddmm = false;
#endif
const char* const kOpName = kIsSddmm ? "SDDMM" : "SpMM";
constexpr int kWarmupCalls = 30;
constexpr unsigned kDenseSeed = 1;
constexpr double kCheckTol = 1e-3;

// ---- command line ------------------------------------------------------------

struct Args {
  std::string matrix;
  int n = 0, device = 0, check = 0, repeats = 0;
};

// Whole-string decimal int; the error texts are the reference's.
int to_int(const char* text, const char* what) {
  std::size_t used = 0;
  int value = 0;
  try {
    value = std::stoi(std::string(text), &used);
  } catch (...) {
    throw std::invalid_argument(std::string("Invalid ") + what + ": " + text);
  }
  if (used != std::strlen(text)) throw std::invalid_argument(std::string("Invalid ") + what);
  return value;
}

void usage(const char* prog) {
  std::cerr << "Usage: " << prog << " MATRIX.mtx N DEVICE CHECK REPEATS\n"
            << "CHECK: 0=skip, 1=verify preprocessing and compare with a CPU reference\n"
            << "SpMM and SDDMM benchmark widths are set to N=32 or 128 in main.\n";
}

const char* csv_header() {
  return "algorithm,operator,matrix,rows,cols,nnz,N,device,gpu,compute_capability,"
         "cuda_runtime,cuda_driver,warmup,repeats,seed,check,preprocess_ms,ms,gflops";
}

std::string quoted(const std::string& s) {
  std::string q;
  q.reserve(s.size() + 2);
  q.push_back('"');
  for (char c : s) {
    q.push_back(c);
    if (c == '"') q.push_back('"');
  }
  q.push_back('"');
  return q;
}

// ---- device memory -----------------------------------------------------------

struct CudaFree {
  void operator()(void* p) const { cudaFree(p); }
};
template <typename T>
using DevicePtr = std::unique_ptr<T, CudaFree>;

template <typename T>
DevicePtr<T> device_alloc(std::size_t count) {
  T* p = nullptr;
  if (count) CUDA_CALL(cudaMalloc(reinterpret_cast<void**>(&p), count * sizeof(T)));
  return DevicePtr<T>(p);
}

template <typename T>
DevicePtr<T> device_copy(const std::vector<T>& host) {
  DevicePtr<T> d = device_alloc<T>(host.size());
  if (!host.empty()) CUDA_CALL(cudaMemcpy(d.get(), host.data(), host.size() * sizeof(T), cudaMemcpyHostToDevice));
  return d;
}

template <typename T>
std::vector<T> host_copy(const T* device, std::size_t count) {
  std::vector<T> h(count);
  if (count) CUDA_CALL(cudaMemcpy(h.data(), device, count * sizeof(T), cudaMemcpyDeviceToHost));
  return h;
}

// ---- the operator under test -------------------------------------------------

// The matrix, its dense inputs, outputs and streams, and the reference operator
// call on them.
class Bench {
 public:
  Bench(const CsrMatrix& csr, int n) : csr_(csr), n_(n) {
    CUDA_CALL(cudaDeviceSynchronize());
    const auto t0 = std::chrono::steady_clock::now();
    matrix_ = std::make_unique<PowerSparse::PowerSparseMatrixGPU>(csr.rows, csr.cols, csr.nnz(), csr.row_ptr.data(),
                                                                  csr.col_ind.data(), csr.values.data());
    CUDA_CALL(cudaDeviceSynchronize());
    preprocess_ms_ = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    const int S = matrix_->GroupTypeNum();
    residue_offset_ = host_copy(matrix_->ResidueOffset(), std::size_t(matrix_->GroupNum()[0]) + 1);
    std::mt19937 draw(kDenseSeed);
    auto fill = [&draw](std::size_t count) {
      std::vector<float> v(count);
      std::generate(v.begin(), v.end(), [&draw] { return float(draw() % 3) / 10.0f; });
      return v;
    };
    if (kIsSddmm) lhs_ = fill(std::size_t(csr.rows) * n);
    rhs_ = fill(std::size_t(csr.cols) * n);
    d_lhs_ = device_copy(lhs_);
    d_rhs_ = device_copy(rhs_);
    if (kIsSddmm) {
      for (int s = 0; s < S; ++s) {
        outputs_.push_back(device_alloc<float>(workset_elems(s)));
        output_ptrs_.push_back(outputs_.back().get());
      }
    } else {
      outputs_.push_back(device_alloc<float>(std::size_t(csr.rows) * n));
    }
    streams_.assign(std::size_t(S), nullptr);
    if (S > 1)
      for (auto& s : streams_) CUDA_CALL(cudaStreamCreate(&s));
  }
  ~Bench() {
    for (auto s : streams_)
      if (s) cudaStreamDestroy(s);
  }
  Bench(const Bench&) = delete;
  Bench& operator=(const Bench&) = delete;

  double preprocess_ms() const { return preprocess_ms_; }

  std::size_t workset_elems(int s) const {
    return s == 0 ? std::size_t(residue_offset_.back()) : std::size_t(matrix_->GroupNum()[s]) * GROUP_SIZE(s);
  }

  void clear_outputs() {
    for (int i = 0; i < int(outputs_.size()); ++i) {
      const std::size_t count = kIsSddmm ? workset_elems(i) : std::size_t(csr_.rows) * n_;
      if (count) CUDA_CALL(cudaMemset(outputs_[i].get(), 0, count * sizeof(float)));
    }
    CUDA_CALL(cudaDeviceSynchronize());
  }

  void call() {
    const int S = int(streams_.size());
    if (kIsSddmm)
      PowerSparse::SDDMM(*matrix_, n_, d_lhs_.get(), d_rhs_.get(), output_ptrs_.data(), S, streams_.data());
    else
      PowerSparse::SpMM(*matrix_, n_, d_rhs_.get(), outputs_[0].get(), S, streams_.data());
  }

  // CHECK=1: the layout and one operator call.
  void verify() {
    verify_layout();
    clear_outputs();
    call();
    CUDA_CALL(cudaDeviceSynchronize());
    if (kIsSddmm) verify_sddmm();
    else verify_spmm();
  }

 private:
  struct Group {  // one group of the layout: destination row and element range
    int row;
    std::size_t begin, end;
  };
  std::vector<Group> groups_of(int s) const {
    const int count = matrix_->GroupNum()[s];
    const std::vector<int> rows = host_copy(matrix_->GroupDestination()[s], std::size_t(count));
    std::vector<Group> g(static_cast<std::size_t>(count));
    for (int i = 0; i < count; ++i) {
      const std::size_t b = s == 0 ? std::size_t(residue_offset_[i]) : std::size_t(i) * GROUP_SIZE(s);
      const std::size_t e = s == 0 ? std::size_t(residue_offset_[i + 1]) : b + GROUP_SIZE(s);
      g[std::size_t(i)] = {rows[std::size_t(i)], b, e};
    }
    return g;
  }

  // Every row of the layout, gathered from all worksets, must hold the same
  // (column, value bits) multiset as the input row.
  void verify_layout() const {
    const int rows = csr_.rows;
    std::vector<long long> start(std::size_t(rows) + 1, 0);
    std::vector<std::vector<Group>> all;
    std::vector<std::vector<int>> cols;
    std::vector<std::vector<float>> vals;
    for (int s = 0; s < matrix_->GroupTypeNum(); ++s) {
      all.push_back(groups_of(s));
      cols.push_back(host_copy(matrix_->WorksetColInd()[s], workset_elems(s)));
      vals.push_back(host_copy(matrix_->WorksetSpData()[s], workset_elems(s)));
      for (const Group& g : all.back()) {
        if (g.row < 0 || g.row >= rows) throw std::runtime_error("Preprocessing changed the sparse matrix");
        start[std::size_t(g.row) + 1] += (long long)(g.end - g.begin);
      }
    }
    for (int r = 0; r < rows; ++r) start[std::size_t(r) + 1] += start[std::size_t(r)];
    if (start.back() != csr_.nnz()) throw std::runtime_error("Preprocessing changed the sparse matrix");
    std::vector<std::pair<int, uint32_t>> laid(std::size_t(csr_.nnz()));
    std::vector<long long> cursor(start.begin(), start.end() - 1);
    for (std::size_t s = 0; s < all.size(); ++s)
      for (const Group& g : all[s])
        for (std::size_t p = g.begin; p < g.end; ++p) {
          uint32_t bits;
          std::memcpy(&bits, &vals[s][p], 4);
          laid[std::size_t(cursor[std::size_t(g.row)]++)] = {cols[s][p], bits};
        }
    std::vector<std::pair<int, uint32_t>> given;
    for (int r = 0; r < rows; ++r) {
      const auto b = laid.begin() + start[std::size_t(r)], e = laid.begin() + start[std::size_t(r) + 1];
      given.clear();
      for (int p = csr_.row_ptr[r]; p < csr_.row_ptr[r + 1]; ++p) {
        uint32_t bits;
        std::memcpy(&bits, &csr_.values[std::size_t(p)], 4);
        given.emplace_back(csr_.col_ind[std::size_t(p)], bits);
      }
      std::sort(b, e);
      std::sort(given.begin(), given.end());
      if (!std::equal(b, e, given.begin(), given.end()))
        throw std::runtime_error("Preprocessing changed the sparse matrix");
    }
  }

  static bool near(float got, double want) {
    return std::isfinite(got) && std::isfinite(want) && std::abs(double(got) - want) <= kCheckTol * (1.0 + std::abs(want));
  }

  void verify_spmm() const {
    const std::vector<float> out = host_copy(outputs_[0].get(), std::size_t(csr_.rows) * n_);
    std::vector<double> acc(static_cast<std::size_t>(n_));
    for (int r = 0; r < csr_.rows; ++r) {
      std::fill(acc.begin(), acc.end(), 0.0);
      for (int p = csr_.row_ptr[r]; p < csr_.row_ptr[r + 1]; ++p) {
        const float* b = rhs_.data() + std::size_t(csr_.col_ind[std::size_t(p)]) * n_;
        const double v = csr_.values[std::size_t(p)];
        for (int j = 0; j < n_; ++j) acc[std::size_t(j)] += v * b[j];
      }
      const float* got = out.data() + std::size_t(r) * n_;
      for (int j = 0; j < n_; ++j)
        if (!near(got[j], acc[std::size_t(j)]))
          throw std::runtime_error("SpMM mismatch at row " + std::to_string(r) + ", feature " + std::to_string(j));
    }
  }

  void verify_sddmm() const {
    for (int s = 0; s < matrix_->GroupTypeNum(); ++s) {
      const std::vector<int> cols = host_copy(matrix_->WorksetColInd()[s], workset_elems(s));
      const std::vector<float> vals = host_copy(matrix_->WorksetSpData()[s], workset_elems(s));
      const std::vector<float> out = host_copy(output_ptrs_[std::size_t(s)], workset_elems(s));
      for (const Group& g : groups_of(s)) {
        const float* x = lhs_.data() + std::size_t(g.row) * n_;
        for (std::size_t p = g.begin; p < g.end; ++p) {
          const float* y = rhs_.data() + std::size_t(cols[p]) * n_;
          double dot = 0.0;
          for (int j = 0; j < n_; ++j) dot += double(x[j]) * y[j];
          if (!near(out[p], dot * vals[p]))
            throw std::runtime_error("SDDMM mismatch in workset " + std::to_string(s) + ", position " +
                                     std::to_string(p));
        }
      }
    }
  }

  const CsrMatrix& csr_;
  int n_;
  std::unique_ptr<PowerSparse::PowerSparseMatrixGPU> matrix_;
  double preprocess_ms_ = 0.0;
  std::vector<int> residue_offset_;
  std::vector<float> lhs_, rhs_;
  DevicePtr<float> d_lhs_, d_rhs_;
  std::vector<DevicePtr<float>> outputs_;
  std::vector<float*> output_ptrs_;
  std::vector<cudaStream_t> streams_;
};

// Average milliseconds of `repeats` back-to-back calls between two events.
double time_calls(Bench& bench, int repeats) {
  cudaEvent_t ev[2];
  CUDA_CALL(cudaEventCreate(&ev[0]));
  CUDA_CALL(cudaEventCreate(&ev[1]));
  float total = 0.f;
  CUDA_CALL(cudaEventRecord(ev[0]));
  for (int i = 0; i < repeats; ++i) bench.call();  // outputs accumulate, as in the reference harness
  CUDA_CALL(cudaEventRecord(ev[1]));
  CUDA_CALL(cudaEventSynchronize(ev[1]));
  CUDA_CALL(cudaEventElapsedTime(&total, ev[0], ev[1]));
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  return double(total) / repeats;
}

int benchmark(const Args& a) {
  if (a.device < 0 || (a.check != 0 && a.check != 1) || a.repeats <= 0)
    throw std::invalid_argument("DEVICE must be nonnegative, CHECK 0 or 1, and REPEATS positive");
  CUDA_CALL(cudaSetDevice(a.device));
  CUDA_CALL(cudaFree(nullptr));
  cudaDeviceProp prop{};
  CUDA_CALL(cudaGetDeviceProperties(&prop, a.device));
  if (prop.major < 10) throw std::runtime_error("These kernels require an sm_100 (Blackwell B200) GPU");
  int runtime = 0, driver = 0;
  CUDA_CALL(cudaRuntimeGetVersion(&runtime));
  CUDA_CALL(cudaDriverGetVersion(&driver));
  std::cerr << kOpName << ": " << a.matrix << ", N=" << a.n << ", GPU=" << prop.name << '\n';

  const CsrMatrix csr = ReadMatrixMarket(a.matrix);
  Bench bench(csr, a.n);
  bench.clear_outputs();
  if (a.check) {
    bench.verify();
    std::cerr << "Preprocessing and CPU reference checks passed (atol=rtol=1e-3).\n";
    bench.clear_outputs();
  }
  for (int i = 0; i < kWarmupCalls; ++i) bench.call();
  CUDA_CALL(cudaDeviceSynchronize());
  bench.clear_outputs();
  const double ms = time_calls(bench, a.repeats);
  if (!(ms > 0) || !std::isfinite(ms)) throw std::runtime_error("Invalid measured latency");

  std::ostringstream row;
  row << std::setprecision(10) << "PowerSparse," << kOpName << ',' << quoted(a.matrix) << ',' << csr.rows << ','
      << csr.cols << ',' << csr.nnz() << ',' << a.n << ',' << a.device << ',' << quoted(prop.name) << ','
      << prop.major << '.' << prop.minor << ',' << runtime << ',' << driver << ',' << kWarmupCalls << ','
      << a.repeats << ',' << kDenseSeed << ',' << (a.check ? "passed" : "skipped") << ',' << bench.preprocess_ms()
      << ',' << ms << ',' << 2.0 * csr.nnz() * a.n / (ms * 1e6);
  std::cout << row.str() << '\n';
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    if (argc == 2 && std::strcmp(argv[1], "--header") == 0) {
      std::cout << csv_header() << '\n';
      return 0;
    }
    if (argc != 6) {
      usage(argv[0]);
      return 2;
    }
    Args a;
    a.matrix = argv[1];
    a.n = to_int(argv[2], "N");
    if (a.n != 32 && a.n != 128) {
      std::cerr << kOpName << " benchmark: N=" << a.n << " was not selected in main; please use N=32 or N=128.\n";
      return 2;
    }
    a.device = to_int(argv[3], "DEVICE");
    a.check = to_int(argv[4], "CHECK");
    a.repeats = to_int(argv[5], "REPEATS");
    return benchmark(a);
  } catch (const std::exception& e) {
    std::cerr << "Error: " << e.what() << '\n';
    return 1;
  }
}
