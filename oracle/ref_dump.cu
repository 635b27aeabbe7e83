// Harness around the reference library (TEST INFRASTRUCTURE ONLY).
//
// Links the reference's own PowerSparseMatrixGPU / SpMM / SDDMM (built from its
// sources by oracle/Makefile) and writes what they produce, so that golden
// fixtures and the reference's GPU timings come from the reference itself.
//
//   ps_ref_dump layout IN.csr OUTDIR
//   ps_ref_dump spmm   IN.csr N B.f32 OUT.f32 [REPEATS]
//   ps_ref_dump sddmm  IN.csr N LHS.f32 RHS.f32 OUTPREFIX [REPEATS]
//
// IN.csr is the binary CSR written by powersparse_b200.synth.write_csr_bin.  A
// dense operand given as "@rand:SEED" is generated on the device instead of read
// (uniform in [-1, 1) from a counter hash; for timing runs), and an output path
// "-" writes nothing.
// With REPEATS > 0 the operator is also timed the way benchmarks/benchmark.cu
// does it (30 warm-up calls, outputs zeroed, REPEATS back-to-back calls under
// one event pair) and one JSON line is printed.
#include "PowerSparse_SDDMM/PowerSparse_SDDMM.h"
#include "PowerSparse_SpMM/PowerSparse_SpMM.h"
#include "utils/cuda_utils.h"

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

struct Csr {
  int64_t rows = 0, cols = 0, nnz = 0;
  std::vector<int> row_ptr, col_ind;
  std::vector<float> values;
};

Csr read_csr(const std::string& path) {
  std::ifstream in(path, std::ios::binary);
  if (!in) throw std::runtime_error("cannot open " + path);
  char magic[8];
  in.read(magic, 8);
  if (std::memcmp(magic, "PSCSR001", 8) != 0) throw std::runtime_error("bad CSR magic");
  Csr m;
  in.read(reinterpret_cast<char*>(&m.rows), 8);
  in.read(reinterpret_cast<char*>(&m.cols), 8);
  in.read(reinterpret_cast<char*>(&m.nnz), 8);
  m.row_ptr.resize(m.rows + 1);
  m.col_ind.resize(m.nnz);
  m.values.resize(m.nnz);
  in.read(reinterpret_cast<char*>(m.row_ptr.data()), 4 * (m.rows + 1));
  in.read(reinterpret_cast<char*>(m.col_ind.data()), 4 * m.nnz);
  in.read(reinterpret_cast<char*>(m.values.data()), 4 * m.nnz);
  if (!in) throw std::runtime_error("truncated CSR " + path);
  return m;
}

template <typename T>
std::vector<T> read_raw(const std::string& path, size_t count) {
  std::vector<T> v(count);
  std::ifstream in(path, std::ios::binary);
  if (!in) throw std::runtime_error("cannot open " + path);
  in.read(reinterpret_cast<char*>(v.data()), sizeof(T) * count);
  if (!in) throw std::runtime_error("short file " + path);
  return v;
}

template <typename T>
void write_raw(const std::string& path, const T* data, size_t count) {
  std::ofstream out(path, std::ios::binary);
  out.write(reinterpret_cast<const char*>(data), sizeof(T) * count);
  if (!out) throw std::runtime_error("cannot write " + path);
}

template <typename T>
std::vector<T> download(const T* d, size_t count) {
  std::vector<T> h(count);
  if (count) CUDA_CALL(cudaMemcpy(h.data(), d, sizeof(T) * count, cudaMemcpyDeviceToHost));
  return h;
}

template <typename T>
T* upload(const std::vector<T>& h) {
  T* d = nullptr;
  CUDA_CALL(cudaMalloc(&d, sizeof(T) * (h.empty() ? 1 : h.size())));
  if (!h.empty()) CUDA_CALL(cudaMemcpy(d, h.data(), sizeof(T) * h.size(), cudaMemcpyHostToDevice));
  return d;
}

// Counter hash (splitmix64 finalizer) to [-1, 1): dense operands for timing runs.
__global__ void fill_uniform(float* out, size_t count, unsigned long long seed) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < count; i += size_t(gridDim.x) * blockDim.x) {
    unsigned long long z = i + 0x9E3779B97F4A7C15ull * (seed + 1);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    out[i] = float((z >> 40) * (1.0 / 16777216.0)) * 2.0f - 1.0f;
  }
}

float* dense_input(const std::string& spec, size_t count) {
  if (spec.rfind("@rand:", 0) == 0) {
    float* d = nullptr;
    CUDA_CALL(cudaMalloc(&d, sizeof(float) * (count ? count : 1)));
    fill_uniform<<<1024, 256>>>(d, count, std::stoull(spec.substr(6)));
    CUDA_CALL(cudaGetLastError());
    CUDA_CALL(cudaDeviceSynchronize());
    return d;
  }
  return upload(read_raw<float>(spec, count));
}

size_t workset_size(const PowerSparse::PowerSparseMatrixGPU& m, int s, const std::vector<int>& res) {
  return s == 0 ? size_t(res.back()) : size_t(m.GroupNum()[s]) * GROUP_SIZE(s);
}

struct Streams {
  std::vector<cudaStream_t> s;
  explicit Streams(int count) : s(count, nullptr) {
    if (count > 1) for (auto& x : s) CUDA_CALL(cudaStreamCreate(&x));
  }
  ~Streams() { for (auto x : s) if (x) cudaStreamDestroy(x); }
};

int run(int argc, char** argv) {
  if (argc < 4) {
    std::cerr << "usage: ps_ref_dump {layout|spmm|sddmm} IN.csr ...\n";
    return 2;
  }
  const std::string mode = argv[1];
  const Csr csr = read_csr(argv[2]);
  CUDA_CALL(cudaFree(nullptr));
  CUDA_CALL(cudaDeviceSynchronize());
  const auto t0 = std::chrono::steady_clock::now();
  PowerSparse::PowerSparseMatrixGPU m(int(csr.rows), int(csr.cols), int(csr.nnz), csr.row_ptr.data(),
                                      csr.col_ind.data(), csr.values.data());
  CUDA_CALL(cudaDeviceSynchronize());
  const double pre_ms =
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  const int S = m.GroupTypeNum();
  const auto res = download(m.ResidueOffset(), size_t(m.GroupNum()[0]) + 1);

  if (mode == "layout") {
    const std::string dir = argv[3];
    std::ofstream meta(dir + "/meta.txt");
    meta << S << ' ' << m.GroupFineSize();
    for (int s = 0; s < S; ++s) meta << ' ' << m.GroupNum()[s];
    meta << '\n';
    for (int s = 0; s < S; ++s) {
      const size_t n = workset_size(m, s, res);
      const auto col = download(m.WorksetColInd()[s], n);
      const auto val = download(m.WorksetSpData()[s], n);
      const auto des = download(m.GroupDestination()[s], size_t(m.GroupNum()[s]));
      write_raw(dir + "/ws" + std::to_string(s) + ".col.i32", col.data(), col.size());
      write_raw(dir + "/ws" + std::to_string(s) + ".val.f32", val.data(), val.size());
      write_raw(dir + "/ws" + std::to_string(s) + ".des.i32", des.data(), des.size());
    }
    write_raw(dir + "/res_off.i32", res.data(), res.size());
    std::vector<unsigned char> atomic(m.GroupNum()[0]);
    if (!atomic.empty()) {
      static_assert(sizeof(bool) == 1, "bool flags are copied bytewise");
      CUDA_CALL(cudaMemcpy(atomic.data(), m.ResidueAtomic(), atomic.size(), cudaMemcpyDeviceToHost));
      for (auto& a : atomic) a = a ? 1 : 0;
    }
    write_raw(dir + "/res_atomic.u8", atomic.data(), atomic.size());
    std::printf("{\"mode\":\"layout\",\"S\":%d,\"preprocess_ms\":%.3f}\n", S, pre_ms);
    return 0;
  }

  Streams streams(S);
  const int n = std::stoi(argv[3]);
  int repeats = 0;
  std::vector<float*> outs;
  std::vector<size_t> out_sizes;
  float* d_lhs = nullptr;
  float* d_rhs = nullptr;
  float* d_c = nullptr;
  std::function<void()> invoke;
  std::string out_path;
  if (mode == "spmm") {
    if (argc < 6) return 2;
    d_rhs = dense_input(argv[4], size_t(csr.cols) * n);
    out_path = argv[5];
    if (argc > 6) repeats = std::stoi(argv[6]);
    CUDA_CALL(cudaMalloc(&d_c, sizeof(float) * size_t(csr.rows) * n));
    outs.push_back(d_c);
    out_sizes.push_back(size_t(csr.rows) * n);
    invoke = [&] { PowerSparse::SpMM(m, n, d_rhs, d_c, S, streams.s.data()); };
  } else if (mode == "sddmm") {
    if (argc < 7) return 2;
    d_lhs = dense_input(argv[4], size_t(csr.rows) * n);
    d_rhs = dense_input(argv[5], size_t(csr.cols) * n);
    out_path = argv[6];
    if (argc > 7) repeats = std::stoi(argv[7]);
    for (int s = 0; s < S; ++s) {
      const size_t cnt = workset_size(m, s, res);
      float* d = nullptr;
      if (cnt) CUDA_CALL(cudaMalloc(&d, sizeof(float) * cnt));
      outs.push_back(d);
      out_sizes.push_back(cnt);
    }
    invoke = [&] { PowerSparse::SDDMM(m, n, d_lhs, d_rhs, outs.data(), S, streams.s.data()); };
  } else {
    return 2;
  }
  auto reset = [&] {
    for (size_t i = 0; i < outs.size(); ++i)
      if (out_sizes[i]) CUDA_CALL(cudaMemset(outs[i], 0, sizeof(float) * out_sizes[i]));
    CUDA_CALL(cudaDeviceSynchronize());
  };
  reset();
  invoke();
  CUDA_CALL(cudaDeviceSynchronize());
  if (out_path == "-") {
    // timing run: nothing written
  } else if (mode == "spmm") {
    const auto c = download(d_c, out_sizes[0]);
    write_raw(out_path, c.data(), c.size());
  } else {
    for (int s = 0; s < S; ++s) {
      const auto o = download(outs[s], out_sizes[s]);
      write_raw(out_path + ".ws" + std::to_string(s) + ".f32", o.data(), o.size());
    }
  }
  double ms = 0;
  if (repeats > 0) {
    for (int i = 0; i < 30; ++i) invoke();
    CUDA_CALL(cudaDeviceSynchronize());
    reset();
    cudaEvent_t a, b;
    CUDA_CALL(cudaEventCreate(&a));
    CUDA_CALL(cudaEventCreate(&b));
    CUDA_CALL(cudaEventRecord(a));
    for (int i = 0; i < repeats; ++i) invoke();
    CUDA_CALL(cudaEventRecord(b));
    CUDA_CALL(cudaEventSynchronize(b));
    float t = 0;
    CUDA_CALL(cudaEventElapsedTime(&t, a, b));
    ms = double(t) / repeats;
  }
  std::printf(
      "{\"mode\":\"%s\",\"N\":%d,\"S\":%d,\"rows\":%lld,\"cols\":%lld,\"nnz\":%lld,"
      "\"preprocess_ms\":%.3f,\"repeats\":%d,\"ms\":%.6f,\"gflops\":%.3f}\n",
      mode.c_str(), n, S, (long long)csr.rows, (long long)csr.cols, (long long)csr.nnz, pre_ms,
      repeats, ms, repeats > 0 ? 2.0 * double(csr.nnz) * n / (ms * 1e6) : 0.0);
  for (auto p : outs) cudaFree(p);
  cudaFree(d_lhs);
  cudaFree(d_rhs);
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    return run(argc, argv);
  } catch (const std::exception& e) {
    std::cerr << "Error: " << e.what() << '\n';
    return 1;
  }
}
