// Layout cache: the preprocessed matrix written to / read from a file, so that a
// repeated run skips the preprocessing (a few hundred ms to seconds per matrix).
// No reference counterpart: the reference rebuilds the layout in every
// PowerSparseMatrixGPU constructor (utils/matrix_utils.cu:470-663).
//
// File (little-endian, no padding):
//   char[8]  magic "PSLAYT01"
//   int32    rows, cols, nnz, S, fine, sm_count, signature_len
//   int32    group_num[S]
//   int64    ws_size[S]
//   per workset s:  int32 col_ind[ws_size[s]], float sp_data[ws_size[s]],
//                   int32 group_des[group_num[s]], int32 csr_pos[ws_size[s]]
//   int32    residue_offset[group_num[0] + 1]
//   uint8    residue_atomic[group_num[0]]
// The layout arrays are the reference's, bit for bit; the residue rows, wide rows
// and task lists are derived again on load (finish_matrix).
#include "ps_common.cuh"
#include "ps_matrix.h"

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace psb {
namespace {

constexpr char kMagic[8] = {'P', 'S', 'L', 'A', 'Y', 'T', '0', '1'};

struct File {
  std::FILE* f = nullptr;
  std::string path;
  File(const std::string& p, const char* mode) : f(std::fopen(p.c_str(), mode)), path(p) {}
  ~File() {
    if (f) std::fclose(f);
  }
};

void put(File& out, const void* data, size_t bytes) {
  if (bytes && std::fwrite(data, 1, bytes, out.f) != bytes)
    throw std::runtime_error("Cannot write the layout file " + out.path);
}

void get(File& in, void* data, size_t bytes) {
  if (bytes && std::fread(data, 1, bytes, in.f) != bytes)
    throw std::invalid_argument("Truncated layout file " + in.path);
}

template <typename T>
void put_device(File& out, const T* d, long long count) {
  if (count <= 0) return;
  std::vector<T> h(static_cast<size_t>(count));
  PSB_CUDA(cudaMemcpy(h.data(), d, sizeof(T) * h.size(), cudaMemcpyDeviceToHost));
  put(out, h.data(), sizeof(T) * h.size());
}

template <typename T>
std::vector<T> get_vector(File& in, long long count) {
  std::vector<T> h(static_cast<size_t>(count > 0 ? count : 0));
  get(in, h.data(), sizeof(T) * h.size());
  return h;
}

template <typename T>
T* upload(const std::vector<T>& h) {
  if (h.empty()) return nullptr;
  DeviceArray<T> d(h.size());
  PSB_CUDA(cudaMemcpy(d.get(), h.data(), sizeof(T) * h.size(), cudaMemcpyHostToDevice));
  return d.release_ownership();
}

// File -> device through two pinned staging buffers: the read of one chunk
// overlaps the copy of the previous one.
class Stager {
 public:
  static constexpr size_t kChunkBytes = size_t(32) << 20;
  explicit Stager(File& in) : in_(in) {
    PSB_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    for (int i = 0; i < 2; ++i) PSB_CUDA(cudaEventCreateWithFlags(&done_[i], cudaEventDisableTiming));
    PSB_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&buf_), 2 * kChunkBytes, cudaHostAllocDefault));
  }
  ~Stager() {
    if (stream_) cudaStreamSynchronize(stream_);
    cudaFreeHost(buf_);
    for (auto e : done_)
      if (e) cudaEventDestroy(e);
    if (stream_) cudaStreamDestroy(stream_);
  }
  Stager(const Stager&) = delete;
  Stager& operator=(const Stager&) = delete;

  template <typename T>
  T* read(long long count) {
    if (count <= 0) return nullptr;
    DeviceArray<T> d(static_cast<size_t>(count));
    const size_t bytes = sizeof(T) * size_t(count);
    try {
      for (size_t at = 0; at < bytes; at += kChunkBytes) {
        const size_t n = std::min(kChunkBytes, bytes - at);
        char* b = buf_ + cur_ * kChunkBytes;
        PSB_CUDA(cudaEventSynchronize(done_[cur_]));  // this buffer's previous copy has finished
        get(in_, b, n);
        PSB_CUDA(cudaMemcpyAsync(reinterpret_cast<char*>(d.get()) + at, b, n, cudaMemcpyHostToDevice, stream_));
        PSB_CUDA(cudaEventRecord(done_[cur_], stream_));
        cur_ ^= 1;
      }
    } catch (...) {
      cudaStreamSynchronize(stream_);  // no copy into `d` may outlive it
      throw;
    }
    return d.release_ownership();
  }
  void finish() { PSB_CUDA(cudaStreamSynchronize(stream_)); }
  cudaStream_t stream() const { return stream_; }

 private:
  File& in_;
  cudaStream_t stream_ = nullptr;
  cudaEvent_t done_[2] = {nullptr, nullptr};
  char* buf_ = nullptr;
  int cur_ = 0;
};

// Error bits of the device-side validation.
enum : int { kBadColumn = 1, kBadRow = 2, kBadPosition = 4, kRepeatedPosition = 8 };

__global__ void check_range(const int* __restrict__ v, long long n, int hi, int bit, int* __restrict__ bad) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int x = v[i];
    if (x < 0 || x >= hi) atomicOr(bad, bit);
  }
}

// Positions must be a permutation of [0, nnz): in range and each set once.
__global__ void mark_positions(const int* __restrict__ pos, long long n, int nnz, unsigned* __restrict__ seen,
                               int* __restrict__ bad) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int p = pos[i];
    if (p < 0 || p >= nnz) {
      atomicOr(bad, kBadPosition);
      continue;
    }
    const unsigned bit = 1u << (p & 31);
    if (atomicOr(&seen[p >> 5], bit) & bit) atomicOr(bad, kRepeatedPosition);
  }
}

unsigned blocks_for(long long n) { return unsigned(std::max<long long>(1, std::min<long long>((n + 255) / 256, 8LL * device_sms()))); }

}  // namespace

void save_matrix(const Matrix& m, const std::string& path) {
  File out(path, "wb");
  if (!out.f) throw std::invalid_argument("Cannot open the layout file " + path + " for writing");
  put(out, kMagic, sizeof(kMagic));
  const int head[7] = {m.rows, m.cols, m.nnz, m.S, m.fine, m.sm_count, m.signature_len};
  put(out, head, sizeof(head));
  put(out, m.group_num.data(), sizeof(int) * size_t(m.S));
  put(out, m.ws_size.data(), sizeof(long long) * size_t(m.S));
  for (int s = 0; s < m.S; ++s) {
    put_device(out, m.col_ind[s], m.ws_size[s]);
    put_device(out, m.sp_data[s], m.ws_size[s]);
    put_device(out, m.group_des[s], m.group_num[s]);
    put_device(out, m.csr_pos[s], m.ws_size[s]);
  }
  put_device(out, m.residue_offset, (long long)m.group_num[0] + 1);
  put_device(out, reinterpret_cast<const unsigned char*>(m.residue_atomic), m.group_num[0]);
  if (std::fflush(out.f) != 0) throw std::runtime_error("Cannot write the layout file " + path);
}

Matrix* load_matrix(const std::string& path) {
  const auto t0 = std::chrono::steady_clock::now();
  File in(path, "rb");
  if (!in.f) throw std::invalid_argument("Cannot open the layout file " + path);
  char magic[8];
  get(in, magic, sizeof(magic));
  if (std::memcmp(magic, kMagic, sizeof(kMagic)) != 0)
    throw std::invalid_argument("Not a PowerSparse layout file: " + path);
  int head[7];
  get(in, head, sizeof(head));
  std::unique_ptr<Matrix> m(new Matrix());
  m->rows = head[0];
  m->cols = head[1];
  m->nnz = head[2];
  m->S = head[3];
  m->fine = head[4];
  m->sm_count = head[5];
  m->signature_len = head[6];
  const int S = m->S;
  // Group sizes 32 << (s - 1) fit an int for s <= 26, the most build_matrix makes.
  if (m->rows <= 0 || m->cols <= 0 || m->nnz <= 0 || S < 1 || S > 27 || m->fine != kFineGroupSize)
    throw std::invalid_argument("Corrupt layout file header: " + path);
  PSB_CUDA(cudaGetDevice(&m->device));
  m->group_num.resize(S);
  m->ws_size.resize(S);
  get(in, m->group_num.data(), sizeof(int) * size_t(S));
  get(in, m->ws_size.data(), sizeof(long long) * size_t(S));
  long long total = 0;
  for (int s = 0; s < S; ++s) {
    const long long expect = s == 0 ? -1 : (long long)m->group_num[s] * group_size(s);
    if (m->group_num[s] < 0 || m->ws_size[s] < 0 || (s > 0 && m->ws_size[s] != expect))
      throw std::invalid_argument("Corrupt layout file header: " + path);
    total += m->ws_size[s];
  }
  if (total != m->nnz) throw std::invalid_argument("Corrupt layout file header: " + path);
  m->col_ind.assign(S, nullptr);
  m->sp_data.assign(S, nullptr);
  m->group_des.assign(S, nullptr);
  m->csr_pos.assign(S, nullptr);
  {
    // Arrays go to the device as read; the checks run there before any operator
    // can see them (the matrix is freed if one fails).
    Stager stager(in);
    for (int s = 0; s < S; ++s) {
      m->col_ind[s] = stager.read<int>(m->ws_size[s]);
      m->sp_data[s] = stager.read<float>(m->ws_size[s]);
      m->group_des[s] = stager.read<int>(m->group_num[s]);
      m->csr_pos[s] = stager.read<int>(m->ws_size[s]);
    }
    stager.finish();
    DeviceArray<int> bad(1);
    DeviceArray<unsigned> seen((size_t(m->nnz) + 31) / 32);
    cudaStream_t st = stager.stream();
    PSB_CUDA(cudaMemsetAsync(bad.get(), 0, sizeof(int), st));
    PSB_CUDA(cudaMemsetAsync(seen.get(), 0, sizeof(unsigned) * ((size_t(m->nnz) + 31) / 32), st));
    for (int s = 0; s < S; ++s) {
      if (m->ws_size[s] > 0) {
        check_range<<<blocks_for(m->ws_size[s]), 256, 0, st>>>(m->col_ind[s], m->ws_size[s], m->cols, kBadColumn,
                                                               bad.get());
        mark_positions<<<blocks_for(m->ws_size[s]), 256, 0, st>>>(m->csr_pos[s], m->ws_size[s], m->nnz, seen.get(),
                                                                  bad.get());
      }
      if (m->group_num[s] > 0)
        check_range<<<blocks_for(m->group_num[s]), 256, 0, st>>>(m->group_des[s], m->group_num[s], m->rows, kBadRow,
                                                                 bad.get());
      PSB_LAUNCH_CHECK();
    }
    int h_bad = 0;
    PSB_CUDA(cudaMemcpyAsync(&h_bad, bad.get(), sizeof(int), cudaMemcpyDeviceToHost, st));
    stager.finish();
    if (h_bad & kBadColumn) throw std::invalid_argument("Corrupt layout file (column index): " + path);
    if (h_bad & kBadRow) throw std::invalid_argument("Corrupt layout file (group destination): " + path);
    if (h_bad & (kBadPosition | kRepeatedPosition))
      throw std::invalid_argument("Corrupt layout file (CSR position): " + path);
  }
  const int G0 = m->group_num[0];
  const std::vector<int> h_res_off = get_vector<int>(in, (long long)G0 + 1);
  std::vector<unsigned char> atomic = get_vector<unsigned char>(in, G0);
  for (auto& a : atomic) a = a ? 1 : 0;  // stored as bool on the device
  const int max_group = S == 1 ? m->fine : 31;
  if (h_res_off.front() != 0 || h_res_off.back() != m->ws_size[0])
    throw std::invalid_argument("Corrupt layout file (residue offsets): " + path);
  for (int g = 0; g < G0; ++g) {
    const int size = h_res_off[g + 1] - h_res_off[g];
    if (size < 1 || size > max_group) throw std::invalid_argument("Corrupt layout file (residue offsets): " + path);
  }
  m->residue_offset = upload(h_res_off);
  m->residue_atomic = reinterpret_cast<bool*>(upload(atomic));
  char extra;
  if (std::fread(&extra, 1, 1, in.f) != 0) throw std::invalid_argument("Trailing data in layout file " + path);
  finish_matrix(*m, h_res_off);
  m->preprocess_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  return m.release();
}

}  // namespace psb
