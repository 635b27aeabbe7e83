// GPU preprocessing: host CSR -> PowerSparse block/residue worksets (sm_100a).
//
// Produces, bit for bit, the layout of the reference constructor
// PowerSparseMatrixGPU::PowerSparseMatrixGPU (utils/matrix_utils.cu:470-663):
//
//   step                               reference                  here
//   S from the SM count                AnalyzeMatrix :31-63        workset_size_counts (1 pass)
//   column histogram                   host OpenMP :508-514        col_histogram
//   (row asc, col_nnz desc) stable     thrust::sort NNZPoint :522  64-bit key LSD radix sort
//   groups per workset / metadata      host loops :132-208         row_group_counts + scans + scatter
//   column -> signature bit            GenerateSigBit :65-128      same host std::sort call
//   group signatures                   Get*Signature :261-327      group_signatures (all worksets)
//   signature order (stable, per word) thrust::stable_sort :590    32-bit key LSD radix per word
//   per-group column order (stable)    thrust::sort NNZPoint2 :616 (group, col) key LSD radix sort
//   permuted offsets / final arrays    :451-464, :619-656          permute + gather kernels
//
// Every reference sort is stable with an integer key, so each becomes a radix
// sort over exactly the bits in use; the resulting orders are identical.
#include "ps_common.cuh"
#include "ps_matrix.h"
#include "ps_ops.h"
#include "ps_sort.cuh"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <future>
#include <limits>
#include <memory>
#include <mutex>
#include <numeric>
#include <stdexcept>
#include <string>
#include <thread>
#include <utility>

namespace psb {

Matrix::~Matrix() {
  for (auto p : col_ind) cudaFree(p);
  for (auto p : sp_data) cudaFree(p);
  for (auto p : group_des) cudaFree(p);
  for (auto p : csr_pos) cudaFree(p);
  cudaFree(residue_offset);
  cudaFree(residue_atomic);
  for (auto p : block_tasks) cudaFree(p);
  for (auto p : residue_tasks) cudaFree(p);
  cudaFree(residue_row);
  cudaFree(row_ptr);
  cudaFree(wide_row);
  cudaFree(wide_acc);
  for (auto p : wide_acc_retired) cudaFree(p);
  if (wide_ready) cudaEventDestroy(wide_ready);
  for (auto p : push_count) cudaFree(p);
  cudaFree(push_pending);
  cudaFree(quiet_rows);
  if (push_ready) cudaEventDestroy(push_ready);
}

namespace {

constexpr int kSizeClasses = 26;  // group sizes 32 << k, k < 26, cover every 32-bit row length

struct WorksetArrays {
  int* des[kMaxWorksets];
  int* start[kMaxWorksets];
  uint32_t* sig[kMaxWorksets];
  int groups[kMaxWorksets];
};

__device__ __forceinline__ int dev_group_size(int s) { return 32 << (s - 1); }

// Sum over rows of floor(len / (32 << k)) for every k (AnalyzeMatrix's counts).
__global__ void workset_size_counts(const int* __restrict__ row_ptr, int rows,
                                    unsigned long long* __restrict__ counts) {
  unsigned long long local[kSizeClasses];
#pragma unroll
  for (int k = 0; k < kSizeClasses; ++k) local[k] = 0;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const unsigned len = unsigned(row_ptr[r + 1] - row_ptr[r]);
#pragma unroll
    for (int k = 0; k < kSizeClasses; ++k) local[k] += len >> (5 + k);
  }
#pragma unroll
  for (int k = 0; k < kSizeClasses; ++k) {
    unsigned long long v = local[k];
    for (int d = 16; d > 0; d >>= 1) v += __shfl_down_sync(0xffffffffu, v, d);
    if ((threadIdx.x & 31) == 0 && v) atomicAdd(&counts[k], v);
  }
}

__global__ void col_histogram(const int* __restrict__ col_ind, long long nnz, int* __restrict__ col_nnz) {
  for (long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x; p < nnz;
       p += (long long)gridDim.x * blockDim.x)
    atomicAdd(&col_nnz[col_ind[p]], 1);
}

// Sort-A keys: (row << wc) | (maxcnt - col_nnz[col]); ascending = row asc, frequency desc.
__global__ void freq_sort_keys(const int* __restrict__ row_ptr, int rows, const int* __restrict__ col_ind,
                               const int* __restrict__ col_nnz, int maxcnt, int wc,
                               uint64_t* __restrict__ keys, uint32_t* __restrict__ vals) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const int end = row_ptr[r + 1];
    for (int p = row_ptr[r] + lane; p < end; p += 32) {
      keys[p] = (uint64_t(r) << wc) | uint64_t(maxcnt - col_nnz[col_ind[p]]);
      vals[p] = uint32_t(p);
    }
  }
}

// Groups of each row per workset (GetGroupNumArray, utils/matrix_utils.cu:132-156).
__global__ void row_group_counts(const int* __restrict__ row_ptr, int rows, int S, int fine,
                                 int* __restrict__ counts /* [S][rows] */) {
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const int len = row_ptr[r + 1] - row_ptr[r];
    if (S == 1) {
      counts[r] = (len + fine - 1) / fine;
      continue;
    }
    int rest = len;
    for (int s = S - 1; s > 0; --s) {
      const int g = rest / dev_group_size(s);
      counts[size_t(s) * rows + r] = g;
      rest -= g * dev_group_size(s);
    }
    counts[r] = rest > 0 ? 1 : 0;
  }
}

// Source metadata of every group, in the reference's unpermuted group order
// (GetGroupMetaInfo, utils/matrix_utils.cu:158-208): destination row, first
// element in frequency-sorted order, and for the residue its size and atomic flag.
__global__ void group_metadata(const int* __restrict__ row_ptr, int rows, int S, int fine,
                               const int* __restrict__ prefix /* [S][rows+1] */, WorksetArrays wa,
                               int* __restrict__ res_size, unsigned char* __restrict__ res_atomic) {
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const int beg = row_ptr[r];
    const int len = row_ptr[r + 1] - beg;
    if (S == 1) {
      const int groups = (len + fine - 1) / fine;
      const int g0 = prefix[r];
      for (int k = 0; k < groups; ++k) {
        wa.des[0][g0 + k] = r;
        wa.start[0][g0 + k] = beg + k * fine;
        res_size[g0 + k] = min(len - k * fine, fine);
        res_atomic[g0 + k] = groups > 1;
      }
      continue;
    }
    int at = beg, rest = len;
    for (int s = S - 1; s > 0; --s) {
      const int G = dev_group_size(s);
      const int c = rest / G;
      const int g0 = prefix[size_t(s) * (rows + 1) + r];
      for (int k = 0; k < c; ++k) {
        wa.des[s][g0 + k] = r;
        wa.start[s][g0 + k] = at;
        at += G;
      }
      rest -= c * G;
    }
    if (rest) {
      const int g = prefix[r];
      wa.des[0][g] = r;
      wa.start[0][g] = at;
      res_size[g] = rest;
      res_atomic[g] = len > 32;
    }
  }
}

// Signature bits of every group of every workset (GetResidueSignature /
// GetBlockSignature, utils/matrix_utils.cu:261-327).  One warp per row; element k
// of the row (frequency order) belongs to the workset whose span contains it.
__global__ void group_signatures(const int* __restrict__ row_ptr, int rows, int S, int fine,
                                 const int* __restrict__ prefix, const uint32_t* __restrict__ perm,
                                 const int* __restrict__ col_ind, const int* __restrict__ sigbit,
                                 WorksetArrays wa) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const int beg = row_ptr[r];
    const int len = row_ptr[r + 1] - beg;
    for (int k = lane; k < len; k += 32) {
      int s = 0, g;
      if (S == 1) {
        g = prefix[r] + k / fine;
      } else {
        int rest = len, off = k;
        g = -1;
        for (int t = S - 1; t > 0; --t) {
          const int G = dev_group_size(t);
          const int c = rest / G;
          if (off < c * G) {
            s = t;
            g = prefix[size_t(t) * (rows + 1) + r] + off / G;
            break;
          }
          off -= c * G;
          rest -= c * G;
        }
        if (g < 0) g = prefix[r];
      }
      const int b = sigbit[col_ind[perm[beg + k]]];
      atomicOr(&wa.sig[s][size_t(b >> 5) * wa.groups[s] + g], 1u << (31 - (b & 31)));
    }
  }
}

// Keys of one signature word in the current group order.  The order and the keys
// live in whichever buffer pair *side names (the sort's device-side record).
__global__ void signature_word_keys(const uint32_t* __restrict__ sig_word, const uint32_t* __restrict__ idx0,
                                    const uint32_t* __restrict__ idx1, const int* __restrict__ side, int n,
                                    uint32_t* __restrict__ keys0, uint32_t* __restrict__ keys1) {
  const bool alt = *side != 0;
  const uint32_t* __restrict__ idx = alt ? idx1 : idx0;
  uint32_t* __restrict__ keys = alt ? keys1 : keys0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    keys[i] = ~sig_word[idx[i]];  // ascending complement = descending word
}

__global__ void permute_residue_meta(const uint32_t* __restrict__ order, int G, const int* __restrict__ size,
                                     const unsigned char* __restrict__ atomic_src, const int* __restrict__ des_src,
                                     int* __restrict__ size_perm, bool* __restrict__ atomic_out,
                                     int* __restrict__ des_out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < G; i += gridDim.x * blockDim.x) {
    const uint32_t j = order[i];
    size_perm[i] = size[j];
    atomic_out[i] = atomic_src[j] != 0;
    des_out[i] = des_src[j];
  }
}

__global__ void permute_block_des(const uint32_t* __restrict__ order, int G, const int* __restrict__ des_src,
                                  int* __restrict__ des_out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < G; i += gridDim.x * blockDim.x)
    des_out[i] = des_src[order[i]];
}

// Element keys of one workset in final group order: (dst group << wcol) | col,
// value = CSR position, written in frequency order within each group so that a
// stable sort leaves equal columns in that order (thrust::sort of NNZPoint2).
__global__ void gather_group_elements(const uint32_t* __restrict__ order, int G, int group_len,
                                      const int* __restrict__ res_off, const int* __restrict__ res_size,
                                      const int* __restrict__ start, const uint32_t* __restrict__ perm,
                                      const int* __restrict__ col_ind, int wcol,
                                      uint64_t* __restrict__ keys, uint32_t* __restrict__ vals) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < G; i += warps) {
    const uint32_t j = order[i];
    const long long dst = res_off ? (long long)res_off[i] : (long long)i * group_len;
    const int size = res_off ? res_size[j] : group_len;
    const int src = start[j];
    for (int k = lane; k < size; k += 32) {
      const uint32_t p = perm[src + k];
      keys[dst + k] = (uint64_t(i) << wcol) | uint64_t(uint32_t(col_ind[p]));
      vals[dst + k] = p;
    }
  }
}

// lens[des[g]] += size of group g (group_len for block groups, from res_off for the residue).
__global__ void add_group_lengths(const int* __restrict__ des, int groups, int group_len,
                                  const int* __restrict__ res_off, int* __restrict__ lens) {
  for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < groups; g += gridDim.x * blockDim.x)
    atomicAdd(&lens[des[g]], res_off ? res_off[g + 1] - res_off[g] : group_len);
}

// Row word of every residue element: its group's destination row, with bit 31 set
// when the group adds atomically (residue_atomic).
__global__ void residue_rows(const int* __restrict__ res_off, const int* __restrict__ des,
                             const bool* __restrict__ atomic, int groups, int* __restrict__ row_of) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; g < groups; g += warps) {
    const int w = int(unsigned(des[g]) | (atomic[g] ? 0x80000000u : 0u));
    for (int e = res_off[g] + lane; e < res_off[g + 1]; e += 32) row_of[e] = w;
  }
}

// The sorted (key, CSR position) pairs are in whichever buffer pair *side names.
__global__ void finalize_workset(const uint64_t* __restrict__ keys0, const uint32_t* __restrict__ vals0,
                                 const uint64_t* __restrict__ keys1, const uint32_t* __restrict__ vals1,
                                 const int* __restrict__ side, long long n, uint64_t col_mask,
                                 const float* __restrict__ sp_data, int* __restrict__ col_out,
                                 float* __restrict__ val_out, int* __restrict__ pos_out) {
  const bool alt = *side != 0;
  const uint64_t* __restrict__ keys = alt ? keys1 : keys0;
  const uint32_t* __restrict__ vals = alt ? vals1 : vals0;
  for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < n;
       q += (long long)gridDim.x * blockDim.x) {
    col_out[q] = int(keys[q] & col_mask);
    val_out[q] = sp_data[vals[q]];
    pos_out[q] = int(vals[q]);
  }
}

unsigned grid_for(long long work, int per_block, int max_blocks) {
  long long b = (work + per_block - 1) / per_block;
  if (b < 1) b = 1;
  if (b > max_blocks) b = max_blocks;
  return unsigned(b);
}

// GenerateSigBit in FFC mode, ffc = 2 (utils/matrix_utils.cu:65-128, mode fixed at :55-60).
// The column order comes from the same libstdc++ std::sort (introsort, not stable)
// on the same input, so columns with equal frequency receive the same bits.  The
// sort runs over (frequency, column) pairs compared by frequency alone: it makes the
// same comparisons with the same outcomes, so it moves the pairs exactly as the
// reference's sort of column ids compared through col_nnz moves the ids, and the
// keys sit next to the ids instead of behind an indirection.
void signature_bits(int cols, const std::vector<int>& col_nnz, std::vector<int>& bit, int& len) {
  std::vector<std::pair<int, int>> by_freq(cols);  // (col_nnz[c], c)
  for (int c = 0; c < cols; ++c) by_freq[c] = {col_nnz[c], c};
  std::sort(by_freq.begin(), by_freq.end(),
            [](const std::pair<int, int>& a, const std::pair<int, int>& b) { return a.first > b.first; });
  bit.assign(cols, 0);
  const int top = std::min(2, cols);
  int next = 0;
  long long budget = 0;
  for (; next < top; ++next) {
    bit[by_freq[next].second] = 0;
    budget += by_freq[next].first;
  }
  int pos = 1;
  while (next < cols) {
    const int first = next;
    long long run = 0;
    while (next < cols) {
      run += by_freq[next].first;
      if (run < budget || next == first) {
        bit[by_freq[next].second] = pos;
        ++next;
      } else {
        break;
      }
    }
    ++pos;
  }
  len = pos;
  if (len < 32) len = 32;
  else if (len % 32 < 16) len = (len / 32) * 32;
  else len = (len / 32 + (len % 32 != 0)) * 32;
  for (int c = 0; c < cols; ++c) bit[c] = std::min(bit[c], len - 1);
}

// True if any_in(begin, end) is true for a part of [0, n); the parts run on up to
// hardware_concurrency host threads (one call below 2^20 items per thread).
template <typename F>
bool parallel_any(long long n, const F& any_in) {
  const long long threads =
      std::min<long long>(std::max(1u, std::thread::hardware_concurrency()), std::max(1LL, n >> 20));
  if (threads <= 1) return any_in(0LL, n);
  std::vector<char> hit(size_t(threads), 0);
  std::vector<std::thread> pool;
  for (long long t = 0; t < threads; ++t)
    pool.emplace_back([&, t] { hit[size_t(t)] = any_in(n * t / threads, n * (t + 1) / threads) ? 1 : 0; });
  for (auto& th : pool) th.join();
  return std::find(hit.begin(), hit.end(), 1) != hit.end();
}

struct HostCopy {
  void* dst;        // device
  const void* src;  // pageable host
  size_t bytes;
};

// Synchronous host-to-device copy of pageable host arrays.  A pageable cudaMemcpy
// goes through the driver's staging at ~11 GB/s on the B200 box; here up to 16 host
// threads each copy 4 MiB pieces into a pinned buffer of their own and start the
// transfer from it on a stream of their own, so host copies and transfers of
// different pieces overlap (config 5's 8.2 GB: 730 -> ~300 ms).  Taking pinned
// memory is slow (with the buffers taken per call, config 2's 0.5 GB took 135-210 ms
// against 48 ms pageable), so the buffers are taken once, on the first staged upload
// of the process, and kept until it exits (64 MiB of host memory), and inputs below
// 1 GiB in total use the plain copy.
struct PinnedPool {
  std::mutex mu;  // one staged upload at a time
  std::vector<void*> bufs;
};
PinnedPool& pinned_pool() {
  static PinnedPool* pool = new PinnedPool();  // never destroyed: CUDA may be gone at exit
  return *pool;
}

void upload_pageable(const std::vector<HostCopy>& copies, cudaStream_t st) {
  size_t total = 0;
  for (const auto& c : copies) total += c.bytes;
  if (total < (size_t(1) << 30)) {
    for (const auto& c : copies)
      if (c.bytes) PSB_CUDA(cudaMemcpyAsync(c.dst, c.src, c.bytes, cudaMemcpyHostToDevice, st));
    PSB_CUDA(cudaStreamSynchronize(st));
    return;
  }
  constexpr size_t kPiece = size_t(4) << 20;
  struct Piece {
    char* dst;
    const char* src;
    size_t bytes;
  };
  std::vector<Piece> pieces;
  for (const auto& c : copies)
    for (size_t off = 0; off < c.bytes; off += kPiece)
      pieces.push_back({static_cast<char*>(c.dst) + off, static_cast<const char*>(c.src) + off,
                        std::min(kPiece, c.bytes - off)});
  const int threads = int(std::min<size_t>({size_t(16), std::max<size_t>(1, std::thread::hardware_concurrency()),
                                            pieces.size()}));
  int device = 0;
  PSB_CUDA(cudaGetDevice(&device));
  PSB_CUDA(cudaStreamSynchronize(st));  // the destinations are ready
  PinnedPool& pool = pinned_pool();
  std::lock_guard<std::mutex> lock(pool.mu);
  while (pool.bufs.size() < size_t(threads)) {
    void* p = nullptr;
    PSB_CUDA(cudaHostAlloc(&p, kPiece, cudaHostAllocPortable));
    pool.bufs.push_back(p);
  }
  std::vector<std::string> errors(static_cast<size_t>(threads));
  auto worker = [&](int t) {
    void* pin = pool.bufs[size_t(t)];
    cudaStream_t s = nullptr;
    cudaEvent_t done = nullptr;
    try {
      PSB_CUDA(cudaSetDevice(device));  // a new thread starts on device 0
      PSB_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
      PSB_CUDA(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
      bool pending = false;
      for (size_t i = size_t(t); i < pieces.size(); i += size_t(threads)) {
        if (pending) PSB_CUDA(cudaEventSynchronize(done));  // the pinned buffer is free again
        std::memcpy(pin, pieces[i].src, pieces[i].bytes);
        PSB_CUDA(cudaMemcpyAsync(pieces[i].dst, pin, pieces[i].bytes, cudaMemcpyHostToDevice, s));
        PSB_CUDA(cudaEventRecord(done, s));
        pending = true;
      }
      PSB_CUDA(cudaStreamSynchronize(s));
    } catch (const std::exception& e) {
      errors[size_t(t)] = e.what();
      if (s) cudaStreamSynchronize(s);
    }
    if (done) cudaEventDestroy(done);
    if (s) cudaStreamDestroy(s);
  };
  std::vector<std::thread> team;
  for (int t = 0; t < threads; ++t) team.emplace_back(worker, t);
  for (auto& th : team) th.join();
  for (const auto& e : errors)
    if (!e.empty()) throw CudaError(cudaErrorUnknown, "staged upload: " + e);
}

void validate_csr(int rows, int cols, int nnz, const int* row_ptr, const int* col_ind, const float* vals) {
  // Same checks, order and messages as utils/matrix_utils.cu:475-488 (each message
  // names a class of error, not a position, so the scans may run in parallel).
  if (rows <= 0 || cols <= 0 || nnz <= 0 || rows > std::numeric_limits<int>::max() - 32 ||
      nnz > std::numeric_limits<int>::max() - 32 || !row_ptr || !col_ind || !vals)
    throw std::invalid_argument("Expected a nonempty CSR matrix with 32-bit indices");
  if (row_ptr[0] != 0 || row_ptr[rows] != nnz) throw std::invalid_argument("Invalid CSR row-pointer endpoints");
  if (parallel_any(rows, [&](long long b, long long e) {
        for (long long r = b; r < e; ++r)
          if (row_ptr[r] < 0 || row_ptr[r] > row_ptr[r + 1]) return true;
        return false;
      }))
    throw std::invalid_argument("CSR row pointers must be nondecreasing");
  if (parallel_any(nnz, [&](long long b, long long e) {
        for (long long p = b; p < e; ++p)
          if (col_ind[p] < 0 || col_ind[p] >= cols || !std::isfinite(vals[p])) return true;
        return false;
      }))
    throw std::invalid_argument("Invalid CSR column index or sparse value");
}

// Block tasks of about kTaskElems elements, largest group sizes first (the
// reference launches worksets S-1 down to 0), in one of the two BlockOrders.
//
// Why two orders (measured on B200, configurations 2-4): a row's most frequent
// columns sit in its largest groups and each group's columns are ascending, so
// slice k of the groups of one workset gathers from largely the same hot rows of
// the dense operand.  Running those slices side by side (kSliceOrder) turns that
// into L1/L2 hits when the dense operand does not fit L2 (N = 128: -4% to -10%
// time; N = 32 on configurations 2-3: -1% to -3%).  When it does fit (config 4 at
// N = 32), the same order concentrates the requests of every SM on a few lines at
// once and row order is 6% faster.
// `slot_of[s][g]`: wide-row slot of block group g of workset s (empty: none).
std::vector<Task> build_block_tasks(const Matrix& m, BlockOrder order, const std::vector<std::vector<int>>& slot_of,
                                    const std::vector<char>& slot_sum) {
  auto slot = [&](int s, int g) { return slot_of[s].empty() ? -1 : slot_of[s][g]; };
  auto sum = [&](int s, int g) { const int k = slot(s, g); return k >= 0 ? int(slot_sum[size_t(k)]) : 0; };
  std::vector<Task> tasks;
  size_t count = 0;
  for (int s = 1; s < m.S; ++s) {
    const int G = group_size(s);
    count += G >= kTaskElems ? size_t(m.group_num[s]) * size_t(G / kTaskElems)
                             : size_t(ceil_div(m.group_num[s], kTaskElems / G));
  }
  tasks.reserve(count);
  for (int s = m.S - 1; s >= 1; --s) {
    const int G = group_size(s);
    const int groups = m.group_num[s];
    if (G >= kTaskElems && order == kRowOrder) {
      for (int g = 0; g < groups; ++g)
        for (int off = 0; off < G; off += kTaskElems)
          tasks.push_back({s, g * G + off, g * G + std::min(G, off + kTaskElems), g, slot(s, g), sum(s, g)});
    } else if (G >= kTaskElems) {
      for (int off = 0; off < G; off += kTaskElems)
        for (int g = 0; g < groups; ++g)
          tasks.push_back({s, g * G + off, g * G + std::min(G, off + kTaskElems), g, slot(s, g), sum(s, g)});
    } else {
      const int per = kTaskElems / G;
      for (int g = 0; g < groups; g += per) {
        const int ge = std::min(groups, g + per);
        tasks.push_back({s, g * G, ge * G, g, -1, 0});
      }
    }
  }
  return tasks;
}

// Residue tasks: runs of whole residue groups of at most `elems` elements.  The
// residue runs last in a launch; at N < 128 shorter tasks (kFineResidue) drain
// that tail sooner (config 4 SpMM N = 32: -5%), at N >= 128 they cost ~3%.
std::vector<Task> build_residue_tasks(const Matrix& m, const std::vector<int>& h_res_off, int elems) {
  std::vector<Task> tasks;
  const int G0 = m.group_num[0];
  tasks.reserve(std::min<size_t>(size_t(G0), size_t(h_res_off[G0]) / size_t(elems) * 2 + 16));
  int g = 0;
  while (g < G0) {
    const int first = g;
    const int begin = h_res_off[g];
    while (g < G0 && h_res_off[g + 1] - begin <= elems) ++g;
    if (g == first) ++g;  // a single group longer than a task (cannot happen: <= 31 or 16)
    tasks.push_back({0, begin, h_res_off[g], first, -1, 0});
  }
  return tasks;
}

}  // namespace

void finish_matrix(Matrix& mat, const std::vector<int>& h_res_off) {
  Matrix* m = &mat;
  const int S = m->S, G0 = m->group_num[0];
  const int kBlocks = 16 * device_sms();
  cudaStream_t st = nullptr;
  if (!m->row_ptr) {
    // A loaded layout: the row pointer from the group sizes of every row.
    DeviceArray<int> lens(size_t(m->rows)), rp(size_t(m->rows) + 1);
    PSB_CUDA(cudaMemsetAsync(lens.get(), 0, sizeof(int) * size_t(m->rows), st));
    for (int s = 0; s < S; ++s) {
      if (m->group_num[s] == 0) continue;
      add_group_lengths<<<grid_for(m->group_num[s], 256, kBlocks), 256, 0, st>>>(
          m->group_des[s], m->group_num[s], s == 0 ? 0 : group_size(s), s == 0 ? m->residue_offset : nullptr,
          lens.get());
      PSB_LAUNCH_CHECK();
    }
    exclusive_scan<int32_t>(lens.get(), rp.get(), size_t(m->rows), st);
    m->row_ptr = rp.release_ownership();
  }
  if (m->ws_size[0] > 0) {
    DeviceArray<int> rows_of(size_t(m->ws_size[0]));
    residue_rows<<<grid_for(G0, 8, kBlocks), 256, 0, st>>>(m->residue_offset, m->group_des[0], m->residue_atomic,
                                                           G0, rows_of.get());
    PSB_LAUNCH_CHECK();
    m->residue_row = rows_of.release_ownership();
  }

  // Wide rows (kWideRowSlices): block slices per row, counted over the groups of
  // the worksets whose groups are cut into slices; slots in row order.
  std::vector<std::vector<int>> slot_of(S);
  std::vector<char> slot_sum;  // per wide-row slot: its WideSum
  {
    std::vector<std::vector<int>> h_des(S);
    std::vector<int> slices(size_t(m->rows), 0);
    for (int s = 1; s < S; ++s) {
      const int G = group_size(s);
      if (G < kTaskElems || m->group_num[s] == 0) continue;
      h_des[s].resize(m->group_num[s]);
      PSB_CUDA(cudaMemcpy(h_des[s].data(), m->group_des[s], sizeof(int) * h_des[s].size(), cudaMemcpyDeviceToHost));
      for (int r : h_des[s]) slices[r] += G / kTaskElems;
    }
    std::vector<int> slot_of_row(size_t(m->rows), -1), h_wide_row;
    for (int r = 0; r < m->rows; ++r) {
      if (slices[r] >= kWideRowSlices) {
        slot_of_row[r] = int(h_wide_row.size());
        h_wide_row.push_back(r);
        slot_sum.push_back(char(slices[r] >= kExactRowSlices ? kWideExact : kWideQuad));
      }
    }
    m->wide_rows = int(h_wide_row.size());
    if (m->wide_rows > 0) {
      for (int s = 1; s < S; ++s) {
        if (h_des[s].empty()) continue;
        slot_of[s].resize(h_des[s].size());
        for (size_t g = 0; g < h_des[s].size(); ++g) slot_of[s][g] = slot_of_row[h_des[s][g]];
      }
      PSB_CUDA(cudaMalloc(reinterpret_cast<void**>(&m->wide_row), sizeof(int) * h_wide_row.size()));
      PSB_CUDA(cudaMemcpy(m->wide_row, h_wide_row.data(), sizeof(int) * h_wide_row.size(), cudaMemcpyHostToDevice));
      PSB_CUDA(cudaEventCreateWithFlags(&m->wide_ready, cudaEventDisableTiming));
    }
  }
  // The four task lists are independent: built on host threads, uploaded in turn.
  auto upload_tasks = [](const std::vector<Task>& tasks, Task** dst, int* count) {
    *count = int(tasks.size());
    if (tasks.empty()) return;
    PSB_CUDA(cudaMalloc(reinterpret_cast<void**>(dst), sizeof(Task) * tasks.size()));
    PSB_CUDA(cudaMemcpy(*dst, tasks.data(), sizeof(Task) * tasks.size(), cudaMemcpyHostToDevice));
  };
  auto row_order = std::async(std::launch::async,
                              [&] { return build_block_tasks(*m, kRowOrder, slot_of, slot_sum); });
  auto slice_order = std::async(std::launch::async,
                                [&] { return build_block_tasks(*m, kSliceOrder, slot_of, slot_sum); });
  auto fine = std::async(std::launch::async,
                         [&] { return build_residue_tasks(*m, h_res_off, kFineResidueTaskElems); });
  const std::vector<Task> coarse = build_residue_tasks(*m, h_res_off, kTaskElems);
  upload_tasks(row_order.get(), &m->block_tasks[kRowOrder], &m->num_block_tasks[kRowOrder]);
  upload_tasks(slice_order.get(), &m->block_tasks[kSliceOrder], &m->num_block_tasks[kSliceOrder]);
  upload_tasks(fine.get(), &m->residue_tasks[kFineResidue], &m->num_residue_tasks[kFineResidue]);
  upload_tasks(coarse, &m->residue_tasks[kCoarseResidue], &m->num_residue_tasks[kCoarseResidue]);
  int l2 = 0;
  PSB_CUDA(cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, m->device));
  m->l2_bytes = l2;
  noalloc_prepare(m->device);
  PSB_CUDA(cudaDeviceSynchronize());
  trim_scratch_pool();
}

// Non-blocking streams that start after the work queued so far on `parent`;
// join() makes `parent` wait for everything queued on them (the destructor joins
// too, if join() was not reached, and then destroys the streams).
class StreamSet {
 public:
  StreamSet(int n, cudaStream_t parent) : parent_(parent), streams_(size_t(n), nullptr) {
    cudaEvent_t start = nullptr;
    PSB_CUDA(cudaEventCreateWithFlags(&start, cudaEventDisableTiming));
    EventGuard g{start};
    PSB_CUDA(cudaEventRecord(start, parent_));
    for (auto& s : streams_) {
      PSB_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
      PSB_CUDA(cudaStreamWaitEvent(s, start, 0));
    }
  }
  StreamSet(const StreamSet&) = delete;
  StreamSet& operator=(const StreamSet&) = delete;
  ~StreamSet() {
    if (!joined_) {
      try {
        join();
      } catch (...) {
      }
    }
    for (auto s : streams_)
      if (s) cudaStreamDestroy(s);
  }
  cudaStream_t operator[](int i) const { return streams_[size_t(i)]; }
  void join() {
    joined_ = true;
    for (auto s : streams_) {
      if (!s) continue;
      cudaEvent_t done = nullptr;
      PSB_CUDA(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
      EventGuard g{done};
      PSB_CUDA(cudaEventRecord(done, s));
      PSB_CUDA(cudaStreamWaitEvent(parent_, done, 0));
    }
  }

 private:
  struct EventGuard {
    cudaEvent_t e;
    ~EventGuard() { cudaEventDestroy(e); }
  };
  cudaStream_t parent_;
  std::vector<cudaStream_t> streams_;
  bool joined_ = false;
};

// Phases of build_matrix.  With the environment variable PSB_PREPROCESS_TRACE set,
// every phase ends with a device synchronization and the wall time of each phase
// is printed to stderr on one line when the build ends; otherwise it does nothing.
class PhaseTrace {
 public:
  PhaseTrace() : on_(std::getenv("PSB_PREPROCESS_TRACE") != nullptr), last_(std::chrono::steady_clock::now()) {}
  ~PhaseTrace() {
    if (on_) std::fprintf(stderr, "psb preprocess:%s\n", line_.c_str());
  }
  void mark(const char* phase) {
    if (!on_) return;
    cudaDeviceSynchronize();
    const auto now = std::chrono::steady_clock::now();
    char buf[96];
    std::snprintf(buf, sizeof(buf), " %s=%.1f", phase, std::chrono::duration<double, std::milli>(now - last_).count());
    line_ += buf;
    last_ = now;
  }

 private:
  bool on_;
  std::chrono::steady_clock::time_point last_;
  std::string line_;
};

Matrix* build_matrix(int rows, int cols, int nnz, const int* row_ptr, const int* col_ind,
                     const float* sp_data, int sm_count) {
  // The time covers the whole constructor, validation included, as the reference's
  // benchmark times it (benchmarks/benchmark.cu:128-134).
  const auto t0 = std::chrono::steady_clock::now();
  PhaseTrace trace;
  struct TrimOnExit {
    ~TrimOnExit() { trim_scratch_pool(); }
  } trim_on_exit;  // declared before every StreamArray, so it runs after their frees
  validate_csr(rows, cols, nnz, row_ptr, col_ind, sp_data);
  trace.mark("validate");
  std::unique_ptr<Matrix> m(new Matrix());
  m->rows = rows;
  m->cols = cols;
  m->nnz = nnz;
  PSB_CUDA(cudaGetDevice(&m->device));
  if (sm_count <= 0) PSB_CUDA(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, m->device));
  m->sm_count = sm_count;
  cudaStream_t st = nullptr;  // preprocessing is synchronous, like the reference constructor
  const int kBlocks = 16 * device_sms();

  // Temporaries come from the scratch pool (stream-ordered, no cudaMalloc / cudaFree
  // and the device-wide waits cudaFree implies); arrays the matrix keeps are cudaMalloc'd.
  DeviceArray<int> d_row_ptr(size_t(rows) + 1);
  StreamArray<int> d_col(nnz, st);
  StreamArray<float> d_val(nnz, st);
  upload_pageable({{d_row_ptr.get(), row_ptr, sizeof(int) * (size_t(rows) + 1)},
                   {d_col.get(), col_ind, sizeof(int) * size_t(nnz)},
                   {d_val.get(), sp_data, sizeof(float) * size_t(nnz)}},
                  st);
  trace.mark("upload");

  // --- Number of worksets (AnalyzeMatrix).
  {
    StreamArray<unsigned long long> counts(kSizeClasses, st);
    PSB_CUDA(cudaMemsetAsync(counts.get(), 0, sizeof(unsigned long long) * kSizeClasses, st));
    workset_size_counts<<<grid_for(rows, 256, kBlocks), 256, 0, st>>>(d_row_ptr.get(), rows, counts.get());
    PSB_LAUNCH_CHECK();
    unsigned long long h[kSizeClasses];
    PSB_CUDA(cudaMemcpy(h, counts.get(), sizeof(h), cudaMemcpyDeviceToHost));
    const unsigned long long threshold = 8ULL * unsigned(sm_count) * 4ULL;
    int S = 0;
    unsigned long long groups = threshold + 1;
    while (groups >= threshold) {
      groups = S < kSizeClasses ? h[S] : 0;
      ++S;
    }
    if (S > kMaxWorksets) throw std::runtime_error("too many worksets");
    m->S = S;
  }
  const int S = m->S, fine = m->fine;
  trace.mark("worksets");

  // --- Column frequencies.
  StreamArray<int> d_col_nnz(cols, st);
  PSB_CUDA(cudaMemsetAsync(d_col_nnz.get(), 0, sizeof(int) * size_t(cols), st));
  col_histogram<<<grid_for(nnz, 256, kBlocks), 256, 0, st>>>(d_col.get(), nnz, d_col_nnz.get());
  PSB_LAUNCH_CHECK();
  std::vector<int> h_col_nnz(cols);
  PSB_CUDA(cudaMemcpy(h_col_nnz.data(), d_col_nnz.get(), sizeof(int) * size_t(cols), cudaMemcpyDeviceToHost));
  const int maxcnt = *std::max_element(h_col_nnz.begin(), h_col_nnz.end());
  // GenerateSigBit needs only the column frequencies: its host sort runs on another
  // thread while the device sorts the rows and builds the groups.
  std::vector<int> h_sigbit;
  int signature_len = 0;
  std::future<void> sig_job =
      std::async(std::launch::async, [&] { signature_bits(cols, h_col_nnz, h_sigbit, signature_len); });
  trace.mark("col_freq");

  // --- Within-row order: frequency descending, stable (thrust::sort of NNZPoint).
  // perm[i] = CSR position of the i-th element in frequency order; it lives in one of
  // the two value buffers of the sort (both stay until the column sorts are done).
  StreamArray<uint32_t> perm_a(nnz, st), perm_b(nnz, st);
  uint32_t* perm = nullptr;
  {
    StreamArray<uint64_t> keys(nnz, st), keys_alt(nnz, st);
    const int wc = bits_for(unsigned(maxcnt));
    const int wr = bits_for(unsigned(rows - 1));
    freq_sort_keys<<<grid_for(rows, 8, kBlocks), 256, 0, st>>>(d_row_ptr.get(), rows, d_col.get(),
                                                               d_col_nnz.get(), maxcnt, wc, keys.get(),
                                                               perm_a.get());
    PSB_LAUNCH_CHECK();
    const bool alt = radix_sort_pairs<uint64_t>(keys.get(), perm_a.get(), keys_alt.get(), perm_b.get(),
                                                size_t(nnz), 0, wc + wr, st);
    perm = alt ? perm_b.get() : perm_a.get();
  }
  d_col_nnz.release();
  trace.mark("freq_sort");

  // --- Groups per workset and their source metadata.
  StreamArray<int> counts(size_t(S) * rows, st), prefix(size_t(S) * (size_t(rows) + 1), st);
  row_group_counts<<<grid_for(rows, 256, kBlocks), 256, 0, st>>>(d_row_ptr.get(), rows, S, fine, counts.get());
  PSB_LAUNCH_CHECK();
  m->group_num.assign(S, 0);
  for (int s = 0; s < S; ++s) {
    int* pre = prefix.get() + size_t(s) * (size_t(rows) + 1);
    exclusive_scan<int32_t>(counts.get() + size_t(s) * rows, pre, size_t(rows), st);
    PSB_CUDA(cudaMemcpy(&m->group_num[s], pre + rows, sizeof(int), cudaMemcpyDeviceToHost));
  }
  counts.release();
  const int G0 = m->group_num[0];
  std::vector<std::unique_ptr<StreamArray<int>>> src_des(S), src_start(S);
  StreamArray<int> res_size(G0, st);
  StreamArray<unsigned char> res_atomic_src(G0, st);
  WorksetArrays wa{};
  for (int s = 0; s < S; ++s) {
    src_des[s].reset(new StreamArray<int>(m->group_num[s], st));
    src_start[s].reset(new StreamArray<int>(m->group_num[s], st));
    wa.des[s] = src_des[s]->get();
    wa.start[s] = src_start[s]->get();
    wa.groups[s] = m->group_num[s];
  }
  group_metadata<<<grid_for(rows, 256, kBlocks), 256, 0, st>>>(d_row_ptr.get(), rows, S, fine, prefix.get(), wa,
                                                               res_size.get(), res_atomic_src.get());
  PSB_LAUNCH_CHECK();
  trace.mark("groups");

  // --- Signatures (GenerateSigBit on the host, bits on the device).
  sig_job.get();
  m->signature_len = signature_len;
  trace.mark("sig_bits_wait");
  const int words = m->signature_len / 32;
  StreamArray<int> d_sigbit(cols, st);
  PSB_CUDA(cudaMemcpyAsync(d_sigbit.get(), h_sigbit.data(), sizeof(int) * size_t(cols), cudaMemcpyHostToDevice, st));
  std::vector<std::unique_ptr<StreamArray<uint32_t>>> sig(S);
  for (int s = 0; s < S; ++s) {
    sig[s].reset(new StreamArray<uint32_t>(size_t(words) * m->group_num[s], st));
    if (m->group_num[s])
      PSB_CUDA(cudaMemsetAsync(sig[s]->get(), 0, sizeof(uint32_t) * size_t(words) * m->group_num[s], st));
    wa.sig[s] = sig[s]->get();
  }
  group_signatures<<<grid_for(rows, 8, kBlocks), 256, 0, st>>>(d_row_ptr.get(), rows, S, fine, prefix.get(),
                                                               perm, d_col.get(), d_sigbit.get(), wa);
  PSB_LAUNCH_CHECK();
  prefix.release();
  d_sigbit.release();
  trace.mark("signatures");

  // --- Signature order of the groups of every workset: stable, lexicographically
  // descending over words (LSD: last word first, as utils/matrix_utils.cu:590-592).
  // The worksets are independent, so each sorts on its own stream; within one, all
  // word passes are queued without a host round trip (the buffer side of every
  // pass is kept on the device), and the order ends in order[s].
  std::vector<std::unique_ptr<StreamArray<uint32_t>>> order(S);
  for (int s = 0; s < S; ++s) order[s].reset(new StreamArray<uint32_t>(m->group_num[s], st));
  {
    StreamSet streams(S, st);
    for (int s = 0; s < S; ++s) {
      const int G = m->group_num[s];
      if (G == 0) continue;
      const cudaStream_t ss = streams[s];
      const int per_word = radix_passes(size_t(G), 0, 32);
      StreamArray<uint32_t> keys(2 * size_t(G), ss), idx_alt(G, ss);
      StreamArray<int> side(size_t(words) * per_word + 1, ss);
      PSB_CUDA(cudaMemsetAsync(side.get(), 0, sizeof(int), ss));
      uint32_t* ord = order[s]->get();
      iota_u32(ord, G, ss);
      int pass = 0;
      for (int w = words - 1; w >= 0; --w) {
        signature_word_keys<<<grid_for(G, 256, kBlocks), 256, 0, ss>>>(
            sig[s]->get() + size_t(w) * G, ord, idx_alt.get(), side.get() + pass, G, keys.get(), keys.get() + G);
        PSB_LAUNCH_CHECK();
        radix_sort_pairs_async<uint32_t>(keys.get(), ord, keys.get() + G, idx_alt.get(), size_t(G), 0, 32,
                                         side.get() + pass, ss);
        pass += per_word;
      }
      take_from_alt(side.get() + pass, idx_alt.get(), ord, size_t(G), ss);
    }
    streams.join();
  }
  for (int s = 0; s < S; ++s) sig[s]->release();
  trace.mark("sig_sort");

  // --- Final worksets.
  m->col_ind.assign(S, nullptr);
  m->sp_data.assign(S, nullptr);
  m->group_des.assign(S, nullptr);
  m->csr_pos.assign(S, nullptr);
  m->ws_size.assign(S, 0);
  DeviceArray<int> res_off(size_t(G0) + 1);
  {
    StreamArray<int> size_perm(G0, st);
    DeviceArray<bool> atomic_out(G0);
    DeviceArray<int> des_out(G0);
    if (G0) {
      permute_residue_meta<<<grid_for(G0, 256, kBlocks), 256, 0, st>>>(order[0]->get(), G0, res_size.get(),
                                                                        res_atomic_src.get(), src_des[0]->get(),
                                                                        size_perm.get(), atomic_out.get(),
                                                                        des_out.get());
      PSB_LAUNCH_CHECK();
    }
    exclusive_scan<int32_t>(size_perm.get(), res_off.get(), size_t(G0), st);
    m->residue_atomic = atomic_out.release_ownership();
    m->group_des[0] = des_out.release_ownership();
  }
  std::vector<int> h_res_off(size_t(G0) + 1);
  PSB_CUDA(cudaMemcpy(h_res_off.data(), res_off.get(), sizeof(int) * (size_t(G0) + 1), cudaMemcpyDeviceToHost));
  trace.mark("residue_meta");
  const int wcol = bits_for(unsigned(cols - 1));
  for (int s = 0; s < S; ++s) {
    const int G = m->group_num[s];
    const long long n = s == 0 ? (long long)h_res_off[G0] : (long long)G * group_size(s);
    m->ws_size[s] = n;
    if (s > 0 && G) {
      DeviceArray<int> des_out(G);
      permute_block_des<<<grid_for(G, 256, kBlocks), 256, 0, st>>>(order[s]->get(), G, src_des[s]->get(),
                                                                   des_out.get());
      PSB_LAUNCH_CHECK();
      m->group_des[s] = des_out.release_ownership();
    }
    if (n == 0) continue;
    const int wg = bits_for(unsigned(G - 1));
    const int passes = radix_passes(size_t(n), 0, wcol + wg);
    StreamArray<uint64_t> keys(n, st), keys_alt(n, st);
    StreamArray<uint32_t> vals(n, st), vals_alt(n, st);
    StreamArray<int> side(size_t(passes) + 1, st);
    PSB_CUDA(cudaMemsetAsync(side.get(), 0, sizeof(int), st));
    gather_group_elements<<<grid_for(G, 8, kBlocks), 256, 0, st>>>(
        order[s]->get(), G, s == 0 ? 0 : group_size(s), s == 0 ? res_off.get() : nullptr,
        s == 0 ? res_size.get() : nullptr, src_start[s]->get(), perm, d_col.get(), wcol, keys.get(),
        vals.get());
    PSB_LAUNCH_CHECK();
    radix_sort_pairs_async<uint64_t>(keys.get(), vals.get(), keys_alt.get(), vals_alt.get(), size_t(n), 0,
                                     wcol + wg, side.get(), st);
    DeviceArray<int> col_out(n), pos_out(n);
    DeviceArray<float> val_out(n);
    finalize_workset<<<grid_for(n, 256, kBlocks), 256, 0, st>>>(
        keys.get(), vals.get(), keys_alt.get(), vals_alt.get(), side.get() + passes, n,
        (uint64_t(1) << wcol) - 1, d_val.get(), col_out.get(), val_out.get(), pos_out.get());
    PSB_LAUNCH_CHECK();
    m->col_ind[s] = col_out.release_ownership();
    m->sp_data[s] = val_out.release_ownership();
    m->csr_pos[s] = pos_out.release_ownership();
  }
  m->residue_offset = res_off.release_ownership();
  m->row_ptr = d_row_ptr.release_ownership();
  trace.mark("col_sort");
  finish_matrix(*m, h_res_off);
  trace.mark("tasks");
  m->preprocess_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  return m.release();
}

}  // namespace psb
