// The preprocessed matrix owned by the library (behind the opaque ps_matrix handle).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

namespace psb {

constexpr int kMaxWorksets = 32;
constexpr int kFineGroupSize = 16;  // utils/matrix_utils.cu:56 of the reference

// GROUP_SIZE(s) of the reference (utils/matrix_utils.h:8): 32 * 2^(s-1) for s >= 1.
inline int group_size(int s) { return 32 << (s - 1); }

// A unit of SpMM/SDDMM work: elements [begin, end) of workset `ws`, starting in
// group `group`.  Residue tasks cover whole groups; block tasks cover whole
// groups, or one slice of a group when the group is longer than a task.
// `slot` >= 0 marks a slice of a wide row (see Matrix::wide_rows); `sum` is then
// how the slice sums its products (WideSum, chosen by the row's length).
struct Task {
  int ws;
  int begin;
  int end;
  int group;
  int slot;
  int sum;
};

// A launch runs the block tasks (largest groups first), then the residue tasks.
// Each part is kept in two variants and the operators combine one of each:
//   block order   kRowOrder    a group's slices consecutive;
//                 kSliceOrder  per workset, slice k of every group before slice k+1;
//   residue cut   kFineResidue tasks of at most kFineResidueTaskElems elements;
//                 kCoarseResidue at most kTaskElems.
enum BlockOrder { kRowOrder = 0, kSliceOrder = 1 };
enum ResidueCut { kFineResidue = 0, kCoarseResidue = 1 };

struct Matrix {
  int device = 0;
  int rows = 0, cols = 0, nnz = 0;
  int S = 0;                     // GroupTypeNum(): worksets including the residue
  int fine = kFineGroupSize;     // GroupFineSize()
  int sm_count = 0;              // SM count the workset heuristic used
  int signature_len = 32;
  double preprocess_ms = 0.0;

  // The reference-visible layout (utils/matrix_utils.h:30-40).
  std::vector<int> group_num;          // host [S]
  std::vector<int*> col_ind;           // device, per workset (nullptr when empty)
  std::vector<float*> sp_data;         // device, per workset
  std::vector<int*> group_des;         // device, per workset
  std::vector<long long> ws_size;      // elements per workset
  int* residue_offset = nullptr;       // device [G0 + 1]
  bool* residue_atomic = nullptr;      // device [G0], nullptr when G0 == 0
  // Row pointer of the constructor's CSR (device, rows + 1): edge softmax rows.
  int* row_ptr = nullptr;
  // CSR position (index into the constructor's col_ind / sp_data) of every
  // workset element: SDDMM in CSR order writes through it.
  std::vector<int*> csr_pos;           // device, per workset

  // Work decomposition for the fused SpMM / SDDMM kernels (not part of the
  // reference layout; derived from it).
  // Device task lists: block tasks per BlockOrder, residue tasks per ResidueCut.
  Task* block_tasks[2] = {};
  int num_block_tasks[2] = {};
  Task* residue_tasks[2] = {};
  int num_residue_tasks[2] = {};
  long long l2_bytes = 0;              // L2 size of the device (picks the block order)
  // Row word of every residue element: its group's destination row, bit 31 set when
  // the group adds atomically (its row has other groups).  Residue groups are short,
  // so SDDMM reads the lhs row per element and SpMM finds group ends by comparing
  // neighbouring words, instead of switching through group metadata.
  int* residue_row = nullptr;          // device [ws_size[0]]

  // Wide rows: rows split into at least kWideRowSlices block-slice tasks.  SpMM
  // sums their slices in FP64 (one slot of N doubles per row) and folds the sum
  // into C once, instead of adding every slice to C in FP32.
  int wide_rows = 0;
  int* wide_row = nullptr;             // device [wide_rows]: row of each slot
  // FP64 scratch of the wide rows, grown on demand to wide_rows * N doubles and
  // all-zero between calls.  Eager calls that use it are ordered by `wide_ready`.
  // Buffers replaced by a larger one stay allocated until the matrix is destroyed
  // (a captured CUDA graph may still use them).
  mutable double* wide_acc = nullptr;
  mutable long long wide_acc_cap = 0;  // doubles
  mutable std::vector<double*> wide_acc_retired;
  mutable cudaEvent_t wide_ready = nullptr;
  mutable std::mutex wide_mutex;

  // SpMM with a push epilogue (ps_spmm_push), built by its first call per residue
  // cut: push_count[cut][r] = how many times one launch adds into row r of C (0 for
  // wide rows, which the fold kernel finishes); push_pending is the per-call
  // countdown; quiet_rows lists the rows nothing adds into (not wide, no elements).
  mutable int* push_count[2] = {nullptr, nullptr};
  mutable int* push_pending = nullptr;
  mutable int* quiet_rows = nullptr;
  mutable int num_quiet_rows = -1;     // -1: not built yet
  mutable cudaEvent_t push_ready = nullptr;  // orders eager push calls (they share push_pending)
  mutable std::mutex push_mutex;

  Matrix() = default;
  Matrix(const Matrix&) = delete;
  Matrix& operator=(const Matrix&) = delete;
  ~Matrix();
};

// Derives what the operators need beyond the reference layout (residue rows,
// wide rows, the task lists) from a matrix whose layout arrays, group counts,
// workset sizes and residue offsets (device, and h_res_off on the host) are set.
// Used by build_matrix and by load_matrix.
void finish_matrix(Matrix& m, const std::vector<int>& h_res_off);

// Builds the layout on the current device from host CSR.  Throws
// std::invalid_argument on an invalid CSR (same checks and messages as
// utils/matrix_utils.cu:475-488) and psb::CudaError on CUDA failures.
// sm_count <= 0 uses the device's multiprocessor count.
Matrix* build_matrix(int rows, int cols, int nnz, const int* row_ptr, const int* col_ind,
                     const float* sp_data, int sm_count);

// Layout cache (ps_cache.cu): writes the layout arrays to `path` / reads them
// back onto the current device, validating every index, and derives the rest.
// Errors: std::invalid_argument (unreadable, truncated or corrupt file),
// std::runtime_error (write failure), psb::CudaError.
void save_matrix(const Matrix& m, const std::string& path);
Matrix* load_matrix(const std::string& path);

// Task sizes in elements used by build_matrix.
constexpr int kTaskElems = 256;
constexpr int kFineResidueTaskElems = 64;
// Rows with at least this many block slices are wide rows (FP64 slice sums).
// A slice partial is rounded once per FP32 add into C; with k adds of a running
// sum of magnitude R the rounding drift is about sqrt(k) * 2^-24 * R, which for
// k >= 8 (rows of >= 2048 elements, R ~ sqrt(row length)) reaches 1e-5, the
// absolute tolerance, on outputs whose exact value is near zero.
constexpr int kWideRowSlices = 8;
// Summation of a wide-row slice, by the row's block slices (rows of L products;
// the tolerance bites at 1e-5 absolute, on outputs whose exact value is near zero):
//   < kExactRowSlices  kWideQuad: chains of 4 FP32 FMAs, the first starting from the
//                      compensation, each chain added to the slice sum by a Kahan
//                      step (1.75 operations per product); what it keeps is each
//                      chain's own rounding, a drift of order sqrt(L) * 2^-24 * |v * b|;
//   otherwise          kWideExact: exact FP64 products (an FP32 x FP32 product is
//                      exact in FP64) summed in FP64.
// Worst element on the 300 longest and ~900 sampled long rows of configurations 2-5
// at N = 32 and 128, in units of the tolerance: chains 0.39 (rows of 2048-16383
// products) and 0.46 (16384-65535); a Kahan step per product 0.26 / 0.52 at 2-4% more
// time; plain FP32 chunk sums 0.99 / 1.32; exact products 0.14 on rows of >= 65536.
enum WideSum { kWideQuad = 0, kWideExact = 1 };
constexpr int kExactRowSlices = 256;

// Peer replicas one ps_spmm_push call writes (a node of 8 GPUs: 7 peers).
constexpr int kMaxPushPeers = 7;

}  // namespace psb
