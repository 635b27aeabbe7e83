// CPU oracle for the PowerSparse hot path.  TEST INFRASTRUCTURE ONLY.
//
// This file restates, on the host and step by step, what the reference's
// preprocessing and CPU checks compute.  It is the checker for the CUDA
// library in powersparse_b200/: only tests/, __graft_entry__.smoke() and the
// cpu_baseline / reference legs of bench.py may load it.  The product never
// links or calls it.
//
// Citations are paths inside the ParCIS/PowerSparse source tree.
//
//   * layout construction  utils/matrix_utils.cu:470-663 (constructor)
//       - S from the SM count          AnalyzeMatrix       :31-63
//       - column histogram             ctor                :508-514
//       - (row asc, col_nnz desc) sort NNZPoint + sort     :210-223, 522-524
//       - groups per workset           GetGroupNumArray    :132-156
//       - residue offsets / atomics    GetGroupMetaInfo    :158-208
//       - column -> signature bit      GenerateSigBit      :65-128
//       - group signatures             Get*Signature       :261-327
//       - signature order              stable_sort x words :567-594
//       - per-group column order       GetSrc*Workset+sort :329-392, 596-618
//       - final permutation            Get*Workset         :403-464, 619-656
//   * SpMM check  benchmarks/benchmark.cu:64-77  (FP64, CSR order)
//   * SDDMM check benchmarks/benchmark.cu:79-96  (FP64, workset order)
//
// thrust::sort / thrust::stable_sort with a user comparator run CUB's merge
// sort in CUDA 12.9 (thrust/system/cuda/detail/sort.h:139-164), which keeps
// equal keys in input order; every such sort is restated as std::stable_sort.
// The one std::sort of the reference (GenerateSigBit, :72-75) is restated as
// the same libstdc++ std::sort call on the same input, so ties resolve
// identically.  The LSD sequence of stable per-word sorts (:590-592) equals one
// stable sort by the whole signature, lexicographically descending.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <stdexcept>
#include <string>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

inline int group_size(int s) { return 32 * (1 << (s - 1)); }  // utils/matrix_utils.h:8

struct Layout {
  int rows = 0, cols = 0, nnz = 0;
  int S = 0, fine = 16, signature_len = 32;
  std::vector<int> group_num;                  // [S]
  std::vector<std::vector<int>> col_ind;       // [S][workset size]
  std::vector<std::vector<int>> csr_pos;       // [S][workset size]: CSR position of each element
  std::vector<std::vector<float>> sp_data;     // [S][workset size]
  std::vector<std::vector<int>> group_des;     // [S][group_num[s]]
  std::vector<int> residue_offset;             // [G0 + 1], permuted order
  std::vector<unsigned char> residue_atomic;   // [G0], permuted order
  std::vector<std::vector<int>> order;         // [S][group_num[s]] sorted source index
};

// AnalyzeMatrix (utils/matrix_utils.cu:31-63): one workset for the residue plus one
// per consecutive size 32, 64, ... whose floor-count reaches 32 * SMs.
int analyze(int rows, const int* row_ptr, int sm_count) {
  const long long threshold = 8LL * sm_count * 4;
  int S = 0;
  long long groups = threshold + 1;
  while (groups >= threshold) {
    const long long size = 32LL << S;
    groups = 0;
    for (int r = 0; r < rows; ++r) groups += (row_ptr[r + 1] - row_ptr[r]) / size;
    ++S;
  }
  return S;
}

// GenerateSigBit in FFC mode with ffc = 2 (utils/matrix_utils.cu:65-128; the
// constructor hard-wires FFC, :55-60).
void signature_bits(int cols, const std::vector<int>& col_nnz, std::vector<int>& bit, int& len) {
  std::vector<int> by_freq(cols);
  std::iota(by_freq.begin(), by_freq.end(), 0);
  std::sort(by_freq.begin(), by_freq.end(),
            [&col_nnz](const int& a, const int& b) { return col_nnz[a] > col_nnz[b]; });
  bit.assign(cols, 0);
  const int top = std::min(2, cols);
  int next = 0, pos = 0;
  long long budget = 0;
  for (; next < top; ++next) {
    bit[by_freq[next]] = pos;
    budget += col_nnz[by_freq[next]];
  }
  pos = 1;
  while (next < cols) {
    const int first = next;
    long long run = 0;
    while (next < cols) {
      run += col_nnz[by_freq[next]];
      if (run < budget || next == first) {
        bit[by_freq[next]] = pos;
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

Layout build(int rows, int cols, int nnz, const int* row_ptr, const int* col_ind,
             const float* vals, int sm_count) {
  // Constructor validation (utils/matrix_utils.cu:475-488).
  if (rows <= 0 || cols <= 0 || nnz <= 0 || rows > 2147483647 - 32 || nnz > 2147483647 - 32 ||
      !row_ptr || !col_ind || !vals)
    throw std::invalid_argument("Expected a nonempty CSR matrix with 32-bit indices");
  if (row_ptr[0] != 0 || row_ptr[rows] != nnz)
    throw std::invalid_argument("Invalid CSR row-pointer endpoints");
  for (int r = 0; r < rows; ++r)
    if (row_ptr[r] < 0 || row_ptr[r] > row_ptr[r + 1])
      throw std::invalid_argument("CSR row pointers must be nondecreasing");
  for (int p = 0; p < nnz; ++p)
    if (col_ind[p] < 0 || col_ind[p] >= cols || !std::isfinite(vals[p]))
      throw std::invalid_argument("Invalid CSR column index or sparse value");

  Layout L;
  L.rows = rows; L.cols = cols; L.nnz = nnz;
  L.S = analyze(rows, row_ptr, sm_count);
  const int S = L.S, fine = L.fine;

  std::vector<int> col_nnz(cols, 0);
  for (int p = 0; p < nnz; ++p) ++col_nnz[col_ind[p]];

  // Within each row: column frequency descending, ties in CSR order.
  std::vector<int> perm(nnz);
  std::iota(perm.begin(), perm.end(), 0);
  for (int r = 0; r < rows; ++r)
    std::stable_sort(perm.begin() + row_ptr[r], perm.begin() + row_ptr[r + 1],
                     [&](int a, int b) { return col_nnz[col_ind[a]] > col_nnz[col_ind[b]]; });

  // Group counts and the unpermuted group metadata (GetGroupNumArray / GetGroupMetaInfo).
  L.group_num.assign(S, 0);
  std::vector<std::vector<int>> des(S);
  std::vector<std::vector<int>> first_pos(S);  // position (in perm) of each source group
  std::vector<int> res_size;
  std::vector<unsigned char> res_atomic;
  for (int r = 0; r < rows; ++r) {
    const int len = row_ptr[r + 1] - row_ptr[r];
    int at = row_ptr[r];
    if (S == 1) {
      const int groups = (len + fine - 1) / fine;
      for (int k = 0; k < groups; ++k) {
        des[0].push_back(r);
        first_pos[0].push_back(at + k * fine);
        res_size.push_back(std::min(len - k * fine, fine));
        res_atomic.push_back(groups > 1);
      }
      continue;
    }
    int rest = len;
    for (int s = S - 1; s > 0; --s) {
      const int g = rest / group_size(s);
      for (int k = 0; k < g; ++k) {
        des[s].push_back(r);
        first_pos[s].push_back(at);
        at += group_size(s);
      }
      rest -= g * group_size(s);
    }
    if (rest) {
      des[0].push_back(r);
      first_pos[0].push_back(at);
      res_size.push_back(rest);
      res_atomic.push_back(len > 32);
    }
  }
  for (int s = 0; s < S; ++s) L.group_num[s] = static_cast<int>(des[s].size());
  std::vector<long long> res_off(res_size.size() + 1, 0);
  for (size_t g = 0; g < res_size.size(); ++g) res_off[g + 1] = res_off[g] + res_size[g];
  auto members = [&](int s, int g) -> std::pair<int, int> {
    return {first_pos[s][g], s == 0 ? res_size[g] : group_size(s)};
  };

  // Signatures and the signature order of the groups of every workset.
  std::vector<int> bit;
  signature_bits(cols, col_nnz, bit, L.signature_len);
  const int words = L.signature_len / 32;
  L.order.assign(S, {});
  for (int s = 0; s < S; ++s) {
    const int G = L.group_num[s];
    std::vector<uint32_t> sig(size_t(G) * words, 0u);  // group-major here
    for (int g = 0; g < G; ++g) {
      auto [pos, count] = members(s, g);
      for (int k = 0; k < count; ++k) {
        const int b = bit[col_ind[perm[pos + k]]];
        sig[size_t(g) * words + b / 32] |= 1u << (31 - b % 32);
      }
    }
    std::vector<int>& idx = L.order[s];
    idx.resize(G);
    std::iota(idx.begin(), idx.end(), 0);
    std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) {
      const uint32_t* x = &sig[size_t(a) * words];
      const uint32_t* y = &sig[size_t(b) * words];
      for (int w = 0; w < words; ++w)
        if (x[w] != y[w]) return x[w] > y[w];
      return false;
    });
  }

  // Final worksets: groups in signature order, each group's columns ascending
  // (ties keep the frequency order, which for equal columns is CSR order).
  L.col_ind.assign(S, {});
  L.csr_pos.assign(S, {});
  L.sp_data.assign(S, {});
  L.group_des.assign(S, {});
  for (int s = 0; s < S; ++s) {
    const int G = L.group_num[s];
    std::vector<int>& dc = L.col_ind[s];
    std::vector<float>& dv = L.sp_data[s];
    L.group_des[s].resize(G);
    if (s == 0) {
      L.residue_offset.assign(size_t(G) + 1, 0);
      L.residue_atomic.assign(G, 0);
    }
    std::vector<int> tmp;
    for (int i = 0; i < G; ++i) {
      const int src = L.order[s][i];
      auto [pos, count] = members(s, src);
      tmp.assign(perm.begin() + pos, perm.begin() + pos + count);
      std::stable_sort(tmp.begin(), tmp.end(),
                       [&](int a, int b) { return col_ind[a] < col_ind[b]; });
      for (int p : tmp) {
        dc.push_back(col_ind[p]);
        L.csr_pos[s].push_back(p);
        dv.push_back(vals[p]);
      }
      L.group_des[s][i] = des[s][src];
      if (s == 0) {
        L.residue_offset[i + 1] = L.residue_offset[i] + count;
        L.residue_atomic[i] = res_atomic[src];
      }
    }
  }
  if (L.residue_offset.empty()) L.residue_offset.assign(1, 0);
  return L;
}

thread_local std::string g_error;

}  // namespace

extern "C" {

typedef struct ps_oracle_layout ps_oracle_layout;

const char* ps_oracle_last_error(void) { return g_error.c_str(); }

// Returns nullptr and sets the last error (std::invalid_argument text) on bad CSR.
ps_oracle_layout* ps_oracle_build(int rows, int cols, int nnz, const int* row_ptr,
                                  const int* col_ind, const float* vals, int sm_count) {
  try {
    return reinterpret_cast<ps_oracle_layout*>(
        new Layout(build(rows, cols, nnz, row_ptr, col_ind, vals, sm_count)));
  } catch (const std::exception& e) {
    g_error = e.what();
    return nullptr;
  }
}

void ps_oracle_free(ps_oracle_layout* h) { delete reinterpret_cast<Layout*>(h); }

int ps_oracle_analyze(int rows, const int* row_ptr, int sm_count) {
  return analyze(rows, row_ptr, sm_count);
}

#define L_ (*reinterpret_cast<const Layout*>(h))
int ps_oracle_group_type_num(const ps_oracle_layout* h) { return L_.S; }
int ps_oracle_group_fine_size(const ps_oracle_layout* h) { return L_.fine; }
int ps_oracle_signature_len(const ps_oracle_layout* h) { return L_.signature_len; }
int ps_oracle_group_num(const ps_oracle_layout* h, int s) { return L_.group_num[s]; }
long long ps_oracle_workset_size(const ps_oracle_layout* h, int s) {
  return static_cast<long long>(L_.col_ind[s].size());
}
const int* ps_oracle_col_ind(const ps_oracle_layout* h, int s) { return L_.col_ind[s].data(); }
const int* ps_oracle_csr_pos(const ps_oracle_layout* h, int s) { return L_.csr_pos[s].data(); }
const float* ps_oracle_sp_data(const ps_oracle_layout* h, int s) { return L_.sp_data[s].data(); }
const int* ps_oracle_group_des(const ps_oracle_layout* h, int s) { return L_.group_des[s].data(); }
const int* ps_oracle_residue_offset(const ps_oracle_layout* h) { return L_.residue_offset.data(); }
const unsigned char* ps_oracle_residue_atomic(const ps_oracle_layout* h) {
  return L_.residue_atomic.data();
}
const int* ps_oracle_group_order(const ps_oracle_layout* h, int s) { return L_.order[s].data(); }
#undef L_

// CheckSpmm (benchmarks/benchmark.cu:64-77): C[r, j] = sum_p double(A_p) * B[col_p, j],
// accumulated in CSR order.  Rows are independent, so any thread count gives the
// same bits.
void ps_oracle_spmm(int rows, const int* row_ptr, const int* col_ind, const float* vals,
                    int n, const float* B, double* C, int threads) {
#ifdef _OPENMP
  if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(dynamic, 256)
#endif
  for (int r = 0; r < rows; ++r) {
    double* out = C + size_t(r) * n;
    for (int j = 0; j < n; ++j) out[j] = 0.0;
    for (int p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
      const double a = vals[p];
      const float* b = B + size_t(col_ind[p]) * n;
      for (int j = 0; j < n; ++j) out[j] += a * b[j];
    }
  }
}

// Same, restricted to rows [r0, r1): the bounded CPU-baseline sample.
void ps_oracle_spmm_rows(int r0, int r1, const int* row_ptr, const int* col_ind,
                         const float* vals, int n, const float* B, double* C, int threads) {
#ifdef _OPENMP
  if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(dynamic, 256)
#endif
  for (int r = r0; r < r1; ++r) {
    double* out = C + size_t(r - r0) * n;
    for (int j = 0; j < n; ++j) out[j] = 0.0;
    for (int p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
      const double a = vals[p];
      const float* b = B + size_t(col_ind[p]) * n;
      for (int j = 0; j < n; ++j) out[j] += a * b[j];
    }
  }
}

// CheckSddmm (benchmarks/benchmark.cu:79-96) for one workset given as arrays:
// out[p] = A_p * sum_j double(lhs[row(g), j]) * rhs[col_p, j] for p in group g,
// with group g spanning [offsets[g], offsets[g+1]).
void ps_oracle_sddmm(int groups, const int* group_des, const long long* offsets,
                     const int* col_ind, const float* vals, int n, const float* lhs,
                     const float* rhs, double* out, int threads) {
#ifdef _OPENMP
  if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(dynamic, 256)
#endif
  for (int g = 0; g < groups; ++g) {
    const float* x = lhs + size_t(group_des[g]) * n;
    for (long long p = offsets[g]; p < offsets[g + 1]; ++p) {
      const float* y = rhs + size_t(col_ind[p]) * n;
      double acc = 0.0;
      for (int j = 0; j < n; ++j) acc += double(x[j]) * y[j];
      out[p] = acc * vals[p];
    }
  }
}

int ps_oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"
