// Fused SpMM and SDDMM over the PowerSparse worksets (sm_100a, FP32 CUDA cores).
//
// The reference launches one kernel per workset on its own stream and
// device-synchronizes (PowerSparse_SpMM/spmm_solution.cu:16-33,
// PowerSparse_SDDMM/sddmm_solution.cu:23-49).  Here one launch covers every
// workset: the matrix carries task lists (ps_matrix.h: about kTaskElems
// elements per task, largest groups first) and each lane group runs one task.
//
// Lane groups: LG lanes (8, 16 or 32) handle one sparse element at a time, each
// lane owning 4 consecutive dense columns, so a gathered dense row segment of
// 4*LG floats is one fully coalesced 16*LG-byte load.  A warp holds 32/LG lane
// groups working on different tasks (at N = 32: four elements per warp
// instruction, like the reference's 8-lane "octets").  Column indices and values
// are staged 32 at a time per lane group in shared memory and read back as
// broadcasts; gathers are issued kUnroll at a time.
//
// Design note, from measurements on B200 (configurations 2-4): the gathers are
// latency-bound, and the number of warps per SM matters more than the depth of
// each warp's load batch, so the kernels are written to stay at 64 registers or
// fewer (4 CTAs of 256 threads per SM).  Within that budget SpMM's block path
// keeps 8 gathers in flight per lane group (-1% to -6% against 4) and the residue
// path, with its per-element group checks, 4.  The residue and block paths are
// separate code regions so their registers do not add up.
#include "ps_common.cuh"
#include "ps_matrix.h"
#include "ps_ops.h"

#include <algorithm>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

namespace psb {
namespace {

constexpr int kWarpsPerBlock = 8;
constexpr int kThreads = kWarpsPerBlock * 32;
constexpr int kChunk = 32;        // staged elements per lane group
constexpr int kUnroll = 4;        // gathers in flight per lane group (residue, SDDMM)
constexpr int kBlockUnroll = 8;   // gathers in flight per lane group (SpMM block groups)
// Gathers in flight per lane group on SpMM residue groups: 8 spills at 64 registers
// and measured 7% slower at N=32 (config 2); 4 keeps the row-word bookkeeping free.
constexpr int kResidueUnroll = 4;
static_assert(kChunk % kUnroll == 0 && kChunk % kBlockUnroll == 0 && kChunk % kResidueUnroll == 0 &&
                  kResidueUnroll % 4 == 0,
              "unrolls must divide the staged chunk");

struct WorksetView {
  const int* col[kMaxWorksets];
  const float* val[kMaxWorksets];
  const int* des[kMaxWorksets];
  int group_len[kMaxWorksets];
  int groups[kMaxWorksets];
  long long len[kMaxWorksets];  // elements of the workset
};

// --- Bounds-checked build ------------------------------------------------------
// With PSB_BOUNDS_CHECK defined (lib/libpowersparse_b200_checked.so, built by
// `python -m powersparse_b200.build`), the operator kernels check every index they
// take from the layout, the task lists or a caller's array before following it.  A
// bad task is skipped and a bad index is not followed (the access is dropped or
// redirected to element 0); the first failure is recorded in g_bounds_status, and the
// launcher waits for the launch and raises it as an error.  No assert or trap: the
// context stays usable.  The release library compiles every check away.
#ifdef PSB_BOUNDS_CHECK
constexpr bool kChecked = true;
#else
constexpr bool kChecked = false;
#endif

enum BoundsCode : unsigned {
  kBadTask = 1,      // task outside its workset, or an unknown workset / group / slot
  kBadColumn = 2,    // column index >= cols
  kBadRow = 3,       // destination row >= rows
  kBadGroup = 4,     // group index past the workset's groups
  kBadPosition = 5,  // CSR position >= nnz
  kBadRowPtr = 6,    // row pointer out of order or past nnz
};

__device__ unsigned long long g_bounds_status;  // (code << 32) | low bits of the bad index; 0: none

// True when 0 <= v < limit; otherwise (checked build) records the failure.
__device__ __forceinline__ bool in_range(long long v, long long limit, unsigned code) {
  if constexpr (kChecked) {
    if (v < 0 || v >= limit) {
      atomicCAS(&g_bounds_status, 0ull, ((unsigned long long)code << 32) | (unsigned long long)(v & 0xffffffffLL));
      return false;
    }
  }
  return true;
}

// v when it is in [0, limit); otherwise (checked build) 0, with the failure recorded.
__device__ __forceinline__ long long checked(long long v, long long limit, unsigned code) {
  return in_range(v, limit, code) ? v : 0;
}

__device__ __forceinline__ void fma4(float4& acc, float s, const float4& b) {
  acc.x = fmaf(s, b.x, acc.x);
  acc.y = fmaf(s, b.y, acc.y);
  acc.z = fmaf(s, b.z, acc.z);
  acc.w = fmaf(s, b.w, acc.w);
}

// Kahan step over a chain of four products: s + c tracks sum(v[i] * b_i); the chain
// (FP32 FMAs, starting from -c) is one addend, so the step's three adds cover four
// products.
__device__ __forceinline__ void kahan4(float& s, float& c, const float* v, float b0, float b1, float b2,
                                       float b3) {
  const float y = fmaf(v[3], b3, fmaf(v[2], b2, fmaf(v[1], b1, fmaf(v[0], b0, -c))));
  const float t = s + y;
  c = (t - s) - y;
  s = t;
}

__device__ __forceinline__ float dot4(const float4& a, const float4& b) {
  return fmaf(a.w, b.w, fmaf(a.z, b.z, fmaf(a.y, b.y, a.x * b.x)));
}

__device__ __forceinline__ void emit4(float* dst, const float4& v, bool atomic) {
  if (atomic) atomicAdd(reinterpret_cast<float4*>(dst), v);
  else __stcs(reinterpret_cast<float4*>(dst), v);
}

struct SpmmArgs {
  WorksetView ws;
  const Task* block_tasks;  // tasks [0, num_block)
  int num_block;
  const Task* res_tasks;    // tasks [num_block, num_tasks)
  int num_tasks;
  const int* res_row;       // row word of every residue element (Matrix::residue_row)
  const float* B;
  float* C;
  long long ldb;  // N
  double* wide_acc;  // [wide rows][N] FP64 slice sums (tasks with slot >= 0)
  const int* pos_ws[kMaxWorksets];  // CSR position of every element (kValues)
  const float* values;              // per-call values in CSR order (kValues)
  int S, rows, cols, nnz, wide_rows;  // index limits (checked build)
  // kPush: per-row countdown of the adds into C still to come in this launch, and
  // the peer replicas (other GPUs' copies of C, at this panel's first row).
  int* pending;
  float* peer[kMaxPushPeers];
  int peers;
};

// kPush epilogue of one add into row `row` of C: counts the add down and, in the
// lane group that made the row's last add, stores the finished row segment to every
// peer replica.  Each lane fences its own atomic add before lane 0 counts, so the
// finishing group reads complete sums from L2; no lane ever waits for another group.
template <int LG>
__device__ __forceinline__ void push_if_finished(const SpmmArgs& a, long long row, int colofs, unsigned gm,
                                                 int l) {
  __threadfence();
  __syncwarp(gm);
  int last = 0;
  if (l == 0) last = atomicSub(a.pending + row, 1) == 1;
  last = __shfl_sync(gm, last, 0, LG);
  if (!last) return;
  __threadfence();
  const float4 v = __ldcg(reinterpret_cast<const float4*>(a.C + row * a.ldb + colofs));
  for (int k = 0; k < a.peers; ++k) __stcg(reinterpret_cast<float4*>(a.peer[k] + row * a.ldb + colofs), v);
}

// Checked build: a task must lie inside its workset (begin <= end <= workset length,
// group < groups) and name an existing wide-row slot.
template <typename Args>
__device__ __forceinline__ bool task_ok(const Args& a, const Task& t) {
  if constexpr (kChecked) {
    if (!in_range(t.ws, a.S, kBadTask)) return false;
    const long long len = a.ws.len[t.ws];
    if (!in_range(t.begin, len + 1, kBadTask) || !in_range(t.end, len + 1, kBadTask) ||
        !in_range(t.end - t.begin, len + 1, kBadTask) || !in_range(t.group, max(a.ws.groups[t.ws], 1), kBadTask))
      return false;
    if (t.slot >= 0 && !in_range(t.slot, a.wide_rows, kBadTask)) return false;
  }
  return true;
}

// SpMM, one task per lane group:
//   C[row(g), slab] (+)= sum over elements e of group g of val[e] * B[col[e], slab].
// Block groups always add atomically and residue groups add atomically only when
// their row has other groups, as in spmm_kernel_block.cu:155-161 and
// spmm_kernel_residue.cu:68-81 of the reference.  Block groups accumulate FP32
// per 32-element chunk and carry the running sum in FP64; slices of wide rows add
// that FP64 sum into the row's FP64 scratch instead of into C (Matrix::wide_rows).
// With kValues the value of element e is a.values[csr_pos[e]] (values supplied per
// call in CSR order) instead of the layout's sp_data[e].  With kPush every add into
// C is followed by push_if_finished.
template <int LG, bool kValues = false, bool kPush = false>
__global__ void __launch_bounds__(kThreads, 4) spmm_fused(const SpmmArgs a) {
  constexpr int NG = 32 / LG;
  // Column indices and values of the staged chunk, read back 4 at a time (one
  // 16-byte shared load each); rows of kChunk + 4 words put the lane groups of a
  // warp 4 banks apart.
  // With one lane group per warp (LG = 32) pairs staged as int2 and read one
  // element at a time measure faster (2-4% at N = 128 on B200).
  constexpr bool kPairs = LG == 32;
  constexpr int kStride = kChunk + 4;
  static_assert(kUnroll == 4, "elements are read from shared memory 4 at a time");
  __shared__ __align__(16) int s_col[kWarpsPerBlock][NG][kStride];
  __shared__ __align__(16) float s_val[kWarpsPerBlock][NG][kStride];
  __shared__ int2 s_cv[kPairs ? kWarpsPerBlock : 1][kChunk + 1];
  __shared__ __align__(16) int s_row[kWarpsPerBlock][NG][kStride];  // residue row words (kChunk + 1 used)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = lane / LG, l = lane % LG;
  const unsigned gm = LG == 32 ? 0xffffffffu : (((1u << LG) - 1u) << (q * LG));
  const int task_id = (blockIdx.x * kWarpsPerBlock + warp) * NG + q;
  if (task_id >= a.num_tasks) return;
  const Task t = task_id < a.num_block ? a.block_tasks[task_id] : a.res_tasks[task_id - a.num_block];
  if (!task_ok(a, t)) return;
  const int* __restrict__ col = a.ws.col[t.ws];
  const float* __restrict__ val = a.ws.val[t.ws];
  const int* __restrict__ des = a.ws.des[t.ws];
  const int colofs = blockIdx.y * (4 * LG) + l * 4;
  const float* __restrict__ Bl = a.B + colofs;
  float* __restrict__ Cl = a.C + colofs;
  int* sc = s_col[warp][q];
  float* sv = s_val[warp][q];
  int2* cv = s_cv[kPairs ? warp : 0];
  auto gather = [&](int c) {
    return __ldg(reinterpret_cast<const float4*>(Bl + checked(c, a.cols, kBadColumn) * a.ldb));
  };
  const int* __restrict__ pos = a.pos_ws[t.ws];
  auto value1 = [&](int e) -> float {
    if constexpr (kValues) return __ldg(a.values + checked(__ldcs(pos + e), a.nnz, kBadPosition));
    else return __ldcs(val + e);
  };
  auto value4 = [&](int e0, int k) -> float4 {  // elements e0 + 4k .. e0 + 4k + 3, e0 16-byte aligned
    if constexpr (kValues) {
      const int4 p = __ldcs(reinterpret_cast<const int4*>(pos + e0) + k);
      return make_float4(__ldg(a.values + checked(p.x, a.nnz, kBadPosition)),
                         __ldg(a.values + checked(p.y, a.nnz, kBadPosition)),
                         __ldg(a.values + checked(p.z, a.nnz, kBadPosition)),
                         __ldg(a.values + checked(p.w, a.nnz, kBadPosition)));
    } else {
      return __ldcs(reinterpret_cast<const float4*>(val + e0) + k);
    }
  };
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);

  if (t.ws == 0) {
    // Residue: groups of <= 31 elements.  Every element carries its row word
    // (destination row | atomic << 31, Matrix::residue_row); a group ends where the
    // next element's word differs or the task ends, so a boundary costs one shared
    // compare, and 8 gathers stay in flight as in the block path.  (Consecutive
    // groups of one row, the fine groups when S == 1, are all atomic and are added
    // as one sum.)
    int* sr = s_row[warp][q];
    for (int base = t.begin; base < t.end; base += kChunk) {
      const int n = min(kChunk, t.end - base);
      // Residue tasks start anywhere, so they are staged element by element.
#pragma unroll
      for (int r = 0; r < kChunk / LG; ++r) {
        const int i = l + r * LG;
        if (i < n) {
          sc[i] = __ldcs(col + base + i);
          sv[i] = value1(base + i);
          sr[i] = __ldcs(a.res_row + base + i);
        }
      }
      if (l == 0) sr[n] = base + n < t.end ? __ldcs(a.res_row + base + n) : -1;  // -1: no row has this word
      __syncwarp(gm);
#pragma unroll 1
      for (int j = 0; j < n; j += kResidueUnroll) {
        float4 b[kResidueUnroll];
#pragma unroll
        for (int u = 0; u < kResidueUnroll; u += 4) {
          const int4 c4 = *reinterpret_cast<const int4*>(sc + j + u);
          if (j + u < n) b[u] = gather(c4.x);
          if (j + u + 1 < n) b[u + 1] = gather(c4.y);
          if (j + u + 2 < n) b[u + 2] = gather(c4.z);
          if (j + u + 3 < n) b[u + 3] = gather(c4.w);
        }
#pragma unroll
        for (int u = 0; u < kResidueUnroll; ++u) {
          if (j + u < n) {
            fma4(acc, sv[j + u], b[u]);
            const int w = sr[j + u];
            if (w != sr[j + u + 1]) {
              const int row = w & 0x7fffffff;
              if (in_range(row, a.rows, kBadRow)) {
                emit4(Cl + (long long)row * a.ldb, acc, w < 0);
                if constexpr (kPush) {
                  // A stored group (w >= 0) is its row's only add of the launch (a residue
                  // group never spans two tasks), so `acc` is the finished segment: it goes
                  // to the peers at once, with no fence or countdown.
                  if (w < 0) {
                    push_if_finished<LG>(a, row, colofs, gm, l);
                  } else {
                    for (int k = 0; k < a.peers; ++k)
                      __stcg(reinterpret_cast<float4*>(a.peer[k] + (long long)row * a.ldb + colofs), acc);
                  }
                }
              }
              acc = make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
        }
      }
      __syncwarp(gm);
    }
    return;
  }

  // Block workset: groups of group_len (a multiple of 32) elements; a task is a
  // whole number of 32-element chunks inside one group or a run of whole groups.
  const int G = a.ws.group_len[t.ws];
  int g = t.group;
  double dx = 0.0, dy = 0.0, dz = 0.0, dw = 0.0;
  for (int base = t.begin; base < t.end; base += kChunk) {
    // Block chunks start on 32-element (128-byte) boundaries: 8 lanes stage the
    // 32 column indices with one 16-byte load each, 8 lanes the 32 values.
    if constexpr (kPairs) {
      cv[l] = make_int2(__ldcs(col + base + l), __float_as_int(value1(base + l)));
    } else if constexpr (LG == 8) {
      *reinterpret_cast<int4*>(sc + 4 * l) = __ldcs(reinterpret_cast<const int4*>(col + base) + l);
      *reinterpret_cast<float4*>(sv + 4 * l) = value4(base, l);
    } else if (l < 8) {
      *reinterpret_cast<int4*>(sc + 4 * l) = __ldcs(reinterpret_cast<const int4*>(col + base) + l);
    } else if (l < 16) {
      *reinterpret_cast<float4*>(sv + 4 * (l - 8)) = value4(base, l - 8);
    }
    __syncwarp(gm);
    // The gathers and values of elements j .. j + 3 of the chunk.
    auto load4 = [&](int j, float4* b, float* vv) {
      if constexpr (kPairs) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int2 e = cv[j + u];
          b[u] = gather(e.x);
          vv[u] = __int_as_float(e.y);
        }
      } else {
        const int4 c0 = *reinterpret_cast<const int4*>(sc + j);
        b[0] = gather(c0.x);
        b[1] = gather(c0.y);
        b[2] = gather(c0.z);
        b[3] = gather(c0.w);
        const float4 v0 = *reinterpret_cast<const float4*>(sv + j);
        vv[0] = v0.x; vv[1] = v0.y; vv[2] = v0.z; vv[3] = v0.w;
      }
    };
    if (t.slot >= 0 && t.sum == kWideExact) {
      // Slices of the longest wide rows add exact products (an FP32 x FP32 product
      // is exact in FP64) in FP64.  Four gathers at a time: the FP64 sums hold the
      // registers of the other four.
#pragma unroll 1
      for (int j = 0; j < kChunk; j += 4) {
        float4 b[4];
        float vv[4];
        load4(j, b, vv);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const double v = vv[u];
          dx = fma(v, double(b[u].x), dx);
          dy = fma(v, double(b[u].y), dy);
          dz = fma(v, double(b[u].z), dz);
          dw = fma(v, double(b[u].w), dw);
        }
      }
    } else if (t.slot >= 0) {
      // Other wide-row slices: chains of four products added by Kahan steps (FP32),
      // the sum and its compensation folded into FP64 separately.  Plain FP32 chunk
      // sums would drift by about sqrt(chunks) * 2^-24 * |chunk sum| over rows of
      // thousands of elements, above the 1e-5 absolute tolerance where the exact
      // value is near zero; rows that are not wide hold at most ~2300 elements and
      // keep them.
      float4 ks = make_float4(0.f, 0.f, 0.f, 0.f), kc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
      for (int j = 0; j < kChunk; j += kBlockUnroll) {
        float4 b[kBlockUnroll];
        float vv[kBlockUnroll];
        load4(j, b, vv);
        load4(j + 4, b + 4, vv + 4);
#pragma unroll
        for (int u = 0; u < kBlockUnroll; u += 4) {
          kahan4(ks.x, kc.x, vv + u, b[u].x, b[u + 1].x, b[u + 2].x, b[u + 3].x);
          kahan4(ks.y, kc.y, vv + u, b[u].y, b[u + 1].y, b[u + 2].y, b[u + 3].y);
          kahan4(ks.z, kc.z, vv + u, b[u].z, b[u + 1].z, b[u + 2].z, b[u + 3].z);
          kahan4(ks.w, kc.w, vv + u, b[u].w, b[u + 1].w, b[u + 2].w, b[u + 3].w);
        }
      }
      dx += double(ks.x) - double(kc.x);
      dy += double(ks.y) - double(kc.y);
      dz += double(ks.z) - double(kc.z);
      dw += double(ks.w) - double(kc.w);
    } else {
      float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);  // FP32 sum of this chunk
#pragma unroll 1
      for (int j = 0; j < kChunk; j += kBlockUnroll) {
        float4 b[kBlockUnroll];
        float vv[kBlockUnroll];
        load4(j, b, vv);
        load4(j + 4, b + 4, vv + 4);
#pragma unroll
        for (int u = 0; u < kBlockUnroll; ++u) fma4(sum, vv[u], b[u]);
      }
      dx += sum.x; dy += sum.y; dz += sum.z; dw += sum.w;
    }
    __syncwarp(gm);
    const int next = base + kChunk;
    if (next == t.end || next % G == 0) {
      if (t.slot >= 0) {
        // A slice of a wide row (one group per task): FP64 sum, folded into C
        // by wide_rows_fold after the launch.
        double* row_sum = a.wide_acc + (long long)t.slot * a.ldb + colofs;
        atomicAdd(row_sum, dx);
        atomicAdd(row_sum + 1, dy);
        atomicAdd(row_sum + 2, dz);
        atomicAdd(row_sum + 3, dw);
      } else {
        if (in_range(g, a.ws.groups[t.ws], kBadGroup) && in_range(des[g], a.rows, kBadRow)) {
          emit4(Cl + (long long)des[g] * a.ldb, make_float4(float(dx), float(dy), float(dz), float(dw)), true);
          if constexpr (kPush) push_if_finished<LG>(a, des[g], colofs, gm, l);
        }
      }
      dx = dy = dz = dw = 0.0;
      ++g;
    }
  }
}

struct SddmmArgs {
  WorksetView ws;
  const Task* block_tasks;  // tasks [0, num_block)
  int num_block;
  const Task* res_tasks;    // tasks [num_block, num_tasks)
  int num_tasks;
  const int* res_row;   // destination row of every residue element
  const float* lhs;
  const float* rhs;
  float* out_ws[kMaxWorksets];
  const int* pos_ws[kMaxWorksets];  // CSR position of every element (CSR-order output)
  float* out_csr;                   // CSR-order output, or nullptr
  int S, rows, cols, nnz, wide_rows;  // index limits (checked build)
};

// Reduces BATCH per-lane partial dot products over the LG lanes of a lane group:
// halving steps on the top log2(BATCH) lane bits (each keeps the half of the
// elements selected by one lane bit and adds the partner's copy of it) leave lane
// l with element l / (LG / BATCH); butterflies on the lower bits finish the sum.
template <int LG, int BATCH>
__device__ __forceinline__ float reduce_batch(float (&p)[BATCH], int l, unsigned gm) {
#pragma unroll
  for (int h = BATCH / 2, bit = LG / 2; h >= 1; h >>= 1, bit >>= 1) {
    const bool upper = l & bit;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float send = upper ? p[i] : p[i + h];
      const float keep = upper ? p[i + h] : p[i];
      p[i] = keep + __shfl_xor_sync(gm, send, bit, LG);
    }
  }
  float v = p[0];
#pragma unroll
  for (int bit = LG / (2 * BATCH); bit >= 1; bit >>= 1) v += __shfl_xor_sync(gm, v, bit, LG);
  return v;
}

// SDDMM, one task per lane group:  out[e] (+)= val[e] * <lhs[row(e)], rhs[col[e]]>.
// A lane covers FC chunks of 4 features, chunk c of lane l being features
// [c*4*LG + 4*l, +4), so every chunk of a dense row is one coalesced 16*LG-byte
// segment and N = 4 * LG * FC.  Elements are reduced BATCH at a time.
// Block outputs are stored (sddmm_kernel_block.cu:160-164 of the reference);
// residue outputs are added, as its residue kernels atomically add into a zeroed
// buffer (sddmm_kernel_residue.cu:297-305).  Residue groups are short, so the
// residue path loads each element's lhs row alongside its rhs row (per-element
// rows from the matrix); block groups span whole 32-element chunks, so the block
// path switches lhs rows once per chunk with the next group's row prefetched.
// With kCsr every output goes to out_csr[csr_pos[e]] (a plain store: each CSR
// position is written exactly once) instead of the workset-order buffers.
// 8-lane groups (N = 32) fit 64 registers and run 4 CTAs per SM (-2% to -8% on B200
// against 3); the 16-lane kernel would spill at that bound and runs 3 (80 registers).
template <int LG, int FC, int BATCH, bool kCsr = false>
__global__ void __launch_bounds__(kThreads, LG == 8 ? 4 : 3) sddmm_fused(const SddmmArgs a) {
  static_assert(BATCH <= LG && kChunk % BATCH == 0, "batch must fit the lane group and the chunk");
  constexpr int kLoadGroup = BATCH < kUnroll ? BATCH : kUnroll;  // gathers issued together
  // Reusing a residue element's lhs row for the next element of the same group
  // pays at N = 128 (512-byte rows) and costs more than it saves at N = 32.
  constexpr bool kReuseRows = 4 * LG * FC >= 128;
  static_assert(BATCH % kLoadGroup == 0, "load groups tile the batch");
  constexpr int NG = 32 / LG;
  constexpr int kLanesPerElem = LG / BATCH;
  constexpr int SEG = 4 * LG;
  constexpr long long N = (long long)SEG * FC;
  __shared__ int s_col[kWarpsPerBlock][NG][kChunk + 1];
  __shared__ float s_val[kWarpsPerBlock][NG][kChunk + 1];
  __shared__ int s_row[kWarpsPerBlock][NG][kChunk + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = lane / LG, l = lane % LG;
  const unsigned gm = LG == 32 ? 0xffffffffu : (((1u << LG) - 1u) << (q * LG));
  const int task_id = (blockIdx.x * kWarpsPerBlock + warp) * NG + q;
  if (task_id >= a.num_tasks) return;
  const Task t = task_id < a.num_block ? a.block_tasks[task_id] : a.res_tasks[task_id - a.num_block];
  if (!task_ok(a, t)) return;
  const int* __restrict__ col = a.ws.col[t.ws];
  const float* __restrict__ val = a.ws.val[t.ws];
  float* __restrict__ out = a.out_ws[t.ws];
  const int* __restrict__ pos = a.pos_ws[t.ws];
  const float* __restrict__ rhs_l = a.rhs + 4 * l;
  const float* __restrict__ lhs_l = a.lhs + 4 * l;
  int* sc = s_col[warp][q];
  float* sv = s_val[warp][q];
  int* sr = s_row[warp][q];
  // Segment c of dense row `row` (< limit) of lhs or rhs.
  auto seg = [](const float* base, long long row, int c, long long limit, unsigned code) {
    return __ldg(reinterpret_cast<const float4*>(base + checked(row, limit, code) * N + c * SEG));
  };

  if (t.ws == 0) {
    float4 xc[FC];  // lhs row segments of the last element handled
    for (int base = t.begin; base < t.end; base += kChunk) {
      const int n = min(kChunk, t.end - base);
      const int last_row = base == t.begin ? -1 : sr[kChunk - 1];
      __syncwarp(gm);
#pragma unroll
      for (int r = 0; r < kChunk / LG; ++r) {
        const int i = l + r * LG;
        if (i < n) {
          sc[i] = __ldcs(col + base + i);
          sv[i] = __ldcs(val + base + i);
          sr[i] = __ldcs(a.res_row + base + i) & 0x7fffffff;  // the row (bit 31: SpMM's atomic flag)
        }
      }
      if (l == 0) sr[kChunk] = last_row;
      __syncwarp(gm);
      for (int j = 0; j < n; j += BATCH) {
        float p[BATCH];
#pragma unroll
        for (int u = 0; u < BATCH; ++u) p[u] = 0.f;
#pragma unroll
        for (int c = 0; c < FC; ++c) {
#pragma unroll
          for (int h = 0; h < BATCH; h += kLoadGroup) {
            // Consecutive elements of a group share their lhs row: with kReuseRows,
            // load it only where the row changes (issued with the rhs loads) and
            // copy it otherwise.
            float4 y[kLoadGroup], x[kLoadGroup];
            bool fresh[kLoadGroup];
#pragma unroll
            for (int u = 0; u < kLoadGroup; ++u) {
              const int e = j + h + u;
              fresh[u] = !kReuseRows || sr[e] != (e == 0 ? sr[kChunk] : sr[e - 1]);
              if (e < n) {
                y[u] = seg(rhs_l, sc[e], c, a.cols, kBadColumn);
                if (fresh[u]) x[u] = seg(lhs_l, sr[e], c, a.rows, kBadRow);
              }
            }
#pragma unroll
            for (int u = 0; u < kLoadGroup; ++u) {
              if (j + h + u < n) {
                if (!fresh[u]) x[u] = u == 0 ? xc[c] : x[u - 1];
                p[h + u] += dot4(x[u], y[u]);
              }
            }
            xc[c] = x[kLoadGroup - 1];
          }
        }
        const float dot = reduce_batch<LG, BATCH>(p, l, gm);
        const int jl = j + l / kLanesPerElem;
        if (l % kLanesPerElem == 0 && jl < n) {
          if constexpr (kCsr) a.out_csr[checked(pos[base + jl], a.nnz, kBadPosition)] = dot * sv[jl];
          else atomicAdd(out + base + jl, dot * sv[jl]);
        }
      }
      __syncwarp(gm);
    }
    return;
  }

  const int* __restrict__ des = a.ws.des[t.ws];
  const int G = a.ws.group_len[t.ws];
  const int groups = a.ws.groups[t.ws];
  int g = t.group;
  float4 x[FC], x_next[FC];
#pragma unroll
  for (int c = 0; c < FC; ++c) x[c] = seg(lhs_l, des[g], c, a.rows, kBadRow);
  const bool more = g + 1 < groups && (g + 1) * G < t.end;
  if (more) {
#pragma unroll
    for (int c = 0; c < FC; ++c) x_next[c] = seg(lhs_l, des[g + 1], c, a.rows, kBadRow);
  }
  for (int base = t.begin; base < t.end; base += kChunk) {
    if (base != t.begin && base % G == 0) {  // the chunk starts group g + 1
      ++g;
#pragma unroll
      for (int c = 0; c < FC; ++c) x[c] = x_next[c];
      if (g + 1 < groups && (g + 1) * G < t.end) {
#pragma unroll
        for (int c = 0; c < FC; ++c) x_next[c] = seg(lhs_l, des[g + 1], c, a.rows, kBadRow);
      }
    }
#pragma unroll
    for (int r = 0; r < kChunk / LG; ++r) {
      const int i = l + r * LG;
      sc[i] = __ldcs(col + base + i);
      sv[i] = __ldcs(val + base + i);
    }
    __syncwarp(gm);
#pragma unroll 1
    for (int j = 0; j < kChunk; j += BATCH) {
      float p[BATCH];
#pragma unroll
      for (int u = 0; u < BATCH; ++u) p[u] = 0.f;
#pragma unroll
      for (int c = 0; c < FC; ++c) {
#pragma unroll
        for (int h = 0; h < BATCH; h += kLoadGroup) {
          float4 y[kLoadGroup];
#pragma unroll
          for (int u = 0; u < kLoadGroup; ++u) y[u] = seg(rhs_l, sc[j + h + u], c, a.cols, kBadColumn);
#pragma unroll
          for (int u = 0; u < kLoadGroup; ++u) p[h + u] += dot4(x[c], y[u]);
        }
      }
      const float dot = reduce_batch<LG, BATCH>(p, l, gm);
      const int jl = j + l / kLanesPerElem;
      if (l % kLanesPerElem == 0) {
        if constexpr (kCsr) a.out_csr[checked(pos[base + jl], a.nnz, kBadPosition)] = dot * sv[jl];
        else out[base + jl] = dot * sv[jl];
      }
    }
    __syncwarp(gm);
  }
}

// C[wide_row[slot], :] = float(C + acc[slot, :]) (one rounding), then acc = 0
// so that the scratch is all-zero for the next call.
// The peer replicas of a push call (n = 0 outside ps_spmm_push).
struct PeerSet {
  float* p[kMaxPushPeers];
  int n;
};

// With peers, the finished row is also stored to every peer replica.
__global__ void __launch_bounds__(256) wide_rows_fold(const int* __restrict__ wide_row, int wide_rows, int N,
                                                      double* __restrict__ acc, float* __restrict__ C, int rows,
                                                      const PeerSet peers) {
  const int per_row = N / 4;
  const long long total = (long long)wide_rows * per_row;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long slot = i / per_row;
    const int q = int(i - slot * per_row);
    double2* a2 = reinterpret_cast<double2*>(acc + slot * N + 4 * q);
    const long long off = checked(wide_row[slot], rows, kBadRow) * N + 4 * q;
    float4* c4 = reinterpret_cast<float4*>(C + off);
    const double2 lo = a2[0], hi = a2[1];
    float4 c = *c4;
    c.x = float(double(c.x) + lo.x);
    c.y = float(double(c.y) + lo.y);
    c.z = float(double(c.z) + hi.x);
    c.w = float(double(c.w) + hi.y);
    *c4 = c;
    for (int k = 0; k < peers.n; ++k) __stcg(reinterpret_cast<float4*>(peers.p[k] + off), c);
    a2[0] = make_double2(0.0, 0.0);
    a2[1] = make_double2(0.0, 0.0);
  }
}

// Stores rows `list[i]` of C (N floats each) to every peer replica.
__global__ void __launch_bounds__(256) push_rows(const int* __restrict__ list, int count, int N,
                                                 const float* __restrict__ C, int rows, const PeerSet peers) {
  const int per_row = N / 4;
  const long long total = (long long)count * per_row;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long k = i / per_row;
    const long long off = checked(list[k], rows, kBadRow) * N + 4 * (i - k * per_row);
    const float4 v = *reinterpret_cast<const float4*>(C + off);
    for (int p = 0; p < peers.n; ++p) __stcg(reinterpret_cast<float4*>(peers.p[p] + off), v);
  }
}

// Adds into C per row of one SpMM launch over the task lists of `a`, counted the way
// spmm_fused adds: a block task that is not a wide-row slice adds once per group it
// ends; a residue task once per run of equal row words (and at its end).
__global__ void __launch_bounds__(256) count_row_adds(const SpmmArgs a, int* __restrict__ count) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.num_tasks; i += gridDim.x * blockDim.x) {
    const Task t = i < a.num_block ? a.block_tasks[i] : a.res_tasks[i - a.num_block];
    if (!task_ok(a, t)) continue;
    if (t.ws == 0) {
      if (t.end <= t.begin) continue;
      int prev = a.res_row[t.begin];
      for (int e = t.begin + 1; e < t.end; ++e) {
        const int w = a.res_row[e];
        if (w != prev) {
          if (in_range(prev & 0x7fffffff, a.rows, kBadRow)) atomicAdd(count + (prev & 0x7fffffff), 1);
          prev = w;
        }
      }
      if (in_range(prev & 0x7fffffff, a.rows, kBadRow)) atomicAdd(count + (prev & 0x7fffffff), 1);
    } else if (t.slot < 0) {
      const int G = a.ws.group_len[t.ws];
      const int* des = a.ws.des[t.ws];
      for (int g = t.begin / G; (long long)g * G < t.end; ++g)
        if (in_range(g, a.ws.groups[t.ws], kBadGroup) && in_range(des[g], a.rows, kBadRow))
          atomicAdd(count + des[g], 1);
    }
  }
}

__global__ void __launch_bounds__(256) zero_listed(const int* __restrict__ list, int count, int* __restrict__ v,
                                                   int rows) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x)
    v[checked(list[i], rows, kBadRow)] = 0;
}

// In-place softmax over each row's entries of a CSR-order array (one warp per row):
// v[p] = exp(v[p] - max_row) / sum_row exp(v[q] - max_row).
__global__ void __launch_bounds__(256) edge_softmax_rows(const int* __restrict__ row_ptr, int rows,
                                                         float* __restrict__ v, int nnz) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const int b = row_ptr[r], e = row_ptr[r + 1];
    if (!in_range(b, nnz + 1LL, kBadRowPtr) || !in_range(e, nnz + 1LL, kBadRowPtr) ||
        !in_range(e - b, nnz + 1LL, kBadRowPtr))
      continue;
    if (b == e) continue;
    float mx = -INFINITY;
    for (int p = b + lane; p < e; p += 32) mx = fmaxf(mx, v[p]);
    for (int d = 16; d > 0; d >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, d));
    float sum = 0.f;
    for (int p = b + lane; p < e; p += 32) {
      const float x = expf(v[p] - mx);
      v[p] = x;
      sum += x;
    }
    for (int d = 16; d > 0; d >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, d);
    const float inv = 1.f / sum;
    for (int p = b + lane; p < e; p += 32) v[p] *= inv;
  }
}

unsigned task_blocks(int num_tasks, int lane_group) {
  const long long per_block = (long long)kWarpsPerBlock * (32 / lane_group);
  return unsigned((num_tasks + per_block - 1) / per_block);
}

// Launches sddmm_fused<LG, FC, BATCH, kCsr> for dense rows of N floats.  The kernel
// addresses rows with its compile-time length 4 * LG * FC, so that must be N: a
// shape launched at another N would read and write past the operands.
template <int LG, int FC, int BATCH, bool kCsr>
void launch_sddmm(const SddmmArgs& a, int N, cudaStream_t stream) {
  if (N != 4 * LG * FC)
    throw std::logic_error("SDDMM kernel shape for N=" + std::to_string(4 * LG * FC) + " launched at N=" +
                           std::to_string(N));
  sddmm_fused<LG, FC, BATCH, kCsr><<<task_blocks(a.num_tasks, LG), kThreads, 0, stream>>>(a);
}

WorksetView view_of(const Matrix& m) {
  WorksetView v{};
  for (int s = 0; s < m.S; ++s) {
    v.col[s] = m.col_ind[s];
    v.val[s] = m.sp_data[s];
    v.des[s] = m.group_des[s];
    v.group_len[s] = s == 0 ? 0 : group_size(s);
    v.groups[s] = m.group_num[s];
    v.len[s] = m.ws_size[s];
  }
  return v;
}

// The task lists of a launch over dense rows of N floats (ps_matrix.h): slice-major
// block order when the gathered operand (cols x N floats) is more than half the
// L2, residue tasks of kFineResidueTaskElems below N = 128.  Returns false when
// the matrix has no work.
template <typename Args>
bool set_tasks(Args& a, const Matrix& m, int N) {
  a.S = m.S;
  a.rows = m.rows;
  a.cols = m.cols;
  a.nnz = m.nnz;
  a.wide_rows = m.wide_rows;
  const int o = (long long)m.cols * N * 4 > m.l2_bytes / 2 ? kSliceOrder : kRowOrder;
  const int r = N < 128 ? kFineResidue : kCoarseResidue;
  a.block_tasks = m.block_tasks[o];
  a.num_block = m.num_block_tasks[o];
  a.res_tasks = m.residue_tasks[r];
  a.num_tasks = m.num_block_tasks[o] + m.num_residue_tasks[r];
  return a.num_tasks > 0;
}

}  // namespace

namespace {

// SpMM with the layout's values (values == nullptr) or with per-call values in CSR
// order (kValues).
// Checked build: waits for the launches on `stream` and raises the first index
// failure the kernels recorded (clearing it).  Nothing in the release build.
void check_bounds(cudaStream_t stream) {
  if constexpr (kChecked) {
    PSB_CUDA(cudaStreamSynchronize(stream));
    unsigned long long status = 0;
    PSB_CUDA(cudaMemcpyFromSymbol(&status, g_bounds_status, sizeof(status)));
    if (status == 0) return;
    const unsigned long long zero = 0;
    PSB_CUDA(cudaMemcpyToSymbol(g_bounds_status, &zero, sizeof(zero)));
    static const char* const what[] = {"", "task outside its workset", "column index out of range",
                                       "destination row out of range", "group index out of range",
                                       "CSR position out of range", "row pointer out of range"};
    const unsigned code = unsigned(status >> 32);
    throw std::runtime_error(std::string("bounds check failed in an operator kernel: ") +
                             (code < 7 ? what[code] : "unknown") + " (index " +
                             std::to_string(int(unsigned(status & 0xffffffffu))) + ")");
  }
}

// The pieces of a push call beyond plain SpMM (kPush): the per-row countdown and
// the peer replicas.
struct PushSetup {
  int* pending = nullptr;
  PeerSet peers{};
};

template <bool kValues, bool kPush = false>
void spmm_run(const Matrix& m, int N, const float* B, float* C, const float* values, cudaStream_t stream,
              const PushSetup& push = PushSetup{}) {
  SpmmArgs a{};
  if (!set_tasks(a, m, N)) return;
  a.ws = view_of(m);
  a.res_row = m.residue_row;
  a.B = B;
  a.C = C;
  a.ldb = N;
  if constexpr (kValues) {
    for (int s = 0; s < m.S; ++s) a.pos_ws[s] = m.csr_pos[s];
    a.values = values;
  }
  if constexpr (kPush) {
    a.pending = push.pending;
    for (int k = 0; k < push.peers.n; ++k) a.peer[k] = push.peers.p[k];
    a.peers = push.peers.n;
  }
  auto launch = [&] {
    if (N % 128 == 0) {
      spmm_fused<32, kValues, kPush><<<dim3(task_blocks(a.num_tasks, 32), N / 128), kThreads, 0, stream>>>(a);
    } else if (N % 64 == 0) {
      spmm_fused<16, kValues, kPush><<<dim3(task_blocks(a.num_tasks, 16), N / 64), kThreads, 0, stream>>>(a);
    } else {
      spmm_fused<8, kValues, kPush><<<dim3(task_blocks(a.num_tasks, 8), N / 32), kThreads, 0, stream>>>(a);
    }
    PSB_LAUNCH_CHECK();
  };
  if (m.wide_rows == 0) {
    launch();
    check_bounds(stream);
    return;
  }
  // Wide rows: the matrix's FP64 scratch.  Eager calls that share it are
  // serialized on the device through wide_ready (the scratch is all-zero again
  // when a call's fold kernel ends).  A larger N grows it: the smaller buffer is
  // retired, not freed, because a CUDA graph captured earlier may still hold it;
  // retired buffers are freed with the matrix.  Captured calls skip the event
  // (replays are ordered by the caller, as documented for ps_spmm).
  std::lock_guard<std::mutex> lock(m.wide_mutex);
  const long long need = (long long)m.wide_rows * N;
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  PSB_CUDA(cudaStreamIsCapturing(stream, &capture));
  if (m.wide_acc_cap < need) {
    if (capture != cudaStreamCaptureStatusNone)
      throw std::runtime_error("SpMM at a new N cannot be captured: call it once with this N before capturing");
    if (m.wide_acc) m.wide_acc_retired.push_back(m.wide_acc);
    m.wide_acc = nullptr;
    m.wide_acc_cap = 0;
    PSB_CUDA(cudaMalloc(reinterpret_cast<void**>(&m.wide_acc), sizeof(double) * size_t(need)));
    PSB_CUDA(cudaMemset(m.wide_acc, 0, sizeof(double) * size_t(need)));
    m.wide_acc_cap = need;
  }
  if (capture == cudaStreamCaptureStatusNone) PSB_CUDA(cudaStreamWaitEvent(stream, m.wide_ready, 0));
  a.wide_acc = m.wide_acc;
  launch();
  const long long total = (long long)m.wide_rows * (N / 4);
  const unsigned blocks = unsigned(std::min<long long>((total + 255) / 256, 8LL * device_sms()));
  wide_rows_fold<<<blocks, 256, 0, stream>>>(m.wide_row, m.wide_rows, N, m.wide_acc, C, m.rows,
                                             kPush ? push.peers : PeerSet{});
  PSB_LAUNCH_CHECK();
  if (capture == cudaStreamCaptureStatusNone) PSB_CUDA(cudaEventRecord(m.wide_ready, stream));
  check_bounds(stream);
}

// First push call at a residue cut: the per-row add counts (wide rows zeroed: the
// fold finishes them), the countdown buffer, the list of rows nothing adds into and
// the event that orders eager push calls.  Synchronous; caller holds push_mutex.
void prepare_push(const Matrix& m, int N, cudaStream_t stream) {
  const int cut = N < 128 ? kFineResidue : kCoarseResidue;
  if (m.push_count[cut]) return;
  SpmmArgs a{};
  set_tasks(a, m, N);
  a.ws = view_of(m);
  a.res_row = m.residue_row;
  DeviceArray<int> count(size_t(m.rows));
  PSB_CUDA(cudaMemsetAsync(count.get(), 0, sizeof(int) * size_t(m.rows), stream));
  const unsigned blocks = unsigned(std::max(1LL, std::min<long long>((a.num_tasks + 255) / 256, 8LL * device_sms())));
  count_row_adds<<<blocks, 256, 0, stream>>>(a, count.get());
  PSB_LAUNCH_CHECK();
  if (m.wide_rows > 0) {
    zero_listed<<<unsigned(std::min<long long>((m.wide_rows + 255) / 256, 8LL * device_sms())), 256, 0, stream>>>(
        m.wide_row, m.wide_rows, count.get(), m.rows);
    PSB_LAUNCH_CHECK();
  }
  PSB_CUDA(cudaStreamSynchronize(stream));
  check_bounds(stream);
  if (m.num_quiet_rows < 0) {
    // Rows that no add reaches and that are not wide: no elements at all (the same
    // rows at either residue cut).
    std::vector<int> h_count(size_t(m.rows)), h_wide(size_t(m.wide_rows)), quiet;
    PSB_CUDA(cudaMemcpy(h_count.data(), count.get(), sizeof(int) * h_count.size(), cudaMemcpyDeviceToHost));
    if (m.wide_rows > 0)
      PSB_CUDA(cudaMemcpy(h_wide.data(), m.wide_row, sizeof(int) * h_wide.size(), cudaMemcpyDeviceToHost));
    std::vector<char> wide(size_t(m.rows), 0);
    for (int r : h_wide) wide[size_t(r)] = 1;
    for (int r = 0; r < m.rows; ++r)
      if (h_count[size_t(r)] == 0 && !wide[size_t(r)]) quiet.push_back(r);
    if (!quiet.empty()) {
      DeviceArray<int> d_quiet(quiet.size());
      PSB_CUDA(cudaMemcpy(d_quiet.get(), quiet.data(), sizeof(int) * quiet.size(), cudaMemcpyHostToDevice));
      m.quiet_rows = d_quiet.release_ownership();
    }
    m.num_quiet_rows = int(quiet.size());
  }
  if (!m.push_pending) {
    DeviceArray<int> pending(size_t(m.rows));
    m.push_pending = pending.release_ownership();
  }
  if (!m.push_ready) PSB_CUDA(cudaEventCreateWithFlags(&m.push_ready, cudaEventDisableTiming));
  m.push_count[cut] = count.release_ownership();
}

}  // namespace

void spmm_launch(const Matrix& m, int N, const float* B, float* C, cudaStream_t stream) {
  spmm_run<false>(m, N, B, C, nullptr, stream);
}

void spmm_values_launch(const Matrix& m, int N, const float* values, const float* B, float* C,
                        cudaStream_t stream) {
  spmm_run<true>(m, N, B, C, values, stream);
}

void spmm_push_launch(const Matrix& m, int N, const float* B, float* C, float* const* peers, int n_peers,
                      cudaStream_t stream) {
  if (N != 32 && N != 64 && N != 128)
    throw std::invalid_argument("ps_spmm_push: N must be 32, 64 or 128 (one column slab per row)");
  if (n_peers < 0 || n_peers > kMaxPushPeers)
    throw std::invalid_argument("ps_spmm_push: between 0 and " + std::to_string(kMaxPushPeers) + " peers");
  if (n_peers > 0 && !peers) throw std::invalid_argument("ps_spmm_push: null peer array");
  PushSetup push;
  for (int k = 0; k < n_peers; ++k) {
    if (!peers[k]) throw std::invalid_argument("ps_spmm_push: null peer replica");
    push.peers.p[k] = peers[k];
  }
  push.peers.n = n_peers;
  std::lock_guard<std::mutex> lock(m.push_mutex);
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  PSB_CUDA(cudaStreamIsCapturing(stream, &capture));
  const int cut = N < 128 ? kFineResidue : kCoarseResidue;
  if (!m.push_count[cut]) {
    if (capture != cudaStreamCaptureStatusNone)
      throw std::runtime_error("ps_spmm_push at a new N cannot be captured: call it once with this N first");
    prepare_push(m, N, stream);
  }
  if (capture == cudaStreamCaptureStatusNone) PSB_CUDA(cudaStreamWaitEvent(stream, m.push_ready, 0));
  PSB_CUDA(cudaMemcpyAsync(m.push_pending, m.push_count[cut], sizeof(int) * size_t(m.rows),
                           cudaMemcpyDeviceToDevice, stream));
  push.pending = m.push_pending;
  spmm_run<false, true>(m, N, B, C, nullptr, stream, push);
  if (m.num_quiet_rows > 0 && n_peers > 0) {
    const long long total = (long long)m.num_quiet_rows * (N / 4);
    const unsigned blocks = unsigned(std::min<long long>((total + 255) / 256, 8LL * device_sms()));
    push_rows<<<blocks, 256, 0, stream>>>(m.quiet_rows, m.num_quiet_rows, N, C, m.rows, push.peers);
    PSB_LAUNCH_CHECK();
  }
  if (capture == cudaStreamCaptureStatusNone) PSB_CUDA(cudaEventRecord(m.push_ready, stream));
  check_bounds(stream);
}

void edge_softmax_launch(const Matrix& m, float* values, cudaStream_t stream) {
  const unsigned blocks = unsigned(std::max<long long>(1, std::min<long long>(((long long)m.rows + 7) / 8, 16LL * device_sms())));
  edge_softmax_rows<<<blocks, 256, 0, stream>>>(m.row_ptr, m.rows, values, m.nnz);
  PSB_LAUNCH_CHECK();
  check_bounds(stream);
}

void sddmm_launch(const Matrix& m, int N, const float* lhs, const float* rhs, float* const* out,
                  cudaStream_t stream) {
  SddmmArgs a{};
  if (!set_tasks(a, m, N)) return;
  a.ws = view_of(m);
  for (int s = 0; s < m.S; ++s) a.out_ws[s] = out[s];
  a.res_row = m.residue_row;
  a.lhs = lhs;
  a.rhs = rhs;
  if (N == 128) {
    launch_sddmm<16, 2, 4, false>(a, N, stream);
  } else {
    launch_sddmm<8, 1, 8, false>(a, N, stream);
  }
  PSB_LAUNCH_CHECK();
  check_bounds(stream);
}

void sddmm_csr_launch(const Matrix& m, int N, const float* lhs, const float* rhs, float* out,
                      cudaStream_t stream) {
  SddmmArgs a{};
  if (!set_tasks(a, m, N)) return;
  a.ws = view_of(m);
  for (int s = 0; s < m.S; ++s) a.pos_ws[s] = m.csr_pos[s];
  a.out_csr = out;
  a.res_row = m.residue_row;
  a.lhs = lhs;
  a.rhs = rhs;
  if (N == 128) {
    launch_sddmm<16, 2, 4, true>(a, N, stream);
  } else {
    launch_sddmm<8, 1, 8, true>(a, N, stream);
  }
  PSB_LAUNCH_CHECK();
  check_bounds(stream);
}

// --- SpMM without allocation (ps_spmm_noalloc) -------------------------------
//
// No counterpart in the reference.  For callers that must not allocate device
// memory while they run: engines that reserve the GPU's memory up front and hand
// it out from their own pool (a cudaMalloc at call time fails or escapes their
// accounting), and latency-bound callers that cannot take the device-wide
// synchronization cudaMalloc / cudaFree may imply.  spmm_launch keeps the FP64
// wide-row scratch in the matrix and grows it with cudaMalloc when N grows; this
// variant runs the same kernels with that scratch in a fixed array of this file,
// which every GPU that loads the library holds until the process exits.
static __device__ __align__(256) double g_noalloc_wide_acc[kNoAllocScratchDoubles];

namespace {

std::mutex g_noalloc_mutex;
std::unordered_map<int, double*> g_noalloc_addr;  // device -> address of g_noalloc_wide_acc

// Device address of the array on `device` (the current device), resolved once
// per device.  The host-side name of the array is not a device address.
double* noalloc_scratch(int device) {
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  const auto it = g_noalloc_addr.find(device);
  if (it != g_noalloc_addr.end()) return it->second;
  double* p = nullptr;
  PSB_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_noalloc_wide_acc));
  g_noalloc_addr.emplace(device, p);
  return p;
}

}  // namespace

void noalloc_prepare(int device) {
  noalloc_scratch(device);
  // With lazy loading (the CUDA 12 default) a kernel's code is loaded onto the
  // device at its first use; querying its attributes loads it now, so the first
  // ps_spmm_noalloc call on a device does not.
  cudaFuncAttributes attr;
  PSB_CUDA(cudaFuncGetAttributes(&attr, spmm_fused<8>));
  PSB_CUDA(cudaFuncGetAttributes(&attr, spmm_fused<16>));
  PSB_CUDA(cudaFuncGetAttributes(&attr, spmm_fused<32>));
  PSB_CUDA(cudaFuncGetAttributes(&attr, wide_rows_fold));
}

void spmm_launch_noalloc(const Matrix& m, int N, const float* B, float* C, cudaStream_t stream) {
  const long long need = (long long)m.wide_rows * N;
  if (need > kNoAllocScratchDoubles)
    throw std::invalid_argument("ps_spmm_noalloc: this matrix needs " + std::to_string(need) +
                                " doubles of scratch at N=" + std::to_string(N) + " (" +
                                std::to_string(m.wide_rows) + " wide rows x N), above the fixed " +
                                std::to_string(kNoAllocScratchDoubles) + " (16 MiB); use ps_spmm");
  SpmmArgs a{};
  if (!set_tasks(a, m, N)) return;
  a.ws = view_of(m);
  a.res_row = m.residue_row;
  a.B = B;
  a.C = C;
  a.ldb = N;
  if (m.wide_rows > 0) {
    // The array keeps whatever the previous call (of any matrix) left in it.
    a.wide_acc = noalloc_scratch(m.device);
    PSB_CUDA(cudaMemsetAsync(a.wide_acc, 0, sizeof(double) * size_t(need), stream));
  }
  if (N % 128 == 0) {
    spmm_fused<32><<<dim3(task_blocks(a.num_tasks, 32), N / 128), kThreads, 0, stream>>>(a);
  } else if (N % 64 == 0) {
    spmm_fused<16><<<dim3(task_blocks(a.num_tasks, 16), N / 64), kThreads, 0, stream>>>(a);
  } else {
    spmm_fused<8><<<dim3(task_blocks(a.num_tasks, 8), N / 32), kThreads, 0, stream>>>(a);
  }
  PSB_LAUNCH_CHECK();
  if (m.wide_rows > 0) {
    const long long total = (long long)m.wide_rows * (N / 4);
    const unsigned blocks = unsigned(std::min<long long>((total + 255) / 256, 8LL * device_sms()));
    wide_rows_fold<<<blocks, 256, 0, stream>>>(m.wide_row, m.wide_rows, N, a.wide_acc, C, m.rows, PeerSet{});
    PSB_LAUNCH_CHECK();
  }
  check_bounds(stream);
}

}  // namespace psb
