// Fused SpMM and SDDMM over the PowerSparse worksets (sm_100a, FP32 CUDA cores).
//
// The reference launches one kernel per workset on its own stream and
// device-synchronizes (PowerSparse_SpMM/spmm_solution.cu:16-33,
// PowerSparse_SDDMM/sddmm_solution.cu:23-49).  Here one launch covers every
// workset: the matrix carries a task list (ps_matrix.h) and each warp runs one
// task, a contiguous element range of one workset, largest groups first.
//
// Lane layout: a warp owns a slab of 32*VEC consecutive columns of the dense
// operand and handles one sparse element at a time, so every gathered dense row
// segment is one fully coalesced 128*VEC-byte load (float4 per lane at N=128).
// Column indices and values are staged per warp in shared memory 32 at a time
// and read back as broadcasts.
#include "ps_common.cuh"
#include "ps_matrix.h"
#include "ps_ops.h"

namespace psb {
namespace {

constexpr int kWarpsPerBlock = 8;
constexpr int kThreads = kWarpsPerBlock * 32;

struct WorksetView {
  const int* col[kMaxWorksets];
  const float* val[kMaxWorksets];
  const int* des[kMaxWorksets];
};

template <int VEC> struct VecT;
template <> struct VecT<1> { using T = float; };
template <> struct VecT<2> { using T = float2; };
template <> struct VecT<4> { using T = float4; };

template <int VEC>
__device__ __forceinline__ void load_vec(const float* __restrict__ p, float (&v)[VEC]) {
  if constexpr (VEC == 4) {
    const float4 x = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
  } else if constexpr (VEC == 2) {
    const float2 x = __ldg(reinterpret_cast<const float2*>(p));
    v[0] = x.x; v[1] = x.y;
  } else {
    v[0] = __ldg(p);
  }
}

// Adds (atomic) or stores one lane's VEC outputs.
template <int VEC>
__device__ __forceinline__ void emit(float* __restrict__ dst, const float (&v)[VEC], bool atomic) {
  if (atomic) {
    if constexpr (VEC == 4) {
      atomicAdd(reinterpret_cast<float4*>(dst), make_float4(v[0], v[1], v[2], v[3]));
    } else if constexpr (VEC == 2) {
      atomicAdd(reinterpret_cast<float2*>(dst), make_float2(v[0], v[1]));
    } else {
      atomicAdd(dst, v[0]);
    }
  } else {
    if constexpr (VEC == 4) {
      *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
    } else if constexpr (VEC == 2) {
      *reinterpret_cast<float2*>(dst) = make_float2(v[0], v[1]);
    } else {
      *dst = v[0];
    }
  }
}

struct SpmmArgs {
  WorksetView ws;
  const Task* tasks;
  int num_tasks;
  const int* res_off;
  const bool* res_atomic;
  int res_groups;
  const float* B;
  float* C;
  long long ldb;  // N
  int group_len[kMaxWorksets];
};

// SpMM: C[row(g), :] (+)= sum over elements e of group g of val[e] * B[col[e], :].
// Block groups always add atomically and residue groups add atomically only when
// their row has other groups, as in spmm_kernel_block.cu:155-161 and
// spmm_kernel_residue.cu:68-81 of the reference.  Block groups accumulate FP32
// per 32-element chunk and carry the running sum in FP64.
template <int VEC, int UNROLL>
__global__ void __launch_bounds__(kThreads) spmm_fused(const SpmmArgs a) {
  __shared__ int s_col[kWarpsPerBlock][32];
  __shared__ float s_val[kWarpsPerBlock][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int task_id = blockIdx.x * kWarpsPerBlock + warp;
  if (task_id >= a.num_tasks) return;
  const Task t = a.tasks[task_id];
  const int* __restrict__ col = a.ws.col[t.ws];
  const float* __restrict__ val = a.ws.val[t.ws];
  const int* __restrict__ des = a.ws.des[t.ws];
  const long long colofs = (long long)blockIdx.y * (32 * VEC) + lane * VEC;
  const float* __restrict__ Bl = a.B + colofs;
  float* __restrict__ Cl = a.C + colofs;
  int* sc = s_col[warp];
  float* sv = s_val[warp];

  float acc[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) acc[v] = 0.f;

  if (t.ws == 0) {
    // Residue: groups of <= 31 elements, boundaries from the residue offsets.
    // Lane i holds the metadata of group (wbase + i); it is read by shuffles.
    int wbase = t.group;
    int g_end = 0, g_row = 0, g_atomic = 0;
    {
      const int gi = wbase + lane;
      if (gi < a.res_groups) {
        g_end = a.res_off[gi + 1];
        g_row = des[gi];
        g_atomic = a.res_atomic[gi];
      }
    }
    int widx = 0;
    int cur_end = __shfl_sync(0xffffffffu, g_end, 0);
    int cur_row = __shfl_sync(0xffffffffu, g_row, 0);
    bool cur_atomic = __shfl_sync(0xffffffffu, g_atomic, 0);
    for (int base = t.begin; base < t.end; base += 32) {
      const int n = min(32, t.end - base);
      if (lane < n) {
        sc[lane] = __ldcs(col + base + lane);
        sv[lane] = __ldcs(val + base + lane);
      }
      __syncwarp();
      for (int j = 0; j < n; j += UNROLL) {
        float b[UNROLL][VEC];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
          if (j + u < n) load_vec<VEC>(Bl + (long long)sc[j + u] * a.ldb, b[u]);
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
          if (j + u < n) {
            const int pos = base + j + u;
            if (pos == cur_end) {
              emit<VEC>(Cl + (long long)cur_row * a.ldb, acc, cur_atomic);
#pragma unroll
              for (int v = 0; v < VEC; ++v) acc[v] = 0.f;
              if (++widx == 32) {
                wbase += 32;
                widx = 0;
                const int gi = wbase + lane;
                if (gi < a.res_groups) {
                  g_end = a.res_off[gi + 1];
                  g_row = des[gi];
                  g_atomic = a.res_atomic[gi];
                }
              }
              cur_end = __shfl_sync(0xffffffffu, g_end, widx);
              cur_row = __shfl_sync(0xffffffffu, g_row, widx);
              cur_atomic = __shfl_sync(0xffffffffu, g_atomic, widx);
            }
            const float s = sv[j + u];
#pragma unroll
            for (int v = 0; v < VEC; ++v) acc[v] = fmaf(s, b[u][v], acc[v]);
          }
        }
      }
      __syncwarp();
    }
    emit<VEC>(Cl + (long long)cur_row * a.ldb, acc, cur_atomic);
    return;
  }

  // Block workset: every group has group_len elements, all added atomically.
  const int G = a.group_len[t.ws];
  int g = t.group;
  double accd[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) accd[v] = 0.0;
  for (int base = t.begin; base < t.end; base += 32) {
    sc[lane] = __ldcs(col + base + lane);
    sv[lane] = __ldcs(val + base + lane);
    __syncwarp();
#pragma unroll 1
    for (int j = 0; j < 32; j += UNROLL) {
      float b[UNROLL][VEC];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) load_vec<VEC>(Bl + (long long)sc[j + u] * a.ldb, b[u]);
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const float s = sv[j + u];
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[v] = fmaf(s, b[u][v], acc[v]);
      }
    }
    __syncwarp();
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      accd[v] += double(acc[v]);
      acc[v] = 0.f;
    }
    const int next = base + 32;
    if (next == t.end || next % G == 0) {
      float out[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        out[v] = float(accd[v]);
        accd[v] = 0.0;
      }
      emit<VEC>(Cl + (long long)des[g] * a.ldb, out, true);
      ++g;
    }
  }
}

struct SddmmArgs {
  WorksetView ws;
  const Task* tasks;
  int num_tasks;
  const int* res_off;
  const float* lhs;
  const float* rhs;
  float* out_ws[kMaxWorksets];
  int group_len[kMaxWorksets];
};

// Reduces 32 per-lane partial sums (one per element) across the warp so that lane
// l ends with the full sum of element l: halve the element set each step, keep
// the half selected by the lane bit, add the partner's copy of it (31 shuffles).
__device__ __forceinline__ float transpose_reduce32(float (&p)[32], int lane) {
#pragma unroll
  for (int k = 16; k >= 1; k >>= 1) {
    const bool upper = lane & k;
#pragma unroll
    for (int i = 0; i < k; ++i) {
      const float send = upper ? p[i] : p[i + k];
      const float keep = upper ? p[i + k] : p[i];
      p[i] = keep + __shfl_xor_sync(0xffffffffu, send, k);
    }
  }
  return p[0];
}

// SDDMM: out[e] (+)= val[e] * <lhs[row(g)], rhs[col[e]]> for every element e of
// group g, N = 32 * VEC.  Block outputs are stored (sddmm_kernel_block.cu:160-164);
// residue outputs are added, matching the reference's atomicAdd into a zeroed
// buffer (sddmm_kernel_residue.cu:297-305).
template <int VEC, int UNROLL>
__global__ void __launch_bounds__(kThreads) sddmm_fused(const SddmmArgs a) {
  __shared__ int s_col[kWarpsPerBlock][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int task_id = blockIdx.x * kWarpsPerBlock + warp;
  if (task_id >= a.num_tasks) return;
  const Task t = a.tasks[task_id];
  const int* __restrict__ col = a.ws.col[t.ws];
  const float* __restrict__ val = a.ws.val[t.ws];
  const int* __restrict__ des = a.ws.des[t.ws];
  float* __restrict__ out = a.out_ws[t.ws];
  const long long N = 32 * VEC;
  const float* __restrict__ rhs_l = a.rhs + lane * VEC;
  const float* __restrict__ lhs_l = a.lhs + lane * VEC;
  int* sc = s_col[warp];
  const bool residue = t.ws == 0;
  const int G = residue ? 0 : a.group_len[t.ws];

  int g = t.group;
  int cur_end = residue ? a.res_off[g + 1] : (g + 1) * G;
  float x[VEC];
  load_vec<VEC>(lhs_l + (long long)des[g] * N, x);

  for (int base = t.begin; base < t.end; base += 32) {
    const int n = min(32, t.end - base);
    const float my_val = lane < n ? __ldcs(val + base + lane) : 0.f;
    if (lane < n) sc[lane] = __ldcs(col + base + lane);
    __syncwarp();
    float p[32];
#pragma unroll
    for (int j0 = 0; j0 < 32; j0 += UNROLL) {
      float y[UNROLL][VEC];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        if (j0 + u < n) load_vec<VEC>(rhs_l + (long long)sc[j0 + u] * N, y[u]);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int j = j0 + u;
        float d = 0.f;
        if (j < n) {
          if (base + j == cur_end) {
            ++g;
            cur_end = residue ? a.res_off[g + 1] : (g + 1) * G;
            load_vec<VEC>(lhs_l + (long long)des[g] * N, x);
          }
#pragma unroll
          for (int v = 0; v < VEC; ++v) d = fmaf(x[v], y[u][v], d);
        }
        p[j] = d;
      }
    }
    const float dot = transpose_reduce32(p, lane);
    if (lane < n) {
      const float r = dot * my_val;
      if (residue) atomicAdd(out + base + lane, r);
      else out[base + lane] = r;
    }
    __syncwarp();
  }
}

unsigned task_blocks(int num_tasks) { return unsigned((num_tasks + kWarpsPerBlock - 1) / kWarpsPerBlock); }

}  // namespace

void spmm_launch(const Matrix& m, int N, const float* B, float* C, cudaStream_t stream) {
  if (m.num_tasks == 0) return;
  SpmmArgs a{};
  for (int s = 0; s < m.S; ++s) {
    a.ws.col[s] = m.col_ind[s];
    a.ws.val[s] = m.sp_data[s];
    a.ws.des[s] = m.group_des[s];
    a.group_len[s] = s == 0 ? 0 : group_size(s);
  }
  a.tasks = m.tasks;
  a.num_tasks = m.num_tasks;
  a.res_off = m.residue_offset;
  a.res_atomic = m.residue_atomic;
  a.res_groups = m.group_num[0];
  a.B = B;
  a.C = C;
  a.ldb = N;
  const unsigned gx = task_blocks(m.num_tasks);
  if (N % 128 == 0) {
    spmm_fused<4, 8><<<dim3(gx, N / 128), kThreads, 0, stream>>>(a);
  } else if (N % 64 == 0) {
    spmm_fused<2, 8><<<dim3(gx, N / 64), kThreads, 0, stream>>>(a);
  } else {
    spmm_fused<1, 16><<<dim3(gx, N / 32), kThreads, 0, stream>>>(a);
  }
  PSB_LAUNCH_CHECK();
}

void sddmm_launch(const Matrix& m, int N, const float* lhs, const float* rhs, float* const* out,
                  cudaStream_t stream) {
  if (m.num_tasks == 0) return;
  SddmmArgs a{};
  for (int s = 0; s < m.S; ++s) {
    a.ws.col[s] = m.col_ind[s];
    a.ws.val[s] = m.sp_data[s];
    a.ws.des[s] = m.group_des[s];
    a.group_len[s] = s == 0 ? 0 : group_size(s);
    a.out_ws[s] = out[s];
  }
  a.tasks = m.tasks;
  a.num_tasks = m.num_tasks;
  a.res_off = m.residue_offset;
  a.lhs = lhs;
  a.rhs = rhs;
  const unsigned gx = task_blocks(m.num_tasks);
  if (N == 128) {
    sddmm_fused<4, 8><<<gx, kThreads, 0, stream>>>(a);
  } else {
    sddmm_fused<1, 16><<<gx, kThreads, 0, stream>>>(a);
  }
  PSB_LAUNCH_CHECK();
}

}  // namespace psb
