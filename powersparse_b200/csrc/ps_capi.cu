// extern "C" boundary of libpowersparse_b200.so (declared in include/powersparse_b200.h).
#include "powersparse_b200.h"

#include <cuda.h>

#include "ps_common.cuh"
#include "ps_matrix.h"
#include "ps_ops.h"

#include <algorithm>
#include <cstring>
#include <exception>
#include <new>
#include <stdexcept>
#include <string>

namespace {

thread_local std::string g_last_error;

template <typename F>
int guarded(F&& f) {
  try {
    f();
    g_last_error.clear();
    return PS_OK;
  } catch (const std::invalid_argument& e) {
    g_last_error = e.what();
    return PS_ERR_INVALID_ARGUMENT;
  } catch (const psb::CudaError& e) {
    g_last_error = e.what();
    return PS_ERR_CUDA;
  } catch (const std::bad_alloc&) {
    g_last_error = "host allocation failed";
    return PS_ERR_INTERNAL;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return PS_ERR_INTERNAL;
  } catch (...) {
    g_last_error = "unknown error";
    return PS_ERR_INTERNAL;
  }
}

const psb::Matrix& M(const ps_matrix* h) { return *reinterpret_cast<const psb::Matrix*>(h); }

// cuMemGetAddressRange from the driver, looked up at run time (the library links the
// runtime only): the allocation that holds a device pointer, whose base is what a
// CUDA IPC handle names.
using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
AddressRangeFn address_range() {
  static AddressRangeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    PSB_CUDA(cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !p)
      throw psb::CudaError(cudaErrorNotSupported, "cuMemGetAddressRange is not available from the driver");
    return reinterpret_cast<AddressRangeFn>(p);
  }();
  return fn;
}

void require_device(const psb::Matrix& m) {
  int dev = -1;
  PSB_CUDA(cudaGetDevice(&dev));
  if (dev != m.device)
    throw std::invalid_argument("The matrix lives on CUDA device " + std::to_string(m.device) +
                                " but device " + std::to_string(dev) + " is current");
}

}  // namespace

extern "C" {

const char* ps_last_error(void) { return g_last_error.c_str(); }

const char* ps_version(void) { return "powersparse_b200 0.1 (sm_100a)"; }

int ps_matrix_create_sm(int row_num, int col_num, int nnz_num, const int* row_ptr, const int* col_ind,
                        const float* sp_data, int sm_count, ps_matrix** out) {
  return guarded([&] {
    if (!out) throw std::invalid_argument("ps_matrix_create: null output handle");
    *out = nullptr;
    *out = reinterpret_cast<ps_matrix*>(
        psb::build_matrix(row_num, col_num, nnz_num, row_ptr, col_ind, sp_data, sm_count));
  });
}

int ps_matrix_create(int row_num, int col_num, int nnz_num, const int* row_ptr, const int* col_ind,
                     const float* sp_data, ps_matrix** out) {
  return ps_matrix_create_sm(row_num, col_num, nnz_num, row_ptr, col_ind, sp_data, 0, out);
}

void ps_matrix_destroy(ps_matrix* matrix) { delete reinterpret_cast<psb::Matrix*>(matrix); }

int ps_matrix_save(const ps_matrix* h, const char* path) {
  return guarded([&] {
    if (!h || !path) throw std::invalid_argument("ps_matrix_save: null matrix or path");
    psb::save_matrix(M(h), path);
  });
}

int ps_matrix_load(const char* path, ps_matrix** out) {
  return guarded([&] {
    if (!out || !path) throw std::invalid_argument("ps_matrix_load: null path or output handle");
    *out = nullptr;
    *out = reinterpret_cast<ps_matrix*>(psb::load_matrix(path));
  });
}

// Accessors: host-only reads of the handle; a NULL handle gives 0 / NULL.
int ps_matrix_row(const ps_matrix* h) { return h ? M(h).rows : 0; }
int ps_matrix_col(const ps_matrix* h) { return h ? M(h).cols : 0; }
int ps_matrix_nnz(const ps_matrix* h) { return h ? M(h).nnz : 0; }
int ps_matrix_group_type_num(const ps_matrix* h) { return h ? M(h).S : 0; }
int ps_matrix_group_fine_size(const ps_matrix* h) { return h ? M(h).fine : 0; }
const int* ps_matrix_group_num(const ps_matrix* h) { return h ? M(h).group_num.data() : nullptr; }
const int* const* ps_matrix_workset_col_ind(const ps_matrix* h) {
  return h ? const_cast<const int* const*>(M(h).col_ind.data()) : nullptr;
}
const float* const* ps_matrix_workset_sp_data(const ps_matrix* h) {
  return h ? const_cast<const float* const*>(M(h).sp_data.data()) : nullptr;
}
const int* const* ps_matrix_group_destination(const ps_matrix* h) {
  return h ? const_cast<const int* const*>(M(h).group_des.data()) : nullptr;
}
const int* const* ps_matrix_csr_position(const ps_matrix* h) {
  return h ? const_cast<const int* const*>(M(h).csr_pos.data()) : nullptr;
}
const int* ps_matrix_residue_offset(const ps_matrix* h) { return h ? M(h).residue_offset : nullptr; }
const bool* ps_matrix_residue_atomic(const ps_matrix* h) { return h ? M(h).residue_atomic : nullptr; }
long long ps_matrix_workset_size(const ps_matrix* h, int s) {
  if (!h) return -1;
  const psb::Matrix& m = M(h);
  return (s < 0 || s >= m.S) ? -1 : m.ws_size[s];
}
double ps_matrix_preprocess_ms(const ps_matrix* h) { return h ? M(h).preprocess_ms : 0.0; }
int ps_matrix_device(const ps_matrix* h) { return h ? M(h).device : -1; }
int ps_matrix_wide_rows(const ps_matrix* h) { return h ? M(h).wide_rows : 0; }

int ps_spmm(const ps_matrix* h, int N, const float* B, float* C, void* stream) {
  return guarded([&] {
    if (!h) throw std::invalid_argument("Invalid SpMM buffers or stream count");
    // Same checks as PowerSparse_SpMM/spmm_solution.cu:9-14 (without the 32-bit
    // dense-offset limit, which these kernels do not have).
    if (N <= 0 || N % 32 != 0 || N / 32 > 65535)
      throw std::invalid_argument("SpMM requires N to be a positive multiple of 32, with N/32 <= 65535");
    if (!B || !C) throw std::invalid_argument("Invalid SpMM buffers or stream count");
    const psb::Matrix& m = M(h);
    require_device(m);
    psb::spmm_launch(m, N, B, C, static_cast<cudaStream_t>(stream));
  });
}

int ps_spmm_noalloc(const ps_matrix* h, int N, const float* B, float* C, void* stream) {
  return guarded([&] {
    if (!h) throw std::invalid_argument("Invalid SpMM buffers or stream count");
    if (N <= 0 || N % 32 != 0 || N / 32 > 65535)
      throw std::invalid_argument("SpMM requires N to be a positive multiple of 32, with N/32 <= 65535");
    if (!B || !C) throw std::invalid_argument("Invalid SpMM buffers or stream count");
    const psb::Matrix& m = M(h);
    require_device(m);
    psb::spmm_launch_noalloc(m, N, B, C, static_cast<cudaStream_t>(stream));
  });
}

int ps_sddmm(const ps_matrix* h, int N, const float* lhs, const float* rhs, float* const* out, void* stream) {
  return guarded([&] {
    // Same checks as PowerSparse_SDDMM/sddmm_solution.cu:10-22.
    if (N != 32 && N != 128)
      throw std::invalid_argument("SDDMM dispatcher expects a benchmark width of N=32 or N=128");
    if (!h || !lhs || !rhs || !out) throw std::invalid_argument("Invalid SDDMM buffers or stream count");
    const psb::Matrix& m = M(h);
    for (int s = 0; s < m.S; ++s) {
      if (m.group_num[s] == 0) continue;
      if (!out[s]) throw std::invalid_argument("Missing SDDMM output workset");
    }
    require_device(m);
    psb::sddmm_launch(m, N, lhs, rhs, out, static_cast<cudaStream_t>(stream));
  });
}

int ps_spmm_push(const ps_matrix* h, int N, const float* B, float* C, float* const* peers, int n_peers,
                 void* stream) {
  return guarded([&] {
    if (!h || !B || !C) throw std::invalid_argument("Invalid SpMM buffers or stream count");
    const psb::Matrix& m = M(h);
    require_device(m);
    psb::spmm_push_launch(m, N, B, C, peers, n_peers, static_cast<cudaStream_t>(stream));
  });
}

int ps_ipc_export(const void* ptr, unsigned char* handle, unsigned long long* offset) {
  return guarded([&] {
    if (!ptr || !handle || !offset) throw std::invalid_argument("ps_ipc_export: null argument");
    CUdeviceptr base = 0;
    size_t size = 0;
    const CUresult r = address_range()(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
    if (r != CUDA_SUCCESS)
      throw std::invalid_argument("ps_ipc_export: not a device allocation (cuMemGetAddressRange error " +
                                  std::to_string(int(r)) + ")");
    cudaIpcMemHandle_t h;
    PSB_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    static_assert(sizeof(h) == PS_IPC_HANDLE_BYTES, "CUDA IPC handle size");
    std::memcpy(handle, &h, sizeof(h));
    *offset = static_cast<unsigned long long>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  });
}

int ps_ipc_open(const unsigned char* handle, void** base) {
  return guarded([&] {
    if (!handle || !base) throw std::invalid_argument("ps_ipc_open: null argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    *base = nullptr;
    PSB_CUDA(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
  });
}

int ps_ipc_close(void* base) {
  return guarded([&] {
    if (!base) throw std::invalid_argument("ps_ipc_close: null pointer");
    PSB_CUDA(cudaIpcCloseMemHandle(base));
  });
}

int ps_spmm_values(const ps_matrix* h, int N, const float* values, const float* B, float* C, void* stream) {
  return guarded([&] {
    if (!h) throw std::invalid_argument("Invalid SpMM buffers or stream count");
    if (N <= 0 || N % 32 != 0 || N / 32 > 65535)
      throw std::invalid_argument("SpMM requires N to be a positive multiple of 32, with N/32 <= 65535");
    if (!values || !B || !C) throw std::invalid_argument("Invalid SpMM buffers or stream count");
    const psb::Matrix& m = M(h);
    require_device(m);
    psb::spmm_values_launch(m, N, values, B, C, static_cast<cudaStream_t>(stream));
  });
}

int ps_edge_softmax_csr(const ps_matrix* h, float* values, void* stream) {
  return guarded([&] {
    if (!h || !values) throw std::invalid_argument("ps_edge_softmax_csr: null matrix or values");
    const psb::Matrix& m = M(h);
    require_device(m);
    psb::edge_softmax_launch(m, values, static_cast<cudaStream_t>(stream));
  });
}

int ps_sddmm_csr(const ps_matrix* h, int N, const float* lhs, const float* rhs, float* out, void* stream) {
  return guarded([&] {
    if (N != 32 && N != 128)
      throw std::invalid_argument("SDDMM dispatcher expects a benchmark width of N=32 or N=128");
    if (!h || !lhs || !rhs || !out) throw std::invalid_argument("Invalid SDDMM buffers or stream count");
    const psb::Matrix& m = M(h);
    require_device(m);
    psb::sddmm_csr_launch(m, N, lhs, rhs, out, static_cast<cudaStream_t>(stream));
  });
}

int ps_partition_rows(int row_num, const int* row_ptr, int parts, int* cuts) {
  return guarded([&] {
    if (row_num < 0 || parts <= 0 || !row_ptr || !cuts)
      throw std::invalid_argument("ps_partition_rows: invalid arguments");
    const long long nnz = row_ptr[row_num];
    cuts[0] = 0;
    for (int p = 1; p < parts; ++p) {
      const long long target = (long long)p * nnz / parts;
      const int* at = std::lower_bound(row_ptr, row_ptr + row_num + 1, target,
                                       [](int a, long long b) { return (long long)a < b; });
      int r = int(at - row_ptr);
      r = std::min(std::max(r, cuts[p - 1]), row_num);
      cuts[p] = r;
    }
    cuts[parts] = row_num;
  });
}

}  // extern "C"
