/* C ABI of libpowersparse_b200.so: PowerSparse SpMM / SDDMM for B200 (sm_100a).
 *
 * This is the drop-in boundary.  Every entry point takes plain pointers and
 * sizes; device pointers are CUDA device addresses on the device that was
 * current when the matrix was created, and `stream` is a cudaStream_t (NULL =
 * the legacy default stream).  The C++ operator API of the reference
 * (include/PowerSparse_SpMM/PowerSparse_SpMM.h, include/PowerSparse_SDDMM/
 * PowerSparse_SDDMM.h, include/utils/matrix_utils.h in this tree) is a thin
 * layer over these functions.
 *
 * Each replaced reference interface is cited as path:line inside the
 * ParCIS/PowerSparse source tree.
 *
 * Errors: every int-returning call returns PS_OK (0) or an error code and
 * records a message readable with ps_last_error() (thread-local).
 * PS_ERR_INVALID_ARGUMENT corresponds to the reference throwing
 * std::invalid_argument, PS_ERR_CUDA to std::runtime_error from CUDA_CALL
 * (utils/cuda_utils.h:7-14).
 */
#ifndef POWERSPARSE_B200_H
#define POWERSPARSE_B200_H

#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ps_matrix ps_matrix;

enum {
  PS_OK = 0,
  PS_ERR_INVALID_ARGUMENT = 1,
  PS_ERR_CUDA = 2,
  PS_ERR_INTERNAL = 3
};

/* Message of the last failed call on this thread ("" if none). */
const char* ps_last_error(void);

/* Library version string. */
const char* ps_version(void);

/* Preprocess a host CSR matrix into the block/residue worksets on the current
 * device.  Replaces the constructor PowerSparseMatrixGPU(int row_num, int col_num,
 * int nnz_num, const int* row_ptr, const int* col_ind, const float* sp_data)
 * (utils/matrix_utils.h:22-23, utils/matrix_utils.cu:470-663): same validation,
 * same error texts, bit-identical layout.  Synchronous. */
int ps_matrix_create(int row_num, int col_num, int nnz_num, const int* row_ptr,
                     const int* col_ind, const float* sp_data, ps_matrix** out);

/* As ps_matrix_create, with the SM count of the workset heuristic
 * (utils/matrix_utils.cu:37-42) given explicitly (sm_count <= 0: the device's).
 * The layout then equals the reference's on a GPU with that many SMs. */
int ps_matrix_create_sm(int row_num, int col_num, int nnz_num, const int* row_ptr,
                        const int* col_ind, const float* sp_data, int sm_count,
                        ps_matrix** out);

/* Frees the worksets (~PowerSparseMatrixGPU, utils/matrix_utils.h:24, 43-55).
 * Complete outstanding operator calls first.  NULL is ignored. */
void ps_matrix_destroy(ps_matrix* matrix);

/* Layout cache.  No reference counterpart: the reference preprocesses in every
 * constructor.  ps_matrix_save writes the layout (the reference-visible arrays
 * and the CSR position map) to `path`; ps_matrix_load reads it onto the current
 * device, checks every index against the stored shape (a corrupt, truncated or
 * foreign file is PS_ERR_INVALID_ARGUMENT and never reaches a kernel) and
 * derives the rest, skipping the preprocessing.  The layout keeps the SM count it
 * was built for (its S).  ps_matrix_preprocess_ms of a loaded matrix is the load
 * time.  Synchronous. */
int ps_matrix_save(const ps_matrix* matrix, const char* path);
int ps_matrix_load(const char* path, ps_matrix** out);

/* Accessors of utils/matrix_utils.h:30-40 (same meaning, same pointer kinds:
 * ps_matrix_group_num is a host array; the workset arrays are host arrays of
 * device pointers; residue offset / atomic flags are device arrays).  Host-only;
 * a NULL matrix gives 0, or NULL for the pointer accessors (-1 from
 * ps_matrix_workset_size and ps_matrix_device). */
int ps_matrix_row(const ps_matrix* matrix);             /* MatrixRow()        */
int ps_matrix_col(const ps_matrix* matrix);             /* MatrixCol()        */
int ps_matrix_nnz(const ps_matrix* matrix);             /* MatrixNNZ()        */
int ps_matrix_group_type_num(const ps_matrix* matrix);  /* GroupTypeNum()     */
int ps_matrix_group_fine_size(const ps_matrix* matrix); /* GroupFineSize()    */
const int* ps_matrix_group_num(const ps_matrix* matrix);                   /* GroupNum()         */
const int* const* ps_matrix_workset_col_ind(const ps_matrix* matrix);      /* WorksetColInd()    */
const float* const* ps_matrix_workset_sp_data(const ps_matrix* matrix);    /* WorksetSpData()    */
const int* const* ps_matrix_group_destination(const ps_matrix* matrix);    /* GroupDestination() */
const int* ps_matrix_residue_offset(const ps_matrix* matrix);              /* ResidueOffset()    */
const bool* ps_matrix_residue_atomic(const ps_matrix* matrix);             /* ResidueAtomic()    */

/* Host array of GroupTypeNum() device pointers: for workset s, the CSR position
 * (index into the constructor's col_ind / sp_data) of each of its elements, in
 * workset order.  No reference counterpart (the reference keeps no map back to
 * the input order). */
const int* const* ps_matrix_csr_position(const ps_matrix* matrix);

/* Elements in workset s (residue: ResidueOffset()[GroupNum()[0]]; block s:
 * GroupNum()[s] * GROUP_SIZE(s)), as benchmarks/benchmark.cu:147-154 sizes the
 * SDDMM outputs.  Returns -1 for an invalid s. */
long long ps_matrix_workset_size(const ps_matrix* matrix, int s);

/* Wall time of ps_matrix_create, validation of the CSR included (the scope of the
 * reference benchmark's preprocess_ms, benchmarks/benchmark.cu:128-134), milliseconds. */
double ps_matrix_preprocess_ms(const ps_matrix* matrix);

/* CUDA device the matrix lives on. */
int ps_matrix_device(const ps_matrix* matrix);

/* Rows whose block slices SpMM sums in FP64 before adding them to C (rows cut
 * into at least 8 block slices of 256 elements).  No reference counterpart: the
 * reference adds every block group to C in FP32. */
int ps_matrix_wide_rows(const ps_matrix* matrix);

/* FP32 C (+)= A * B on `stream`, asynchronous.  B is [MatrixCol() x N] and C is
 * [MatrixRow() x N], both row-major device arrays; zero C before each
 * independent call.  N: positive multiple of 32 with N/32 <= 65535.  Replaces
 * the kernel launches of PowerSparse::SpMM (PowerSparse_SpMM/PowerSparse_SpMM.h:14-17,
 * PowerSparse_SpMM/spmm_solution.cu:7-34) with one fused launch.  Dense offsets
 * are 64-bit, so the reference's rows*N, cols*N <= INT_MAX limit
 * (utils/matrix_utils.h:72-76) does not apply.
 * Stream capture: on a matrix with wide rows (ps_matrix_wide_rows > 0) the call
 * uses an FP64 scratch kept in the matrix, allocated by the first call at a
 * larger N than before; that first call cannot be captured (PS_ERR_CUDA), so
 * call once eagerly at each N before capturing.  Eager calls on one matrix are
 * ordered on the device by the library; replays of a captured call are not:
 * order them against other calls on the same matrix (one stream, or events).
 * A scratch buffer replaced by a larger one stays allocated until
 * ps_matrix_destroy, so earlier captures stay valid. */
int ps_spmm(const ps_matrix* matrix, int N, const float* B, float* C, void* stream);

/* ps_spmm that allocates no device memory.  No counterpart in the reference.
 * For callers that cannot allocate while they run: engines that reserve the
 * GPU's memory up front and serve it from their own pool, and latency-bound
 * callers that cannot take the synchronization cudaMalloc / cudaFree may imply.
 * ps_spmm keeps an FP64 scratch for wide rows (ps_matrix_wide_rows) in the
 * matrix and grows it with cudaMalloc when N grows; this entry point uses a
 * fixed 16 MiB device array instead (2^21 doubles, held by every GPU that
 * loads the library until exit) and fails with PS_ERR_INVALID_ARGUMENT when
 * ps_matrix_wide_rows(matrix) * N exceeds 2^21.  Same inputs, outputs and
 * results as ps_spmm.  The array's device address is resolved when a matrix is
 * created or loaded on a device (ps_matrix_create / ps_matrix_load): that is
 * where the library's operator code, the array among it, is loaded onto the
 * device and allocated, so the calls themselves allocate nothing.  All calls
 * share the array and it keeps what the last call left in it (each call clears
 * the part it uses): calls that overlap on the GPU (other streams, other
 * matrices) race and give wrong results. */
int ps_spmm_noalloc(const ps_matrix* matrix, int N, const float* B, float* C, void* stream);

/* FP32 SDDMM on `stream`, asynchronous: for every element e of workset s,
 * out[s][e] (+)= A_e * <lhs[row(e), :], rhs[col(e), :]>, outputs in workset order.
 * lhs is [MatrixRow() x N], rhs [MatrixCol() x N], row-major device arrays; `out`
 * is a HOST array of GroupTypeNum() device pointers, each sized
 * ps_matrix_workset_size(s) (may be NULL for an empty workset); zero them before
 * each independent call.  N is 32 or 128.  Replaces the kernel launches of
 * PowerSparse::SDDMM (PowerSparse_SDDMM/PowerSparse_SDDMM.h:14-18,
 * PowerSparse_SDDMM/sddmm_solution.cu:7-50) with one fused launch. */
int ps_sddmm(const ps_matrix* matrix, int N, const float* lhs, const float* rhs,
             float* const* out, void* stream);

/* SDDMM with its output in the constructor's CSR order, asynchronous on `stream`:
 * out[p] = sp_data[p] * <lhs[row(p), :], rhs[col_ind[p], :]> for p in [0, nnz),
 * `out` a device array of MatrixNNZ() floats.  Every position is written once
 * (a store, so `out` needs no zeroing).  N is 32 or 128.  No reference
 * counterpart: the reference returns workset order only
 * (PowerSparse_SDDMM/PowerSparse_SDDMM.h:12); this is the same fused kernel
 * writing through ps_matrix_csr_position, with no separate permutation pass. */
int ps_sddmm_csr(const ps_matrix* matrix, int N, const float* lhs, const float* rhs, float* out,
                 void* stream);

/* SpMM with per-call edge values: C (+)= A' * B, where A' has the matrix's sparsity
 * and the entry at CSR position p is values[p] (device, MatrixNNZ() floats, the
 * constructor's CSR order) instead of sp_data[p].  Same B, C, N and stream rules as
 * ps_spmm.  With ps_sddmm_csr and ps_edge_softmax_csr it forms the attention chain
 * out = softmax_rows(A ⊙ (X Yᵀ)) · B.  No reference counterpart. */
int ps_spmm_values(const ps_matrix* matrix, int N, const float* values, const float* B, float* C,
                   void* stream);

/* In place, for every row r of the matrix: values[p] = exp(values[p] - m_r) /
 * sum_q exp(values[q] - m_r) over the row's CSR positions (m_r the row maximum);
 * empty rows are untouched.  values: device, MatrixNNZ() floats, CSR order.  The
 * row structure is the matrix's own.  No reference counterpart. */
int ps_edge_softmax_csr(const ps_matrix* matrix, float* values, void* stream);

/* SpMM fused with the all-gather of its result across GPUs.  No reference
 * counterpart (the reference is single-GPU).  For row panels on several GPUs whose
 * results every GPU needs whole (the next layer's dense operand): instead of SpMM
 * and then an all-gather, each finished row of C is stored straight into the other
 * GPUs' copies while the kernel still runs.  C (+)= A * B exactly as ps_spmm (same
 * B, C, stream rules), and every row of C, once its last contribution of this call
 * has been added, is also stored to peers[k] + row * N for k < n_peers.  peers is a
 * host array of n_peers (0..7) device pointers that this GPU can write (another
 * GPU's buffer opened with ps_ipc_open, or a buffer of this GPU), each pointing at
 * the row of that replica that corresponds to this matrix's row 0.  N is 32, 64 or
 * 128.  The first call at N < 128 and the first at N = 128 each count, once, how
 * many contributions every row receives (allocates, synchronous, cannot be
 * captured).  Eager calls on one matrix are ordered on the device by the library.
 * A peer's replica is complete once every GPU's call has completed (for example
 * after a collective that follows the call on every GPU); the caller must not let a
 * peer read or overwrite those rows while calls that write them may run. */
int ps_spmm_push(const ps_matrix* matrix, int N, const float* B, float* C, float* const* peers, int n_peers,
                 void* stream);

/* CUDA IPC for ps_spmm_push's peer replicas.  ps_ipc_export writes the IPC handle
 * (PS_IPC_HANDLE_BYTES bytes) of the device allocation that holds `ptr` and ptr's
 * byte offset in it; another process opens the handle with ps_ipc_open (the
 * allocation's base address in that process, peer access enabled on demand) and
 * releases it with ps_ipc_close.  No reference counterpart. */
#define PS_IPC_HANDLE_BYTES 64
int ps_ipc_export(const void* ptr, unsigned char* handle, unsigned long long* offset);
int ps_ipc_open(const unsigned char* handle, void** base);
int ps_ipc_close(void* base);

/* nnz-balanced contiguous row panels for `parts` GPUs: writes cuts[0..parts]
 * with cuts[0] = 0, cuts[parts] = row_num, nondecreasing, panel p = rows
 * [cuts[p], cuts[p+1]).  Cut p is the first row whose row_ptr reaches
 * p * nnz / parts.  Host only.  No reference counterpart (the reference is
 * single-GPU; its only device choice is benchmarks/benchmark.cu:116). */
int ps_partition_rows(int row_num, const int* row_ptr, int parts, int* cuts);

#ifdef __cplusplus
}
#endif

#endif /* POWERSPARSE_B200_H */
