"""PowerSparse SpMM / SDDMM for B200, Python view of the C ABI.

This module binds ``lib/libpowersparse_b200.so`` (declared in
``include/powersparse_b200.h``) with ctypes and mirrors the reference's C++
operator API for Python callers and tests:

    PowerSparseMatrixGPU(row_num, col_num, nnz_num, row_ptr, col_ind, sp_data)
        (utils/matrix_utils.h:22-40 of ParCIS/PowerSparse)
    SpMM(matrix, N, B, C, stream=None)             (PowerSparse_SpMM/PowerSparse_SpMM.h:14-17)
    SDDMM(matrix, N, lhs, rhs, outputs, stream=None) (PowerSparse_SDDMM/PowerSparse_SDDMM.h:14-18)

and the additions after the path (no reference counterpart):

    SDDMM_csr(matrix, N, lhs, rhs, out)        SDDMM written in the input's CSR order
    edge_softmax_csr(matrix, values)           per-row softmax of CSR-order edge values
    SpMM_values(matrix, N, values, B, C)       SpMM with per-call CSR-order edge values
    PowerSparseMatrixGPU.save(path) / .load(path)   layout cache
    partition_rows(row_ptr, parts)             nnz-balanced row panels (multi-GPU)

``powersparse_b200.torch_ops`` registers the operators as ``torch.ops.powersparse.*``
and ``powersparse_b200.distributed`` shards them by row panels over torch.distributed.

Errors raise ``ValueError`` where the reference throws std::invalid_argument and
``RuntimeError`` where it throws std::runtime_error.  Dense operands are CUDA
torch tensors (or raw device addresses as ints); every computation runs in the
CUDA library: if the library is missing this module raises instead of
computing anything on the host.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import numpy as np

__all__ = [
    "PowerSparseMatrixGPU", "SpMM", "SDDMM", "SDDMM_csr", "SpMM_values", "edge_softmax_csr", "partition_rows",
    "load_library", "LIB_PATH",
    "GROUP_SIZE", "PS_OK", "PS_ERR_INVALID_ARGUMENT", "PS_ERR_CUDA",
]

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libpowersparse_b200.so")

PS_OK, PS_ERR_INVALID_ARGUMENT, PS_ERR_CUDA, PS_ERR_INTERNAL = 0, 1, 2, 3

_i32p = ctypes.POINTER(ctypes.c_int)
_f32p = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p
_lib = None

# (name, restype, argtypes) of every entry point in include/powersparse_b200.h.
_SIGNATURES = [
    ("ps_last_error", ctypes.c_char_p, []),
    ("ps_version", ctypes.c_char_p, []),
    ("ps_matrix_create", ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _i32p, _i32p, _f32p,
                                        ctypes.POINTER(_vp)]),
    ("ps_matrix_create_sm", ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _i32p, _i32p, _f32p,
                                           ctypes.c_int, ctypes.POINTER(_vp)]),
    ("ps_matrix_destroy", None, [_vp]),
    ("ps_matrix_save", ctypes.c_int, [_vp, ctypes.c_char_p]),
    ("ps_matrix_load", ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    ("ps_matrix_row", ctypes.c_int, [_vp]),
    ("ps_matrix_col", ctypes.c_int, [_vp]),
    ("ps_matrix_nnz", ctypes.c_int, [_vp]),
    ("ps_matrix_group_type_num", ctypes.c_int, [_vp]),
    ("ps_matrix_group_fine_size", ctypes.c_int, [_vp]),
    ("ps_matrix_group_num", _i32p, [_vp]),
    ("ps_matrix_workset_col_ind", ctypes.POINTER(_vp), [_vp]),
    ("ps_matrix_workset_sp_data", ctypes.POINTER(_vp), [_vp]),
    ("ps_matrix_group_destination", ctypes.POINTER(_vp), [_vp]),
    ("ps_matrix_csr_position", ctypes.POINTER(_vp), [_vp]),
    ("ps_matrix_residue_offset", _vp, [_vp]),
    ("ps_matrix_residue_atomic", _vp, [_vp]),
    ("ps_matrix_workset_size", ctypes.c_longlong, [_vp, ctypes.c_int]),
    ("ps_matrix_preprocess_ms", ctypes.c_double, [_vp]),
    ("ps_matrix_device", ctypes.c_int, [_vp]),
    ("ps_matrix_wide_rows", ctypes.c_int, [_vp]),
    ("ps_spmm", ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _vp]),
    ("ps_spmm_noalloc", ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _vp]),
    ("ps_sddmm", ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, ctypes.POINTER(_vp), _vp]),
    ("ps_sddmm_csr", ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _vp, _vp]),
    ("ps_spmm_values", ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _vp, _vp]),
    ("ps_edge_softmax_csr", ctypes.c_int, [_vp, _vp, _vp]),
    ("ps_partition_rows", ctypes.c_int, [ctypes.c_int, _i32p, ctypes.c_int, _i32p]),
    ("ps_spmm_push", ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, ctypes.POINTER(_vp), ctypes.c_int, _vp]),
    ("ps_ipc_export", ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_ulonglong)]),
    ("ps_ipc_open", ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    ("ps_ipc_close", ctypes.c_int, [_vp]),
]

PS_IPC_HANDLE_BYTES = 64


def GROUP_SIZE(s: int) -> int:
    """32 * 2^(s-1), the element count of a block group of workset s (utils/matrix_utils.h:8)."""
    return 32 * (1 << (s - 1))


def load_library(path: Optional[str] = None):
    """Load the CUDA library (raises if it has not been built).  ``path`` defaults to
    the ``PSB_LIBRARY`` environment variable, else ``lib/libpowersparse_b200.so``
    (``lib/libpowersparse_b200_checked.so`` is the bounds-checked debug build)."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or os.environ.get("PSB_LIBRARY") or LIB_PATH
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `python -m powersparse_b200.build` "
                           "(there is no host fallback)")
    lib = ctypes.CDLL(path)
    for name, restype, argtypes in _SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def _check(status: int) -> None:
    if status == PS_OK:
        return
    msg = load_library().ps_last_error().decode()
    if status == PS_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise RuntimeError(msg)


def _dev_ptr(x) -> Optional[int]:
    """Device address of a CUDA tensor / int / None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        if not x.is_cuda:
            raise ValueError("dense operands must be CUDA tensors")
        if not x.is_contiguous():
            raise ValueError("dense operands must be contiguous row-major tensors")
        return int(x.data_ptr())
    raise TypeError(f"cannot take a device address of {type(x).__name__}")


def _stream_ptr(stream) -> Optional[int]:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


class PowerSparseMatrixGPU:
    """Preprocessed block/residue layout on the current CUDA device.

    Same arguments, accessors and errors as the reference class
    (utils/matrix_utils.h:20-69); ``sm_count`` optionally fixes the SM count of
    the workset heuristic (default: the device's).
    """

    def __init__(self, row_num: int, col_num: int, nnz_num: int, row_ptr, col_ind, sp_data,
                 sm_count: Optional[int] = None):
        lib = load_library()
        rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
        ci = np.ascontiguousarray(col_ind, dtype=np.int32)
        va = np.ascontiguousarray(sp_data, dtype=np.float32)
        if rp.shape[0] < row_num + 1 or ci.shape[0] < nnz_num or va.shape[0] < nnz_num:
            raise ValueError("CSR arrays are shorter than the given dimensions")
        h = _vp()
        self._h = None
        _check(lib.ps_matrix_create_sm(row_num, col_num, nnz_num, rp.ctypes.data_as(_i32p),
                                       ci.ctypes.data_as(_i32p), va.ctypes.data_as(_f32p),
                                       int(sm_count or 0), ctypes.byref(h)))
        self._h = h.value

    # -- layout cache (ps_matrix_save / ps_matrix_load)
    def save(self, path: str) -> None:
        """Write the preprocessed layout to ``path`` (load it back with ``PowerSparseMatrixGPU.load``)."""
        _check(load_library().ps_matrix_save(self.handle, os.fsencode(path)))

    @classmethod
    def load(cls, path: str) -> "PowerSparseMatrixGPU":
        """A matrix from a layout file, on the current device, without preprocessing."""
        h = _vp()
        _check(load_library().ps_matrix_load(os.fsencode(path), ctypes.byref(h)))
        self = cls.__new__(cls)
        self._h = h.value
        return self

    # -- lifetime
    def close(self) -> None:
        if self._h:
            load_library().ps_matrix_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self) -> int:
        if not self._h:
            raise ValueError("matrix has been released")
        return self._h

    # -- accessors (utils/matrix_utils.h:30-40)
    def MatrixRow(self) -> int:
        return load_library().ps_matrix_row(self.handle)

    def MatrixCol(self) -> int:
        return load_library().ps_matrix_col(self.handle)

    def MatrixNNZ(self) -> int:
        return load_library().ps_matrix_nnz(self.handle)

    def GroupTypeNum(self) -> int:
        return load_library().ps_matrix_group_type_num(self.handle)

    def GroupFineSize(self) -> int:
        return load_library().ps_matrix_group_fine_size(self.handle)

    def GroupNum(self) -> list:
        p = load_library().ps_matrix_group_num(self.handle)
        return [p[s] for s in range(self.GroupTypeNum())]

    def _ptrs(self, fn) -> list:
        p = fn(self.handle)
        return [p[s] or 0 for s in range(self.GroupTypeNum())]

    def WorksetColInd(self) -> list:
        return self._ptrs(load_library().ps_matrix_workset_col_ind)

    def WorksetSpData(self) -> list:
        return self._ptrs(load_library().ps_matrix_workset_sp_data)

    def GroupDestination(self) -> list:
        return self._ptrs(load_library().ps_matrix_group_destination)

    def CsrPosition(self) -> list:
        """Per workset: device pointer to the CSR position of each element (ps_matrix_csr_position)."""
        return self._ptrs(load_library().ps_matrix_csr_position)

    def ResidueOffset(self) -> int:
        return load_library().ps_matrix_residue_offset(self.handle) or 0

    def ResidueAtomic(self) -> int:
        return load_library().ps_matrix_residue_atomic(self.handle) or 0

    # -- extras
    def workset_size(self, s: int) -> int:
        return int(load_library().ps_matrix_workset_size(self.handle, s))

    @property
    def preprocess_ms(self) -> float:
        return float(load_library().ps_matrix_preprocess_ms(self.handle))

    @property
    def device(self) -> int:
        return int(load_library().ps_matrix_device(self.handle))

    @property
    def wide_rows(self) -> int:
        """Rows whose block slices SpMM sums in FP64 (ps_matrix_wide_rows)."""
        return int(load_library().ps_matrix_wide_rows(self.handle))

    def download(self) -> dict:
        """Copy the layout to host numpy arrays (ReadWorkset of benchmarks/benchmark.cu:29-41)."""
        import torch
        S = self.GroupTypeNum()
        gn = self.GroupNum()
        out = {"S": S, "fine": self.GroupFineSize(), "group_num": gn}
        res = _device_array(self.ResidueOffset(), gn[0] + 1, torch.int32)
        out["res_off"] = res
        out["res_atomic"] = _device_array(self.ResidueAtomic(), gn[0], torch.uint8)
        cols, vals, des = self.WorksetColInd(), self.WorksetSpData(), self.GroupDestination()
        for s in range(S):
            n = self.workset_size(s)
            out[f"ws{s}_col"] = _device_array(cols[s], n, torch.int32)
            out[f"ws{s}_val"] = _device_array(vals[s], n, torch.float32)
            out[f"ws{s}_des"] = _device_array(des[s], gn[s], torch.int32)
            out[f"ws{s}_pos"] = _device_array(self.CsrPosition()[s], n, torch.int32)
        return out


class _CudaArrayView:
    """Minimal __cuda_array_interface__ over a raw device address (no copy)."""

    def __init__(self, ptr: int, count: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (count,), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def _device_array(ptr: int, count: int, dtype) -> np.ndarray:
    import torch
    np_dtype = {torch.int32: np.int32, torch.float32: np.float32, torch.uint8: np.uint8}[dtype]
    if count == 0 or not ptr:
        return np.zeros(0, dtype=np_dtype)
    typestr = {torch.int32: "<i4", torch.float32: "<f4", torch.uint8: "|u1"}[dtype]
    t = torch.as_tensor(_CudaArrayView(ptr, count, typestr), device="cuda")
    return t.cpu().numpy().copy()


def SpMM(matrix: PowerSparseMatrixGPU, N: int, B, C, stream=None) -> None:
    """C (+)= A·B on ``stream`` (asynchronous).  Zero C before each independent call."""
    _check(load_library().ps_spmm(matrix.handle, int(N), _dev_ptr(B), _dev_ptr(C), _stream_ptr(stream)))


def SDDMM(matrix: PowerSparseMatrixGPU, N: int, lhs, rhs, outputs: Sequence, stream=None) -> None:
    """out[s] (+)= A_e·<lhs[row], rhs[col]> per workset, in workset order (asynchronous)."""
    S = matrix.GroupTypeNum()
    if len(outputs) != S:
        raise ValueError("Invalid SDDMM buffers or stream count")
    arr = (_vp * S)(*[_dev_ptr(o) for o in outputs])
    _check(load_library().ps_sddmm(matrix.handle, int(N), _dev_ptr(lhs), _dev_ptr(rhs), arr,
                                   _stream_ptr(stream)))


def SDDMM_csr(matrix: PowerSparseMatrixGPU, N: int, lhs, rhs, out, stream=None) -> None:
    """out[p] = A_p·<lhs[row(p)], rhs[col(p)]> in the constructor's CSR order (``out``: nnz floats)."""
    _check(load_library().ps_sddmm_csr(matrix.handle, int(N), _dev_ptr(lhs), _dev_ptr(rhs), _dev_ptr(out),
                                       _stream_ptr(stream)))


def SpMM_values(matrix: PowerSparseMatrixGPU, N: int, values, B, C, stream=None) -> None:
    """C (+)= A'·B with per-call edge values ``values`` (nnz floats, CSR order) in A's pattern."""
    _check(load_library().ps_spmm_values(matrix.handle, int(N), _dev_ptr(values), _dev_ptr(B), _dev_ptr(C),
                                         _stream_ptr(stream)))


def edge_softmax_csr(matrix: PowerSparseMatrixGPU, values, stream=None) -> None:
    """In place: softmax over each row's edge values (nnz floats, CSR order)."""
    _check(load_library().ps_edge_softmax_csr(matrix.handle, _dev_ptr(values), _stream_ptr(stream)))


def SpMM_push(matrix: PowerSparseMatrixGPU, N: int, B, C, peers: Sequence[int], stream=None) -> None:
    """C (+)= A·B as SpMM, with every finished row of C also stored to each peer replica
    (``peers``: device addresses of the replicas' rows matching this matrix's row 0)."""
    arr = (_vp * max(1, len(peers)))(*[_vp(int(p)) for p in peers])
    _check(load_library().ps_spmm_push(matrix.handle, int(N), _dev_ptr(B), _dev_ptr(C), arr, len(peers),
                                       _stream_ptr(stream)))


def ipc_export(tensor) -> tuple:
    """(CUDA IPC handle bytes, byte offset) of the device allocation holding ``tensor``."""
    handle = ctypes.create_string_buffer(PS_IPC_HANDLE_BYTES)
    offset = ctypes.c_ulonglong(0)
    _check(load_library().ps_ipc_export(_dev_ptr(tensor), handle, ctypes.byref(offset)))
    return handle.raw, int(offset.value)


def ipc_open(handle: bytes) -> int:
    """Opens a handle from ipc_export in another process; returns the allocation's base address."""
    if len(handle) != PS_IPC_HANDLE_BYTES:
        raise ValueError("an IPC handle is %d bytes" % PS_IPC_HANDLE_BYTES)
    base = _vp()
    _check(load_library().ps_ipc_open(handle, ctypes.byref(base)))
    return int(base.value)


def ipc_close(base: int) -> None:
    """Releases a mapping made by ipc_open."""
    _check(load_library().ps_ipc_close(_vp(int(base))))


def partition_rows(row_ptr, parts: int) -> np.ndarray:
    """nnz-balanced contiguous row panels: cut points [parts + 1] (host)."""
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    cuts = np.zeros(parts + 1, dtype=np.int32)
    _check(load_library().ps_partition_rows(len(rp) - 1, rp.ctypes.data_as(_i32p), int(parts),
                                            cuts.ctypes.data_as(_i32p)))
    return cuts
