"""ctypes view of the CPU oracle (ps_oracle.cpp).  TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference
legs import this module, as the checker.  The product (``powersparse_b200``)
never imports it.
"""
from __future__ import annotations

import ctypes
import dataclasses
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libps_oracle.so")

_i32p = ctypes.POINTER(ctypes.c_int)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64p = ctypes.POINTER(ctypes.c_longlong)
_u8p = ctypes.POINTER(ctypes.c_ubyte)

_lib = None


def build() -> None:
    """Compile libps_oracle.so from ps_oracle.cpp (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.ps_oracle_build.restype = ctypes.c_void_p
        L.ps_oracle_build.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _i32p, _i32p, _f32p,
                                      ctypes.c_int]
        L.ps_oracle_last_error.restype = ctypes.c_char_p
        L.ps_oracle_free.argtypes = [ctypes.c_void_p]
        L.ps_oracle_analyze.argtypes = [ctypes.c_int, _i32p, ctypes.c_int]
        for name in ("group_type_num", "group_fine_size", "signature_len"):
            getattr(L, f"ps_oracle_{name}").argtypes = [ctypes.c_void_p]
        L.ps_oracle_group_num.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.ps_oracle_workset_size.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.ps_oracle_workset_size.restype = ctypes.c_longlong
        for name, rt in (("col_ind", _i32p), ("sp_data", _f32p), ("group_des", _i32p),
                         ("group_order", _i32p), ("csr_pos", _i32p)):
            f = getattr(L, f"ps_oracle_{name}")
            f.argtypes = [ctypes.c_void_p, ctypes.c_int]
            f.restype = rt
        L.ps_oracle_residue_offset.argtypes = [ctypes.c_void_p]
        L.ps_oracle_residue_offset.restype = _i32p
        L.ps_oracle_residue_atomic.argtypes = [ctypes.c_void_p]
        L.ps_oracle_residue_atomic.restype = _u8p
        L.ps_oracle_spmm.argtypes = [ctypes.c_int, _i32p, _i32p, _f32p, ctypes.c_int, _f32p, _f64p,
                                     ctypes.c_int]
        L.ps_oracle_spmm_rows.argtypes = [ctypes.c_int, ctypes.c_int, _i32p, _i32p, _f32p,
                                          ctypes.c_int, _f32p, _f64p, ctypes.c_int]
        L.ps_oracle_sddmm.argtypes = [ctypes.c_int, _i32p, _i64p, _i32p, _f32p, ctypes.c_int, _f32p,
                                      _f32p, _f64p, ctypes.c_int]
        L.ps_oracle_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def _arr(ptr, n: int, dtype) -> np.ndarray:
    if n == 0:
        return np.zeros(0, dtype=dtype)
    return np.ctypeslib.as_array(ptr, shape=(n,)).astype(dtype, copy=True)


@dataclasses.dataclass
class Layout:
    """The reference layout as the oracle restates it (all arrays host numpy)."""
    S: int
    fine: int
    signature_len: int
    group_num: list
    col_ind: list       # per workset int32
    sp_data: list       # per workset float32
    group_des: list     # per workset int32
    residue_offset: np.ndarray
    residue_atomic: np.ndarray
    group_order: list   # per workset: source group index of each final group
    csr_pos: list       # per workset int32: CSR position of each element

    def offsets(self, s: int) -> np.ndarray:
        """Start offsets (int64, length G+1) of the groups of workset ``s``."""
        if s == 0:
            return self.residue_offset.astype(np.int64)
        g = 32 << (s - 1)
        return np.arange(self.group_num[s] + 1, dtype=np.int64) * g


def analyze(row_ptr: np.ndarray, sm_count: int) -> int:
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    return lib().ps_oracle_analyze(len(rp) - 1, _p(rp, _i32p), sm_count)


def build_layout(rows: int, cols: int, row_ptr, col_ind, values, sm_count: int) -> Layout:
    """Restated PowerSparseMatrixGPU constructor; raises ValueError on invalid CSR."""
    L = lib()
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_ind, dtype=np.int32)
    va = np.ascontiguousarray(values, dtype=np.float32)
    h = L.ps_oracle_build(rows, cols, len(ci), _p(rp, _i32p), _p(ci, _i32p), _p(va, _f32p), sm_count)
    if not h:
        raise ValueError(L.ps_oracle_last_error().decode())
    try:
        S = L.ps_oracle_group_type_num(h)
        gn = [L.ps_oracle_group_num(h, s) for s in range(S)]
        sizes = [L.ps_oracle_workset_size(h, s) for s in range(S)]
        return Layout(
            S=S, fine=L.ps_oracle_group_fine_size(h), signature_len=L.ps_oracle_signature_len(h),
            group_num=gn,
            col_ind=[_arr(L.ps_oracle_col_ind(h, s), sizes[s], np.int32) for s in range(S)],
            sp_data=[_arr(L.ps_oracle_sp_data(h, s), sizes[s], np.float32) for s in range(S)],
            group_des=[_arr(L.ps_oracle_group_des(h, s), gn[s], np.int32) for s in range(S)],
            residue_offset=_arr(L.ps_oracle_residue_offset(h), gn[0] + 1, np.int32),
            residue_atomic=_arr(L.ps_oracle_residue_atomic(h), gn[0], np.uint8),
            group_order=[_arr(L.ps_oracle_group_order(h, s), gn[s], np.int32) for s in range(S)],
            csr_pos=[_arr(L.ps_oracle_csr_pos(h, s), sizes[s], np.int32) for s in range(S)],
        )
    finally:
        L.ps_oracle_free(h)


def spmm(row_ptr, col_ind, values, B: np.ndarray, threads: int = 0) -> np.ndarray:
    """FP64 C = A·B accumulated in CSR order (the reference's CheckSpmm)."""
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_ind, dtype=np.int32)
    va = np.ascontiguousarray(values, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    rows, n = len(rp) - 1, B.shape[1]
    C = np.empty((rows, n), dtype=np.float64)
    threads = threads or lib().ps_oracle_max_threads()
    lib().ps_oracle_spmm(rows, _p(rp, _i32p), _p(ci, _i32p), _p(va, _f32p), n, _p(B, _f32p),
                         _p(C, _f64p), threads)
    return C


def spmm_rows(r0: int, r1: int, row_ptr, col_ind, values, B: np.ndarray, threads: int = 0) -> np.ndarray:
    """Rows [r0, r1) of the FP64 SpMM check."""
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_ind, dtype=np.int32)
    va = np.ascontiguousarray(values, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    n = B.shape[1]
    C = np.empty((r1 - r0, n), dtype=np.float64)
    threads = threads or lib().ps_oracle_max_threads()
    lib().ps_oracle_spmm_rows(r0, r1, _p(rp, _i32p), _p(ci, _i32p), _p(va, _f32p), n, _p(B, _f32p),
                              _p(C, _f64p), threads)
    return C


def sddmm(layout: Layout, lhs: np.ndarray, rhs: np.ndarray, threads: int = 0) -> list:
    """FP64 SDDMM per workset, in workset order (the reference's CheckSddmm)."""
    lhs = np.ascontiguousarray(lhs, dtype=np.float32)
    rhs = np.ascontiguousarray(rhs, dtype=np.float32)
    n = lhs.shape[1]
    threads = threads or lib().ps_oracle_max_threads()
    outs = []
    for s in range(layout.S):
        off = np.ascontiguousarray(layout.offsets(s))
        out = np.empty(int(off[-1]), dtype=np.float64)
        if layout.group_num[s]:
            lib().ps_oracle_sddmm(layout.group_num[s], _p(layout.group_des[s], _i32p),
                                  _p(off, _i64p), _p(layout.col_ind[s], _i32p),
                                  _p(layout.sp_data[s], _f32p), n, _p(lhs, _f32p), _p(rhs, _f32p),
                                  _p(out, _f64p), threads)
        outs.append(out)
    return outs


def close(actual: np.ndarray, expected: np.ndarray, atol: float = 1e-5, rtol: float = 1e-4) -> np.ndarray:
    """Elementwise |a - e| <= atol + rtol*|e| with both finite (the reference's Close form,
    benchmarks/benchmark_utils.h:106-109, at the tolerances this build is held to)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    return np.isfinite(a) & np.isfinite(e) & (np.abs(a - e) <= atol + rtol * np.abs(e))
