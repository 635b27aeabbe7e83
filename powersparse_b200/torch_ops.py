"""PowerSparse operators registered with PyTorch: ``torch.ops.powersparse.*``.

For GNN code that calls operators through the dispatcher.  The ops take the integer
handle of a ``PowerSparseMatrixGPU`` (``matrix.handle``) and CUDA tensors, run on
PyTorch's current stream and copy nothing (the C ABI reads the tensors in place):

    spmm(handle, B) -> C                     C = A·B, fresh [rows, N] tensor
    spmm_(handle, B, C) -> ()                C (+)= A·B in place (the reference's contract)
    sddmm_csr(handle, lhs, rhs) -> out       out[p] = A_p·<lhs[row(p)], rhs[col(p)]>, CSR order
    sddmm_(handle, lhs, rhs, outs) -> ()     per-workset outputs in workset order, in place

Fake (meta) implementations give shapes for tracing; they read the matrix's
dimensions through the C ABI.  Importing this module registers the ops once.
"""
from __future__ import annotations

from typing import List

import torch

from . import SDDMM, SDDMM_csr, SpMM, load_library

__all__ = ["spmm", "spmm_", "sddmm_csr", "sddmm_"]


def _dims(handle: int):
    lib = load_library()
    return lib.ps_matrix_row(handle), lib.ps_matrix_col(handle), lib.ps_matrix_nnz(handle)


class _Handle:
    """Minimal stand-in for a matrix object: the module-level functions want ``.handle``."""

    def __init__(self, handle: int):
        self.handle = handle

    def GroupTypeNum(self) -> int:
        return load_library().ps_matrix_group_type_num(self.handle)


def _require(t: torch.Tensor, name: str):
    if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous float32 CUDA tensor")


@torch.library.custom_op("powersparse::spmm_", mutates_args=("C",))
def spmm_(handle: int, B: torch.Tensor, C: torch.Tensor) -> None:
    _require(B, "B")
    _require(C, "C")
    SpMM(_Handle(handle), B.shape[1], B, C, torch.cuda.current_stream(B.device))


@torch.library.custom_op("powersparse::spmm", mutates_args=())
def spmm(handle: int, B: torch.Tensor) -> torch.Tensor:
    _require(B, "B")
    rows, _, _ = _dims(handle)
    C = torch.zeros((rows, B.shape[1]), dtype=torch.float32, device=B.device)
    SpMM(_Handle(handle), B.shape[1], B, C, torch.cuda.current_stream(B.device))
    return C


@spmm.register_fake
def _(handle: int, B: torch.Tensor) -> torch.Tensor:
    rows, _, _ = _dims(handle)
    return B.new_empty((rows, B.shape[1]))


@torch.library.custom_op("powersparse::sddmm_csr", mutates_args=())
def sddmm_csr(handle: int, lhs: torch.Tensor, rhs: torch.Tensor) -> torch.Tensor:
    _require(lhs, "lhs")
    _require(rhs, "rhs")
    _, _, nnz = _dims(handle)
    out = torch.empty(nnz, dtype=torch.float32, device=lhs.device)
    SDDMM_csr(_Handle(handle), lhs.shape[1], lhs, rhs, out, torch.cuda.current_stream(lhs.device))
    return out


@sddmm_csr.register_fake
def _(handle: int, lhs: torch.Tensor, rhs: torch.Tensor) -> torch.Tensor:
    _, _, nnz = _dims(handle)
    return lhs.new_empty((nnz,))


@torch.library.custom_op("powersparse::sddmm_", mutates_args=("outs",))
def sddmm_(handle: int, lhs: torch.Tensor, rhs: torch.Tensor, outs: List[torch.Tensor]) -> None:
    _require(lhs, "lhs")
    _require(rhs, "rhs")
    SDDMM(_Handle(handle), lhs.shape[1], lhs, rhs, list(outs), torch.cuda.current_stream(lhs.device))
