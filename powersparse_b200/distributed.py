"""Row-panel sharding of PowerSparse SpMM / SDDMM over several GPUs.

The reference is single-GPU (its only device choice is the CLI's DEVICE
argument).  Here one process drives one GPU: every rank cuts the same
nnz-balanced contiguous row panels (``partition_rows``), builds a
``PowerSparseMatrixGPU`` over its own panel (row pointer rebased, columns
global) and multiplies against a replicated dense operand.  Results stay
sharded by rows; ``allgather_rows`` assembles the full result on every rank
when a caller asks for a replicated one (padded all-gather: panels differ in
length).  torch.distributed is the plumbing (NCCL for CUDA tensors, gloo for
CPU tensors).
"""
from __future__ import annotations

from typing import Optional

import numpy as np

from . import PowerSparseMatrixGPU, SDDMM, SpMM, partition_rows
from .synth import Csr

__all__ = ["panel_csr", "ShardedPowerSparse", "allgather_rows"]


def panel_csr(m: Csr, r0: int, r1: int) -> Csr:
    """Rows [r0, r1) of ``m`` as a CSR with its own row pointer; columns stay global."""
    rp = m.row_ptr[r0:r1 + 1].astype(np.int64)
    lo, hi = int(rp[0]), int(rp[-1])
    return Csr(r1 - r0, m.cols, (rp - lo).astype(np.int32), m.col_ind[lo:hi], m.values[lo:hi], m.symmetric)


def allgather_rows(local, cuts, group=None):
    """Concatenate every rank's row panel (``local``: [cuts[r+1]-cuts[r], N]) into the
    full [cuts[-1], N] tensor on every rank.  Panels are padded to the longest one for
    one ``all_gather_into_tensor``; collective order is the same on every rank."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    cuts = [int(c) for c in cuts]
    rows = [cuts[r + 1] - cuts[r] for r in range(world)]
    longest = max(rows)
    n = local.shape[1]
    padded = torch.zeros((longest, n), dtype=local.dtype, device=local.device)
    padded[: local.shape[0]].copy_(local)
    gathered = torch.empty((world * longest, n), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(gathered, padded, group=group)
    return torch.cat([gathered[r * longest: r * longest + rows[r]] for r in range(world)])


class ShardedPowerSparse:
    """One rank's share of a row-partitioned PowerSparse matrix.

    ``global_row_ptr`` (host, all rows) fixes the panel cuts identically on every
    rank; ``panel`` is this rank's rows (``panel_csr`` of the global matrix, or
    generated directly).  ``sm_count`` is forwarded to the workset heuristic.
    """

    def __init__(self, global_row_ptr, panel: Csr, rank: int, world: int, sm_count: Optional[int] = None,
                 cuts=None):
        self.rank, self.world = rank, world
        self.cuts = np.asarray(cuts if cuts is not None else partition_rows(global_row_ptr, world))
        r0, r1 = int(self.cuts[rank]), int(self.cuts[rank + 1])
        if panel.rows != r1 - r0:
            raise ValueError(f"panel has {panel.rows} rows, the cut for rank {rank} has {r1 - r0}")
        self.row_begin, self.row_end = r0, r1
        self.matrix = PowerSparseMatrixGPU(panel.rows, panel.cols, panel.nnz, panel.row_ptr, panel.col_ind,
                                           panel.values, sm_count=sm_count)

    def spmm(self, N: int, B, C_local, stream=None, gather: bool = False, group=None):
        """C_local (+)= A_panel · B; with ``gather`` also return the full C on every rank."""
        SpMM(self.matrix, N, B, C_local, stream)
        if gather:
            return allgather_rows(C_local, self.cuts, group)
        return C_local

    def sddmm(self, N: int, lhs_panel, rhs, outputs, stream=None):
        """Per-workset SDDMM outputs of this panel (lhs_panel holds the panel's rows)."""
        SDDMM(self.matrix, N, lhs_panel, rhs, outputs, stream)
        return outputs

    def close(self):
        self.matrix.close()
