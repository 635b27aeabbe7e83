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

import time
from typing import Optional

import numpy as np

from . import PowerSparseMatrixGPU, SDDMM, SpMM, SpMM_push, ipc_close, ipc_export, ipc_open, partition_rows
from .synth import Csr

__all__ = ["panel_csr", "ShardedPowerSparse", "allgather_rows", "heartbeat", "PeerLost", "Replicas"]


class PeerLost(RuntimeError):
    """A rank of the process group stopped taking part: it failed, left between
    steps, or never reached the step."""


def heartbeat(step: int, timeout_s: float = 10.0, group=None, store=None) -> None:
    """Host-side liveness check at the start of a step, before its launches: every
    rank announces (step, rank) in the process group's key-value store and waits up
    to ``timeout_s`` seconds for the announcements of the others.  A rank that failed
    or left between steps is found here, on the host, before this step issues any
    kernel or collective; raises PeerLost naming the missing ranks.  Every rank must
    call it with the same step numbers."""
    import torch.distributed as dist
    if store is None:
        store = dist.distributed_c10d._get_default_store()
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    store.set(f"psb/heartbeat/{step}/{rank}", "1")
    deadline = time.monotonic() + timeout_s
    missing = list(range(world))
    while True:
        missing = [r for r in missing if not store.check([f"psb/heartbeat/{step}/{r}"])]
        if not missing:
            return
        if time.monotonic() >= deadline:
            raise PeerLost(f"rank(s) {missing} did not reach step {step} within {timeout_s:g} s")
        time.sleep(0.01)


def panel_csr(m: Csr, r0: int, r1: int) -> Csr:
    """Rows [r0, r1) of ``m`` as a CSR with its own row pointer; columns stay global."""
    rp = m.row_ptr[r0:r1 + 1].astype(np.int64)
    lo, hi = int(rp[0]), int(rp[-1])
    return Csr(r1 - r0, m.cols, (rp - lo).astype(np.int32), m.col_ind[lo:hi], m.values[lo:hi], m.symmetric)


def allgather_rows(local, cuts, group=None):
    """Concatenate every rank's row panel (``local``: [cuts[r+1]-cuts[r], N]) into the
    full [cuts[-1], N] tensor on every rank.  Panels are padded to the longest one for
    one ``all_gather_into_tensor``; collective order is the same on every rank.  A
    collective that fails because a rank is gone (the group's timeout, or a closed
    connection) raises PeerLost."""
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
    try:
        dist.all_gather_into_tensor(gathered, padded, group=group)
    except (RuntimeError, dist.DistError) as e:  # a peer failed, left, or the group timed out
        raise PeerLost(f"all-gather of the row panels failed: {e}") from e
    return torch.cat([gathered[r * longest: r * longest + rows[r]] for r in range(world)])


def _current_waits_for(stream, tensor) -> None:
    """Make torch's current stream on ``tensor``'s device wait for ``stream`` (a
    torch.cuda.Stream, a raw cudaStream_t as int, or None for the legacy default
    stream)."""
    import torch
    if not tensor.is_cuda:
        return
    current = torch.cuda.current_stream(tensor.device)
    if stream is None:
        other = torch.cuda.default_stream(tensor.device)
    elif isinstance(stream, torch.cuda.Stream):
        other = stream
    else:
        other = torch.cuda.ExternalStream(int(stream), device=tensor.device)
    if other.cuda_stream != current.cuda_stream:
        current.wait_stream(other)


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
        """C_local (+)= A_panel · B; with ``gather`` also return the full C on every rank.

        The all-gather is ordered after torch's current stream, so when ``stream`` is
        another stream the current one first waits for it (the SpMM has finished
        writing C_local before the gather reads it)."""
        SpMM(self.matrix, N, B, C_local, stream)
        if gather:
            _current_waits_for(stream, C_local)
            return allgather_rows(C_local, self.cuts, group)
        return C_local

    def spmm_replicated(self, N: int, B, replicas: "Replicas", stream=None, group=None):
        """The full C = A · B on every rank in ``replicas.full``: this rank's SpMM writes
        its panel of its own replica and stores every finished row straight into the
        other ranks' replicas over NVLink (ps_spmm_push: the all-gather fused into the
        SpMM, no separate collective moves C).  The panel is accumulated into, as SpMM
        does: zero it first for a fresh product.  Returns after a one-element all-reduce
        queued behind the SpMM, so on return (in stream order) every rank's pushes into
        this rank's replica have completed."""
        import torch
        import torch.distributed as dist
        r0, r1 = self.row_begin, self.row_end
        SpMM_push(self.matrix, N, B, replicas.full[r0:r1], replicas.peer_panels(r0, N), stream)
        _current_waits_for(stream, replicas.full)
        flag = torch.zeros(1, device=replicas.full.device)
        try:
            dist.all_reduce(flag, group=group)
        except (RuntimeError, dist.DistError) as e:
            raise PeerLost(f"the barrier after the fused SpMM all-gather failed: {e}") from e
        return replicas.full

    def sddmm(self, N: int, lhs_panel, rhs, outputs, stream=None):
        """Per-workset SDDMM outputs of this panel (lhs_panel holds the panel's rows)."""
        SDDMM(self.matrix, N, lhs_panel, rhs, outputs, stream)
        return outputs

    def close(self):
        self.matrix.close()


class Replicas:
    """Every rank's full copy (``full``: [rows, N] float32 on this rank's GPU) of a
    row-partitioned result, each opened on every other rank through CUDA IPC, so
    that ps_spmm_push can store a rank's finished rows into all the copies.  Every
    rank of ``group`` constructs it with the same shape (a collective); ``close``
    releases the peers' mappings (every rank must close before any frees ``full``)."""

    def __init__(self, rows: int, N: int, device, group=None):
        import torch
        import torch.distributed as dist
        self.N = N
        self.full = torch.zeros((rows, N), dtype=torch.float32, device=device)
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        handle, offset = ipc_export(self.full)
        shared = [None] * world
        dist.all_gather_object(shared, (handle, offset), group=group)
        self._bases, self._peers = [], []
        try:
            # Peers in ring order from this rank (rank+1, rank+2, ...): the push kernel
            # stores to peers in list order, so at each position every rank sends to a
            # different GPU instead of all of them to the same one.
            for step in range(1, world):
                r = (rank + step) % world
                base = ipc_open(shared[r][0])
                self._bases.append(base)
                self._peers.append(base + shared[r][1])
        except Exception:
            self.close()
            raise

    def peer_panels(self, row0: int, N: int) -> list:
        """Addresses of row ``row0`` in every peer's copy."""
        if N != self.N:
            raise ValueError(f"the replicas hold rows of {self.N} floats, not {N}")
        return [p + row0 * N * 4 for p in self._peers]

    def close(self) -> None:
        for b in self._bases:
            ipc_close(b)
        self._bases, self._peers = [], []
