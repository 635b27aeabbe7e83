"""Benchmark of the PowerSparse hot path on B200: fused SpMM over the block/residue layout.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--n 128]

One step = one SpMM call C = A·B (FP32) over one row panel per GPU.  Workload:
benchmark configuration 2 (symmetric Chung-Lu power-law graph, gamma 2.1,
2.45M nodes, ~61.9M nnz, values U[0,1], B U[-1,1], N = 128) per GPU; with N
GPUs the graph has N x 2.45M nodes with the same degree law, is cut into N
nnz-balanced row panels, and B (all N x 2.45M rows) is replicated (weak
scaling; no collective in the timed region).  Inputs are larger than L2
(B is 1.25 GB per 2.45M rows), so no explicit L2 flush is done.

The JSON line's "extra" object times the other operators of the path (SpMM at
N=32, SDDMM at N=32 and 128) on the same panel with the same rules.

Prints one JSON line (rank 0).  ``--impl reference`` times the reference's CPU
path (its FP64 CheckSpmm loop, benchmarks/benchmark.cu:64-77, restated in
oracle/ps_oracle.cpp) on all host cores on the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "SpMM/SDDMM GFLOPS and HBM GB/s (% of roofline) at N=32/128, 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def measured_peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from a committed ncu summary, if one exists for this workload."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f)[kernel][workload]
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while active."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self.proc = None
        self.thread = None
        self.window = [0.0, 0.0]

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=5)

    def summary(self):
        t0, t1 = self.window
        rows = [s for t, s in self.samples if t0 - 0.06 <= t <= t1 + 0.06] or [s for _, s in self.samples]
        mhz, maxmhz, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            f = [x.strip() for x in r.split(",")]
            if len(f) < 9:
                continue
            try:
                mhz.append(float(f[1]))
                maxmhz.append(float(f[2]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": max(maxmhz), "reasons": sorted(reasons),
                "samples": len(mhz)}


def build_workload(rank: int, world: int, device, workload: str = "cfg2"):
    import powersparse_b200 as psb
    from powersparse_b200 import synth_gpu
    if workload == "cfg5":
        n_nodes, pairs = synth_gpu.config5_pairs(device=device)   # one graph for every N (strong scaling)
    else:
        n_nodes, pairs = synth_gpu.config2_pairs(nodes_scale=world, device=device)
    cuts = psb.partition_rows(synth_gpu.global_row_ptr(pairs, n_nodes).astype(np.int32), world)
    panel = synth_gpu.panel_from_pairs(pairs, n_nodes, int(cuts[rank]), int(cuts[rank + 1]),
                                       seed=5 if workload == "cfg5" else 2)
    del pairs
    return panel, cuts


def dense_B(cols: int, n: int, device):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(102)
    return torch.rand((cols, n), generator=g, device=device, dtype=torch.float32) * 2 - 1


def cpu_spmm_rate(panel, B_host: np.ndarray, min_seconds: float, max_passes: int):
    """FP64 CheckSpmm restatement on all host cores; returns (GFLOP/s, threads, passes, seconds)."""
    from oracle import oracle
    threads = oracle.lib().ps_oracle_max_threads()
    n = B_host.shape[1]
    passes, t = 0, 0.0
    while passes < max_passes and (passes == 0 or t < min_seconds):
        t0 = time.perf_counter()
        oracle.spmm(panel.row_ptr, panel.col_ind, panel.values, B_host, threads=threads)
        t += time.perf_counter() - t0
        passes += 1
    flops = 2.0 * panel.nnz * n * passes
    return flops / t / 1e9, threads, passes, t


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--n", type=int, default=128)
    ap.add_argument("--e2e-steps", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["cfg2", "cfg5"], default="cfg2",
                    help="cfg2: config 2 per GPU (weak scaling, default); cfg5: the config-5 R-MAT graph "
                         "(16.8M nodes, ~1B nnz) split over the GPUs (strong scaling)")
    ap.add_argument("--gather", action="store_true",
                    help="also time the all-gather of the C panels (NCCL) that a replicated result needs")
    args = ap.parse_args()

    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)

    N = args.n
    if args.impl == "reference":
        if rank == 0:
            run_reference_arm(args, world, device)
        if dist:
            dist.destroy_process_group()
        return

    import powersparse_b200 as psb
    panel, cuts = build_workload(rank, world, device, args.workload)
    m = psb.PowerSparseMatrixGPU(panel.rows, panel.cols, panel.nnz, panel.row_ptr, panel.col_ind, panel.values)
    if rank == 0:
        B = dense_B(panel.cols, N, device)
    else:
        B = torch.empty((panel.cols, N), dtype=torch.float32, device=device)
    if dist:
        dist.broadcast(B, 0)  # replicate the dense operand once (setup, untimed)
    C = torch.zeros((panel.rows, N), dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)

    for _ in range(max(args.warmup, 3)):
        psb.SpMM(m, N, B, C, stream)
    torch.cuda.synchronize(device)

    sampler = ClockSampler(local).start()
    time.sleep(0.15)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(device)
    sampler.window[0] = time.time()
    ev0.record(stream)
    for _ in range(args.steps):
        psb.SpMM(m, N, B, C, stream)
    ev1.record(stream)
    torch.cuda.synchronize(device)
    sampler.window[1] = time.time()
    if dist:
        dist.barrier()
    time.sleep(0.1)
    sampler.stop()
    ms_local = ev0.elapsed_time(ev1) / args.steps
    ms = ms_local
    nnz_total = panel.nnz
    if dist:
        t = torch.tensor([ms_local], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        z = torch.tensor([panel.nnz], dtype=torch.float64, device=device)
        dist.all_reduce(z)
        nnz_total = int(z.item())
    gflops = 2.0 * nnz_total * N / (ms * 1e-3) / 1e9

    # Roofline of the fused kernel (per GPU): compulsory bytes 8*nnz + 4*N*(rows + cols).
    alg_bytes = 8.0 * panel.nnz + 4.0 * N * (panel.rows + panel.cols)
    peak, peak_kind = measured_peaks()
    achieved = alg_bytes / (ms_local * 1e-3) / 1e9
    scaling = "strong" if args.workload == "cfg5" else "weak"
    traffic = profile_traffic("spmm_fused", f"{args.workload}_spmm_n{N}") if world == 1 else None
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                "traffic": traffic, "alg_bytes_per_launch": alg_bytes}
    if traffic:
        # The DRAM bytes the ncu capture measured per launch, over this run's launch time:
        # how close the gathers run to the measured HBM peak.
        roofline["dram_achieved"] = round(traffic / (ms_local * 1e-3) / 1e9, 1)
        roofline["dram_frac"] = round(traffic / (ms_local * 1e-3) / 1e9 / peak, 4)
    # Model, not roofline: every element gathers its dense row with no reuse.
    roofline["no_reuse_gather_model_gbs"] = round(
        (8.0 * panel.nnz + 4.0 * N * panel.nnz + 4.0 * N * panel.rows) / (ms_local * 1e-3) / 1e9, 1)

    # The other operators of the path on the same panel (kernel only, same timing rules):
    # SpMM at N=32 and SDDMM at N=32/128 (the reference's N choices).
    extra = {}

    def timed(fn, k):
        for _ in range(3):
            fn()
        if dist:
            dist.barrier()
        torch.cuda.synchronize(device)
        ev0.record(stream)
        for _ in range(k):
            fn()
        ev1.record(stream)
        torch.cuda.synchronize(device)
        t = ev0.elapsed_time(ev1) / k
        if dist:
            tt = torch.tensor([t], dtype=torch.float64, device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    k_extra = max(10, min(args.steps, 50))
    if N != 32:
        B32 = B[:, :32].contiguous()
        C32 = torch.zeros((panel.rows, 32), dtype=torch.float32, device=device)
        ms32 = timed(lambda: psb.SpMM(m, 32, B32, C32, stream), k_extra)
        ab32 = 8.0 * panel.nnz + 4.0 * 32 * (panel.rows + panel.cols)
        extra["spmm_n32"] = {"ms": round(ms32, 4), "gflops": round(2.0 * nnz_total * 32 / (ms32 * 1e-3) / 1e9, 1),
                             "roofline_frac": round(ab32 / (ms32 * 1e-3) / 1e9 / peak, 4)}
        del B32, C32
    outs = [torch.zeros(max(m.workset_size(s), 1), dtype=torch.float32, device=device)
            for s in range(m.GroupTypeNum())]
    for n_sd in (32, 128):
        X = B[: panel.rows, :n_sd].contiguous() if panel.rows <= panel.cols else torch.rand(
            (panel.rows, n_sd), device=device)
        Y = B[:, :n_sd].contiguous()
        ms_sd = timed(lambda: psb.SDDMM(m, n_sd, X, Y, outs, stream), k_extra)
        ab = 12.0 * panel.nnz + 4.0 * n_sd * (panel.rows + panel.cols)
        extra[f"sddmm_n{n_sd}"] = {"ms": round(ms_sd, 4),
                                   "gflops": round(2.0 * nnz_total * n_sd / (ms_sd * 1e-3) / 1e9, 1),
                                   "roofline_frac": round(ab / (ms_sd * 1e-3) / 1e9 / peak, 4)}
        # The same SDDMM with its output in CSR order (one fused launch), next to the
        # unfused alternative: workset-order SDDMM, then a scatter through the map.
        out_csr = torch.empty(panel.nnz, dtype=torch.float32, device=device)
        ms_csr = timed(lambda: psb.SDDMM_csr(m, n_sd, X, Y, out_csr, stream), k_extra)
        pos = [torch.as_tensor(psb._CudaArrayView(p, m.workset_size(s), "<i4"), device=device).long()
               for s, p in enumerate(m.CsrPosition()) if m.workset_size(s) > 0]
        src = [o[: m.workset_size(s)] for s, o in enumerate(outs) if m.workset_size(s) > 0]

        def unfused():  # `stream` is torch's current stream, so the scatter follows in order
            psb.SDDMM(m, n_sd, X, Y, outs, stream)
            for p_s, o_s in zip(pos, src):
                out_csr.index_copy_(0, p_s, o_s)

        ms_unf = timed(unfused, k_extra)
        extra[f"sddmm_csr_n{n_sd}"] = {"ms": round(ms_csr, 4),
                                       "gflops": round(2.0 * nnz_total * n_sd / (ms_csr * 1e-3) / 1e9, 1),
                                       "unfused_ms": round(ms_unf, 4)}
        del X, Y, out_csr, pos, src
    del outs
    # SpMM with per-call edge values (CSR order) and the edge softmax of the attention
    # chain, on the same panel.
    w_csr = torch.rand(panel.nnz, dtype=torch.float32, device=device)
    C_v = torch.zeros_like(C)
    ms_v = timed(lambda: psb.SpMM_values(m, N, w_csr, B, C_v, stream), k_extra)
    extra[f"spmm_values_n{N}"] = {"ms": round(ms_v, 4),
                                  "gflops": round(2.0 * nnz_total * N / (ms_v * 1e-3) / 1e9, 1)}
    ms_sm = timed(lambda: psb.edge_softmax_csr(m, w_csr, stream), k_extra)
    extra["edge_softmax"] = {"ms": round(ms_sm, 4),
                             "gb_per_s": round(panel.nnz * 4 * 5 / (ms_sm * 1e-3) / 1e9, 1)}
    del w_csr, C_v

    if args.gather and world > 1:
        # Replicated result: all-gather the C panels over NCCL (outside the timed steps).
        from powersparse_b200.distributed import allgather_rows
        full = allgather_rows(C, cuts)
        tg = timed(lambda: allgather_rows(C, cuts), 5)
        extra["allgather_c"] = {"ms": round(tg, 3), "bytes_per_gpu_in": int(full.numel() * 4 - C.numel() * 4)}
        del full

    # End to end through the public API with host buffers, pipelined the way a serving
    # loop runs it: every step copies its B in from pinned host memory, zeroes C, runs
    # SpMM and copies its C back out; two buffer sets on three streams let step i+1's
    # upload overlap step i's readback (PCIe is full duplex).  Per-step bytes are
    # unchanged.
    hB = B.cpu().pin_memory()
    hC = [torch.empty((panel.rows, N), dtype=torch.float32).pin_memory() for _ in range(2)]
    dB = [torch.empty_like(B) for _ in range(2)]
    dC = [torch.empty_like(C) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev = lambda: torch.cuda.Event()
    in_done, comp_done, out_done = [ev(), ev()], [ev(), ev()], [ev(), ev()]

    def e2e_step(i):
        j = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(comp_done[j])      # SpMM of step i-2 has read dB[j]
            dB[j].copy_(hB, non_blocking=True)
            in_done[j].record(s_in)
        stream.wait_event(in_done[j])
        stream.wait_event(out_done[j])         # readback of step i-2 has read dC[j]
        dC[j].zero_()
        psb.SpMM(m, N, dB[j], dC[j], stream)
        comp_done[j].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(comp_done[j])
            hC[j].copy_(dC[j], non_blocking=True)
            out_done[j].record(s_out)

    def drain():
        for e in out_done + in_done:
            stream.wait_event(e)

    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    for i in range(2):
        e2e_step(i)
    drain()
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    e0.record(stream)
    for i in range(args.e2e_steps):
        e2e_step(i)
    drain()
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = e0.elapsed_time(e1) / args.e2e_steps
    if dist:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": round(2.0 * nnz_total * N / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GFLOP/s",
           "h2d_bytes_per_step": int(hB.numel() * 4), "d2h_bytes_per_step": int(hC[0].numel() * 4),
           "ms_per_step": round(e2e_ms, 3), "steps": args.e2e_steps}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, threads, passes, secs = cpu_spmm_rate(panel, hB.numpy(), min_seconds=10.0, max_passes=40)
        cpu = {"value": round(rate, 2), "unit": "GFLOP/s", "cores": threads, "kind": "port",
               "sample": f"full cfg2 SpMM N={N} (FP64 CheckSpmm restatement, OpenMP), {passes} passes, {secs:.1f} s"}

    if rank == 0:
        clocks = sampler.summary()
        line = {
            "metric": METRIC, "value": round(gflops, 1), "unit": "GFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": (f"cfg2: SpMM N={N}, symmetric Chung-Lu gamma=2.1, {world}x2.45M nodes, "
                                    f"nnz-balanced row panel per GPU, B replicated") if args.workload == "cfg2" else
                                   (f"cfg5: SpMM N={N}, R-MAT scale 24 edge factor 64 symmetrised, split into {world} "
                                    f"nnz-balanced row panels, B replicated"),
                       "rows_per_gpu": panel.rows, "cols": panel.cols, "nnz_per_gpu_rank0": panel.nnz,
                       "nnz_total": nnz_total, "N": N, "S": m.GroupTypeNum(),
                       "parallelism": f"row-panel x{world}", "l2": "inputs larger than L2 (B >= 1.25 GB), no flush",
                       "preprocess_ms": round(m.preprocess_ms, 1)},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            # per step: spmm_fused, plus wide_rows_fold when the panel has wide rows
            "gpu_launches": args.steps * (2 if m.wide_rows > 0 else 1),
            "clocks": clocks, "extra": extra,
        }
        print(json.dumps(line), flush=True)
    m.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_reference_arm(args, world: int, device) -> None:
    """The reference's CPU path (FP64 CheckSpmm, restated: no separately callable CPU
    SpMM exists in the reference) on all host cores, on rank 0's panel of the same workload."""
    panel, _ = build_workload(0, world, device, args.workload)
    N = args.n
    B = dense_B(panel.cols, N, device).cpu().numpy()
    from oracle import oracle
    threads = oracle.lib().ps_oracle_max_threads()
    for _ in range(min(args.warmup, 1)):
        oracle.spmm(panel.row_ptr, panel.col_ind, panel.values, B, threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.spmm(panel.row_ptr, panel.col_ind, panel.values, B, threads=threads)
        times.append(time.perf_counter() - t0)
        if sum(times) > 120:
            break
    ms = 1e3 * sum(times) / len(times)
    v = 2.0 * panel.nnz * N / (ms * 1e-3) / 1e9
    line = {"metric": METRIC, "value": round(v, 2), "unit": "GFLOP/s", "n_gpus": world, "steps": len(times),
            "warmup": min(args.warmup, 1), "ms_per_step": round(ms, 2), "higher_is_better": True,
            "scaling": "strong" if args.workload == "cfg5" else "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": f"{args.workload}: SpMM N={N}, rank-0 row panel ({world} panels)",
                       "rows": panel.rows, "nnz": panel.nnz, "N": N},
            "cpu_baseline": {"value": round(v, 2), "unit": "GFLOP/s", "cores": threads, "kind": "port",
                             "sample": f"one row panel ({panel.nnz} nnz) per step, FP64 CheckSpmm restatement"},
            "e2e": {"value": round(v, 2), "unit": "GFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
