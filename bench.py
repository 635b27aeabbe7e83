"""Benchmark of the PowerSparse hot path on B200: fused SpMM over the block/residue layout.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--n 128]

One step = one SpMM call C = A·B (FP32) over one row panel per GPU.  Workload:
benchmark configuration 2 (symmetric Chung-Lu power-law graph, gamma 2.1,
2.45M nodes, ~61.9M nnz, values U[0,1], B U[-1,1], N = 128) per GPU; with N
GPUs the graph has N x 2.45M nodes with the same degree law, is cut into N
nnz-balanced row panels, and B (all N x 2.45M rows) is replicated (weak
scaling; no collective in the timed region).  Inputs are larger than L2
(B is 1.25 GB per 2.45M rows), so no explicit L2 flush is done.

After the timed steps every rank checks a seeded sample of its panel's rows
against an FP64 product computed on the host with numpy ("check").  The JSON
line's "extra" object times the other operators of the path (SpMM at N=32,
SDDMM at N=32 and 128, the CSR-order and attention-chain additions) on the same
panel with the same rules, and configuration 5 (R-MAT, 16.8M nodes, ~1B nnz)
split over the N GPUs (strong scaling), with its own sampled check and the
all-gather of C.  "e2e" is the same SpMM through the library with host buffers:
at one GPU B is uploaded whole every step; at N GPUs every rank uploads 1/N of
B and the GPUs all-gather it over NVLink (NCCL) before the SpMM, and every rank
reads back its own C panel.

``--impl reference`` times the reference's CPU path (its FP64 CheckSpmm loop,
benchmarks/benchmark.cu:64-77, restated in oracle/ps_oracle.cpp) on all host
cores, on row samples of the same global workload, and -- at one GPU, when the
reference was compiled from its sources into oracle/_ref -- the reference's own
GPU kernels on the same matrix ("extra.ref_gpu").
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "SpMM/SDDMM GFLOPS and HBM GB/s (% of roofline) at N=32/128, 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
KERNEL_SOURCE = os.path.join(ROOT, "powersparse_b200", "csrc", "ps_ops.cu")
ATOL, RTOL = 1e-5, 1e-4  # |a - e| <= ATOL + RTOL * |e| against FP64


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def measured_peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def kernel_source_digest() -> str:
    with open(KERNEL_SOURCE, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()[:16]


def profile_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from profiles/traffic.json, used only when the capture was
    taken from this build's kernel source (its ps_ops.cu digest); else (None, reason)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            entry = json.load(f)[kernel][workload]
    except Exception:
        return None, "no capture for this workload"
    if not isinstance(entry, dict) or entry.get("ps_ops_sha") != kernel_source_digest():
        return None, "capture is of another build of ps_ops.cu"
    return float(entry["bytes"]), f"ncu capture of this build ({entry.get('command', '')})"


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


def partition_rows_np(row_ptr: np.ndarray, parts: int) -> np.ndarray:
    """nnz-balanced contiguous row panels (the rule of ps_partition_rows, in numpy):
    cut p is the first row whose row_ptr reaches p * nnz / parts."""
    rp = np.asarray(row_ptr, dtype=np.int64)
    rows, nnz = len(rp) - 1, int(rp[-1])
    cuts = np.zeros(parts + 1, dtype=np.int64)
    for p in range(1, parts):
        r = int(np.searchsorted(rp, p * nnz // parts, side="left"))
        cuts[p] = min(max(r, int(cuts[p - 1])), rows)
    cuts[parts] = rows
    return cuts


def global_graph(workload: str, world: int, device):
    """(nodes, unique pairs on `device`) of the benchmark graph for this world size:
    config 2's degree law with world x 2.45M nodes, or the config-5 R-MAT graph."""
    from powersparse_b200 import synth_gpu
    if workload == "cfg5":
        return synth_gpu.config5_pairs(device=device)
    return synth_gpu.config2_pairs(nodes_scale=world, device=device)


def build_workload(rank: int, world: int, device, workload: str = "cfg2"):
    import powersparse_b200 as psb
    from powersparse_b200 import synth_gpu
    n_nodes, pairs = global_graph(workload, world, device)
    grp = synth_gpu.global_row_ptr(pairs, n_nodes)
    cuts = psb.partition_rows(grp.astype(np.int32), world)
    panel = synth_gpu.panel_from_pairs(pairs, n_nodes, int(cuts[rank]), int(cuts[rank + 1]),
                                       seed=5 if workload == "cfg5" else 2)
    del pairs
    return panel, cuts, int(grp[-1])


def dense_B(cols: int, n: int, device, seed: int = 102):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.rand((cols, n), generator=g, device=device, dtype=torch.float32) * 2 - 1


def sampled_check(panel, B, C, rows: int = 2048, seed: int = 7) -> dict:
    """Rows of C (device) against an FP64 product computed on the host for a seeded
    sample of the panel's rows: C[r] = sum_p values[p] * B[col_ind[p]] over row r."""
    import torch
    rng = np.random.default_rng(seed)
    r = np.unique(rng.integers(0, panel.rows, size=min(rows, panel.rows)))
    rp = panel.row_ptr.astype(np.int64)
    lens = rp[r + 1] - rp[r]
    idx = np.concatenate([np.arange(rp[x], rp[x + 1]) for x in r]) if lens.sum() else np.zeros(0, np.int64)
    dev = B.device
    expected = np.zeros((len(r), B.shape[1]), dtype=np.float64)
    if len(idx):
        cols = torch.from_numpy(panel.col_ind[idx].astype(np.int64)).to(dev)
        Bg = B.index_select(0, cols).double().cpu().numpy()
        prod = panel.values[idx].astype(np.float64)[:, None] * Bg
        nz = lens > 0
        starts = np.concatenate([[0], np.cumsum(lens)[:-1]])[nz]
        expected[nz] = np.add.reduceat(prod, starts, axis=0)
    actual = C.index_select(0, torch.from_numpy(r.astype(np.int64)).to(dev)).double().cpu().numpy()
    bad = int((~(np.isfinite(actual) & (np.abs(actual - expected) <= ATOL + RTOL * np.abs(expected)))).sum())
    return {"rows": int(len(r)), "elements": int(actual.size), "bad": bad}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--n", type=int, default=128)
    ap.add_argument("--e2e-steps", type=int, default=8)
    ap.add_argument("--e2e-chunks", type=int, default=1,
                    help="row chunks (one stream each) per host<->device copy of the e2e pipeline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cfg5", action="store_true", help="skip the configuration-5 extra")
    ap.add_argument("--workload", choices=["cfg2", "cfg5"], default="cfg2",
                    help="cfg2: config 2 per GPU (weak scaling, default); cfg5: the config-5 R-MAT graph "
                         "(16.8M nodes, ~1B nnz) split over the GPUs (strong scaling)")
    ap.add_argument("--profile-op", choices=["spmm", "sddmm", "spmm_push"], default=None,
                    help="only build the workload and run this operator at --n, --warmup + --steps times "
                         "(a small, single-kernel process for profilers; spmm_push pushes every finished "
                         "row to one replica on this GPU); prints one short JSON line")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        # Rank 0 alone runs the reference's CPU path; the other ranks have no work.
        if rank == 0:
            run_reference_arm(args, world, local)
        return

    import torch
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)

    import powersparse_b200 as psb
    N = args.n
    panel, cuts, nnz_total = build_workload(rank, world, device, args.workload)
    m = psb.PowerSparseMatrixGPU(panel.rows, panel.cols, panel.nnz, panel.row_ptr, panel.col_ind, panel.values)
    if args.profile_op:
        profile_op(psb, m, panel, args, device)
        m.close()
        if dist:
            dist.destroy_process_group()
        return
    if rank == 0:
        B = dense_B(panel.cols, N, device)
    else:
        B = torch.empty((panel.cols, N), dtype=torch.float32, device=device)
    if dist:
        dist.broadcast(B, 0)  # replicate the dense operand once (setup, untimed)
    C = torch.zeros((panel.rows, N), dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)

    def max_over_ranks(x: float) -> float:
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x: int) -> int:
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t)
        return int(t.item())

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
        return max_over_ranks(ev0.elapsed_time(ev1) / k)

    def check_all(panel_, B_, C_, N_, m_):
        """One fresh SpMM into C_, then every rank's sampled FP64 check; totals over ranks."""
        C_.zero_()
        psb.SpMM(m_, N_, B_, C_, stream)
        torch.cuda.synchronize(device)
        c = sampled_check(panel_, B_, C_)
        tot = {k: sum_over_ranks(v) for k, v in c.items()}
        tot["status"] = "passed" if tot["bad"] == 0 else "failed"
        return tot

    for _ in range(max(args.warmup, 3)):
        psb.SpMM(m, N, B, C, stream)
    torch.cuda.synchronize(device)

    sampler = ClockSampler(local).start()
    time.sleep(0.15)
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
    ms = max_over_ranks(ms_local)
    gflops = 2.0 * nnz_total * N / (ms * 1e-3) / 1e9
    check = check_all(panel, B, C, N, m)

    # Roofline of the fused kernel (per GPU): compulsory bytes 8*nnz + 4*N*(rows + cols).
    alg_bytes = 8.0 * panel.nnz + 4.0 * N * (panel.rows + panel.cols)
    peak, peak_kind = measured_peaks()
    achieved = alg_bytes / (ms_local * 1e-3) / 1e9
    scaling = "strong" if args.workload == "cfg5" else "weak"
    traffic, traffic_note = (profile_traffic("spmm_fused", f"{args.workload}_spmm_n{N}") if world == 1
                             else (None, "no capture for multi-GPU panels"))
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                "traffic": traffic, "traffic_source": traffic_note, "alg_bytes_per_launch": alg_bytes}
    if traffic:
        roofline["dram_achieved"] = round(traffic / (ms_local * 1e-3) / 1e9, 1)
        roofline["dram_frac"] = round(traffic / (ms_local * 1e-3) / 1e9 / peak, 4)
    # Model, not roofline: every element gathers its dense row with no reuse.
    roofline["no_reuse_gather_model_gbs"] = round(
        (8.0 * panel.nnz + 4.0 * N * panel.nnz + 4.0 * N * panel.rows) / (ms_local * 1e-3) / 1e9, 1)

    # The other operators of the path on the same panel (kernel only, same timing rules).
    extra = {}
    k_extra = max(10, min(args.steps, 50))
    if N != 32:
        B32 = B[:, :32].contiguous()
        C32 = torch.zeros((panel.rows, 32), dtype=torch.float32, device=device)
        ms32 = timed(lambda: psb.SpMM(m, 32, B32, C32, stream), k_extra)
        ab32 = 8.0 * panel.nnz + 4.0 * 32 * (panel.rows + panel.cols)
        extra["spmm_n32"] = {"ms": round(ms32, 4), "gflops": round(2.0 * nnz_total * 32 / (ms32 * 1e-3) / 1e9, 1),
                             "roofline_frac": round(ab32 / (ms32 * 1e-3) / 1e9 / peak, 4),
                             "check": check_all(panel, B32, C32, 32, m)["status"]}
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

    if world > 1:
        # Replicated result: all-gather the C panels over NCCL (outside the timed steps).
        from powersparse_b200.distributed import allgather_rows
        full = allgather_rows(C, cuts)
        tg = timed(lambda: allgather_rows(C, cuts), 5)
        extra["allgather_c"] = {"ms": round(tg, 3), "bytes_per_gpu_in": int(full.numel() * 4 - C.numel() * 4)}
        del full
        extra["spmm_allgather_fused"] = fused_allgather(psb, m, B, C, N, cuts, rank, device, stream, dist, timed,
                                                        allgather_rows)

    if world == 1:
        e2e = e2e_whole(psb, m, panel, B, C, N, device, stream, args.e2e_steps, nnz_total, args.e2e_chunks)
    else:
        e2e = e2e_sharded(psb, m, panel, B, N, rank, world, device, stream, dist, args.e2e_steps, nnz_total,
                          max_over_ranks, args.e2e_chunks)

    cpu = None
    hB = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        hB = B.cpu().numpy()
        rate, threads, passes, secs = cpu_spmm_rate(panel, hB, min_seconds=10.0, max_passes=40)
        cpu = {"value": round(rate, 2), "unit": "GFLOP/s", "cores": threads, "kind": "port",
               "sample": f"full cfg2 SpMM N={N} (FP64 CheckSpmm restatement, OpenMP), {passes} passes, {secs:.1f} s"}
    launches = args.steps * (2 if m.wide_rows > 0 else 1)  # spmm_fused (+ wide_rows_fold) per step
    rows_per_gpu, cols, nnz_rank0, S, pre_ms = panel.rows, panel.cols, panel.nnz, m.GroupTypeNum(), m.preprocess_ms
    m.close()
    del B, C, panel, hB
    torch.cuda.empty_cache()

    if args.workload == "cfg2" and not args.no_cfg5:
        extra["cfg5"] = run_cfg5(psb, rank, world, device, stream, timed, check_all, dist)

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
                       "rows_per_gpu": rows_per_gpu, "cols": cols, "nnz_per_gpu_rank0": nnz_rank0,
                       "nnz_total": nnz_total, "N": N, "S": S,
                       "parallelism": f"row-panel x{world}", "l2": "inputs larger than L2 (B >= 1.25 GB), no flush",
                       "preprocess_ms": round(pre_ms, 1)},
            "check": check["status"], "check_detail": check,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks, "extra": extra,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def profile_op(psb, m, panel, args, device) -> None:
    """One operator on the panel, --warmup + --steps calls and nothing else on the
    device but its operands: the process profilers capture (e.g. ncu -k ... -s W -c 1)."""
    import torch
    N = args.n
    B = dense_B(panel.cols, N, device)
    if args.profile_op == "spmm":
        C = torch.zeros((panel.rows, N), dtype=torch.float32, device=device)
        run = lambda: psb.SpMM(m, N, B, C)
    elif args.profile_op == "spmm_push":
        C = torch.zeros((panel.rows, N), dtype=torch.float32, device=device)
        replica = torch.zeros_like(C)
        run = lambda: psb.SpMM_push(m, N, B, C, [replica.data_ptr()])
    else:
        X = dense_B(panel.rows, N, device, seed=202)
        outs = [torch.zeros(max(m.workset_size(s), 1), dtype=torch.float32, device=device)
                for s in range(m.GroupTypeNum())]
        run = lambda: psb.SDDMM(m, N, X, B, outs)
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        run()
    e1.record()
    torch.cuda.synchronize(device)
    print(json.dumps({"profile_op": args.profile_op, "N": N, "nnz": panel.nnz, "calls": args.warmup + args.steps,
                      "ms": round(e0.elapsed_time(e1) / max(args.steps, 1), 4)}), flush=True)


def cpu_spmm_rate(panel, B_host: np.ndarray, min_seconds: float, max_passes: int):
    """FP64 CheckSpmm restatement on all host cores; returns (GFLOP/s, threads, passes, seconds)."""
    from oracle import oracle
    threads = host_cores()
    n = B_host.shape[1]
    passes, t = 0, 0.0
    while passes < max_passes and (passes == 0 or t < min_seconds):
        t0 = time.perf_counter()
        oracle.spmm(panel.row_ptr, panel.col_ind, panel.values, B_host, threads=threads)
        t += time.perf_counter() - t0
        passes += 1
    flops = 2.0 * panel.nnz * n * passes
    return flops / t / 1e9, threads, passes, t


class _ChunkedCopy:
    """A host<->device copy of the rows of a tensor, cut into `k` row chunks that
    copy on `k` streams (`done[j]`: the chunks' events for buffer set j).  Measured
    in the config-2 e2e pipeline (1.25 GB each way per step): 28.4 ms per step with
    one chunk, 29.1 with 2, 29.8 with 4, 30.0 with 8, so the default is one."""

    def __init__(self, device, k: int):
        import torch
        self.streams = [torch.cuda.Stream(device) for _ in range(k)]
        self.done = [[torch.cuda.Event() for _ in range(k)] for _ in range(2)]

    def run(self, dst, src, j: int, after) -> None:
        import torch
        rows, k = src.shape[0], len(self.streams)
        for c, s in enumerate(self.streams):
            lo, hi = rows * c // k, rows * (c + 1) // k
            for e in after:
                s.wait_event(e)
            with torch.cuda.stream(s):
                dst[lo:hi].copy_(src[lo:hi], non_blocking=True)
            self.done[j][c].record(s)

    def wait(self, stream, j: int) -> None:
        for e in self.done[j]:
            stream.wait_event(e)

    def events(self) -> list:
        return [e for pair in self.done for e in pair]


def e2e_whole(psb, m, panel, B, C, N, device, stream, steps, nnz_total, chunks) -> dict:
    """One GPU, end to end through the public API with host buffers: every step copies
    its B in from pinned host memory, zeroes C, runs SpMM and copies C back out; two
    buffer sets let step i+1's upload overlap step i's readback (PCIe is full
    duplex), each copy cut into `chunks` row chunks on their own streams.  Per-step
    bytes are unchanged by the overlap."""
    import torch
    hB = B.cpu().pin_memory()
    hC = [torch.empty((panel.rows, N), dtype=torch.float32).pin_memory() for _ in range(2)]
    dB = [torch.empty_like(B) for _ in range(2)]
    dC = [torch.empty_like(C) for _ in range(2)]
    up, down = _ChunkedCopy(device, chunks), _ChunkedCopy(device, chunks)
    comp_done = [torch.cuda.Event(), torch.cuda.Event()]

    def step(i):
        j = i % 2
        up.run(dB[j], hB, j, [comp_done[j]])   # after SpMM of step i-2 has read dB[j]
        up.wait(stream, j)
        down.wait(stream, j)                   # readback of step i-2 has read dC[j]
        dC[j].zero_()
        psb.SpMM(m, N, dB[j], dC[j], stream)
        comp_done[j].record(stream)
        down.run(hC[j], dC[j], j, [comp_done[j]])

    ms = _run_pipeline(step, up.events() + down.events() + comp_done, stream, device, steps, None)
    return {"value": round(2.0 * nnz_total * N / (ms * 1e-3) / 1e9, 2), "unit": "GFLOP/s",
            "h2d_bytes_per_step": int(hB.numel() * 4), "d2h_bytes_per_step": int(hC[0].numel() * 4),
            "ms_per_step": round(ms, 3), "steps": steps, "copy_chunks": chunks}


def e2e_sharded(psb, m, panel, B, N, rank, world, device, stream, dist, steps, nnz_total, max_over_ranks,
                chunks) -> dict:
    """N GPUs, end to end: every rank uploads its 1/N slice of B from pinned host
    memory, the ranks all-gather B over NVLink (NCCL), each runs SpMM on its panel and
    reads back only its own C panel.  Two buffer sets; upload, all-gather, SpMM and
    readback of consecutive steps overlap, the copies cut into `chunks` row chunks on
    their own streams."""
    import torch
    cols = B.shape[0]
    per = -(-cols // world)
    lo, hi = rank * per, min(cols, (rank + 1) * per)
    h_slice = torch.zeros((per, N), dtype=torch.float32).pin_memory()
    if hi > lo:
        h_slice[: hi - lo].copy_(B[lo:hi].cpu())
    d_slice = [torch.empty((per, N), dtype=torch.float32, device=device) for _ in range(2)]
    d_full = [torch.empty((per * world, N), dtype=torch.float32, device=device) for _ in range(2)]
    dC = [torch.empty((panel.rows, N), dtype=torch.float32, device=device) for _ in range(2)]
    hC = [torch.empty((panel.rows, N), dtype=torch.float32).pin_memory() for _ in range(2)]
    s_comm = torch.cuda.Stream(device)
    up, down = _ChunkedCopy(device, chunks), _ChunkedCopy(device, chunks)
    gathered, comp_done = ([torch.cuda.Event(), torch.cuda.Event()] for _ in range(2))

    def step(i):
        j = i % 2
        up.run(d_slice[j], h_slice, j, [gathered[j]])  # after the all-gather of step i-2 has read d_slice[j]
        up.wait(s_comm, j)
        s_comm.wait_event(comp_done[j])        # SpMM of step i-2 has read d_full[j]
        with torch.cuda.stream(s_comm):
            dist.all_gather_into_tensor(d_full[j], d_slice[j])
        gathered[j].record(s_comm)
        stream.wait_event(gathered[j])
        down.wait(stream, j)                   # readback of step i-2 has read dC[j]
        dC[j].zero_()
        psb.SpMM(m, N, d_full[j], dC[j], stream)
        comp_done[j].record(stream)
        down.run(hC[j], dC[j], j, [comp_done[j]])

    ms = max_over_ranks(_run_pipeline(step, up.events() + down.events() + gathered + comp_done, stream, device,
                                      steps, dist))
    # Correctness of the assembled operand: the gathered B equals the replicated one.
    same = bool(torch.equal(d_full[(steps - 1) % 2][:cols], B))
    return {"value": round(2.0 * nnz_total * N / (ms * 1e-3) / 1e9, 2), "unit": "GFLOP/s",
            "h2d_bytes_per_step": int(h_slice.numel() * 4), "d2h_bytes_per_step": int(hC[0].numel() * 4),
            "bytes_per": "rank", "h2d_bytes_per_step_all_ranks": int(h_slice.numel() * 4 * world),
            "allgather_bytes_in_per_rank": int((world - 1) * per * N * 4),
            "gathered_B_matches": same, "ms_per_step": round(ms, 3), "steps": steps, "copy_chunks": chunks}


def fused_allgather(psb, m, B, C, N, cuts, rank, device, stream, dist, timed, allgather_rows) -> dict:
    """SpMM with the all-gather of C fused in (ps_spmm_push over CUDA IPC: each rank's
    finished rows go straight into every other rank's replica from the kernel; a
    one-element all-reduce after it marks every replica complete), timed against
    SpMM followed by the NCCL all-gather of the panels.  The replica after one fused
    call is checked against the all-gathered result of a plain SpMM."""
    import torch
    from powersparse_b200.distributed import Replicas
    rows_total = int(cuts[-1])
    r0, r1 = int(cuts[rank]), int(cuts[rank + 1])
    reps = Replicas(rows_total, N, device)
    peers = reps.peer_panels(r0, N)
    flag = torch.zeros(1, device=device)
    panel_out = reps.full[r0:r1]

    def fused():
        psb.SpMM_push(m, N, B, panel_out, peers, stream)
        dist.all_reduce(flag)

    def separate():
        psb.SpMM(m, N, B, C, stream)
        allgather_rows(C, cuts)

    ms_fused = timed(fused, 5)
    ms_sep = timed(separate, 5)
    reps.full.zero_()
    C.zero_()
    torch.cuda.synchronize(device)
    dist.barrier()
    fused()
    psb.SpMM(m, N, B, C, stream)
    ref = allgather_rows(C, cuts)
    torch.cuda.synchronize(device)
    ok = torch.tensor([1.0 if bool(torch.allclose(reps.full, ref, rtol=1e-4, atol=1e-5)) else 0.0], device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    torch.cuda.synchronize(device)
    dist.barrier()  # no rank frees its replica while a peer still maps it
    reps.close()
    dist.barrier()
    del ref
    return {"ms": round(ms_fused, 3), "separate_ms": round(ms_sep, 3),
            "replica_bytes_out_per_gpu": int((r1 - r0) * N * 4 * (dist.get_world_size() - 1)),
            "replicas_match_allgather": bool(ok.item() == 1.0)}


def _run_pipeline(step, events, stream, device, steps, dist) -> float:
    import torch
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)

    def drain():
        for e in events:
            stream.wait_event(e)

    for i in range(2):
        step(i)
    drain()
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
        torch.cuda.synchronize(device)
    e0.record(stream)
    for i in range(steps):
        step(i)
    drain()
    e1.record(stream)
    torch.cuda.synchronize(device)
    return e0.elapsed_time(e1) / steps


def run_cfg5(psb, rank, world, device, stream, timed, check_all, dist, steps: int = 20) -> dict:
    """Configuration 5 (R-MAT scale 24, edge factor 64, ~1B nnz) split into `world`
    nnz-balanced row panels (strong scaling): SpMM N=128 per step, its sampled check,
    and the all-gather of the C panels into a replicated result."""
    import torch
    t0 = time.time()
    panel, cuts, nnz_total = build_workload(rank, world, device, "cfg5")
    torch.cuda.empty_cache()
    m = psb.PowerSparseMatrixGPU(panel.rows, panel.cols, panel.nnz, panel.row_ptr, panel.col_ind, panel.values)
    B = dense_B(panel.cols, 128, device, seed=105)  # the same replicated B on every rank (same seed)
    C = torch.zeros((panel.rows, 128), dtype=torch.float32, device=device)
    ms = timed(lambda: psb.SpMM(m, 128, B, C, stream), steps)
    check = check_all(panel, B, C, 128, m)
    out = {"workload": "cfg5: R-MAT scale 24 (16,777,216 nodes), edge factor 64, symmetrised, "
                       f"{world} row panels, SpMM N=128, B replicated",
           "scaling": "strong", "nnz_total": nnz_total, "nnz_rank0": panel.nnz, "rows_rank0": panel.rows,
           "ms": round(ms, 4), "gflops": round(2.0 * nnz_total * 128 / (ms * 1e-3) / 1e9, 1),
           "preprocess_ms_rank0": round(m.preprocess_ms, 1), "check": check["status"], "check_detail": check,
           "steps": steps}
    if world > 1:
        from powersparse_b200.distributed import allgather_rows
        full = allgather_rows(C, cuts)
        out["allgather_c_ms"] = round(timed(lambda: allgather_rows(C, cuts), 3), 3)
        out["allgather_bytes_in_per_gpu"] = int(full.numel() * 4 - C.numel() * 4)
        del full
    out["setup_s"] = round(time.time() - t0, 1)
    m.close()
    del B, C, panel
    torch.cuda.empty_cache()
    return out


def run_reference_arm(args, world: int, local: int) -> None:
    """The reference's CPU path (FP64 CheckSpmm, restated: the reference has no
    separately callable CPU SpMM) on all host cores.  The workload is the repo arm's
    global graph at this world size (every rank's panel); each step multiplies a
    bounded sample of it: from every nnz-balanced panel a contiguous block of rows
    (rotating from step to step), about 16M nonzeros in total, against the full B.
    Inputs are generated with torch on GPU `local`; the product library is not loaded."""
    import torch
    from oracle import oracle
    from powersparse_b200 import synth_gpu
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    N = args.n
    threads = host_cores()
    n_nodes, pairs = global_graph(args.workload, world, device)
    full = synth_gpu.panel_from_pairs(pairs, n_nodes, 0, n_nodes, seed=5 if args.workload == "cfg5" else 2)
    del pairs
    torch.cuda.empty_cache()
    cuts = partition_rows_np(full.row_ptr, world)
    B = dense_B(n_nodes, N, device).cpu().numpy()
    rp = full.row_ptr.astype(np.int64)
    target = 16_000_000 // world

    def blocks(step: int):
        out = []
        for p in range(world):
            r0, r1 = int(cuts[p]), int(cuts[p + 1])
            if r1 <= r0:
                continue
            span = r1 - r0
            start = r0 + (step * 7919 * 1031) % span
            end = int(np.searchsorted(rp, rp[start] + target, side="left"))
            out.append((start, max(start + 1, min(end, r1))))
        return out

    def run(step: int):
        nnz = 0
        for r0, r1 in blocks(step):
            oracle.spmm_rows(r0, r1, full.row_ptr, full.col_ind, full.values, B, threads=threads)
            nnz += int(rp[r1] - rp[r0])
        return nnz

    for w in range(min(args.warmup, 1)):
        run(10_000 + w)
    times, nnzs = [], []
    for s in range(args.steps):
        t0 = time.perf_counter()
        nnzs.append(run(s))
        times.append(time.perf_counter() - t0)
        if sum(times) > 60:
            break
    secs = sum(times)
    v = 2.0 * sum(nnzs) * N / secs / 1e9
    ms = 1e3 * secs / len(times)
    scaling = "strong" if args.workload == "cfg5" else "weak"
    sample = (f"{len(times)} steps; each multiplies ~16M nonzeros: from each of the {world} nnz-balanced panels of "
              f"the {int(rp[-1])}-nnz graph a contiguous row block (rotating), against the full B "
              f"({n_nodes} x {N}); FP64 CheckSpmm restatement, OpenMP")
    line = {"metric": METRIC, "value": round(v, 2), "unit": "GFLOP/s", "n_gpus": world, "steps": len(times),
            "warmup": min(args.warmup, 1), "ms_per_step": round(ms, 2), "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "f64", "data": "synthetic", "impl": "reference",
            "config": {"workload": (f"cfg2: SpMM N={N}, symmetric Chung-Lu gamma=2.1, {world}x2.45M nodes, "
                                    f"{world} nnz-balanced row panels") if args.workload == "cfg2" else
                                   f"cfg5: SpMM N={N}, R-MAT scale 24 edge factor 64, {world} row panels",
                       "nnz_total": int(rp[-1]), "N": N, "threads": threads},
            "cpu_baseline": {"value": round(v, 2), "unit": "GFLOP/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 2), "unit": "GFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if world == 1 and args.workload == "cfg2":
        line["extra"] = {"ref_gpu": reference_gpu_times(full)}
    print(json.dumps(line), flush=True)


def reference_gpu_times(csr) -> dict:
    """The reference's own GPU kernels (compiled from its sources into oracle/_ref,
    called through its public API by oracle/_ref/ps_ref_dump) on the same matrix,
    timed with the reference's protocol (30 warm-up calls, outputs zeroed, 20 timed
    calls under one event pair); dense operands generated on the device."""
    exe = os.path.join(ROOT, "oracle", "_ref", "ps_ref_dump")
    if not os.path.exists(exe):
        return {"unavailable": "oracle/_ref/ps_ref_dump was not built (no reference checkout at build time)"}
    from powersparse_b200 import synth
    out = {}
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "a.csr")
        synth.write_csr_bin(path, csr)
        for op, n in (("spmm", 32), ("spmm", 128), ("sddmm", 32), ("sddmm", 128)):
            cmd = [exe, op, path, str(n), "@rand:1"] + (["@rand:2"] if op == "sddmm" else []) + ["-", "20"]
            try:
                r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
                rec = json.loads(r.stdout.strip().splitlines()[-1]) if r.returncode == 0 else None
            except Exception as e:  # noqa: BLE001 - reported, not raised
                rec, r = None, None
                out[f"{op}_n{n}"] = {"error": str(e)[:200]}
                continue
            if rec is None:
                out[f"{op}_n{n}"] = {"error": (r.stderr or r.stdout).strip()[-200:]}
            else:
                out[f"{op}_n{n}"] = {"ms": round(rec["ms"], 4), "gflops": round(rec["gflops"], 1),
                                     "preprocess_ms": round(rec["preprocess_ms"], 1)}
    return out


if __name__ == "__main__":
    main()
