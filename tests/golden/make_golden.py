"""Generate golden fixtures from the reference itself.

Run on a machine with a GPU, after ``make -C oracle ref`` has built
``oracle/_ref/ps_ref_dump`` from the reference's sources:

    python tests/golden/make_golden.py OUTDIR

For every case below it writes the case's CSR and dense inputs, runs the
reference's own PowerSparseMatrixGPU constructor, SpMM and SDDMM through
``ps_ref_dump``, and packs inputs and outputs into ``OUTDIR/<case>.npz``.
Small cases keep every array; the medium case keeps SHA-256 digests of the
layout arrays only (its full arrays would not be a small fixture).

The case inputs are built here from fixed seeds; the small cases also store
their CSR so the fixtures never depend on a generator's random stream.
Dense operands come from ``dense_inputs`` (a counter hash, no RNG state).
"""
from __future__ import annotations

import hashlib
import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from powersparse_b200 import synth  # noqa: E402

DUMP = os.path.join(ROOT, "oracle", "_ref", "ps_ref_dump")


def dense_inputs(rows: int, n: int, seed: int) -> np.ndarray:
    """Row-major float32 [rows, n] in [-1, 1) from a counter hash of (seed, index)."""
    idx = np.arange(rows * n, dtype=np.uint64)
    return (2.0 * synth._hash01(idx, seed) - 1.0).astype(np.float32).reshape(rows, n)


def edge_matrix() -> synth.Csr:
    """Hand-shaped 200 x 60 CSR: empty rows, rows around every group boundary
    (16, 31, 32, 33, 63, 64, 65, ...), rows longer than the column count (so
    duplicate columns), and skewed column frequencies with many ties."""
    rng = np.random.default_rng(5)
    cycle = [0, 1, 16, 17, 31, 32, 33, 63, 64, 65, 96, 127, 128, 200, 5, 3]
    rows, cols = 200, 60
    weights = np.repeat([8.0, 4.0, 2.0, 1.0], 15)
    weights /= weights.sum()
    col_lists = []
    for r in range(rows):
        k = cycle[r % len(cycle)]
        col_lists.append(rng.choice(cols, size=k, replace=True, p=weights))
    row_ptr = np.zeros(rows + 1, dtype=np.int64)
    row_ptr[1:] = np.cumsum([len(c) for c in col_lists])
    col_ind = np.concatenate(col_lists).astype(np.int32)
    values = rng.uniform(-1, 1, size=len(col_ind)).astype(np.float32)
    return synth.Csr(rows, cols, row_ptr.astype(np.int32), col_ind, values)


def cases() -> dict:
    """name -> (matrix, forced SM count or None, [(op, N)], keep_full)."""
    cl = synth.chung_lu(3000, 14, 600, 2.1, seed=7)
    return {
        "cfg1": (synth.config_matrix(1), None, [("spmm", 32), ("sddmm", 32)], True),
        "cl3k_sm1": (cl, 1, [("spmm", 32), ("spmm", 128), ("sddmm", 32), ("sddmm", 128)], True),
        "cl3k_sm2": (cl, 2, [("spmm", 64)], True),
        "cl3k_sm148": (cl, 148, [("spmm", 32), ("sddmm", 128)], True),
        "edge_sm1": (edge_matrix(), 1, [("spmm", 32), ("spmm", 96), ("sddmm", 32), ("sddmm", 128)], True),
        "edge_sm148": (edge_matrix(), 148, [("spmm", 32), ("sddmm", 32)], True),
        "cl30k_natural": (synth.chung_lu(30000, 40, 3000, 2.1, seed=11), None, [("spmm", 128)], False),
    }


def _digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def csr_digest(m: synth.Csr) -> str:
    h = hashlib.sha256()
    for a in (m.row_ptr.astype("<i4"), m.col_ind.astype("<i4"), m.values.astype("<f4")):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


HEAD_ROWS = 512


def trim_outputs(out: dict) -> dict:
    """Keep fixtures small: a dense SpMM output above 64K elements is stored as its
    first HEAD_ROWS rows plus the FP64 sum of every row."""
    for k in [k for k in out if k.startswith("spmm") and not k.endswith(("_sum", "_head", "_rowsum"))]:
        C = np.asarray(out[k])
        if C.ndim == 2 and C.size > (1 << 16):
            out[f"{k}_head"] = C[:HEAD_ROWS]
            out[f"{k}_rowsum"] = C.astype(np.float64).sum(axis=1)
            del out[k]
    return out


def run_case(name: str, spec, work: str, outdir: str) -> dict:
    m, sm, ops, keep_full = spec
    os.makedirs(work, exist_ok=True)
    csr_path = os.path.join(work, f"{name}.csr")
    synth.write_csr_bin(csr_path, m)
    env = dict(os.environ)
    env.pop("PS_REF_SM_COUNT", None)
    if sm is not None:
        env["PS_REF_SM_COUNT"] = str(sm)
    lay = os.path.join(work, f"{name}.layout")
    os.makedirs(lay, exist_ok=True)
    subprocess.run([DUMP, "layout", csr_path, lay], check=True, env=env)
    meta = open(os.path.join(lay, "meta.txt")).read().split()
    S, fine = int(meta[0]), int(meta[1])
    group_num = [int(x) for x in meta[2:2 + S]]
    out = {"name": name, "sm_count": -1 if sm is None else sm, "S": S, "fine": fine,
           "group_num": np.array(group_num, dtype=np.int64), "csr_sha256": csr_digest(m)}
    arrays = {}
    for s in range(S):
        arrays[f"ws{s}_col"] = np.fromfile(os.path.join(lay, f"ws{s}.col.i32"), dtype="<i4")
        arrays[f"ws{s}_val"] = np.fromfile(os.path.join(lay, f"ws{s}.val.f32"), dtype="<f4")
        arrays[f"ws{s}_des"] = np.fromfile(os.path.join(lay, f"ws{s}.des.i32"), dtype="<i4")
    arrays["res_off"] = np.fromfile(os.path.join(lay, "res_off.i32"), dtype="<i4")
    arrays["res_atomic"] = np.fromfile(os.path.join(lay, "res_atomic.u8"), dtype=np.uint8)
    if keep_full:
        out.update(rows=m.rows, cols=m.cols, row_ptr=m.row_ptr, col_ind=m.col_ind, values=m.values)
        out.update(arrays)
    else:
        out["rows"], out["cols"], out["nnz"] = m.rows, m.cols, m.nnz
        for k, v in arrays.items():
            out[f"sha_{k}"] = _digest(v)
    for op, n in ops:
        if op == "spmm":
            B = dense_inputs(m.cols, n, 1000 + n)
            bp = os.path.join(work, f"{name}.B{n}.f32")
            B.tofile(bp)
            cp = os.path.join(work, f"{name}.spmm{n}.f32")
            subprocess.run([DUMP, "spmm", csr_path, str(n), bp, cp], check=True, env=env)
            C = np.fromfile(cp, dtype="<f4").reshape(m.rows, n)
            if keep_full:
                out[f"spmm{n}"] = C
            else:
                out[f"spmm{n}_sum"] = C.astype(np.float64).sum(axis=1)
        else:
            X = dense_inputs(m.rows, n, 2000 + n)
            Y = dense_inputs(m.cols, n, 3000 + n)
            xp = os.path.join(work, f"{name}.X{n}.f32")
            yp = os.path.join(work, f"{name}.Y{n}.f32")
            X.tofile(xp)
            Y.tofile(yp)
            pre = os.path.join(work, f"{name}.sddmm{n}")
            subprocess.run([DUMP, "sddmm", csr_path, str(n), xp, yp, pre], check=True, env=env)
            for s in range(S):
                o = np.fromfile(f"{pre}.ws{s}.f32", dtype="<f4")
                if keep_full:
                    out[f"sddmm{n}_ws{s}"] = o
                else:
                    out[f"sddmm{n}_ws{s}_sum"] = np.array([o.astype(np.float64).sum()])
    np.savez_compressed(os.path.join(outdir, f"{name}.npz"), **trim_outputs(out))
    return {"name": name, "S": S, "group_num": group_num, "nnz": m.nnz}


def trim_existing(paths) -> None:
    for p in paths:
        z = np.load(p, allow_pickle=False)
        np.savez_compressed(p, **trim_outputs({k: z[k] for k in z.files}))


def main() -> None:
    if len(sys.argv) > 2 and sys.argv[1] == "--trim":
        trim_existing(sys.argv[2:])
        return
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py OUTDIR   (run on a GPU host; copy OUTDIR/*.npz here)  |  --trim FILES")
    outdir = sys.argv[1]
    work = os.path.join(outdir, "_work")
    os.makedirs(outdir, exist_ok=True)
    summary = [run_case(name, spec, work, outdir) for name, spec in cases().items()]
    with open(os.path.join(outdir, "summary.json"), "w") as f:
        json.dump(summary, f, indent=1)
    print(json.dumps(summary))


if __name__ == "__main__":
    main()
