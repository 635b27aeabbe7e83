"""Seeded synthetic sparse matrices standing in for PowerSparse's graph dataset.

The reference benchmarks real graphs from an external archive (its
``dataset/README.md:3``), which is not available here.  These generators make
seeded power-law graphs with the shapes and value distributions of the five
benchmark configurations.  Every generator returns a ``Csr`` whose rows list
their columns in ascending order: the same CSR the reference's MatrixMarket
reader (``benchmarks/matrix_market.cpp:97-134``) builds from the canonical
``.mtx`` file that ``write_mtx`` writes (a symmetric file stores the lower
triangle sorted by (row, col), which expands to ascending columns per row).

Graph seeds are the configuration number; dense operands use ``100 + config``.
"""
from __future__ import annotations

import dataclasses
import os
import struct

import numpy as np

__all__ = [
    "Csr", "uniform_rows", "chung_lu", "lognormal_graph", "rmat", "config_matrix",
    "dense", "write_mtx", "write_csr_bin", "read_csr_bin", "CONFIGS",
]


@dataclasses.dataclass
class Csr:
    rows: int
    cols: int
    row_ptr: np.ndarray  # int32 [rows + 1]
    col_ind: np.ndarray  # int32 [nnz]
    values: np.ndarray   # float32 [nnz]
    symmetric: bool = False

    @property
    def nnz(self) -> int:
        return int(self.col_ind.shape[0])

    def row_lengths(self) -> np.ndarray:
        return np.diff(self.row_ptr)


def _csr_from_coo(rows: int, cols: int, r: np.ndarray, c: np.ndarray, v: np.ndarray,
                  symmetric: bool) -> Csr:
    key = r.astype(np.int64) * cols + c.astype(np.int64)
    order = np.argsort(key, kind="stable")
    r = r[order]
    row_ptr = np.zeros(rows + 1, dtype=np.int64)
    np.cumsum(np.bincount(r, minlength=rows), out=row_ptr[1:])
    if row_ptr[-1] > np.iinfo(np.int32).max - 32:
        raise ValueError("matrix exceeds 32-bit CSR indices")
    return Csr(rows, cols, row_ptr.astype(np.int32), c[order].astype(np.int32),
               v[order].astype(np.float32), symmetric)


def uniform_rows(rows: int = 4096, cols: int = 4096, per_row: int = 16, seed: int = 1) -> Csr:
    """Config 1: every row holds exactly ``per_row`` distinct uniform columns, values U[-1,1]."""
    rng = np.random.default_rng(seed)
    c = np.empty((rows, per_row), dtype=np.int64)
    for r in range(rows):
        c[r] = rng.choice(cols, size=per_row, replace=False)
    c.sort(axis=1)
    v = rng.uniform(-1.0, 1.0, size=(rows, per_row)).astype(np.float32)
    row_ptr = (np.arange(rows + 1, dtype=np.int64) * per_row).astype(np.int32)
    return Csr(rows, cols, row_ptr, c.reshape(-1).astype(np.int32), v.reshape(-1), False)


def _hash01(key: np.ndarray, seed: int) -> np.ndarray:
    """Deterministic U[0,1) float64 per uint64 key (splitmix64 finaliser, 24-bit mantissa)."""
    z = key.astype(np.uint64) + np.uint64((0x9E3779B97F4A7C15 * (seed + 1)) & 0xFFFFFFFFFFFFFFFF)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    z = z ^ (z >> np.uint64(31))
    return (z >> np.uint64(40)).astype(np.float64) * (1.0 / (1 << 24))


def _symmetric_from_pairs(n: int, u: np.ndarray, v: np.ndarray, seed: int,
                          lo: float, hi: float) -> Csr:
    """Drop self loops and duplicate undirected pairs, mirror, and give each pair one value.

    The value of pair {i, j} is a hash of (min, max) so both directions carry it.
    """
    keep = u != v
    u, v = u[keep].astype(np.int64), v[keep].astype(np.int64)
    key = np.minimum(u, v) * n + np.maximum(u, v)
    del u, v
    key.sort()
    first = np.ones(key.shape[0], dtype=bool)
    first[1:] = key[1:] != key[:-1]
    key = key[first]
    a, b = np.divmod(key, n)
    directed = np.concatenate([key, b * n + a])
    del a, b
    directed.sort()
    r, c = np.divmod(directed, n)
    pair = np.minimum(r, c) * n + np.maximum(r, c)
    val = (lo + (hi - lo) * _hash01(pair, seed)).astype(np.float32)
    del pair, directed
    row_ptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(np.bincount(r, minlength=n), out=row_ptr[1:])
    if row_ptr[-1] > np.iinfo(np.int32).max - 32:
        raise ValueError("matrix exceeds 32-bit CSR indices")
    return Csr(n, n, row_ptr.astype(np.int32), c.astype(np.int32), val, True)


def _sample_pairs(weights: np.ndarray, m: int, rng: np.random.Generator) -> tuple[np.ndarray, np.ndarray]:
    """``m`` independent endpoint pairs, each endpoint drawn with probability ∝ weight.

    Endpoint counts are multinomial; pairing the sorted first endpoints with a random
    permutation of the second endpoints gives the same joint law as drawing each pair
    independently.
    """
    p = weights / weights.sum()
    idx = np.arange(len(weights), dtype=np.int32)
    u = np.repeat(idx, rng.multinomial(m, p))
    v = rng.permutation(np.repeat(idx, rng.multinomial(m, p)))
    return u, v


def _powerlaw_weights(n: int, mean: float, dmax: float, gamma: float) -> np.ndarray:
    """Expected degrees C*(i+i0)^(-1/(gamma-1)), clipped below at 1, max ``dmax``, mean ``mean``."""
    alpha = 1.0 / (gamma - 1.0)
    i = np.arange(n, dtype=np.float64)
    lo, hi = 1e-6, 1e12
    for _ in range(90):
        i0 = (lo * hi) ** 0.5
        c = dmax * i0 ** alpha
        avg = np.maximum(c * (i + i0) ** -alpha, 1.0).mean()
        if avg > mean:
            hi = i0
        else:
            lo = i0
    c = dmax * i0 ** alpha
    return np.maximum(c * (i + i0) ** -alpha, 1.0)


def chung_lu(n: int, mean_degree: float, max_degree: float, gamma: float, seed: int,
             oversample: float = 1.0, values: tuple[float, float] = (0.0, 1.0)) -> Csr:
    """Symmetric Chung-Lu power-law graph with randomly permuted node labels."""
    rng = np.random.default_rng(seed)
    w = _powerlaw_weights(n, mean_degree, max_degree, gamma)
    w = w[rng.permutation(n)]
    m = int(round(n * mean_degree / 2 * oversample))
    u, v = _sample_pairs(w, m, rng)
    return _symmetric_from_pairs(n, u, v, seed, *values)


def lognormal_graph(n: int, mean_degree: float, sigma: float, cap: float, seed: int,
                    oversample: float = 1.0, values: tuple[float, float] = (-1.0, 1.0)) -> Csr:
    """Symmetric Chung-Lu graph with lognormal expected degrees capped at ``cap``."""
    rng = np.random.default_rng(seed)
    z = rng.standard_normal(n)
    lo, hi = -10.0, 20.0
    for _ in range(80):
        mu = 0.5 * (lo + hi)
        if np.minimum(np.exp(mu + sigma * z), cap).mean() > mean_degree:
            hi = mu
        else:
            lo = mu
    w = np.maximum(np.minimum(np.exp(mu + sigma * z), cap), 1.0)
    m = int(round(n * mean_degree / 2 * oversample))
    u, v = _sample_pairs(w, m, rng)
    return _symmetric_from_pairs(n, u, v, seed, *values)


def rmat(scale: int, edge_factor: int, seed: int, abcd=(0.57, 0.19, 0.19, 0.05),
         values: tuple[float, float] = (0.0, 1.0), chunk: int = 1 << 22) -> Csr:
    """R-MAT graph (2^scale nodes, edge_factor*2^scale/2 sampled undirected pairs), symmetrised."""
    rng = np.random.default_rng(seed)
    n = 1 << scale
    m = edge_factor * n // 2
    a, b, c, _ = abcd
    us, vs = [], []
    left = m
    while left > 0:
        k = min(chunk, left)
        u = np.zeros(k, dtype=np.int64)
        v = np.zeros(k, dtype=np.int64)
        for bit in range(scale):
            x = rng.random(k)
            right = (x >= a) & (x < a + b) | (x >= a + b + c)
            down = x >= a + b
            u |= down.astype(np.int64) << bit
            v |= right.astype(np.int64) << bit
        us.append(u)
        vs.append(v)
        left -= k
    perm = rng.permutation(n)
    u = perm[np.concatenate(us)]
    v = perm[np.concatenate(vs)]
    return _symmetric_from_pairs(n, u, v, seed, *values)


# Per-configuration parameters.  ``oversample`` compensates for the pairs removed by
# deduplication so that the realised nnz lands near the configuration's figure.
CONFIGS = {
    1: dict(kind="uniform", rows=4096, cols=4096, per_row=16),
    2: dict(kind="chung_lu", n=2_450_000, mean=25.27, dmax=17_000, gamma=2.1, oversample=1.0135,
            values=(0.0, 1.0)),
    3: dict(kind="chung_lu", n=1_570_000, mean=168.2, dmax=40_000, gamma=2.0, oversample=1.0,
            values=(0.0, 1.0)),
    4: dict(kind="lognormal", n=233_000, mean=490.0, sigma=1.2, cap=20_000, oversample=1.0,
            values=(-1.0, 1.0)),
    5: dict(kind="rmat", scale=24, edge_factor=64, values=(0.0, 1.0)),
}


def config_matrix(cfg: int, scale: float = 1.0) -> Csr:
    """The seeded matrix of benchmark configuration ``cfg`` (graph seed = ``cfg``).

    ``scale`` < 1 shrinks the node count (and, for R-MAT, the scale) while keeping
    the degree distribution, for parity tests that must finish quickly.
    """
    p = CONFIGS[cfg]
    if p["kind"] == "uniform":
        return uniform_rows(p["rows"], p["cols"], p["per_row"], seed=cfg)
    if p["kind"] == "chung_lu":
        n = max(64, int(p["n"] * scale))
        dmax = min(p["dmax"], max(8.0, n / 4))
        return chung_lu(n, p["mean"], dmax, p["gamma"], seed=cfg,
                        oversample=p["oversample"], values=p["values"])
    if p["kind"] == "lognormal":
        n = max(64, int(p["n"] * scale))
        cap = min(p["cap"], max(8.0, n / 4))
        return lognormal_graph(n, p["mean"] if scale == 1.0 else min(p["mean"], n / 8),
                               p["sigma"], cap, seed=cfg, oversample=p["oversample"],
                               values=p["values"])
    if p["kind"] == "rmat":
        s = p["scale"] if scale == 1.0 else max(8, int(round(p["scale"] + np.log2(scale))))
        return rmat(s, p["edge_factor"], seed=cfg, values=p["values"])
    raise ValueError(cfg)


def dense(rows: int, n: int, seed: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    """Row-major float32 [rows, n] drawn U[lo, hi] from ``seed``."""
    rng = np.random.default_rng(seed)
    return rng.uniform(lo, hi, size=(rows, n)).astype(np.float32)


def write_mtx(path: str, m: Csr) -> None:
    """Canonical MatrixMarket file: lower triangle of a symmetric matrix, sorted by (row, col)."""
    r = np.repeat(np.arange(m.rows, dtype=np.int64), m.row_lengths())
    c = m.col_ind.astype(np.int64)
    v = m.values
    if m.symmetric:
        keep = c <= r
        r, c, v = r[keep], c[keep], v[keep]
        sym = "symmetric"
    else:
        sym = "general"
    with open(path, "w") as f:
        f.write(f"%%MatrixMarket matrix coordinate real {sym}\n")
        f.write(f"{m.rows} {m.cols} {len(r)}\n")
        step = 1 << 20
        for s in range(0, len(r), step):
            block = np.column_stack([r[s:s + step] + 1, c[s:s + step] + 1])
            lines = [f"{a} {b} {float(x)!r}" for (a, b), x in zip(block.tolist(), v[s:s + step].tolist())]
            f.write("\n".join(lines))
            f.write("\n")


_MAGIC = b"PSCSR001"


def write_csr_bin(path: str, m: Csr) -> None:
    """Binary CSR: magic, int64 rows/cols/nnz, int32 row_ptr, int32 col_ind, float32 values."""
    with open(path, "wb") as f:
        f.write(_MAGIC)
        f.write(struct.pack("<qqq", m.rows, m.cols, m.nnz))
        f.write(np.ascontiguousarray(m.row_ptr, dtype="<i4").tobytes())
        f.write(np.ascontiguousarray(m.col_ind, dtype="<i4").tobytes())
        f.write(np.ascontiguousarray(m.values, dtype="<f4").tobytes())


def read_csr_bin(path: str) -> Csr:
    with open(path, "rb") as f:
        if f.read(8) != _MAGIC:
            raise ValueError(f"{path}: not a binary CSR file")
        rows, cols, nnz = struct.unpack("<qqq", f.read(24))
        row_ptr = np.frombuffer(f.read(4 * (rows + 1)), dtype="<i4").copy()
        col_ind = np.frombuffer(f.read(4 * nnz), dtype="<i4").copy()
        values = np.frombuffer(f.read(4 * nnz), dtype="<f4").copy()
    return Csr(int(rows), int(cols), row_ptr, col_ind, values)


def _cli() -> None:
    import argparse
    ap = argparse.ArgumentParser(description="write a seeded benchmark matrix")
    ap.add_argument("config", type=int)
    ap.add_argument("out")
    ap.add_argument("--scale", type=float, default=1.0)
    a = ap.parse_args()
    m = config_matrix(a.config, a.scale)
    if a.out.endswith(".mtx"):
        write_mtx(a.out, m)
    else:
        write_csr_bin(a.out, m)
    print(os.path.basename(a.out), m.rows, m.cols, m.nnz)


if __name__ == "__main__":
    _cli()
