"""Seeded power-law graphs generated on the GPU, for benchmark-sized inputs.

Same model as ``synth.chung_lu`` (symmetric Chung-Lu, expected degrees
C*(i+i0)^(-1/(gamma-1)) clipped at 1, random node labels, duplicate pairs and
self loops dropped, one value per undirected pair from a counter hash), but
sampled with torch on the GPU so that a config-2-sized graph takes about a
second and a multi-GPU job can cut out one nnz-balanced row panel of a larger
graph.  Every rank draws the same global sample from the same seed, so the
panels of all ranks partition one graph.

This is input generation, not the hot path: it only produces host CSR arrays
that are then handed to the library like any caller's matrix.
"""
from __future__ import annotations

import numpy as np
import torch

from . import synth


def _weights(n: int, mean: float, dmax: float, gamma: float, device) -> torch.Tensor:
    alpha = 1.0 / (gamma - 1.0)
    i = torch.arange(n, dtype=torch.float64, device=device)
    lo, hi = 1e-6, 1e12
    for _ in range(90):
        i0 = (lo * hi) ** 0.5
        c = dmax * i0 ** alpha
        avg = torch.clamp(c * (i + i0) ** -alpha, min=1.0).mean().item()
        if avg > mean:
            hi = i0
        else:
            lo = i0
    c = dmax * i0 ** alpha
    return torch.clamp(c * (i + i0) ** -alpha, min=1.0)


def _hash01(key: torch.Tensor, seed: int) -> torch.Tensor:
    """Same counter hash as synth._hash01, on int64 tensors (two's-complement wraparound)."""
    def u64(x):
        return int(np.uint64(x).astype(np.int64)) if x >= (1 << 63) else x
    k = key + u64((0x9E3779B97F4A7C15 * (seed + 1)) & 0xFFFFFFFFFFFFFFFF)
    k = (k ^ ((k >> 30) & ((1 << 34) - 1))) * u64(0xBF58476D1CE4E5B9)
    k = (k ^ ((k >> 27) & ((1 << 37) - 1))) * u64(0x94D049BB133111EB)
    k = k ^ ((k >> 31) & ((1 << 33) - 1))
    return ((k >> 40) & ((1 << 24) - 1)).to(torch.float64) * (1.0 / (1 << 24))


def chung_lu_pairs(n: int, mean: float, dmax: float, gamma: float, seed: int, oversample: float,
                   device="cuda") -> torch.Tensor:
    """Unique undirected pairs (sorted int64 keys a*n+b, a<b) of the global graph."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    w = _weights(n, mean, dmax, gamma, device)
    perm = torch.randperm(n, generator=gen, device=device)
    return _pairs_by_weight(w[perm], int(round(n * mean / 2 * oversample)), gen)


def lognormal_pairs(n: int, mean: float, sigma: float, cap: float, seed: int, oversample: float,
                    device="cuda") -> torch.Tensor:
    """Unique undirected pairs of a Chung-Lu graph with lognormal expected degrees
    capped at ``cap`` (the model of ``synth.lognormal_graph``)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    z = torch.randn(n, generator=gen, device=device, dtype=torch.float64)
    lo, hi = -10.0, 20.0
    for _ in range(80):
        mu = 0.5 * (lo + hi)
        if torch.clamp(torch.exp(mu + sigma * z), max=cap).mean().item() > mean:
            hi = mu
        else:
            lo = mu
    w = torch.clamp(torch.exp(mu + sigma * z), min=1.0, max=cap)
    return _pairs_by_weight(w, int(round(n * mean / 2 * oversample)), gen)


def _pairs_by_weight(w: torch.Tensor, m: int, gen: torch.Generator) -> torch.Tensor:
    """``m`` endpoint pairs drawn with probability proportional to ``w`` (self loops
    dropped), as unique sorted keys a*n+b with a < b."""
    n = w.numel()
    device = w.device
    cdf = torch.cumsum(w, 0)
    cdf /= cdf[-1].clone()
    keys = []
    chunk = 1 << 26
    for s in range(0, m, chunk):
        k = min(chunk, m - s)
        u = torch.searchsorted(cdf, torch.rand(k, generator=gen, device=device, dtype=torch.float64))
        v = torch.searchsorted(cdf, torch.rand(k, generator=gen, device=device, dtype=torch.float64))
        u.clamp_(max=n - 1)
        v.clamp_(max=n - 1)
        keep = u != v
        u, v = u[keep], v[keep]
        keys.append(torch.minimum(u, v) * n + torch.maximum(u, v))
    return torch.unique(torch.cat(keys))


def panel_from_pairs(pairs: torch.Tensor, n: int, r0: int, r1: int, seed: int,
                     values=(0.0, 1.0)) -> synth.Csr:
    """Rows [r0, r1) of the symmetric matrix of ``pairs`` as a host CSR (columns global)."""
    a = torch.div(pairs, n, rounding_mode="floor")
    b = pairs - a * n
    parts_r, parts_c, parts_k = [], [], []
    for x, y in ((a, b), (b, a)):
        sel = (x >= r0) & (x < r1)
        parts_r.append(x[sel])
        parts_c.append(y[sel])
        parts_k.append(pairs[sel])
    r = torch.cat(parts_r)
    c = torch.cat(parts_c)
    k = torch.cat(parts_k)
    order = torch.argsort(r * n + c)
    r, c, k = r[order], c[order], k[order]
    lo, hi = values
    val = (lo + (hi - lo) * _hash01(k, seed)).to(torch.float32)
    counts = torch.bincount(r - r0, minlength=r1 - r0)
    row_ptr = torch.zeros(r1 - r0 + 1, dtype=torch.int64, device=pairs.device)
    row_ptr[1:] = torch.cumsum(counts, 0)
    return synth.Csr(r1 - r0, n, row_ptr.to(torch.int32).cpu().numpy(), c.to(torch.int32).cpu().numpy(),
                     val.cpu().numpy(), True)


def global_row_ptr(pairs: torch.Tensor, n: int) -> np.ndarray:
    """row_ptr of the full symmetric matrix (for nnz-balanced panel cuts)."""
    a = torch.div(pairs, n, rounding_mode="floor")
    b = pairs - a * n
    deg = torch.bincount(a, minlength=n) + torch.bincount(b, minlength=n)
    rp = torch.zeros(n + 1, dtype=torch.int64, device=pairs.device)
    rp[1:] = torch.cumsum(deg, 0)
    return rp.cpu().numpy()


def rmat_pairs(scale: int, edge_factor: int, seed: int, abcd=(0.57, 0.19, 0.19, 0.05), device="cuda",
               chunk: int = 1 << 25) -> tuple[int, torch.Tensor]:
    """Unique undirected pairs of an R-MAT graph (2^scale nodes, edge_factor * 2^scale / 2
    sampled pairs, self loops dropped, node labels randomly permuted), as sorted keys."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    n = 1 << scale
    m = edge_factor * n // 2
    a, b, c, _ = abcd
    perm = torch.randperm(n, generator=gen, device=device)
    keys = []
    for s0 in range(0, m, chunk):
        k = min(chunk, m - s0)
        u = torch.zeros(k, dtype=torch.int64, device=device)
        v = torch.zeros(k, dtype=torch.int64, device=device)
        for bit in range(scale):
            x = torch.rand(k, generator=gen, device=device)
            down = x >= a + b
            right = ((x >= a) & (x < a + b)) | (x >= a + b + c)
            u |= down.to(torch.int64) << bit
            v |= right.to(torch.int64) << bit
        u = perm[u]
        v = perm[v]
        keep = u != v
        u, v = u[keep], v[keep]
        keys.append(torch.unique(torch.minimum(u, v) * n + torch.maximum(u, v)))
    return n, torch.unique(torch.cat(keys))


def config5_pairs(device="cuda"):
    """Configuration 5: R-MAT scale 24, edge factor 64, (a,b,c,d) = (.57,.19,.19,.05)."""
    p = synth.CONFIGS[5]
    return rmat_pairs(p["scale"], p["edge_factor"], seed=5, device=device)


def config_pairs(cfg: int, device="cuda"):
    """(nodes, unique pairs) of benchmark configuration 2, 3, 4 or 5 at full size
    (graph seed = configuration number; the GPU sampler, not synth.config_matrix's
    numpy stream, so the graphs differ from the CPU generator's but share its law)."""
    if cfg == 5:
        return config5_pairs(device=device)
    p = synth.CONFIGS[cfg]
    if p["kind"] == "chung_lu":
        return p["n"], chung_lu_pairs(p["n"], p["mean"], p["dmax"], p["gamma"], seed=cfg,
                                      oversample=p["oversample"], device=device)
    if p["kind"] == "lognormal":
        return p["n"], lognormal_pairs(p["n"], p["mean"], p["sigma"], p["cap"], seed=cfg,
                                       oversample=p["oversample"], device=device)
    raise ValueError(f"configuration {cfg} has no GPU generator")


def config_matrix(cfg: int, device="cuda") -> synth.Csr:
    """The whole matrix of configuration ``cfg`` (2-5) as a host CSR, generated on the GPU."""
    n, pairs = config_pairs(cfg, device=device)
    return panel_from_pairs(pairs, n, 0, n, seed=cfg, values=synth.CONFIGS[cfg]["values"])


def config2_pairs(nodes_scale: int = 1, device="cuda"):
    """Config 2's degree law (synth.CONFIGS[2]); ``nodes_scale`` multiplies the node count."""
    p = synth.CONFIGS[2]
    n = p["n"] * nodes_scale
    return n, chung_lu_pairs(n, p["mean"], p["dmax"], p["gamma"], seed=2, oversample=p["oversample"],
                             device=device)
