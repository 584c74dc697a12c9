"""Seeded synthetic graphs and features with the shapes of the benchmark workloads.

No dataset content is used: Cora, ogbn-arxiv and ogbn-products are absent here
(gnnc/ingress.py:52-83 would download them), so each workload is a seeded graph
with the real dataset's node/edge counts and a degree distribution of the
stated kind. The generators are deterministic functions of (shape, seed).

  c1  2-layer GCN, fp32. Configuration model, power-law exponent 2.5, 2,708
      nodes, exactly 5,278 undirected (10,556 directed) edges, no loops or
      duplicates; X in {0,1}^{2708x1433} ~ Bernoulli(0.0127); 1433-16-7.
  c2  2-layer GAT on the c1 graph and features: 8 heads x 8 (concat, ELU), then
      1 head x 7; slope 0.2.
  c3  3-layer GAT on an R-MAT graph (a,b,c,d = .57,.19,.19,.05), 169,343 nodes,
      exactly 1,166,243 unique directed non-loop edges, symmetrised; X ~ N(0,1)
      [N,128]; 4x64 hidden (concat), 40 classes; fp32 (c3) or bf16 features
      with fp32 accumulation (c3-bf16).
  c4  3-layer GCN / GAT on a configuration-model graph, exponent 2.1,
      2,449,029 nodes, exactly 30,929,570 undirected (61,859,140 directed)
      edges; X ~ N(0,1) bf16 [N,100]; hidden 256 (GAT 4x64), 47 classes.
  c5  fused SDDMM -> LeakyReLU -> softmax -> SpMM microbenchmark on R-MAT
      scale 24 (16,777,216 nodes, 2^28 edges as generated, duplicates kept),
      h [N, 4x64] bf16 ~ N(0,1), a_src / a_dst ~ N(0, 0.1).

Configuration model: degrees d_i = min(cap, floor(x_min * U_i^(-1/(gamma-1))))
with the structural cutoff cap = sqrt(2m) and x_min chosen by bisection so
that the stub count is ~1.1 x 2m; stubs are shuffled and paired, self-loops
and duplicates dropped, and the edge set trimmed (uniformly) or topped up
(stub-weighted pairs) to exactly m undirected edges.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

__all__ = [
    "CONFIGS",
    "WorkloadConfig",
    "config_model_edges",
    "rmat_edges",
    "rmat_unique_symmetric",
    "make_features",
]


@dataclass(frozen=True)
class WorkloadConfig:
    name: str
    model: str  # "gcn", "gat" or "fused"
    graph: str  # "config" or "rmat"
    num_nodes: int
    num_edges: int  # undirected edges (config), unique directed (rmat, c3) or raw (c5)
    in_channels: int
    hidden: int
    out_channels: int
    num_layers: int
    heads: int = 1
    exponent: float = 2.5
    features: str = "normal"  # "bernoulli" or "normal"
    density: float = 0.0
    feature_dtype: torch.dtype = torch.float32
    seed: int = 0
    rmat: tuple[float, float, float, float] = (0.57, 0.19, 0.19, 0.05)
    notes: dict = field(default_factory=dict)


CONFIGS: dict[str, WorkloadConfig] = {
    "c1": WorkloadConfig("c1", "gcn", "config", 2708, 5278, 1433, 16, 7, 2, exponent=2.5,
                         features="bernoulli", density=0.0127),
    "c2": WorkloadConfig("c2", "gat", "config", 2708, 5278, 1433, 8, 7, 2, heads=8,
                         exponent=2.5, features="bernoulli", density=0.0127),
    "c3": WorkloadConfig("c3", "gat", "rmat", 169343, 1166243, 128, 64, 40, 3, heads=4),
    "c3-bf16": WorkloadConfig("c3-bf16", "gat", "rmat", 169343, 1166243, 128, 64, 40, 3,
                              heads=4, feature_dtype=torch.bfloat16),
    "c4-gcn": WorkloadConfig("c4-gcn", "gcn", "config", 2449029, 30929570, 100, 256, 47, 3,
                             exponent=2.1, feature_dtype=torch.bfloat16),
    "c4-gat": WorkloadConfig("c4-gat", "gat", "config", 2449029, 30929570, 100, 64, 47, 3,
                             heads=4, exponent=2.1, feature_dtype=torch.bfloat16),
    "c5": WorkloadConfig("c5", "fused", "rmat", 1 << 24, 1 << 28, 256, 64, 64, 1, heads=4,
                         feature_dtype=torch.bfloat16),
}


def _degree_sequence(n: int, m: int, exponent: float, rng: np.random.Generator) -> np.ndarray:
    u = 1.0 - rng.random(n)  # (0, 1]
    tail = u ** (-1.0 / (exponent - 1.0))
    cap = max(1, int(math.sqrt(2.0 * m)))
    target = 1.1 * 2.0 * m

    def stubs(x_min: float) -> np.ndarray:
        return np.minimum(cap, np.floor(x_min * tail)).astype(np.int64)

    lo, hi = 1e-3, float(cap)
    for _ in range(60):
        mid = 0.5 * (lo + hi)
        if stubs(mid).sum() < target:
            lo = mid
        else:
            hi = mid
    d = stubs(hi)
    if d.sum() % 2:
        d[int(rng.integers(n))] += 1
    return d


def _unique_pairs(u: np.ndarray, v: np.ndarray, n: int) -> torch.Tensor:
    """Sorted unique keys min(u,v)*n + max(u,v) of the non-loop pairs."""
    tu, tv = torch.from_numpy(u), torch.from_numpy(v)
    keep = tu != tv
    a = torch.minimum(tu[keep], tv[keep])
    b = torch.maximum(tu[keep], tv[keep])
    return torch.unique(a * n + b)


def config_model_edges(
    n: int, m: int, exponent: float, seed: int = 0
) -> torch.Tensor:
    """Symmetric edge_index [2, 2m] (int64): exactly m undirected edges, no loops/dups."""
    rng = np.random.Generator(np.random.PCG64(seed))
    d = _degree_sequence(n, m, exponent, rng)
    stubs = np.repeat(np.arange(n, dtype=np.int64), d)
    rng.shuffle(stubs)
    if stubs.size % 2:
        stubs = stubs[:-1]
    keys = _unique_pairs(stubs[0::2], stubs[1::2], n)
    while keys.numel() < m:
        need = int((m - keys.numel()) * 1.3) + 16
        a = stubs[rng.integers(0, stubs.size, need)]
        b = stubs[rng.integers(0, stubs.size, need)]
        keys = torch.unique(torch.cat([keys, _unique_pairs(a, b, n)]))
    if keys.numel() > m:
        pick = torch.from_numpy(rng.permutation(keys.numel())[:m])
        keys = torch.sort(keys[pick]).values
    u = keys // n
    v = keys % n
    return torch.stack([torch.cat([u, v]), torch.cat([v, u])])


def rmat_edges(
    scale: int,
    n_edges: int,
    probs: tuple[float, float, float, float] = (0.57, 0.19, 0.19, 0.05),
    seed: int = 0,
    device: str | torch.device = "cpu",
) -> torch.Tensor:
    """Raw R-MAT edge list [2, n_edges] on `device` (duplicates and loops kept).

    Level i picks the quadrant (a: src 0 / dst 0, b: 0/1, c: 1/0, d: 1/1) of
    bit scale-1-i. The stream comes from a torch.Generator seeded with `seed`
    on `device` (the graph is a function of seed and device type)."""
    a, b, c, _ = probs
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    src = torch.zeros(n_edges, dtype=torch.int64, device=device)
    dst = torch.zeros(n_edges, dtype=torch.int64, device=device)
    for lvl in range(scale):
        r = torch.rand(n_edges, generator=g, device=device)
        bit = 1 << (scale - 1 - lvl)
        sbit = r >= (a + b)
        dbit = ((r >= a) & (r < a + b)) | (r >= a + b + c)
        src |= sbit.to(torch.int64) * bit
        dst |= dbit.to(torch.int64) * bit
        del r, sbit, dbit
    return torch.stack([src, dst])


def rmat_unique_symmetric(
    n: int, m: int, probs=(0.57, 0.19, 0.19, 0.05), seed: int = 0
) -> tuple[torch.Tensor, int]:
    """R-MAT graph with exactly m unique directed non-loop edges among n nodes,
    then symmetrised (union with the reverse). Returns (edge_index, m)."""
    scale = max(1, math.ceil(math.log2(n)))
    keys = np.empty(0, dtype=np.int64)
    first = np.empty(0, dtype=np.int64)
    batch = 0
    while keys.size < m:
        ei = rmat_edges(scale, int(m * 1.6) + 1024, probs, seed=seed * 1000 + batch).numpy()
        s, d = ei[0], ei[1]
        ok = (s < n) & (d < n) & (s != d)
        k = s[ok] * n + d[ok]
        order = np.arange(k.size, dtype=np.int64) + batch * (1 << 40)
        allk = torch.from_numpy(np.concatenate([keys, k]))
        allo = torch.from_numpy(np.concatenate([first, order]))
        # first occurrence of each key: stable sort by key, keep run starts
        sk, perm = torch.sort(allk, stable=True)
        start = torch.ones_like(sk, dtype=torch.bool)
        start[1:] = sk[1:] != sk[:-1]
        keys, first = sk[start].numpy(), allo[perm[start]].numpy()
        batch += 1
    take = np.argsort(first, kind="stable")[:m]
    k = torch.from_numpy(keys[take])
    s, d = k // n, k % n
    sym = torch.unique(torch.cat([s * n + d, d * n + s]))
    return torch.stack([sym // n, sym % n]), m


def make_features(cfg: WorkloadConfig, seed: int = 1) -> torch.Tensor:
    """Node features [N, in_channels] (host, fp32 or bf16 per cfg)."""
    g = torch.Generator()
    g.manual_seed(seed)
    shape = (cfg.num_nodes, cfg.in_channels)
    if cfg.features == "bernoulli":
        x = (torch.rand(shape, generator=g) < cfg.density).to(torch.float32)
    else:
        x = torch.randn(shape, generator=g)
    return x.to(cfg.feature_dtype)


def make_graph(cfg: WorkloadConfig) -> torch.Tensor:
    """edge_index [2, E] int64 (host) for cfg (c5 is generated by rmat_edges on the GPU)."""
    if cfg.graph == "config":
        return config_model_edges(cfg.num_nodes, cfg.num_edges, cfg.exponent, cfg.seed)
    if cfg.name.startswith("c3"):
        return rmat_unique_symmetric(cfg.num_nodes, cfg.num_edges, cfg.rmat, cfg.seed)[0]
    scale = int(math.log2(cfg.num_nodes))
    return rmat_edges(scale, cfg.num_edges, cfg.rmat, cfg.seed)
