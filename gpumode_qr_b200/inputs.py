"""Seeded input generators: the five workload configs, the reference's GPUMODE
shapes and its stress structures.

All generation happens on the CPU with ``torch.Generator`` seeds so that the
CPU oracle and the GPU see bit-identical inputs; callers move the result to the
device themselves.

* :data:`CONFIGS` — the workload configs (iid N(0,1), or ``U diag(s) V^T`` with
  Haar U, V and log-spaced singular values). The Haar recipe: one generator
  seeded with the config seed draws ``Z_U`` then ``Z_V`` (N(0,1), FP64,
  ``[b, n, n]``); ``Q, R = qr(Z)``, ``U = Q diag(sign(diag R))`` (sign 0 -> +1);
  ``A = (U diag(s)) V^T`` in FP64, cast to FP32.
* :data:`BENCHMARK_SHAPES`, :func:`column_scaled_dense` — the reference's
  ranked shapes and its dense generator (``src/qrbench/inputs.py:20-28,
  :52-60``): N(0,1) with columns scaled by ``logspace(0, -cond, n)``.
* :func:`stress_cases` — the reference's nine stress structures
  (``src/qrbench/inputs.py:84-135``), drawn in the same order from one CPU
  generator.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class Config:
    index: int
    batch: int
    n: int
    kind: str  # "iid" | "haar"
    seed: int
    log10_cond: float = 0.0  # singular values logspace(0, log10_cond, n) for "haar"
    parity: bool = True  # elementwise parity vs geqrf is asserted (cond <= 1e2)

    @property
    def name(self) -> str:
        return f"cfg{self.index}_b{self.batch}_n{self.n}"

    @property
    def bytes(self) -> int:
        """Algorithmic HBM bytes: read A once, write H once (tau ignored)."""
        return 2 * self.batch * self.n * self.n * 4

    @property
    def flops(self) -> float:
        """Algorithmic FLOPs of Householder QR of square matrices: 4/3 n^3 each."""
        return 4.0 / 3.0 * self.n**3 * self.batch


CONFIGS: list[Config] = [
    Config(1, 8, 64, "iid", 0),
    Config(2, 4096, 32, "iid", 1),
    Config(3, 640, 512, "haar", 2, 2.0),
    Config(4, 64, 1024, "haar", 3, 4.0, parity=False),
    Config(5, 8, 4096, "iid", 4),
]


def config(index: int) -> Config:
    return CONFIGS[index - 1]


def _haar(z: torch.Tensor) -> torch.Tensor:
    q, r = torch.linalg.qr(z)
    d = torch.diagonal(r, dim1=-2, dim2=-1)
    s = torch.where(d < 0, -torch.ones_like(d), torch.ones_like(d))
    return q * s.unsqueeze(-2)


def make_config_input(cfg: Config, batch: int | None = None) -> torch.Tensor:
    """CPU float32 ``[batch, n, n]`` input of a config (first ``batch`` matrices).

    The first ``batch`` matrices are exactly the leading matrices of the full
    config batch only for "iid" configs; "haar" inputs with a smaller batch are
    drawn from the same recipe and seed at that batch size.
    """
    b = cfg.batch if batch is None else batch
    g = torch.Generator().manual_seed(cfg.seed)
    n = cfg.n
    if cfg.kind == "iid":
        return torch.randn(b, n, n, generator=g, dtype=torch.float32)
    zu = torch.randn(b, n, n, generator=g, dtype=torch.float64)
    zv = torch.randn(b, n, n, generator=g, dtype=torch.float64)
    u = _haar(zu)
    v = _haar(zv)
    s = torch.logspace(0.0, cfg.log10_cond, n, dtype=torch.float64)
    a = (u * s.unsqueeze(-2)) @ v.transpose(-2, -1)
    return a.to(torch.float32)


# ---------------------------------------------------------------------------
# The reference's benchmark shapes and stress structures
# ---------------------------------------------------------------------------

BENCHMARK_SHAPES: list[dict] = [
    {"batch": 20, "cond": 1, "n": 32},
    {"batch": 40, "cond": 1, "n": 176},
    {"batch": 40, "cond": 1, "n": 352},
    {"batch": 640, "cond": 2, "n": 512},
    {"batch": 60, "cond": 2, "n": 1024},
    {"batch": 8, "cond": 1, "n": 2048},
    {"batch": 2, "cond": 1, "n": 4096},
]


@dataclass
class Problem:
    name: str
    tensor: torch.Tensor
    meta: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return self.tensor.shape[0]

    @property
    def n(self) -> int:
        return self.tensor.shape[-1]


def column_scaled_dense(batch: int, n: int, cond: float, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(batch, n, n, generator=g, dtype=torch.float32)
    scale = torch.logspace(0, -float(cond), n, dtype=torch.float32)
    return a * scale


def make_benchmark_problem(shape: dict, seed: int = 0) -> Problem:
    t = column_scaled_dense(shape["batch"], shape["n"], shape["cond"], seed)
    name = f"b{shape['batch']}_n{shape['n']}_cond{shape['cond']}"
    return Problem(name=name, tensor=t, meta=dict(shape))


def stress_cases(n: int, batch: int = 4, seed: int = 1234) -> list[Problem]:
    g = torch.Generator().manual_seed(seed)
    out: list[Problem] = []
    f32 = torch.float32

    def add(name, t, **meta):
        out.append(Problem(name=f"{name}_n{n}", tensor=t.contiguous(), meta=meta))

    def dense(cond):
        a = torch.randn(batch, n, n, generator=g, dtype=f32)
        return a * torch.logspace(0, -float(cond), n, dtype=f32)

    add("dense_cond1", dense(1), kind="dense", cond=1)
    add("dense_cond4", dense(4), kind="dense", cond=4)
    r = max(1, n // 2)
    u = torch.randn(batch, n, r, generator=g, dtype=f32)
    v = torch.randn(batch, r, n, generator=g, dtype=f32)
    add("rank_deficient", u @ v, kind="rank_deficient", rank=r)
    tiny = 1e-6 * torch.randn(batch, n, n, generator=g, dtype=f32)
    add("near_rank_deficient", u @ v + tiny, kind="near_rank_deficient", rank=r)
    full = torch.randn(batch, n, n, generator=g, dtype=f32)
    bw = max(1, n // 16)
    idx = torch.arange(n)
    add("banded", full * ((idx[None, :] - idx[:, None]).abs() <= bw), kind="banded", bandwidth=bw)
    base = torch.randn(batch, n, n, generator=g, dtype=f32)
    add("row_scaled", base * torch.logspace(0, -6, n, dtype=f32).view(1, n, 1), kind="row_scaled")
    direction = torch.randn(batch, n, 1, generator=g, dtype=f32)
    perturb = 1e-4 * torch.randn(batch, n, n, generator=g, dtype=f32)
    add("near_collinear", direction + perturb, kind="near_collinear")
    add("upper_triangular", torch.triu(torch.randn(batch, n, n, generator=g, dtype=f32)),
        kind="upper_triangular")
    clustered = torch.randn(batch, n, n, generator=g, dtype=f32)
    cscale = torch.ones(n, dtype=f32)
    cscale[n // 2:] = 1e-5
    add("clustered_scale", clustered * cscale, kind="clustered_scale")
    return out
