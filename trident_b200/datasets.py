"""Seeded synthetic stand-ins for the reference's datasets (SIFT-, GIST- and Deep-shaped).

The benchmark configurations name synthetic distributions of the reference datasets' shapes; the
real datasets (SIFT1M/GIST1M/Deep10M/SIFT100M) are not used. Two generators produce the same
distributions: NumPy PCG64 on the host (tests, fixtures, CPU-sized cases) and torch's Philox on a
CUDA device (benchmark-sized cases). They draw different numbers; the stored arrays, not the
generator, are the ground truth every check uses.

Seeds: base rows 0, queries 1, k-means 2, PCA sample 3; mixture centres 100. The centres are always
drawn by NumPy (PCG64, seed 100), whichever generator draws the rows, so base rows generated on the
GPU and queries generated on the host come from the same mixture.
"""
from dataclasses import dataclass, field
from typing import Optional, Tuple

import numpy as np

SEED_BASE, SEED_QUERY, SEED_KMEANS, SEED_PCA, SEED_CENTRES = 0, 1, 2, 3, 100


@dataclass(frozen=True)
class Config:
    name: str
    N: int
    D: int
    nlist: int
    nprobe: int
    K: int
    B: int
    kind: str                 # "int_mixture" | "decay" | "norm_mixture"
    n_comp: int = 0
    sigma: float = 0.0
    alpha: float = 0.7
    kmeans_sample: int = 0    # 0 -> min(N, 64 * nlist)
    extra: dict = field(default_factory=dict)

    def sample_size(self) -> int:
        return self.kmeans_sample or min(self.N, 64 * self.nlist)


# The five configurations of the benchmark (configs[0..4]).
CONFIGS = {
    "c1": Config("c1", 100_000, 128, 256, 16, 10, 1000, "int_mixture", n_comp=256, sigma=20.0, kmeans_sample=20_000),
    "c2": Config("c2", 1_000_000, 960, 1024, 64, 10, 1000, "decay", alpha=0.7),
    "c3": Config("c3", 10_000_000, 96, 4096, 32, 10, 10_000, "norm_mixture", n_comp=1024, sigma=0.25,
                 extra={"nprobe": (32, 128), "K": (1, 10, 50, 100), "B": (1, 100, 10_000)}),
    "c4": Config("c4", 100_000_000, 128, 65_536, 256, 10, 10_000, "int_mixture", n_comp=4096, sigma=25.0),
    "c5": Config("c5", 1_000_000_000, 128, 262_144, 512, 10, 10_000, "int_mixture", n_comp=16_384, sigma=25.0),
}


def scaled(cfg: Config, N: Optional[int] = None, nlist: Optional[int] = None, B: Optional[int] = None,
           nprobe: Optional[int] = None, K: Optional[int] = None, D: Optional[int] = None) -> Config:
    """A smaller case of the same distribution (used by tests and the oracle)."""
    kw = dict(cfg.__dict__)
    for k, v in (("N", N), ("nlist", nlist), ("B", B), ("nprobe", nprobe), ("K", K), ("D", D)):
        if v is not None:
            kw[k] = v
    kw["name"] = f"{cfg.name}_small"
    if N is not None and cfg.kmeans_sample:
        kw["kmeans_sample"] = min(cfg.kmeans_sample, N)
    return Config(**kw)


# ----------------------------------------------------------------------------------------------
# NumPy generator (host)
# ----------------------------------------------------------------------------------------------
def _np_centres(cfg: Config) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(SEED_CENTRES))
    if cfg.kind == "int_mixture":
        return rng.uniform(0.0, 255.0, size=(cfg.n_comp, cfg.D))
    if cfg.kind == "norm_mixture":
        return rng.standard_normal((cfg.n_comp, cfg.D))
    return np.zeros((0, cfg.D))


def generate_np(cfg: Config, n: int, seed: int, chunk: int = 65_536) -> np.ndarray:
    """n rows of cfg's distribution as float32 [n, D] (host)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = np.empty((n, cfg.D), np.float32)
    centres = _np_centres(cfg)
    scale = (np.arange(cfg.D, dtype=np.float64) + 1.0) ** (-cfg.alpha)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        m = e - s
        if cfg.kind == "int_mixture":
            comp = rng.integers(0, cfg.n_comp, size=m)
            x = centres[comp] + rng.normal(0.0, cfg.sigma, size=(m, cfg.D))
            out[s:e] = np.clip(np.rint(x), 0.0, 255.0)
        elif cfg.kind == "decay":
            x = np.abs(rng.standard_normal((m, cfg.D))) * scale
            out[s:e] = x / x.sum(axis=1, keepdims=True)
        elif cfg.kind == "norm_mixture":
            comp = rng.integers(0, cfg.n_comp, size=m)
            x = centres[comp] + cfg.sigma * rng.standard_normal((m, cfg.D))
            out[s:e] = x / np.linalg.norm(x, axis=1, keepdims=True)
        else:
            raise ValueError(cfg.kind)
    return out


# ----------------------------------------------------------------------------------------------
# torch generator (CUDA device)
# ----------------------------------------------------------------------------------------------
def _torch_centres(cfg: Config, device):
    """The mixture centres of the NumPy generator (PCG64, seed SEED_CENTRES), moved to `device`: rows
    drawn on the GPU and queries drawn on the host must come from the same mixture."""
    import torch

    if cfg.kind not in ("int_mixture", "norm_mixture"):
        return None
    return torch.from_numpy(_np_centres(cfg)).to(device)


TORCH_CHUNK = 1 << 20  # rows per generator call; regeneration must use the same chunking


def iter_torch_chunks(cfg: Config, n: int, seed: int, device="cuda", chunk: int = TORCH_CHUNK):
    """Yields (start, end, rows [end - start, D] float32 on `device`) for rows [0, n) of cfg's
    distribution, in order. The draws depend only on (cfg, seed, chunk), so a second pass yields the
    same rows: a process can regenerate the rows it needs instead of keeping them."""
    for s, e, x in _torch_rows(cfg, n, seed, device, chunk):
        yield s, e, x


def generate_torch(cfg: Config, n: int, seed: int, device="cuda", chunk: int = TORCH_CHUNK, out=None):
    """n rows of cfg's distribution as a float32 tensor [n, D] on `device` (or written into `out`)."""
    import torch

    if out is None:
        out = torch.empty((n, cfg.D), dtype=torch.float32, device=device)
    for s, e, x in _torch_rows(cfg, n, seed, device, chunk):
        out[s:e].copy_(x)
    return out


def _torch_rows(cfg: Config, n: int, seed: int, device, chunk: int):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    centres = _torch_centres(cfg, device)
    scale = (torch.arange(cfg.D, device=device, dtype=torch.float64) + 1.0) ** (-cfg.alpha)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        m = e - s
        if cfg.kind == "int_mixture":
            comp = torch.randint(0, cfg.n_comp, (m,), generator=g, device=device)
            x = centres[comp] + cfg.sigma * torch.randn((m, cfg.D), generator=g, device=device, dtype=torch.float64)
            x = torch.clamp(torch.round(x), 0.0, 255.0)
        elif cfg.kind == "decay":
            x = torch.randn((m, cfg.D), generator=g, device=device, dtype=torch.float64).abs_() * scale
            x = x / x.sum(dim=1, keepdim=True)
        elif cfg.kind == "norm_mixture":
            comp = torch.randint(0, cfg.n_comp, (m,), generator=g, device=device)
            x = centres[comp] + cfg.sigma * torch.randn((m, cfg.D), generator=g, device=device, dtype=torch.float64)
            x = x / torch.linalg.norm(x, dim=1, keepdim=True)
        else:
            raise ValueError(cfg.kind)
        yield s, e, x.to(torch.float32)


def make_dataset(cfg: Config, device=None) -> Tuple[object, object]:
    """(base rows, queries) for cfg: NumPy arrays when device is None, else CUDA tensors."""
    if device is None:
        return generate_np(cfg, cfg.N, SEED_BASE), generate_np(cfg, cfg.B, SEED_QUERY)
    return generate_torch(cfg, cfg.N, SEED_BASE, device), generate_torch(cfg, cfg.B, SEED_QUERY, device)
