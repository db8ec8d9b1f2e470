"""Seeded synthetic detector events for benchmarks and tests.

No public dataset ships with this package; these generators produce inputs
with the shapes and value distributions of the benchmark configurations:

* positions: x, y uniform in a disc of radius 500 m, z uniform in
  [-500, 500] m; time uniform in [0, 20000] ns, sorted within each event;
* q, k, v ~ N(0, 1); W ``[Dh, C]`` ~ N(0, 1/C); b ``[Dh]`` ~ N(0, 0.02^2);
* event lengths: lognormal (median, sigma) clipped to a range, or uniform.

With raw metre/nanosecond coordinates the spacetime interval of every
distinct pair exceeds the clip (|I| >= 16), so only the diagonal takes the
unclipped branch; ``scaled=True`` divides positions by 500 m and times by
3e4 ns (the encoder's own normalisation) so most pairs take the sqrt branch.
"""

from typing import Dict, List, Optional, Sequence

import torch
from torch import Tensor


def lognormal_lengths(n: int, median: float, sigma: float, lo: int, hi: int,
                      gen: torch.Generator) -> Tensor:
    z = torch.randn(n, generator=gen, dtype=torch.float64)
    return (median * torch.exp(sigma * z)).round().clamp(lo, hi).to(torch.int64)


def uniform_lengths(n: int, lo: int, hi: int, gen: torch.Generator) -> Tensor:
    return torch.randint(lo, hi + 1, (n,), generator=gen, dtype=torch.int64)


def detector_coords(lengths: Sequence[int], gen: torch.Generator, scaled: bool = False) -> Tensor:
    """Packed ``[T, 4]`` float32 coordinates (x, y, z, t), time-sorted per event."""
    total = int(sum(int(n) for n in lengths))
    r = 500.0 * torch.rand(total, generator=gen, dtype=torch.float64).sqrt()
    phi = 2 * torch.pi * torch.rand(total, generator=gen, dtype=torch.float64)
    z = 1000.0 * torch.rand(total, generator=gen, dtype=torch.float64) - 500.0
    t = 20000.0 * torch.rand(total, generator=gen, dtype=torch.float64)
    chunks = []
    start = 0
    for n in lengths:
        n = int(n)
        chunks.append(torch.sort(t[start:start + n]).values)
        start += n
    t = torch.cat(chunks) if chunks else t
    out = torch.stack((r * torch.cos(phi), r * torch.sin(phi), z, t), -1)
    if scaled:
        out[:, :3] /= 500.0
        out[:, 3] /= 3e4
    return out.to(torch.float32)


def projection(dim: int, channels: int, gen: torch.Generator) -> Dict[str, Tensor]:
    """W ``[Dh, C]`` ~ N(0, 1/C) and b ``[Dh]`` ~ N(0, 0.02^2), float32."""
    w = torch.randn(dim, channels, generator=gen) / channels**0.5
    b = 0.02 * torch.randn(dim, generator=gen)
    return {"weight": w, "bias": b}


def padded_batch(lengths: Sequence[int], length: int, heads: int, dim: int, channels: int,
                 dtype: torch.dtype, device: torch.device, seed: int,
                 scaled: bool = False) -> Dict[str, Tensor]:
    """A padded ``[B, H, L, Dh]`` batch; padding rows of q/k/v hold N(0,1) junk too."""
    gen = torch.Generator().manual_seed(seed)
    batch = len(lengths)
    coords = detector_coords([length] * batch, gen, scaled).view(batch, length, 4)
    proj = projection(dim, channels, gen)
    dgen = torch.Generator(device=device).manual_seed(seed + 1)
    shape = (batch, heads, length, dim)
    out = {
        name: torch.randn(shape, generator=dgen, device=device, dtype=torch.float32).to(dtype)
        for name in ("q", "k", "v", "grad")
    }
    out["feats"] = coords.to(device)
    out["weight"] = proj["weight"].to(device)
    out["bias"] = proj["bias"].to(device)
    out["seqlens"] = torch.as_tensor(list(lengths), dtype=torch.int32, device=device)
    return out


def packed_batch(lengths: Sequence[int], heads: int, dim: int, channels: int,
                 dtype: torch.dtype, device: torch.device, seed: int,
                 scaled: bool = False) -> Dict[str, Tensor]:
    """A packed ``[T, H, Dh]`` batch with int32 ``cu_seqlens``."""
    gen = torch.Generator().manual_seed(seed)
    total = int(sum(int(n) for n in lengths))
    coords = detector_coords(lengths, gen, scaled)
    proj = projection(dim, channels, gen)
    dgen = torch.Generator(device=device).manual_seed(seed + 1)
    shape = (total, heads, dim)
    out = {
        name: torch.randn(shape, generator=dgen, device=device, dtype=torch.float32).to(dtype)
        for name in ("q", "k", "v", "grad")
    }
    out["feats"] = coords.to(device)
    out["weight"] = proj["weight"].to(device)
    out["bias"] = proj["bias"].to(device)
    cu = torch.zeros(len(lengths) + 1, dtype=torch.int64)
    cu[1:] = torch.cumsum(torch.as_tensor(list(lengths), dtype=torch.int64), 0)
    out["cu_seqlens"] = cu.to(torch.int32).to(device)
    return out


def pair_flops(lengths: Sequence[int], heads: int, dim: int, channels: int) -> Dict[str, float]:
    """Algorithmic FLOPs over valid pairs: fwd 4Dh+4C, bwd 10Dh+8C per pair-head."""
    l2 = float(sum(int(n) * int(n) for n in lengths))
    return {
        "pairs": l2,
        "fwd": l2 * heads * (4 * dim + 4 * channels),
        "bwd": l2 * heads * (10 * dim + 8 * channels),
        "total": l2 * heads * (14 * dim + 12 * channels),
    }


def lengths_for(config: str, n_events: Optional[int], seed: int) -> List[int]:
    """Event lengths of a named benchmark configuration."""
    gen = torch.Generator().manual_seed(seed)
    if config == "config1":
        return lognormal_lengths(n_events or 256, 120.0, 1.2, 1, 768, gen).tolist()
    if config == "config3":
        n = n_events or 16384
        lens = lognormal_lengths(n, 80.0, 1.2, 1, 3000, gen)
        single = torch.rand(n, generator=gen) < 0.02
        lens[single] = 1
        return lens.tolist()
    if config == "config4":
        return uniform_lengths(n_events or 2048, 2048, 16384, gen).tolist()
    if config == "config0":
        return uniform_lengths(n_events or 4, 16, 128, gen).tolist()
    raise ValueError(f"unknown config {config!r}")
