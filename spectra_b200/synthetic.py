"""Seeded synthetic inputs for the W4A16 linear path.

The reference publishes no dataset for this path; its own unit tests and
benchmark configs draw Gaussian weights/activations from a fixed seed
(tests/test_kernels.py:12-14).  These helpers draw from torch's CPU generator
so every test, fixture and bench run sees the same bytes on every machine.

Distributions:
  "n1"   -- N(0, 1)
  "n002" -- N(0, 0.02^2), the scale of a random-initialised LLM linear
  "t3"   -- Student-t with 3 degrees of freedom rescaled to std 0.02
            (heavy-tailed columns that stress outlier isolation)
"""
from __future__ import annotations

import torch


def draw_weight(N: int, K: int, seed: int, dist: str = "n002", dtype=torch.float16) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    if dist == "n1":
        w = torch.randn(N, K, generator=g)
    elif dist == "n002":
        w = torch.randn(N, K, generator=g) * 0.02
    elif dist == "t3":
        z = torch.randn(N, K, generator=g)
        chi2 = torch.zeros(N, K)
        for _ in range(3):
            chi2 += torch.randn(N, K, generator=g) ** 2
        t = z / torch.sqrt(chi2 / 3.0)
        w = t / t.std() * 0.02
    else:
        raise ValueError(f"unknown distribution {dist!r}")
    return w.to(dtype)


def draw_act(M: int, K: int, seed: int, dtype=torch.bfloat16) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(M, K, generator=g).to(dtype)
