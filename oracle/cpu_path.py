"""CPU path of the W4A16 linear layer, for the timed CPU baseline.

TEST / BASELINE INFRASTRUCTURE ONLY: used by ``bench.py``'s ``cpu_baseline``
leg and by ``bench.py --impl reference``; never by the product path.

The reference (NeuraCryption/SPECTRA) has no CPU implementation of its
linear kernels -- ``SpectraFusedLinear.forward`` always launches Triton
(spectra/engine.py:90-124).  Its CPU-side formula for the same layer is the
dequantise-then-matmul used by its own unit tests (tests/test_kernels.py:31-39)
and its embedding module (spectra/engine.py:177-206): unpack the nibbles,
``(q - z) * s`` in fp32, then a dense matmul.  This module restates that
formula with torch ops (multi-threaded BLAS) and adds the outlier columns and
bias exactly as the kernels do (spectra/kernels.py:102-124).
"""
from __future__ import annotations

import torch


def dequant(packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, marlin: bool = True) -> torch.Tensor:
    """fp32 ``(q - z) * s`` of a [N, K/2] packed matrix (tests/test_kernels.py:31-36)."""
    N, Kh = packed.shape
    K = 2 * Kh
    G = K // 32
    lo = (packed & 0x0F).to(torch.float32)
    hi = ((packed >> 4) & 0x0F).to(torch.float32)
    if marlin:
        q = torch.cat([lo.reshape(N, G, 16), hi.reshape(N, G, 16)], dim=-1)
    else:
        q = torch.stack([lo, hi], dim=-1).reshape(N, G, 32)
    z = zeros[:, :G].to(torch.float32).unsqueeze(-1)
    s = scales[:, :G].to(torch.float32).unsqueeze(-1)
    return ((q - z) * s).reshape(N, K)


def linear(x: torch.Tensor, packed, scales, zeros, outlier_idx=None, outlier_w=None, bias=None,
           marlin: bool = True) -> torch.Tensor:
    """y = x @ W^T (+ x[:, idx] @ ow^T) (+ bias) in fp32, x [M, K]."""
    xf = x.to(torch.float32)
    y = xf @ dequant(packed, scales, zeros, marlin).t()
    if outlier_idx is not None and outlier_w is not None and outlier_idx.numel():
        y = y + xf[:, outlier_idx] @ outlier_w.to(torch.float32).t()
    if bias is not None:
        y = y + bias.to(torch.float32)
    return y
