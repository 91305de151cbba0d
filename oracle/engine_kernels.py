"""The reference's operator API (``spectra.kernels``) restated with torch ops,
for running the reference engine without the CUDA kernels of this package.

TEST INFRASTRUCTURE ONLY: the tiny-model engine fixtures are produced by the
reference engine running on the CPU with this module injected as
``spectra.kernels`` (the reference's own kernels are Triton and need a GPU),
and the GPU engine test compares this package's kernels with it.

Both functions keep the reference wrappers' signatures and output-dtype
rules (spectra/kernels.py:132-184, :333-389) and compute with the dequant
formula of the reference's unit test (tests/test_kernels.py:31-39): exact
``(q - z) * s`` in fp32, fp32 matmul, outlier columns added from the exact
outlier weights, one rounding at the end.
"""
from __future__ import annotations

import types
from typing import Optional

import torch

from . import cpu_path


def fused_w4a16_gemv_hdsq(x: torch.Tensor, packed_w: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                          bias: Optional[torch.Tensor] = None, outlier_idx: Optional[torch.Tensor] = None,
                          outlier_w: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                          marlin_layout: bool = False) -> torch.Tensor:
    orig_dim = x.ndim
    x2 = x.unsqueeze(0) if orig_dim == 1 else x
    y = cpu_path.linear(x2, packed_w, scales, zeros, outlier_idx, outlier_w, bias, marlin=marlin_layout)
    compute = torch.bfloat16 if x.dtype == torch.bfloat16 else torch.float16
    y = y.to(compute)
    if out is not None:
        out.copy_(y)
        y = out
    return y.squeeze(0) if orig_dim == 1 else y


def batched_w4a16_gemm(a: torch.Tensor, packed_b: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                       outlier_idx: Optional[torch.Tensor] = None, outlier_w: Optional[torch.Tensor] = None,
                       marlin_layout: bool = False) -> torch.Tensor:
    K = a.shape[-1]
    a2 = a.reshape(-1, K)
    c = cpu_path.linear(a2, packed_b, scales, zeros, outlier_idx, outlier_w, None, marlin=marlin_layout)
    compute = torch.bfloat16 if a.dtype == torch.bfloat16 else torch.float16
    return c.to(compute).reshape(a.shape[:-1] + (packed_b.shape[0],)).to(a.dtype)


def as_module() -> types.ModuleType:
    """A stand-in ``spectra.kernels`` module with the two operators."""
    m = types.ModuleType("spectra.kernels")
    m.fused_w4a16_gemv_hdsq = fused_w4a16_gemv_hdsq
    m.batched_w4a16_gemm = batched_w4a16_gemm
    return m
