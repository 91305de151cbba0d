"""The reference's operator API (``spectra.kernels``) restated with torch ops,
for running the reference engine without the CUDA kernels of this package.

TEST INFRASTRUCTURE ONLY: the tiny-model engine fixtures are produced by the
reference engine running on the CPU with this module injected as
``spectra.kernels`` (the reference's own kernels are Triton and need a GPU),
and the GPU engine test compares this package's kernels with it.

Both functions keep the reference wrappers' signatures and output-dtype
rules (spectra/kernels.py:132-184, :333-389) and compute with the dequant
formula of the reference's unit test (tests/test_kernels.py:31-39), exact
``(q - z) * s`` in fp32: the GEMV multiplies the exact weights and
activations in fp32 (the reference GEMV's arithmetic), the GEMM the operands
rounded to the compute dtype (the reference GEMM's tensor-core operands);
both accumulate in fp32 and round once at the end.
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
    """The reference GEMM feeds its tensor-core dot the dequantised weights,
    the activations and the outlier weights rounded to the compute dtype (bf16
    for bf16 activations, else fp16; spectra/kernels.py:256-261, :315-317)."""
    K = a.shape[-1]
    compute = torch.bfloat16 if a.dtype == torch.bfloat16 else torch.float16
    a2 = a.reshape(-1, K).to(compute).float()
    w = cpu_path.dequant(packed_b, scales, zeros, marlin_layout).to(compute).float()
    c = a2 @ w.t()
    if outlier_idx is not None and outlier_w is not None and outlier_idx.numel():
        c = c + a2[:, outlier_idx] @ outlier_w.to(compute).float().t()
    return c.to(compute).reshape(a.shape[:-1] + (packed_b.shape[0],)).to(a.dtype)


def as_module() -> types.ModuleType:
    """A stand-in ``spectra.kernels`` module with the two operators."""
    m = types.ModuleType("spectra.kernels")
    m.fused_w4a16_gemv_hdsq = fused_w4a16_gemv_hdsq
    m.batched_w4a16_gemm = batched_w4a16_gemm
    return m
