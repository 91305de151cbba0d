"""Minimal drivers for profiling one kernel shape under ncu.

    python -m tests.prof_cases gemv K N n_out iters [--dtype bf16|f16]
    python -m tests.prof_cases gemm M K N n_out iters [--dtype bf16|f16]

Builds random tensors in SPECTRA's weight format of that shape on cuda:0
(codes uniform 0..15, fp16 scales in the range the compressor produces for
N(0, 0.02) weights, n_out outlier columns) and calls the public API `iters`
times, so a capture with ``-s <warm-ups> -c 1`` sees one warm launch.
"""
from __future__ import annotations

import argparse

import torch


def _weights(N: int, K: int, n_out: int, dt, dev):
    g = torch.Generator(device=dev).manual_seed(0)
    p = torch.randint(0, 256, (N, K // 2), generator=g, device=dev, dtype=torch.uint8)
    s = (torch.rand(N, K // 32, generator=g, device=dev) * 0.018 + 0.002).to(torch.float16)
    z = torch.randint(0, 16, (N, K // 32), generator=g, device=dev, dtype=torch.uint8)
    idx = torch.randperm(K, generator=g, device=dev)[:n_out].sort().values
    ow = (torch.randn(N, n_out, generator=g, device=dev) * 0.05).to(dt)
    return p, s, z, idx, ow


def main() -> None:
    from spectra_b200 import kernels as SK
    ap = argparse.ArgumentParser()
    ap.add_argument("op", choices=["gemv", "gemm"])
    ap.add_argument("dims", type=int, nargs="+", help="gemv: K N n_out iters; gemm: M K N n_out iters")
    ap.add_argument("--dtype", choices=["bf16", "f16"], default="bf16")
    a = ap.parse_args()
    dt = torch.bfloat16 if a.dtype == "bf16" else torch.float16
    dev = torch.device("cuda", 0)
    if a.op == "gemv":
        K, N, n_out, iters = a.dims
        M = 1
    else:
        M, K, N, n_out, iters = a.dims
    p, s, z, idx, ow = _weights(N, K, n_out, dt, dev)
    x = torch.randn(M, K, device=dev).to(dt)
    for _ in range(iters):
        if a.op == "gemv":
            y = SK.fused_w4a16_gemv_hdsq(x, p, s, z, outlier_idx=idx, outlier_w=ow, marlin_layout=True)
        else:
            y = SK.batched_w4a16_gemm(x, p, s, z, outlier_idx=idx, outlier_w=ow, marlin_layout=True)
    torch.cuda.synchronize()
    print(f"{a.op} M={M} K={K} N={N} n_out={n_out}: ok, |y|_1={float(y.float().abs().sum()):.4g}")


if __name__ == "__main__":
    main()
