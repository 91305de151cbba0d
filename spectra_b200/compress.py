"""Device-side weight compressor: the tensors SPECTRA's compressor writes for
one linear layer, produced on the GPU.

It restates, in its own code, the algorithm of ``SpectraCompressor``:
  * group-32 asymmetric min/max INT4 codes (spectra/compressor.py:72-156):
    the CUDA kernel ``spectra_quantize_group32`` (csrc/format.cu) -- fp32
    arithmetic in the reference's operation order, round half to even,
    correctly rounded divisions, Marlin packing; bit-identical to the
    reference run on a CPU;
  * kurtosis-adaptive outlier columns (spectra/compressor.py:158-215): fp32
    column L2 norms, ratio = clamp(0.01*(1+0.15*log1p(max(0, kurt-3))),
    0.005, 0.03), top-k columns sorted ascending, zeroed before quantisation
    and kept exactly in the source dtype (torch reductions on the device:
    a K-long vector, not the hot path);
  * the load-time zero-point unpack (spectra/engine.py:1007-1012): the CUDA
    kernel ``spectra_unpack_zeros``.
The kernels need CUDA tensors; there is no CPU path (the numpy restatement in
``oracle/`` is the checker).  Only the column-norm reduction order can differ
from the reference, which matters only for exact near-ties between norms.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib as L

GROUP = 32

_DT = {torch.float16: L.DT_F16, torch.bfloat16: L.DT_BF16, torch.float32: L.DT_F32,
       torch.int32: L.DT_I32, torch.int64: L.DT_I64}


@dataclass
class CompressedLinear:
    packed: torch.Tensor        # u8 [N, K/2], Marlin nibble order
    scales: torch.Tensor        # fp16 [N, K/32]
    zeros: torch.Tensor         # u8 [N, K/32] (unpacked, as the engine binds them)
    packed_zeros: torch.Tensor  # u8 [N, ceil(K/64)] (the on-disk form)
    outlier_idx: torch.Tensor   # int64 [n_out], ascending
    outlier_w: torch.Tensor     # [N, n_out] in the source dtype
    ratio: float
    kurtosis: float


def _cuda(name: str, t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"spectra_b200.compress: {name} must be a CUDA tensor (no CPU path), got {t.device}")


def quantize_group32(w: torch.Tensor, outlier_idx: Optional[torch.Tensor] = None, marlin_layout: bool = True):
    """Group-32 INT4 codes of ``w`` [N, K] (fp16/bf16/fp32, CUDA), columns in
    ``outlier_idx`` read as zero.

    Returns (packed u8 [N,K/2], scales fp16 [N,K/32], zeros u8 [N,K/32],
    packed_zeros u8 [N,ceil(G/2)]).
    """
    _cuda("w", w)
    if w.dim() != 2 or w.shape[1] % GROUP:
        raise ValueError("w must be [N, K] with K a multiple of 32")
    if w.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError(f"unsupported weight dtype {w.dtype}")
    if w.stride(1) != 1:
        w = w.contiguous()
    N, K = w.shape
    G = K // GROUP
    dev = w.device
    packed = torch.empty(N, K // 2, dtype=torch.uint8, device=dev)
    scales = torch.empty(N, G, dtype=torch.float16, device=dev)
    zeros = torch.empty(N, G, dtype=torch.uint8, device=dev)
    pz = torch.empty(N, (G + 1) // 2, dtype=torch.uint8, device=dev)
    idx = None
    if outlier_idx is not None and outlier_idx.numel():
        _cuda("outlier_idx", outlier_idx)
        idx = outlier_idx.reshape(-1)
        if idx.dtype not in (torch.int32, torch.int64):
            idx = idx.to(torch.int64)
        idx = idx.contiguous()
    if N == 0:
        return packed, scales, zeros, pz
    with torch.cuda.device(dev):
        st = L.lib().spectra_quantize_group32(
            w.data_ptr(), _DT[w.dtype], w.stride(0),
            idx.data_ptr() if idx is not None else None, _DT[idx.dtype] if idx is not None else 0,
            idx.numel() if idx is not None else 0,
            packed.data_ptr(), packed.stride(0), scales.data_ptr(), scales.stride(0),
            zeros.data_ptr(), zeros.stride(0), pz.data_ptr(), pz.stride(0),
            N, K, L.LAYOUT_MARLIN if marlin_layout else L.LAYOUT_EVEN_ODD,
            torch.cuda.current_stream(dev).cuda_stream)
    L.check("spectra_quantize_group32", st)
    return packed, scales, zeros, pz


def unpack_zeros(packed_zeros: torch.Tensor, K: int) -> torch.Tensor:
    """Two zero points per byte -> one u8 per group (spectra/engine.py:1007-1012), on the GPU."""
    _cuda("packed_zeros", packed_zeros)
    if packed_zeros.dtype != torch.uint8 or packed_zeros.dim() != 2:
        raise TypeError("packed_zeros must be a 2-D uint8 tensor")
    pz = packed_zeros if packed_zeros.stride(1) == 1 else packed_zeros.contiguous()
    N = pz.shape[0]
    G = K // GROUP
    if pz.shape[1] * 2 < G:
        raise ValueError(f"packed_zeros has {pz.shape[1]} bytes per row; K={K} needs {(G + 1) // 2}")
    z = torch.empty(N, G, dtype=torch.uint8, device=pz.device)
    if N == 0 or G == 0:
        return z
    with torch.cuda.device(pz.device):
        st = L.lib().spectra_unpack_zeros(pz.data_ptr(), pz.stride(0), z.data_ptr(), z.stride(0), N, G,
                                          torch.cuda.current_stream(pz.device).cuda_stream)
    L.check("spectra_unpack_zeros", st)
    return z


def select_outliers(w: torch.Tensor, norm_vector: Optional[torch.Tensor] = None,
                    base_ratio: float = 0.01, adaptive: bool = True):
    """Outlier input columns of ``w`` [N, K]: (idx int64 ascending, ratio, kurtosis)."""
    N, K = w.shape
    if N > 4096:
        sq = torch.zeros(K, dtype=torch.float32, device=w.device)
        for r0 in range(0, N, 4096):
            c = w[r0:r0 + 4096].to(torch.float32)
            sq += (c * c).sum(dim=0)
        norms = sq.sqrt()
    else:
        norms = torch.linalg.vector_norm(w.to(torch.float32), dim=0)
    sal = norms if (norm_vector is None or norm_vector.numel() != K) else norm_vector.to(norms) * norms
    d = sal - sal.mean()
    var = (d * d).mean() + 1e-8
    kurt = max(1.0, float((d ** 4).mean() / (var * var)))
    if adaptive:
        mult = 1.0 + 0.15 * math.log1p(max(0.0, kurt - 3.0))
        ratio = float(torch.tensor(base_ratio * mult, dtype=torch.float32).clamp(0.005, 0.03))
    else:
        ratio = base_ratio
    n_out = max(1, int(round(K * ratio)))
    idx = torch.topk(sal, n_out, largest=True).indices.sort().values
    return idx.to(torch.int64), ratio, kurt


def compress_linear(w: torch.Tensor, norm_vector: Optional[torch.Tensor] = None) -> CompressedLinear:
    """Everything ``SpectraFusedLinear.set_weights`` receives for weight ``w`` (CUDA)."""
    _cuda("w", w)
    idx, ratio, kurt = select_outliers(w, norm_vector)
    ow = w[:, idx].contiguous()
    packed, scales, zeros, pz = quantize_group32(w, idx)
    return CompressedLinear(packed, scales, zeros, pz, idx, ow, ratio, kurt)
