"""Device-side weight compressor: the tensors SPECTRA's compressor writes for
one linear layer, produced with torch ops on whatever device the weight lives
on (a CUDA device in the bench, the CPU in the tests).

It restates, in its own code, the algorithm of ``SpectraCompressor``:
  * group-32 asymmetric min/max INT4 codes (spectra/compressor.py:72-112):
    s = (max-min)/15 (constant groups: |min| or 1), z = clamp(round(-min/s)),
    q = clamp(round((w + z*s)/s)), fp32 arithmetic, round-half-to-even;
    Marlin packing (k in the low nibble, k+16 in the high nibble);
  * kurtosis-adaptive outlier columns (spectra/compressor.py:158-215): fp32
    column L2 norms, ratio = clamp(0.01*(1+0.15*log1p(max(0, kurt-3))),
    0.005, 0.03), top-k columns sorted ascending, zeroed before quantisation
    and kept exactly in the source dtype;
  * the load-time zero-point unpack (spectra/engine.py:1007-1012).
Every elementwise step is an IEEE fp32 operation in the same order as the
reference, so codes, scales and zero points are bit-identical to it; only
the column-norm reduction order can differ, which matters only for exact
near-ties between column norms.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

GROUP = 32


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


def quantize_group32(w: torch.Tensor):
    """Group-32 INT4 codes of ``w`` [N, K] (any float dtype).

    Returns (packed u8 [N,K/2], scales fp16 [N,K/32], packed_zeros u8 [N,ceil(G/2)]).
    """
    N, K = w.shape
    if K % GROUP:
        raise ValueError("K must be a multiple of 32")
    G = K // GROUP
    wg = w.reshape(N, G, GROUP).to(torch.float32)
    lo = wg.amin(dim=-1, keepdim=True)
    hi = wg.amax(dim=-1, keepdim=True)
    span = hi - lo
    flat = span < 1e-8
    one = torch.ones_like(lo)
    # tensor / tensor: a division by a Python scalar may be lowered to a
    # multiplication by its reciprocal on some devices, which rounds differently
    s = torch.where(flat, torch.where(lo == 0, one, lo.abs()), span / torch.full_like(span, 15.0)).clamp(min=1e-8)
    z_live = torch.round(-lo / s).clamp(0, 15)
    z = torch.where(flat, (lo < 0).to(torch.float32), z_live)
    q_live = torch.round((wg - (-(z * s))) / s).clamp(0, 15)
    q = torch.where(flat, (lo > 0).to(torch.float32).expand_as(wg), q_live).to(torch.uint8)
    packed = (q[..., :16] | (q[..., 16:] << 4)).reshape(N, K // 2)
    zb = z.to(torch.uint8).reshape(N, G)
    if G % 2:
        zb = torch.nn.functional.pad(zb, (0, 1))
    packed_zeros = zb[:, 0::2] | (zb[:, 1::2] << 4)
    return packed.contiguous(), s.reshape(N, G).to(torch.float16).contiguous(), packed_zeros.contiguous()


def unpack_zeros(packed_zeros: torch.Tensor, K: int) -> torch.Tensor:
    """Two zero points per byte -> one u8 per group (spectra/engine.py:1007-1012)."""
    lo = packed_zeros & 0x0F
    hi = (packed_zeros >> 4) & 0x0F
    z = torch.stack([lo, hi], dim=-1).reshape(packed_zeros.shape[0], -1)
    return z[:, : K // GROUP].contiguous()


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
    """Everything ``SpectraFusedLinear.set_weights`` receives for weight ``w``."""
    idx, ratio, kurt = select_outliers(w, norm_vector)
    ow = w[:, idx].contiguous()
    wz = w.clone()
    wz[:, idx] = 0
    packed, scales, pz = quantize_group32(wz)
    return CompressedLinear(packed, scales, unpack_zeros(pz, w.shape[1]), pz, idx, ow, ratio, kurt)
