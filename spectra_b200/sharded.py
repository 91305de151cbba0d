"""N-sharded SPECTRA linear layer across the GPUs of one node.

A large linear (N output features) is split by weight rows: rank r of g holds
rows [r*Ns, min(N, (r+1)*Ns)) with Ns = ceil(N / g) of the packed codes,
scales, zero points, outlier weights and bias; ``outlier_idx`` (columns of x)
and the activations x are replicated.  Each rank computes its [M, Ns] slice
with the same kernels as the unsharded layer (the M=1 GEMV with bias fused,
else the tensor-core GEMM plus bias, exactly as ``SpectraFusedLinear.forward``
routes them, spectra/engine.py:90-124), then one all-gather over the process
group assembles [M, N].  This is the only collective: the slices are
independent.

The gathered buffer is laid out [g, M, Ns]; for M = 1 it already is the output
row (no copy), for M > 1 one transpose copy makes it [M, N].  Rows of the last
shard past N are zero and dropped.

The reference has no multi-GPU path (no collective call sites); this module is
the sharding the hot path's large layers (lm_head, 8192 x 28672) need on an
8 x B200 NVSwitch node.  Sharding small layers is slower than one GPU once the
gather latency is counted, so callers shard only large layers.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def shard_bounds(N: int, world: int, rank: int):
    """(Ns, lo, hi): shard width and this rank's row range [lo, hi)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    ns = -(-N // world)
    lo = min(N, rank * ns)
    hi = min(N, lo + ns)
    return ns, lo, hi


def _kernel_local(x2d, packed, scales, zeros, outlier_idx, outlier_w, bias, marlin_layout):
    """This rank's slice with the production kernels (spectra/engine.py:97-124 routing)."""
    from . import kernels as SK
    if x2d.shape[0] == 1:
        return SK.fused_w4a16_gemv_hdsq(x2d, packed, scales, zeros, bias=bias, outlier_idx=outlier_idx,
                                        outlier_w=outlier_w, marlin_layout=marlin_layout)
    y = SK.batched_w4a16_gemm(x2d, packed, scales, zeros, outlier_idx=outlier_idx, outlier_w=outlier_w,
                              marlin_layout=marlin_layout)
    return y + bias if bias is not None else y


class ShardedW4A16Linear:
    """Row-sharded W4A16 linear; ``forward(x)`` returns the full [..., N] output on
    every rank.

    ``packed``/``scales``/``zeros``/``outlier_w``/``bias`` are the FULL layer
    tensors (any device); the constructor keeps this rank's rows, moved to
    ``device``.  ``local_fn`` computes one rank's slice; it defaults to the CUDA
    kernels (tests on CPU pass a reference implementation instead).
    """

    def __init__(self, packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                 outlier_idx: Optional[torch.Tensor] = None, outlier_w: Optional[torch.Tensor] = None,
                 bias: Optional[torch.Tensor] = None, marlin_layout: bool = False,
                 group: Optional[dist.ProcessGroup] = None, device: Optional[torch.device] = None,
                 local_fn: Optional[Callable] = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.N = packed.shape[0]
        self.in_features = packed.shape[1] * 2
        self.ns, lo, hi = shard_bounds(self.N, self.world, self.rank)
        self.rows = hi - lo
        dev = device if device is not None else packed.device
        self.device = dev

        def take(t):
            return None if t is None else t[lo:hi].contiguous().to(dev)
        self.packed, self.scales, self.zeros = take(packed), take(scales), take(zeros)
        self.outlier_w = take(outlier_w) if outlier_idx is not None else None
        self.outlier_idx = outlier_idx.to(dev) if outlier_idx is not None and outlier_w is not None else None
        self.bias = take(bias)
        self.marlin_layout = marlin_layout
        self.local_fn = local_fn or _kernel_local

    def local(self, x2d: torch.Tensor) -> torch.Tensor:
        """[M, Ns] slice of this rank (rows past the layer's end are zero)."""
        M = x2d.shape[0]
        out = torch.zeros(M, self.ns, device=x2d.device, dtype=x2d.dtype) if self.rows < self.ns else None
        if self.rows == 0:
            return out
        y = self.local_fn(x2d, self.packed, self.scales, self.zeros, self.outlier_idx, self.outlier_w,
                          self.bias, self.marlin_layout)
        if out is None:
            return y.to(x2d.dtype).reshape(M, self.ns)
        out[:, :self.rows] = y.reshape(M, self.rows)
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        orig_shape = x.shape
        M = x.numel() // self.in_features
        x2d = x.reshape(M, self.in_features)
        y_local = self.local(x2d).contiguous()
        if self.world == 1:
            y = y_local[:, :self.N]
        else:
            gathered = torch.empty(self.world * M * self.ns, device=y_local.device, dtype=y_local.dtype)
            dist.all_gather_into_tensor(gathered, y_local.reshape(-1), group=self.group)
            if M == 1:
                y = gathered[:self.N].reshape(1, self.N)
            else:
                y = gathered.view(self.world, M, self.ns).permute(1, 0, 2).reshape(M, self.world * self.ns)
                y = y[:, :self.N]
        return y.reshape(orig_shape[:-1] + (self.N,)).to(x.dtype)

    __call__ = forward
