"""N-sharded SPECTRA linear layer across the GPUs of one node.

A large linear (N output features) is split by weight rows: rank r of g holds
rows [r*Ns, min(N, (r+1)*Ns)) with Ns = ceil(N / g) of the packed codes,
scales, zero points, outlier weights and bias; ``outlier_idx`` (columns of x)
and the activations x are replicated.  Each rank computes its [M, Ns] slice
with the same kernels as the unsharded layer (the M=1 GEMV with bias fused,
else the tensor-core GEMM plus bias, exactly as ``SpectraFusedLinear.forward``
routes them, spectra/engine.py:90-124), writing straight into a persistent
[M, Ns] buffer of this rank (rows past N stay zero: a ragged last shard costs
no extra kernel), then one all-gather assembles [M, N].  This is the only
collective: the slices are independent.

The all-gather, on GPUs of one node, is this package's peer-memory exchange
(spectra_b200.p2p: one kernel pushes the slice into every peer's buffer over
NVLink, flags it, and writes the gathered [M, N] output), with the slice
buffer being the exchange's source, so a call is two kernels; elsewhere (gloo,
or ``exchange="collective"``, or SPECTRA_B200_P2P=0 in the environment) it is
the process group's ``all_gather_into_tensor`` into a [g, M, Ns] buffer, which
for M = 1 already is the output row and for M > 1 takes one transpose copy.

Greedy decode does not need the whole row of logits on every rank:
``greedy(x)`` computes this rank's slice, its first maximum with the argmax
kernel (the layer's row index), and all-gathers one (value, index) pair per
rank -- 16 bytes instead of N logits -- before picking the first maximum in
rank order, which is row order (the engine's temperature-0 sample_token is a
torch.argmax, spectra/engine.py:1690-1713).

The reference has no multi-GPU path (no collective call sites); this module is
the sharding the hot path's large layers (lm_head, 8192 x 28672) need on an
8 x B200 NVSwitch node.  Sharding small layers is slower than one GPU once the
gather latency is counted, so callers shard only large layers.
"""
from __future__ import annotations

import os
from typing import Callable, Dict, Optional, Tuple

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


def _kernel_local(x2d, packed, scales, zeros, outlier_idx, outlier_w, bias, marlin_layout, out):
    """This rank's slice with the production kernels (spectra/engine.py:97-124
    routing), written into ``out`` ([M, rows] view of the rank's buffer)."""
    from . import kernels as SK
    if x2d.shape[0] == 1:
        SK.fused_w4a16_gemv_hdsq(x2d, packed, scales, zeros, bias=bias, outlier_idx=outlier_idx,
                                 outlier_w=outlier_w, out=out, marlin_layout=marlin_layout)
        return
    SK.batched_w4a16_gemm(x2d, packed, scales, zeros, outlier_idx=outlier_idx, outlier_w=outlier_w,
                          marlin_layout=marlin_layout, out=out)
    if bias is not None:
        out += bias


def _kernel_argmax(y: torch.Tensor, offset: int) -> Tuple[torch.Tensor, torch.Tensor]:
    from . import kernels as SK
    idx, val = SK.argmax(y, idx_offset=offset, with_values=True)
    return val, idx


class ShardedW4A16Linear:
    """Row-sharded W4A16 linear; ``forward(x)`` returns the full [..., N] output on
    every rank.

    ``packed``/``scales``/``zeros``/``outlier_w``/``bias`` are the FULL layer
    tensors (any device); the constructor keeps this rank's rows, moved to
    ``device``.  ``local_fn(x2d, packed, scales, zeros, idx, ow, bias, marlin,
    out)`` writes one rank's slice into ``out``; it defaults to the CUDA kernels
    (tests on CPU pass a reference implementation instead), as does
    ``argmax_fn(y, offset) -> (values, indices)``.

    ``exchange``: "auto" (the peer-memory exchange when the group's backend is
    NCCL on CUDA devices and SPECTRA_B200_P2P is not 0, else the group's
    all-gather), "p2p" or "collective".  ``wait_limit_s`` bounds the
    exchange kernel's wait for a peer.  The first call of each M is collective
    (it sets up that shape's exchange buffers on every rank); ``close()``
    releases them, collectively.
    """

    def __init__(self, packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                 outlier_idx: Optional[torch.Tensor] = None, outlier_w: Optional[torch.Tensor] = None,
                 bias: Optional[torch.Tensor] = None, marlin_layout: bool = False,
                 group: Optional[dist.ProcessGroup] = None, device: Optional[torch.device] = None,
                 local_fn: Optional[Callable] = None, argmax_fn: Optional[Callable] = None,
                 exchange: str = "auto", wait_limit_s: float = 5.0):
        if exchange not in ("auto", "p2p", "collective"):
            raise ValueError(f"exchange must be 'auto', 'p2p' or 'collective', not {exchange!r}")
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.N = packed.shape[0]
        self.in_features = packed.shape[1] * 2
        self.ns, lo, hi = shard_bounds(self.N, self.world, self.rank)
        self.row0 = lo
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
        self.argmax_fn = argmax_fn or _kernel_argmax
        self._local_bufs: Dict[Tuple[int, torch.dtype], torch.Tensor] = {}
        self._exchanges: Dict[tuple, object] = {}
        self.wait_limit_s = wait_limit_s
        self.use_p2p = False
        if self.world > 1 and exchange != "collective":
            on_nccl = torch.device(dev).type == "cuda" and "nccl" in str(dist.get_backend(group))
            wanted = exchange == "p2p" or os.environ.get("SPECTRA_B200_P2P", "1") != "0"
            if exchange == "p2p" and not on_nccl:
                raise ValueError("the peer-memory exchange needs an NCCL group on CUDA devices")
            self.use_p2p = on_nccl and wanted

    def _exchange(self, key: tuple, M: int, ns: int, N: int, dtype: torch.dtype):
        """The peer-memory exchange of one gathered shape, set up on first use
        (collectively); None (on every rank alike) when setup failed and
        exchange is "auto", in which case the group's all-gather is used."""
        if key not in self._exchanges:
            from .p2p import PeerExchange
            try:
                self._exchanges[key] = PeerExchange(M, ns, N, dtype, self.device, self.group, self.wait_limit_s)
            except RuntimeError:
                self._exchanges[key] = None
        return self._exchanges[key]

    def _local_buffer(self, M: int, dtype: torch.dtype) -> torch.Tensor:
        """Persistent [M, Ns] slice buffer (the exchange's source when the
        peer-memory exchange is on): zero-filled once, so the rows past the
        layer's end (ragged last shard) stay zero without a kernel per call."""
        if self.use_p2p:
            ex = self._exchange(("y", M, dtype), M, self.ns, self.N, dtype)
            if ex is not None:
                return ex.src
        key = (M, dtype)
        buf = self._local_bufs.get(key)
        if buf is None:
            buf = torch.zeros(M, self.ns, dtype=dtype, device=self.device)
            self._local_bufs[key] = buf
        return buf

    def close(self) -> None:
        """Releases the exchange buffers (collective: every rank calls it)."""
        for ex in self._exchanges.values():
            if ex is not None:
                ex.close()
        self._exchanges = {}

    def local(self, x2d: torch.Tensor) -> torch.Tensor:
        """[M, Ns] slice of this rank (rows past the layer's end are zero)."""
        M = x2d.shape[0]
        compute = torch.bfloat16 if x2d.dtype == torch.bfloat16 else torch.float16
        buf = self._local_buffer(M, compute)
        if self.rows > 0:
            self.local_fn(x2d, self.packed, self.scales, self.zeros, self.outlier_idx, self.outlier_w,
                          self.bias, self.marlin_layout, buf[:, :self.rows])
        return buf

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        orig_shape = x.shape
        M = x.numel() // self.in_features
        x2d = x.reshape(M, self.in_features)
        y_local = self.local(x2d)
        ex = self._exchanges.get(("y", M, y_local.dtype)) if self.use_p2p else None
        if self.world == 1:
            y = y_local[:, :self.N]
        elif ex is not None:
            y = ex.gather()
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

    def greedy(self, x: torch.Tensor) -> torch.Tensor:
        """Index of the first maximum of each output row [..., N] (int64), from
        this rank's slice and one all-gather of (value, index) pairs."""
        orig_shape = x.shape
        M = x.numel() // self.in_features
        x2d = x.reshape(M, self.in_features)
        y_local = self.local(x2d)
        ex = None
        if self.use_p2p:
            ex = self._exchange(("pair", M), M, 2, 2 * self.world, torch.float64)
        pair = ex.src if ex is not None else torch.empty(M, 2, dtype=torch.float64, device=y_local.device)
        if self.rows > 0:
            val, idx = self.argmax_fn(y_local[:, :self.rows], self.row0)
            torch.stack([val.to(torch.float64), idx.to(torch.float64)], dim=1, out=pair)  # [M, 2], exact
        else:  # an empty shard never wins
            pair[:, 0] = float("-inf")
            pair[:, 1] = float(2 ** 53)
        if self.world == 1:
            return pair[:, 1].to(torch.int64).reshape(orig_shape[:-1])
        if ex is not None:
            g = ex.gather().view(M, self.world, 2).transpose(0, 1)
        else:
            gathered = torch.empty(self.world * M * 2, dtype=torch.float64, device=pair.device)
            dist.all_gather_into_tensor(gathered, pair.reshape(-1), group=self.group)
            g = gathered.view(self.world, M, 2)
        # ranks hold increasing row ranges: the first maximum in rank order is the
        # first maximum of the row (torch.argmax: the first NaN counts as maximum)
        r = torch.argmax(g[:, :, 0], dim=0)
        tok = g[:, :, 1].gather(0, r.view(1, M)).view(M)
        return tok.to(torch.int64).reshape(orig_shape[:-1])
