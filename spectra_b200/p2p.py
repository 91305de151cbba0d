"""NVLink peer-memory all-gather (the C entry points spectra_p2p_*), the
exchange step of the sharded layers in spectra_b200.sharded.

Each ``PeerExchange`` serves one gathered shape: every rank's slice is
[M, ns] elements, the gathered output [M, N] with rank r's columns starting
at r*ns.  Setup is collective over the process group: every rank allocates
its exchange buffer (cudaMalloc, zeroed), the 64-byte CUDA IPC handles are
all-gathered over the group, and every rank opens its peers' buffers.  A
rank on which any step fails makes every rank give up (the outcome is agreed
over the group), so callers fall back to the process group's all-gather
together.

``gather()`` launches one kernel: it pushes this rank's slice (``src``, which
the caller fills first) into every peer's buffer with stores over NVLink,
exchanges an epoch flag with every peer and copies the gathered [M, N]
output.  Every rank must call it the same number of times in the same order;
calls may be captured in and replayed from a CUDA graph.  The device-side
wait for a peer is bounded (``wait_limit_s``): a wait that runs out is
counted by ``spectra_b200.kernels.device_timeouts()`` and leaves that call's
output undefined.

The reference has no multi-GPU path; this is the collective of its large
layers column-sharded over the GPUs of one NVSwitch node.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import torch
import torch.distributed as dist

from ._lib import P2P_STATE_INTS, check, lib

HANDLE_BYTES = 64  # sizeof(cudaIpcMemHandle_t)


def _elem_bytes(dtype: torch.dtype) -> int:
    return torch.empty(0, dtype=dtype).element_size()


class PeerExchange:
    """Peer-memory all-gather of [M, ns] slices into [M, N] over ``group``."""

    def __init__(self, M: int, ns: int, N: int, dtype: torch.dtype, device: torch.device,
                 group: Optional[dist.ProcessGroup] = None, wait_limit_s: float = 5.0):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.M, self.ns, self.N, self.dtype, self.device = M, ns, N, dtype, torch.device(device)
        self.wait_limit_ns = int(wait_limit_s * 1e9)
        self.group = group
        L = lib()
        elem = _elem_bytes(dtype)
        self.buffer_bytes = int(L.spectra_p2p_buffer_bytes(M, ns, elem, self.world))
        if self.buffer_bytes < 0:
            raise ValueError(f"unsupported exchange shape M={M} ns={ns} {dtype} over {self.world} ranks")
        self._own: Optional[int] = None
        self._opened: List[int] = []
        handle = ctypes.create_string_buffer(HANDLE_BYTES)
        ok = True
        with torch.cuda.device(self.device):
            ptr = ctypes.c_void_p()
            ok = L.spectra_p2p_alloc(self.buffer_bytes, ctypes.byref(ptr), handle) == 0
            if ok:
                self._own = ptr.value
            handles: List[Optional[bytes]] = [None] * self.world
            dist.all_gather_object(handles, handle.raw if ok else None, group=group)
            peers: List[int] = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    peers.append(self._own or 0)
                    continue
                p = ctypes.c_void_p()
                if ok and h is not None and L.spectra_p2p_open(h, ctypes.byref(p)) == 0:
                    self._opened.append(p.value)
                    peers.append(p.value)
                else:
                    ok = False
                    peers.append(0)
            agreed: List[Optional[bool]] = [None] * self.world
            dist.all_gather_object(agreed, ok, group=group)
        if not all(agreed):
            self.close(barrier=False)
            raise RuntimeError("peer-memory exchange unavailable on this group")
        self._peers = (ctypes.c_void_p * self.world)(*peers)
        self.state = torch.zeros(P2P_STATE_INTS, dtype=torch.int32, device=self.device)
        pitch = -(-M * ns * elem // 16) * 16
        self._src_store = torch.zeros(pitch // elem, dtype=dtype, device=self.device)
        self.src = self._src_store[:M * ns].view(M, ns)  # this rank's slice, written by the caller

    def gather(self, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """[M, N]: every rank's ``src`` side by side (rank r at columns r*ns)."""
        if out is None:
            out = torch.empty(self.M, self.N, dtype=self.dtype, device=self.device)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check("spectra_p2p_allgather", lib().spectra_p2p_allgather(
            self.src.data_ptr(), self._peers, self.buffer_bytes, out.data_ptr(), out.stride(0),
            self.M, self.ns, self.N, _elem_bytes(self.dtype), self.state.data_ptr(), self.rank, self.world,
            self.wait_limit_ns, stream))
        return out

    def close(self, barrier: bool = True) -> None:
        """Unmaps the peers' buffers and frees this rank's (collective when
        ``barrier``: no peer may still be writing here)."""
        if barrier and self._own is not None:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        L = lib()
        with torch.cuda.device(self.device):
            for p in self._opened:
                L.spectra_p2p_close(p)
            self._opened = []
            if self._own is not None:
                L.spectra_p2p_free(self._own)
                self._own = None
