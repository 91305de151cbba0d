"""The peer-memory all-gather kernel on one GPU, with the peers' side staged
by the test: the other ranks' buffers are plain device buffers on the same GPU
whose epoch slots and slices are written beforehand, so the kernel never
waits on another launch (kernels that wait on one another never run as
separate launches on one GPU).  Checked bit for bit: the gathered [M, N]
output (this rank's columns from its source, each peer's from the own
buffer's region of the call's parity), the slice pushed into every peer's
buffer, the epoch flag each peer receives, the state carried from call to
call (parity alternates), ragged and empty last shards, every copy granule.
And the bounded wait: a peer that never signals ends the wait after the
limit, counted by spectra_device_timeouts, with the context still usable.
The exchange between real GPUs is covered by tests/test_sharded_gpu.py."""
import ctypes

import pytest
import torch

from spectra_b200 import _lib as L
from spectra_b200 import kernels as SK

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
SIG = L.P2P_SIGNAL_BYTES
MAX_CTAS = L.P2P_STATE_INTS


def _pitch(M, ns, elem):
    return -(-M * ns * elem // 16) * 16


def _ctas(pitch):
    """The exchange kernel's grid: ~2 16-byte units per thread of 256, at most 128."""
    return max(1, min(MAX_CTAS, -(-(pitch // 16) // 512)))


def _random(M, ns, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    bits = torch.randint(0, 256, (M * ns * torch.empty(0, dtype=dtype).element_size(),), generator=g,
                         device=DEV, dtype=torch.uint8)
    return bits.view(dtype).view(M, ns)


class Staged:
    """World buffers on one GPU; `rank` runs the kernel, the others are staged."""

    def __init__(self, M, ns, N, dtype, world, rank):
        self.M, self.ns, self.N, self.dtype, self.world, self.rank = M, ns, N, dtype, world, rank
        self.elem = torch.empty(0, dtype=dtype).element_size()
        self.bytes = L.lib().spectra_p2p_buffer_bytes(M, ns, self.elem, world)
        assert self.bytes == SIG + 2 * world * _pitch(M, ns, self.elem)
        self.bufs = [torch.zeros(self.bytes, dtype=torch.uint8, device=DEV) for _ in range(world)]
        self.peers = (ctypes.c_void_p * world)(*[b.data_ptr() for b in self.bufs])
        self.state = torch.zeros(MAX_CTAS, dtype=torch.int32, device=DEV)
        self.src_store = torch.zeros(_pitch(M, ns, self.elem) // self.elem, dtype=dtype, device=DEV)
        self.G = _ctas(_pitch(M, ns, self.elem))

    def flags(self, owner, r):
        """Epoch flags of rank r's chunks in `owner`'s buffer."""
        return self.bufs[owner][:SIG].view(torch.int32).view(-1, MAX_CTAS)[r, :self.G]

    def region(self, owner, parity, r):
        p = _pitch(self.M, self.ns, self.elem)
        off = SIG + (parity * self.world + r) * p
        return self.bufs[owner][off:off + self.M * self.ns * self.elem]

    def call(self, epoch, slices, signal=True, wait_ns=10 ** 9, out_rs=None):
        """Stages the peers' slices for `epoch`, runs the kernel as `rank`."""
        for r in range(self.world):
            if r == self.rank:
                self.src_store[:self.M * self.ns].copy_(slices[r].reshape(-1))
                continue
            self.region(self.rank, epoch & 1, r).copy_(slices[r].reshape(-1).view(torch.uint8))
            if signal:
                self.flags(self.rank, r).fill_(epoch)
        rs = out_rs or self.N
        out = torch.full((self.M, rs), float("nan"), dtype=self.dtype, device=DEV) if self.dtype.is_floating_point \
            else torch.zeros(self.M, rs, dtype=self.dtype, device=DEV)
        st = L.lib().spectra_p2p_allgather(self.src_store.data_ptr(), self.peers, self.bytes, out.data_ptr(), rs,
                                           self.M, self.ns, self.N, self.elem, self.state.data_ptr(), self.rank,
                                           self.world, wait_ns, torch.cuda.current_stream().cuda_stream)
        assert st == L.OK, L.lib().spectra_status_string(st)
        torch.cuda.synchronize()
        return out


CASES = [  # (M, ns, N, dtype, world, rank)
    (1, 16032, 128256, torch.bfloat16, 8, 3),    # lm_head over 8 ranks: 16-byte granule
    (1, 2050, 4099, torch.bfloat16, 2, 0),       # ragged last shard: 2-byte granule
    (1, 2050, 4099, torch.float16, 2, 1),        # this rank is the ragged one
    (32, 4096, 8192, torch.bfloat16, 2, 1),      # M > 1, row-interleaved output, 32 CTAs
    (32, 16032, 128256, torch.bfloat16, 8, 7),   # 126 CTAs, 8 ranks
    (3, 12, 30, torch.float16, 3, 2),            # 4-byte granule, ragged, M = 3
    (1, 2, 16, torch.float64, 8, 5),             # (value, index) pairs of the sharded greedy head
    (2, 2, 8, torch.float64, 4, 0),
    (1, 6, 10, torch.float32, 4, 1),             # 8-byte granule; this rank ragged, the last two empty
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"M{c[0]}_ns{c[1]}_N{c[2]}_w{c[4]}r{c[5]}")
def test_staged_allgather_is_bit_exact(case):
    M, ns, N, dtype, world, rank = case
    s = Staged(M, ns, N, dtype, world, rank)
    SK.device_timeouts(reset=True)
    for epoch in (1, 2, 3):  # parities 1, 0, 1: state carries over
        slices = [_random(M, ns, dtype, 100 * epoch + r) for r in range(world)]
        out = s.call(epoch, slices)
        want = torch.cat(slices, dim=1)[:, :N]
        assert torch.equal(out.view(torch.uint8), want.contiguous().view(torch.uint8)), f"epoch {epoch}"
        assert s.state.tolist() == [epoch] * s.G + [0] * (MAX_CTAS - s.G)
        mine = slices[rank].reshape(-1).view(torch.uint8)
        for r in range(world):
            if r == rank:
                continue
            assert torch.equal(s.region(r, epoch & 1, rank), mine), f"push to {r}, epoch {epoch}"
            assert (s.flags(r, rank) == epoch).all()
    assert SK.device_timeouts() == 0


def test_output_row_stride():
    s = Staged(4, 24, 48, torch.bfloat16, 2, 0)
    slices = [_random(4, 24, torch.bfloat16, r) for r in range(2)]
    out = s.call(1, slices, out_rs=64)
    assert torch.equal(out[:, :48].contiguous().view(torch.int16),
                       torch.cat(slices, 1).contiguous().view(torch.int16))
    assert torch.isnan(out[:, 48:].float()).all()  # nothing written past N


def test_silent_peer_times_out_and_the_context_survives():
    s = Staged(1, 1024, 2048, torch.bfloat16, 2, 0)
    SK.device_timeouts(reset=True)
    slices = [_random(1, 1024, torch.bfloat16, r) for r in range(2)]
    s.call(1, slices, signal=False, wait_ns=50 * 10 ** 6)  # nothing ever sets the peer's flags
    assert SK.device_timeouts() == s.G  # one per CTA that gave up
    SK.device_timeouts(reset=True)
    # the pushes and this rank's own flags went out before the wait
    assert torch.equal(s.region(1, 1, 0), slices[0].reshape(-1).view(torch.uint8))
    assert (s.flags(1, 0) == 1).all()
    # the device is fine and the next call (epoch 2) completes normally
    slices = [_random(1, 1024, torch.bfloat16, 10 + r) for r in range(2)]
    out = s.call(2, slices)
    assert torch.equal(out.view(torch.int16), torch.cat(slices, 1).view(torch.int16))
    assert SK.device_timeouts() == 0


def test_ipc_buffer_round_trip_on_one_device():
    """alloc -> handle -> free, and the size the sharded layer asks for."""
    lib = L.lib()
    h = ctypes.create_string_buffer(64)
    p = ctypes.c_void_p()
    n = lib.spectra_p2p_buffer_bytes(1, 16032, 2, 8)
    torch.cuda.init()
    assert lib.spectra_p2p_alloc(n, ctypes.byref(p), h) == L.OK and p.value
    assert any(h.raw)
    assert lib.spectra_p2p_free(p) == L.OK
