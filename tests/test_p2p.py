"""The peer-memory all-gather's C entry points on the host: buffer sizing and
the argument checks that run before any CUDA call (no GPU needed; the
pointers are never dereferenced because every call here is rejected)."""
import ctypes

import pytest

from spectra_b200 import _lib as L


def _size(M, ns, elem, world):
    return L.lib().spectra_p2p_buffer_bytes(M, ns, elem, world)


def test_buffer_bytes_layout():
    # the epoch flags [8 ranks][128 CTAs] (int32), then 2 parities x world
    # regions of the slice rounded up to 16 bytes
    sig = L.P2P_SIGNAL_BYTES
    assert sig == 4096
    assert _size(1, 8, 2, 2) == sig + 2 * 2 * 16
    assert _size(1, 9, 2, 2) == sig + 2 * 2 * 32
    assert _size(32, 16032, 2, 8) == sig + 2 * 8 * 32 * 16032 * 2
    assert _size(1, 2, 8, 8) == sig + 2 * 8 * 16
    for bad in [(0, 8, 2, 2), (1, 0, 2, 2), (1, 8, 3, 2), (1, 8, 2, 0), (1, 8, 2, 9)]:
        assert _size(*bad) == -1, bad


def _call(**kw):
    a = dict(src=0x10000, peers=(ctypes.c_void_p * 2)(0x20000, 0x30000), buffer_bytes=_size(1, 64, 2, 2),
             out=0x40000, out_rs=128, M=1, ns=64, N=128, elem=2, state=0x50000, rank=0, world=2,
             wait=10 ** 9)
    a.update(kw)
    return L.lib().spectra_p2p_allgather(a["src"], a["peers"], a["buffer_bytes"], a["out"], a["out_rs"], a["M"],
                                         a["ns"], a["N"], a["elem"], a["state"], a["rank"], a["world"], a["wait"],
                                         None)


@pytest.mark.parametrize("kw,code", [
    (dict(src=None), L.ERR_NULL_POINTER),
    (dict(peers=None), L.ERR_NULL_POINTER),
    (dict(out=None), L.ERR_NULL_POINTER),
    (dict(state=None), L.ERR_NULL_POINTER),
    (dict(peers=(ctypes.c_void_p * 2)(0x20000, None)), L.ERR_NULL_POINTER),
    (dict(rank=2), L.ERR_SHAPE),
    (dict(world=9), L.ERR_SHAPE),
    (dict(N=129), L.ERR_SHAPE),          # more columns than world * ns
    (dict(M=0), L.ERR_SHAPE),
    (dict(wait=0), L.ERR_SHAPE),
    (dict(elem=3), L.ERR_DTYPE),
    (dict(buffer_bytes=_size(1, 64, 2, 2) - 16), L.ERR_WORKSPACE),
    (dict(out_rs=100), L.ERR_STRIDE),
    (dict(src=0x10008), L.ERR_ALIGNMENT),
    (dict(peers=(ctypes.c_void_p * 2)(0x20000, 0x30008)), L.ERR_ALIGNMENT),
    (dict(out=0x40001), L.ERR_ALIGNMENT),
])
def test_allgather_rejects_bad_arguments_on_host(kw, code):
    assert _call(**kw) == code


def test_ipc_entry_points_reject_null_pointers():
    lib = L.lib()
    h = ctypes.create_string_buffer(64)
    p = ctypes.c_void_p()
    assert lib.spectra_p2p_alloc(1024, None, h) == L.ERR_NULL_POINTER
    assert lib.spectra_p2p_alloc(1024, ctypes.byref(p), None) == L.ERR_NULL_POINTER
    assert lib.spectra_p2p_alloc(0, ctypes.byref(p), h) == L.ERR_SHAPE
    assert lib.spectra_p2p_open(None, ctypes.byref(p)) == L.ERR_NULL_POINTER
    assert lib.spectra_p2p_close(None) == L.ERR_NULL_POINTER
    assert lib.spectra_p2p_free(None) == L.ERR_NULL_POINTER
