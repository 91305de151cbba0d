"""Host-side plan of the small-M GEMM kernel (spectra_gemm_small_m_plan, no
GPU): which calls it takes and the invariants of its configuration."""
import ctypes

import numpy as np
import pytest

from spectra_b200 import _lib as L


def plan(M, N, K, n_out, a_dt=L.DT_BF16, ow_dt=L.DT_BF16, sms=148):
    out = np.zeros(7, np.int64)
    st = L.lib().spectra_gemm_small_m_plan(M, N, K, n_out, a_dt, ow_dt, sms, out.ctypes.data_as(ctypes.c_void_p))
    return st, out


@pytest.mark.parametrize("M,N,K,n_out,taken", [
    (2, 4096, 4096, 41, True), (8, 14336, 4096, 41, True), (8, 1024, 4096, 41, True),
    (4, 4096, 14336, 143, True), (2, 4096, 14336, 143, True), (8, 8192, 8192, 82, True),
    (8, 4096, 14336, 143, False),   # 8 rows of 14336 activations do not fit beside two stages
    (1, 4096, 4096, 41, False),     # M = 1 is the GEMV's
    (16, 4096, 4096, 41, True),     # two token tiles
    (12, 1024, 4096, 41, True),
    (16, 14336, 4096, 41, False),   # 16 rows of activations and the row partials leave no two stages
    (17, 4096, 4096, 41, False),    # above two token tiles: the tcgen05 GEMM
    (4, 4096, 4000, 40, False),     # K not a multiple of 512
])
def test_which_calls_it_takes(M, N, K, n_out, taken):
    st, out = plan(M, N, K, n_out)
    assert st == L.OK
    assert bool(out[0]) == taken
    if not taken:
        assert not out.any()


def test_plan_invariants_over_shapes():
    for M in range(2, 17):
        for K in (512, 1024, 2048, 2560, 4096, 6144, 8192, 14336, 28672):
            for N in (16, 100, 1024, 4099, 14336, 28672, 128256):
                st, out = plan(M, N, K, min(K // 32, 900))
                assert st == L.OK
                if not out[0]:
                    continue
                grid, smem, ns = int(out[1]), int(out[2]), int(out[3])
                nblk = -(-N // 16)
                assert grid == min(nblk, 148)
                assert smem <= 220 * 1024
                units = -(-nblk // grid) * -(-K // 2048)
                assert 1 <= ns <= 8 and ns >= min(2, units)
                assert out[5] in (1, 2)
                assert out[6] == (2 if M > 8 else 1)
                if out[5] == 2:  # two groups alternate stages: an even ring of >= 4
                    assert ns % 2 == 0 and ns >= 4


def test_plan_rejects_bad_arguments():
    out = np.zeros(7, np.int64)
    lib = L.lib()
    assert lib.spectra_gemm_small_m_plan(2, 64, 512, 0, L.DT_BF16, L.DT_BF16, 148, None) == L.ERR_NULL_POINTER
    assert plan(0, 64, 512, 0)[0] == L.ERR_SHAPE
    assert plan(2, 64, 500, 0)[0] == L.ERR_SHAPE
    assert plan(2, 64, 512, 0, a_dt=L.DT_F32)[0] == L.ERR_DTYPE
    assert plan(2, 64, 512, 4, ow_dt=9)[0] == L.ERR_DTYPE
