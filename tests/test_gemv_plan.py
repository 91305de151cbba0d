"""Host logic of the M=1 GEMV dispatcher, without a GPU: which configuration
of the weight-prefetching kernel (spectra_b200/csrc/gemv_pf.cu) each shape
gets, and the invariants the kernel relies on -- an even ring depth with two
compute groups (a group's mbarrier parity wait must never meet a ring slot
whose previous stage belongs to the other group), the shared-memory budgets
that decide residency, and the outlier rows either staged or streamed
through the ring in pieces that fit it."""
import ctypes

import pytest

from spectra_b200 import _lib as L

F16, BF16, F32 = 0, 1, 2
SMS = 148
PAIR_BUDGET, SOLO_BUDGET = 110 * 1024, 200 * 1024
FIELDS = ("taken", "ng", "chunked", "ns", "stage_bytes", "ow_staged", "ow_ring_rows", "smem", "grid", "rb")


def _fn():
    return L.lib().spectra_gemv_pf_plan


def plan(N, K, n_out, x=BF16, ow=F16, sms=SMS):
    out = (ctypes.c_int64 * 10)()
    st = _fn()(N, K, n_out, x, ow, sms, out)
    assert st == 0, st
    return dict(zip(FIELDS, list(out)))


@pytest.mark.parametrize("K,N,n_out,want", [
    # Llama-3.2-1B decoder layer (the bench): one group, whole-row-block stages
    # that hold all of a CTA's rows (copied before the wait), outliers staged.
    (2048, 8192, 21, dict(ng=1, chunked=0, ow_staged=1, rb=4, ns=4)),
    (2048, 512, 21, dict(ng=1, chunked=0, ow_staged=1, rb=1)),
    (2048, 2048, 21, dict(ng=1, chunked=0, ow_staged=1, rb=1)),
    (8192, 2048, 82, dict(ng=1, chunked=0, rb=1, ns=1)),
    # Llama-3-8B / 70B shapes: two groups.
    (4096, 14336, 41, dict(ng=2, chunked=0, rb=7)),
    (14336, 4096, 143, dict(ng=2, chunked=1, rb=2)),
    (8192, 28672, 81, dict(ng=2, chunked=1, rb=13)),
    (8192, 8192, 171, dict(ng=1, chunked=0, rb=4)),
    # one row block per CTA (70B down_proj split 4 ways): the two-per-SM
    # footprint cannot hold two chunk stages next to the staged x
    (28672, 2048, 286, dict(ng=2, chunked=1, rb=1)),
    # outlier rows too large to stage beside a useful ring: streamed
    (28672, 8192, 512, dict(ng=2, chunked=1, ow_staged=0)),
    (8192, 128256, 81, dict(ng=2, chunked=1, ow_staged=0, rb=55)),
])
def test_known_shapes(K, N, n_out, want):
    p = plan(N, K, n_out)
    assert p["taken"] == 1
    for k, v in want.items():
        assert p[k] == v, (k, p)
    if p["ow_staged"] == 0 and n_out > 0 and p["ng"] == 2:
        assert p["ow_ring_rows"] > 0, p


def test_streamed_outliers_keep_a_deep_ring():
    # staging 64 rows x 512 outlier columns would leave 2 stages
    p = plan(8192, 28672, 512)
    assert p["ns"] >= 4 and p["ow_ring_rows"] > 0


@pytest.mark.parametrize("K", [512, 1024, 2048, 3072, 3584, 4096, 5120, 8192, 10240, 14336, 28672])
@pytest.mark.parametrize("N", [1, 16, 100, 2368, 4745, 11849, 28672, 128256])
@pytest.mark.parametrize("n_out,ow", [(0, F16), (9, F16), (-1, F16), (-1, F32), (600, F32)])
def test_plan_invariants(K, N, n_out, ow):
    if n_out < 0:
        n_out = K // 100
    n_out = min(n_out, K)
    p = plan(N, K, n_out, ow=ow)
    if not p["taken"]:
        # e.g. K = 57344 with 55 row blocks per CTA: the staged x (143 KB) and
        # the row partials leave one chunk stage; the register-prefetch kernel runs
        assert all(v == 0 for v in p.values())
        return
    nblk = (N + 15) // 16
    assert p["grid"] == min(nblk, SMS)
    assert p["rb"] == -(-nblk // p["grid"])
    stages_per_rb = -(-K // 2048) if p["chunked"] else 1
    units = p["rb"] * stages_per_rb
    assert 1 <= p["ns"] <= 8
    assert p["ns"] >= min(2, units)
    assert p["ns"] * p["stage_bytes"] < p["smem"] <= SOLO_BUDGET
    if p["rb"] > 1:
        assert p["smem"] > PAIR_BUDGET  # several row blocks: the CTA owns its SM
    if p["ng"] == 2:
        assert p["ns"] % 2 == 0
        assert p["smem"] > PAIR_BUDGET  # two groups only on CTAs that own their SM
    if p["rb"] == 1 and p["smem"] <= PAIR_BUDGET:
        assert p["ng"] == 1
    row_bytes = n_out * (4 if ow == F32 else 2)
    if p["ow_ring_rows"]:
        assert p["ng"] == 2 and p["ow_staged"] == 0 and n_out > 0
        # pieces of whole 64-row passes, or one piece holding every row
        assert p["ow_ring_rows"] % 64 == 0 or p["ow_ring_rows"] == p["rb"] * 16
        assert p["ow_ring_rows"] <= p["rb"] * 16
        assert p["ow_ring_rows"] * row_bytes + 16 <= p["ns"] * p["stage_bytes"]
    if n_out == 0:
        assert p["ow_staged"] == 0 and p["ow_ring_rows"] == 0


@pytest.mark.parametrize("K,x", [(1056, BF16), (2080, BF16), (4096, F32), (96, F16)])
def test_other_layouts_go_to_the_other_kernel(K, x):
    # K not a multiple of 512, or fp32 activations: the register-prefetch kernel
    assert plan(4096, K, 0, x=x)["taken"] == 0


def test_bad_arguments():
    f = _fn()
    out = (ctypes.c_int64 * 10)()
    assert f(0, 2048, 0, BF16, F16, SMS, out) == 2      # SPECTRA_ERR_SHAPE
    assert f(16, 2000, 0, BF16, F16, SMS, out) == 2     # K not a multiple of 32
    assert f(16, 2048, 4096, BF16, F16, SMS, out) == 2  # more outlier columns than features
    assert f(16, 2048, 0, BF16, F16, SMS, None) == 1    # SPECTRA_ERR_NULL_POINTER


@pytest.mark.parametrize("ow_dtype", [3, 4, 9, -1])  # I32, I64, unknown codes
def test_unknown_outlier_weight_dtype_is_rejected_like_the_gemv(ow_dtype):
    # spectra_w4a16_gemv rejects these with SPECTRA_ERR_DTYPE, so the diagnostic must too
    f = _fn()
    out = (ctypes.c_int64 * 10)()
    assert f(4096, 4096, 41, BF16, ow_dtype, SMS, out) == 5  # SPECTRA_ERR_DTYPE
    assert f(4096, 4096, 41, 7, F16, SMS, out) == 5          # unknown x dtype
    # without outlier columns the outlier dtype is not looked at (as in the GEMV)
    assert f(4096, 4096, 0, BF16, ow_dtype, SMS, out) == 0
