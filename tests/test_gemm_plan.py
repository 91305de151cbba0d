"""Host-side plan of the tcgen05 GEMM (spectra_gemm_plan, no GPU): which calls
run on SM pairs (token tiles of >= 128, cta_group::2, opt-in with
SPECTRA_B200_GEMM_PAIR=1, read once per process: checked in a child process)
and the invariants the kernel relies on -- a pair MMA's N (the token tile) a
multiple of 32, an even CTA count per chunk (tiles padded to pairs), all CTAs
in one wave of 148 SMs, splits no more than 256-k code stages, the workspace
the ABI reports."""
import ctypes
import os
import subprocess
import sys
from pathlib import Path

import pytest

from spectra_b200 import _lib as L

ROOT = Path(__file__).resolve().parents[1]

SMS = 148


def plan(M, N, K, n_out=0):
    out = (ctypes.c_int64 * 8)()
    assert L.lib().spectra_gemm_plan(M, N, K, n_out, out) == 0
    keys = ("MT", "chunks", "tiles", "S", "pair", "ctas", "act_stages", "workspace")
    return dict(zip(keys, list(out)))


SHAPES = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (640, 1024), (896, 4096), (128256, 4096),
          (28672, 8192), (8192, 28672)]


def check_pair_plan(M, N, K):
    p = plan(M, N, K, 41)
    assert p["pair"] == 1
    assert p["MT"] % 32 == 0 and 128 <= p["MT"] <= 256
    assert p["chunks"] == -(-M // 256)
    if p["chunks"] == 1:
        assert p["MT"] >= M and p["MT"] - M < 32
    tiles_pad = p["tiles"] + (p["tiles"] & 1)
    assert p["ctas"] == tiles_pad * p["S"] and p["ctas"] % 2 == 0
    assert 1 <= p["S"] <= -(-K // 256)
    if tiles_pad * p["chunks"] <= SMS:
        assert p["ctas"] * p["chunks"] <= SMS  # one wave
    assert p["act_stages"] >= 3
    ws = L.lib().spectra_w4a16_gemm_workspace_bytes(M, N, K, 41)
    assert ws == p["workspace"]
    if p["S"] > 1:
        assert ws >= p["S"] * M * N * 4


def test_pair_plan():
    code = ("import sys; sys.path.insert(0, sys.argv[1]); from tests.test_gemm_plan import SHAPES, check_pair_plan\n"
            "for M in (128, 130, 160, 200, 256, 300, 512, 1024):\n"
            "    for N, K in SHAPES:\n"
            "        check_pair_plan(M, N, K)\n")
    env = dict(os.environ, SPECTRA_B200_GEMM_PAIR="1")
    r = subprocess.run([sys.executable, "-c", code, str(ROOT)], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]


@pytest.mark.skipif(os.environ.get("SPECTRA_B200_GEMM_PAIR") == "1", reason="pair mode switched on")
@pytest.mark.parametrize("M", [128, 256, 1024])
def test_pairs_are_opt_in(M):
    assert plan(M, 4096, 4096)["pair"] == 0


@pytest.mark.parametrize("M", [2, 16, 17, 64, 100, 112])
def test_small_tiles_stay_on_one_sm(M):
    p = plan(M, 4096, 4096)
    assert p["pair"] == 0
    assert p["ctas"] == p["tiles"] * p["S"]
    assert p["MT"] % 16 == 0


def test_plan_rejects_bad_arguments():
    out = (ctypes.c_int64 * 8)()
    assert L.lib().spectra_gemm_plan(0, 4096, 4096, 0, out) != 0
    assert L.lib().spectra_gemm_plan(256, 4096, 4096, 0, None) != 0


@pytest.mark.parametrize("M", [16, 17, 32, 64, 112, 128, 256, 1024])
@pytest.mark.parametrize("n_out", [0, 41, 512])
def test_outlier_gather_workspace(M, n_out):
    """Token tiles of >= 32 with outlier columns: the workspace also holds the
    activations at the outlier columns, gathered once per call ([M, 64 per
    outlier step] 16-bit values after the split-K region and never over the
    1 KB counter region other calls rely on being zero); other calls keep the
    split-K-only size (none when K is not split)."""
    N, K = 4096, 8192
    p = plan(M, N, K, n_out)
    n_os = -(-n_out // 64)
    gathered = M * n_os * 64 * 2
    split = (1024 + p["S"] * M * N * 4) if p["S"] > 1 else 0  # counters (fixed 1 KB), partials
    if n_out and p["MT"] >= 32:
        assert p["workspace"] >= -(-max(split, 1024) // 256) * 256 + gathered  # never over the counters
    else:
        assert p["workspace"] == split
