"""GPU parity of the tcgen05 GEMM's SM-pair mode: token tiles of >= 128 run on
two-CTA clusters (cta_group::2), each CTA loading half of the tokens and the
even one issuing M = 256 MMAs over both SMs' TMEM (opt-in:
SPECTRA_B200_GEMM_PAIR=1, read once per process, so the pair calls run in a
child process).  The pair MMA sums the same products in the same K order as the
single-SM MMA, so the pair calls must give the same bits as the default ones;
both are also held to the tcgen05 GEMM's oracle bar (1e-2*||c||_inf of the operand-rounded exact result, one
output ulp of its rounding).  Cases cover ragged token tiles (MT = 160),
odd tile counts (a rowless pad CTA), split-K, several token chunks, both
nibble orders, bf16 and fp16, outlier columns."""
import ctypes
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import w4a16 as O
from spectra_b200 import _lib as L
from spectra_b200 import kernels as SK
from tests.helpers import act, assert_close_to_oracle, compressed, np_of, out_f64, random_format

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

# (M, N, K, n_out, a dtype, marlin, compressor output)
CASES = [
    (128, 1024, 2048, 0, "bf16", True, False),     # one pair tile width, no outliers
    (130, 640, 1024, 7, "bf16", True, False),      # MT = 160 (80 tokens per CTA), 5 tiles: a pad CTA
    (256, 896, 4096, 41, "bf16", True, False),     # 7 tiles, split-K 16, pad CTA
    (200, 4096, 1024, 13, "f16", False, False),    # even-odd nibbles, fp16, split-K 4
    (300, 512, 2048, 20, "bf16", True, False),     # two token chunks
    (512, 1408, 1024, 0, "f16", True, False),      # two full chunks, 11 tiles
    (256, 2048, 2048, 0, "bf16", True, True),      # compressor output (its outlier columns)
    (256, 14336, 4096, 41, "bf16", True, False),   # Llama-3-8B gate/up at M = 256
]


def _case_inputs(M, N, K, n_out, dt, marlin, real, seed):
    fmt = compressed(N, K, seed) if real else random_format(N, K, n_out, seed)
    a = act(M, K, seed + 1, dt)
    return fmt, a


def _plan(M, N, K, n_out):
    out = (ctypes.c_int64 * 8)()
    assert L.lib().spectra_gemm_plan(M, N, K, n_out, out) == 0
    return list(out)


def _run(fmt, a, marlin):
    t = lambda v: torch.from_numpy(np.ascontiguousarray(v)).cuda()  # noqa: E731
    has = fmt["outlier_idx"].size > 0
    c = SK.batched_w4a16_gemm(a.cuda(), t(fmt["packed"]), t(fmt["scales"]), t(fmt["zeros"]),
                              outlier_idx=t(fmt["outlier_idx"]) if has else None,
                              outlier_w=fmt["outlier_w_t"].cuda() if has else None, marlin_layout=marlin)
    torch.cuda.synchronize()
    return c


CHILD = r"""
import ctypes, sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from spectra_b200 import _lib as L
from spectra_b200 import kernels as SK
d = np.load(sys.argv[2])
n = int(d["n"])
outs = {}
for i in range(n):
    pl = (ctypes.c_int64 * 8)()
    assert L.lib().spectra_gemm_plan(int(d[f"M{i}"]), int(d[f"N{i}"]), int(d[f"K{i}"]), int(d[f"nout{i}"]), pl) == 0
    assert pl[4] == 1, list(pl)  # the pair mode takes the call
    g = lambda k: torch.from_numpy(np.ascontiguousarray(d[f"{k}{i}"])).cuda()
    a = g("a")
    a = a.view(torch.bfloat16) if int(d[f"bf{i}"]) else a.view(torch.float16)
    has = int(d[f"has{i}"])
    ow = g("ow")
    ow = ow if int(d[f"owdt{i}"]) == 0 else ow.view(torch.float16 if int(d[f"owdt{i}"]) == 1 else torch.bfloat16)
    c = SK.batched_w4a16_gemm(a, g("p"), g("s"), g("z"), outlier_idx=g("idx") if has else None,
                              outlier_w=ow if has else None, marlin_layout=bool(int(d[f"marlin{i}"])))
    torch.cuda.synchronize()
    outs[f"c{i}"] = c.view(torch.int16).cpu().numpy()
np.savez(sys.argv[3], **outs)
"""


@pytest.fixture(scope="module")
def pair_outputs(tmp_path_factory):
    """The same calls with the pair mode on, in a child process."""
    tmp = tmp_path_factory.mktemp("pair")
    arrs = {"n": np.int64(len(CASES))}
    for i, (M, N, K, n_out, dt, marlin, real) in enumerate(CASES):
        fmt, a = _case_inputs(M, N, K, n_out, dt, marlin, real, seed=100 + i)
        arrs[f"a{i}"] = a.view(torch.int16).numpy()
        arrs[f"bf{i}"] = np.int64(a.dtype == torch.bfloat16)
        arrs[f"p{i}"], arrs[f"s{i}"], arrs[f"z{i}"] = fmt["packed"], fmt["scales"], fmt["zeros"]
        arrs[f"has{i}"] = np.int64(fmt["outlier_idx"].size > 0)
        arrs[f"idx{i}"] = fmt["outlier_idx"]
        ow_t = fmt["outlier_w_t"]
        arrs[f"owdt{i}"] = np.int64({torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[ow_t.dtype])
        arrs[f"ow{i}"] = ow_t.numpy() if ow_t.dtype == torch.float32 else ow_t.view(torch.int16).numpy()
        arrs[f"marlin{i}"] = np.int64(marlin)
        arrs[f"M{i}"], arrs[f"N{i}"], arrs[f"K{i}"] = np.int64(M), np.int64(N), np.int64(K)
        arrs[f"nout{i}"] = np.int64(fmt["outlier_idx"].size)
    src, dst = tmp / "in.npz", tmp / "out.npz"
    np.savez(src, **arrs)
    env = dict(os.environ, SPECTRA_B200_GEMM_PAIR="1")
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), str(src), str(dst)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-4000:]
    return np.load(dst)


def test_pair_capacity_covers_the_plan():
    n = ctypes.c_int(0)
    assert L.lib().spectra_gemm_pair_capacity(ctypes.byref(n)) == 0
    # the plan puts up to 148 CTAs (74 pairs) in one wave
    assert n.value >= 64, n.value
    print(f"two-CTA clusters resident at once: {n.value}")


@pytest.mark.parametrize("i", range(len(CASES)))
def test_pair_gemm(i, pair_outputs):
    M, N, K, n_out, dt, marlin, real = CASES[i]
    fmt, a = _case_inputs(M, N, K, n_out, dt, marlin, real, seed=100 + i)
    c = _run(fmt, a, marlin)  # the default (one-SM) kernel, here
    # the pair kernel's result bit for bit
    ref = pair_outputs[f"c{i}"]
    got = c.view(torch.int16).cpu().numpy()
    assert got.shape == ref.shape
    assert np.array_equal(got, ref), f"case {i}: {int(np.sum(got != ref))} of {got.size} outputs differ"
    # and within the oracle bar
    an, ad = np_of(a)
    ow, owd = np_of(fmt["outlier_w_t"])
    has = fmt["outlier_idx"].size > 0
    if M * N * K > 2 ** 31:  # the largest case: a row sample keeps the CPU oracle quick
        rows = np.random.default_rng(i).choice(N, size=512, replace=False)
        fmt_s = {k: (v[rows] if k in ("packed", "scales", "zeros") else v) for k, v in fmt.items()}
        ow = ow[rows] if has else ow
        c_exact, c_round, cd = O.gemm(an, ad, fmt_s["packed"], fmt_s["scales"], fmt_s["zeros"],
                                      outlier_idx=fmt["outlier_idx"] if has else None,
                                      outlier_w=ow if has else None, ow_dtype=owd, marlin=marlin)
        got64 = out_f64(c)[:, rows]
    else:
        c_exact, c_round, cd = O.gemm(an, ad, fmt["packed"], fmt["scales"], fmt["zeros"],
                                      outlier_idx=fmt["outlier_idx"] if has else None,
                                      outlier_w=ow if has else None, ow_dtype=owd, marlin=marlin)
        got64 = out_f64(c)
    assert_close_to_oracle(got64.reshape(c_exact.shape), c_exact, c_round, cd, f"pair case {i}")


GRAPH_CHILD = r"""
import ctypes, sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from spectra_b200 import _lib as L
from tests.test_gemm_pair_gpu import graph_replay_check
graph_replay_check()
"""


def test_pair_gemm_graph_replay_and_no_timeouts():
    """Pair-mode calls captured in a CUDA graph and replayed give the eager
    result, and no pipeline wait gave up (child process, pair mode on)."""
    env = dict(os.environ, SPECTRA_B200_GEMM_PAIR="1")
    r = subprocess.run([sys.executable, "-c", GRAPH_CHILD, str(ROOT)], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-4000:]


def graph_replay_check():
    M, N, K = 256, 1024, 2048
    assert _plan(M, N, K, 9)[4] == 1
    fmt = random_format(N, K, 9, seed=7)
    a = act(M, K, 8, "bf16").cuda()
    t = lambda v: torch.from_numpy(np.ascontiguousarray(v)).cuda()  # noqa: E731
    p, s, z, idx, ow = t(fmt["packed"]), t(fmt["scales"]), t(fmt["zeros"]), t(fmt["outlier_idx"]), \
        fmt["outlier_w_t"].cuda()
    eager = SK.batched_w4a16_gemm(a, p, s, z, outlier_idx=idx, outlier_w=ow)
    out = torch.empty_like(eager)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        for _ in range(2):
            out.copy_(SK.batched_w4a16_gemm(a, p, s, z, outlier_idx=idx, outlier_w=ow))
    torch.cuda.current_stream().wait_stream(st)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out.copy_(SK.batched_w4a16_gemm(a, p, s, z, outlier_idx=idx, outlier_w=ow))
    out.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    c = ctypes.c_longlong(-1)
    assert L.lib().spectra_device_timeouts(ctypes.byref(c), 0) == 0
    assert c.value == 0
    del g
