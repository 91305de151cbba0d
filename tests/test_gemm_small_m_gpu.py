"""The small-M GEMM kernel (M = 2..16, gemv_mt.cu) behind batched_w4a16_gemm:
parity with the exact-weights oracle (1 output ulp of the correctly rounded
exact result, floor 2^-16*||c||_inf) and with the reference GEMM's operand
rounding (1e-2*||c||_inf), over token counts, Llama shapes, both nibble orders,
fp16/bf16 activations, outlier dtypes and index widths, ragged N, K that is
not a multiple of the 2048-feature stage, strided activations; plus
determinism, CUDA-graph replay and agreement with the tcgen05 GEMM on the same
rows."""
import numpy as np
import pytest
import torch

from spectra_b200 import kernels as SK
from tests.helpers import (act, assert_close_to_oracle, compressed, gemm_exact_weights, np_of, out_f64,
                           random_format, small_m_path)
from oracle import w4a16 as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _run(fmt, a, marlin=True, idx_dtype=torch.int64, use_out=True):
    p, s, z = _t(fmt["packed"]), _t(fmt["scales"]), _t(fmt["zeros"])
    has = use_out and fmt["outlier_idx"].size
    idx = _t(fmt["outlier_idx"]).to(idx_dtype) if has else None
    ow = fmt["outlier_w_t"].to(DEV) if has else None
    c = SK.batched_w4a16_gemm(a.to(DEV), p, s, z, outlier_idx=idx, outlier_w=ow, marlin_layout=marlin)
    torch.cuda.synchronize()
    return c


def _check(fmt, a, c, marlin=True, use_out=True, what=""):
    an, ad = np_of(a.reshape(-1, a.shape[-1]))
    ow, owd = np_of(fmt["outlier_w_t"])
    has = use_out and fmt["outlier_idx"].size
    kw = dict(outlier_idx=fmt["outlier_idx"] if has else None, outlier_w=ow if has else None, ow_dtype=owd,
              marlin=marlin)
    got = out_f64(c).reshape(a.shape[0], -1)
    assert np.isfinite(got).all(), what
    c_exact, c_round, cd = gemm_exact_weights(an, ad, fmt["packed"], fmt["scales"], fmt["zeros"], **kw)
    assert_close_to_oracle(got, c_exact, c_round, cd, what)
    r_exact, _, _ = O.gemm(an, ad, fmt["packed"], fmt["scales"], fmt["zeros"], **kw)
    assert np.max(np.abs(got - r_exact)) <= 1e-2 * np.max(np.abs(r_exact)), what


def _shape_of(fmt):
    return fmt["packed"].shape[0], fmt["packed"].shape[1] * 2


@pytest.mark.parametrize("M", [2, 3, 4, 5, 6, 7, 8, 9, 12, 15, 16])
@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_token_counts(M, dt):
    fmt = random_format(1000, 2048, 21, seed=M, ow_dtype=dt)
    N, K = _shape_of(fmt)
    assert small_m_path(M, N, K, 21, dt, dt)
    a = act(M, K, seed=M + 100, dtype=dt)
    _check(fmt, a, _run(fmt, a), what=f"M={M} {dt}")


@pytest.mark.parametrize("K,N,M", [(4096, 4096, 8), (4096, 1024, 4), (4096, 14336, 8), (14336, 4096, 2),
                                   (14336, 4096, 4), (8192, 8192, 8), (4096, 4096, 16), (4096, 1024, 13)])
def test_llama_shapes(K, N, M):
    fmt = random_format(N, K, K // 100, seed=K + N + M, ow_dtype="bf16")
    n_out = int(fmt["outlier_idx"].size)
    assert small_m_path(M, N, K, n_out, "bf16", np_of(fmt["outlier_w_t"])[1])
    a = act(M, K, seed=K - M, dtype="bf16")
    c = _run(fmt, a)
    # the oracle on a sample of rows (the first and last row blocks and random rows)
    rng = np.random.default_rng(K ^ N)
    rows = np.unique(np.concatenate([np.arange(16), np.arange(N - 16, N), rng.choice(N, 96, replace=False)]))
    sub = {"packed": fmt["packed"][rows], "scales": fmt["scales"][rows], "zeros": fmt["zeros"][rows],
           "outlier_idx": fmt["outlier_idx"], "outlier_w_t": fmt["outlier_w_t"][torch.from_numpy(rows)]}
    _check(sub, a, c[:, torch.from_numpy(rows).to(DEV)], what=f"{K}x{N} M={M}")


@pytest.mark.parametrize("N,K", [(4099, 1024), (17, 512), (300, 1536), (1000, 2560), (129, 6144)])
@pytest.mark.parametrize("marlin", [True, False])
def test_ragged_shapes_and_layouts(N, K, marlin):
    fmt = random_format(N, K, min(9, K // 64), seed=N + K, ow_dtype="bf16")
    for M in (5, 11):
        assert small_m_path(M, N, K, min(9, K // 64))
        a = act(M, K, seed=N + M, dtype="bf16")
        _check(fmt, a, _run(fmt, a, marlin=marlin), marlin=marlin, what=f"N={N} K={K} M={M} marlin={marlin}")


@pytest.mark.parametrize("ow_dtype", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("idx_dtype", [torch.int32, torch.int64])
def test_outlier_dtypes(ow_dtype, idx_dtype):
    fmt = random_format(512, 1024, 30, seed=7, ow_dtype=ow_dtype)
    a = act(6, 1024, seed=7, dtype="bf16")
    _check(fmt, a, _run(fmt, a, idx_dtype=idx_dtype), what=f"{ow_dtype} {idx_dtype}")


def test_no_outliers():
    fmt = random_format(512, 1024, 0, seed=8, ow_dtype="bf16")
    a = act(3, 1024, seed=8, dtype="f16")
    _check(fmt, a, _run(fmt, a), what="n_out=0")


def test_compressor_output():
    fmt = compressed(512, 2048, seed=21, dist="t3")
    a = act(7, 2048, seed=21, dtype="bf16")
    _check(fmt, a, _run(fmt, a), what="compressed t3")


def test_strided_activations_and_deterministic():
    fmt = random_format(768, 2048, 12, seed=9, ow_dtype="bf16")
    a = act(4, 2048, seed=9, dtype="bf16")
    base = _run(fmt, a)
    wide = torch.zeros(4, 2048 + 64, dtype=torch.bfloat16)
    wide[:, :2048] = a
    assert torch.equal(_run(fmt, wide[:, :2048]), base)  # row pitch 2112 elements
    for _ in range(3):
        assert torch.equal(_run(fmt, a), base)


def test_agrees_with_the_tcgen05_gemm():
    """Rows computed at M = 4 (small-M kernel) and inside M = 20 (tcgen05 GEMM)."""
    fmt = random_format(1024, 4096, 41, seed=10, ow_dtype="bf16")
    a = act(20, 4096, seed=10, dtype="bf16")
    small = _run(fmt, a[:4])
    big = _run(fmt, a)[:4]
    ref = np.abs(out_f64(big)).max()
    assert np.max(np.abs(out_f64(small) - out_f64(big))) <= 1e-2 * ref


def test_graph_replay():
    fmt = random_format(2048, 4096, 41, seed=11, ow_dtype="bf16")
    p, s, z = _t(fmt["packed"]), _t(fmt["scales"]), _t(fmt["zeros"])
    idx, ow = _t(fmt["outlier_idx"]), fmt["outlier_w_t"].to(DEV)
    a = act(8, 4096, seed=11, dtype="bf16").to(DEV)
    SK.batched_w4a16_gemm(a, p, s, z, outlier_idx=idx, outlier_w=ow, marlin_layout=True)
    torch.cuda.synchronize()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        c = SK.batched_w4a16_gemm(a, p, s, z, outlier_idx=idx, outlier_w=ow, marlin_layout=True)
    for seed in (12, 13):
        a.copy_(act(8, 4096, seed=seed, dtype="bf16").to(DEV))
        g.replay()
        torch.cuda.synchronize()
        eager = SK.batched_w4a16_gemm(a, p, s, z, outlier_idx=idx, outlier_w=ow, marlin_layout=True)
        assert torch.equal(c, eager)
    assert SK.device_timeouts() == 0
