"""Parity on the BASELINE configuration shapes with real compressor output.

Weights are drawn on the device (N(0, 0.02) for config 3, Student-t with 3
degrees of freedom rescaled to std 0.02 for config 5) and compressed there by
``spectra_b200.compress`` -- the same path the bench uses.  The matrices are
too large for the CPU oracle to take whole in seconds, so every check runs on
a sample of rows (random rows, plus the first and last row blocks, where the
ragged ends of the kernels' tiles lie):

  * the sampled rows' codes, scales and zero points are bit-identical to the
    oracle quantiser (spectra/compressor.py:72-112) applied to the same source
    rows with the selected outlier columns zeroed (:115-156);
  * the kernel outputs of those rows are within the path's bar of the oracle
    GEMV (spectra/kernels.py:16-129) or GEMM (:191-331): 1e-2*||y||_inf and one
    output ulp of the correctly rounded exact value.
"""
import numpy as np
import pytest
import torch

from oracle import w4a16 as O
from spectra_b200 import compress as C
from spectra_b200 import kernels as SK
from tests.helpers import assert_close_to_oracle, gemm_exact_weights, np_of, out_f64, small_m_path

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def device_weight(N: int, K: int, seed: int, dist: str) -> torch.Tensor:
    g = torch.Generator(device=DEV).manual_seed(seed)
    if dist == "n002":
        return (torch.randn(N, K, generator=g, device=DEV) * 0.02).to(torch.float16)
    # Student-t, 3 degrees of freedom, scaled to std 0.02 (var(t_3) = 3)
    w = torch.empty(N, K, dtype=torch.float16, device=DEV)
    for r0 in range(0, N, 8192):  # bounded temporaries
        n = min(8192, N - r0)
        z = torch.randn(4, n, K, generator=g, device=DEV)
        t = z[0] / torch.sqrt((z[1] ** 2 + z[2] ** 2 + z[3] ** 2) / 3.0)
        w[r0:r0 + n] = (t * (0.02 / 3.0 ** 0.5)).to(torch.float16)
        del z, t
    return w


def sample_rows(N: int, n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    rows = set(range(min(16, N))) | set(range(max(0, N - 16), N))
    rows |= set(rng.choice(N, size=min(n, N), replace=False).tolist())
    return np.array(sorted(rows), np.int64)


def compress_and_pin(N: int, K: int, seed: int, dist: str, rows: np.ndarray):
    """Compress on the device; check the sampled rows against the oracle quantiser."""
    w = device_weight(N, K, seed, dist)
    c = C.compress_linear(w)
    ridx = torch.from_numpy(rows).to(DEV)
    w_rows = w[ridx].cpu().numpy()
    del w
    idx = c.outlier_idx.cpu().numpy()
    packed, scales, pz = O.compute_group32_quant(w_rows, idx)
    assert np.array_equal(c.packed[ridx].cpu().numpy(), packed), "codes differ from the oracle quantiser"
    assert np.array_equal(c.scales[ridx].cpu().numpy().view(np.uint16), scales.view(np.uint16))
    assert np.array_equal(c.zeros[ridx].cpu().numpy(), O.unpack_zeros(pz, K))
    assert np.array_equal(c.outlier_w[ridx].cpu().numpy().view(np.uint16), w_rows[:, idx].view(np.uint16))
    return c


def rows_fmt(c, rows: np.ndarray) -> dict:
    ridx = torch.from_numpy(rows).to(DEV)
    return {"packed": c.packed[ridx].cpu().numpy(), "scales": c.scales[ridx].cpu().numpy(),
            "zeros": c.zeros[ridx].cpu().numpy(), "outlier_idx": c.outlier_idx.cpu().numpy(),
            "ow": c.outlier_w[ridx].cpu()}


def check_gemm_rows(c, a: torch.Tensor, out: torch.Tensor, rows: np.ndarray, what: str):
    """The GEMM's bar on the sampled rows: against the reference's operand
    rounding for the tcgen05 kernel; against the exact dequantised weights
    (1 ulp) and the operand rounding (1e-2*||c||_inf) when the small-M kernel
    (M = 2..8) took the call."""
    f = rows_fmt(c, rows)
    an, ad = np_of(a)
    ow, owd = np_of(f["ow"])
    kw = dict(outlier_idx=f["outlier_idx"], outlier_w=ow, ow_dtype=owd, marlin=True)
    c_exact, c_round, cd = O.gemm(an, ad, f["packed"], f["scales"], f["zeros"], **kw)
    got = out_f64(out[:, torch.from_numpy(rows).to(DEV)])
    assert np.isfinite(got).all(), what
    M, K = a.shape
    if small_m_path(M, int(c.packed.shape[0]), K, int(c.outlier_idx.numel()), ad, owd):
        assert np.max(np.abs(got - c_exact)) <= 1e-2 * np.max(np.abs(c_exact)), what
        c_exact, c_round, cd = gemm_exact_weights(an, ad, f["packed"], f["scales"], f["zeros"], **kw)
    assert_close_to_oracle(got, c_exact, c_round, cd, what)


def check_gemv_rows(c, x: torch.Tensor, y: torch.Tensor, rows: np.ndarray, what: str):
    f = rows_fmt(c, rows)
    xn, xd = np_of(x.reshape(-1))
    ow, owd = np_of(f["ow"])
    y_exact, y_round, od = O.gemv(xn, xd, f["packed"], f["scales"], f["zeros"], outlier_idx=f["outlier_idx"],
                                  outlier_w=ow, ow_dtype=owd, marlin=True)
    got = out_f64(y.reshape(-1)[torch.from_numpy(rows).to(DEV)])
    assert np.isfinite(got).all(), what
    assert_close_to_oracle(got, y_exact, y_round, od, what)


def act(M: int, K: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)


# Llama-3-8B linear shapes (K x N), N(0, 0.02) weights
CONFIG3 = [(4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)]


@pytest.mark.parametrize("K,N", CONFIG3)
def test_config3_gemm_and_gemv(K, N):
    rows = sample_rows(N, 192, seed=K + N)
    c = compress_and_pin(N, K, seed=K * 7 + N, dist="n002", rows=rows)
    for M in (2, 4, 8, 16, 64, 256):  # 2 and 4: the engine's generate_batch; 16-256: config 3
        a = act(M, K, seed=M * 13 + K)
        out = SK.batched_w4a16_gemm(a, c.packed, c.scales, c.zeros, outlier_idx=c.outlier_idx,
                                    outlier_w=c.outlier_w, marlin_layout=True)
        torch.cuda.synchronize()
        assert out.shape == (M, N) and out.dtype == torch.bfloat16
        check_gemm_rows(c, a, out, rows, f"config3 {K}x{N} M={M}")
    x = act(1, K, seed=K - 1)
    y = SK.fused_w4a16_gemv_hdsq(x, c.packed, c.scales, c.zeros, outlier_idx=c.outlier_idx,
                                 outlier_w=c.outlier_w, marlin_layout=True)
    torch.cuda.synchronize()
    check_gemv_rows(c, x, y, rows, f"config3 {K}x{N} M=1")


# Llama-3-70B linear shapes, heavy-tailed weights
CONFIG5 = [(8192, 8192), (8192, 28672), (28672, 8192), (8192, 128256)]


@pytest.mark.parametrize("K,N", CONFIG5)
def test_config5_gemv_m1_and_gemm_m32(K, N):
    rows = sample_rows(N, 160, seed=K ^ N)
    c = compress_and_pin(N, K, seed=5000 + K + N, dist="t3", rows=rows)
    n_out = c.outlier_idx.numel()
    assert 0.005 * K - 1 <= n_out <= 0.03 * K + 1  # the compressor's ratio clamp
    x = act(1, K, seed=K + 3)
    y = SK.fused_w4a16_gemv_hdsq(x, c.packed, c.scales, c.zeros, outlier_idx=c.outlier_idx,
                                 outlier_w=c.outlier_w, marlin_layout=True)
    torch.cuda.synchronize()
    check_gemv_rows(c, x, y, rows, f"config5 {K}x{N} M=1 (n_out={n_out})")
    a = act(32, K, seed=K + 4)
    out = SK.batched_w4a16_gemm(a, c.packed, c.scales, c.zeros, outlier_idx=c.outlier_idx,
                                outlier_w=c.outlier_w, marlin_layout=True)
    torch.cuda.synchronize()
    check_gemm_rows(c, a, out, rows, f"config5 {K}x{N} M=32 (n_out={n_out})")
    del c
    torch.cuda.empty_cache()
