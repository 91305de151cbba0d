"""GPU parity of the M >= 2 GEMM (batched_w4a16_gemm) against the reference's
own outputs and the oracle.  Bar for the tcgen05 kernel: within 1e-2*||c||_inf
of the exact result of the reference's operand rounding, and within 1 output
ulp of its correctly rounded value (floor 2^-16*||c||_inf).  Calls the small-M
kernel takes (M = 2..8, spectra_gemm_small_m_plan) use the exact dequantised
weights instead: the same 1-ulp bar against that exact result, 1e-2*||c||_inf
against the operand-rounded one, and against the reference's own outputs one
output ulp each side plus the most the operand rounding can move a result."""
import numpy as np
import pytest
import torch

from oracle import w4a16 as O
from spectra_b200 import _lib as L
from spectra_b200 import kernels as SK
from tests.helpers import (TORCH_DT, act, assert_close_to_oracle, compressed, gemm_exact_weights, np_of, out_f64,
                           operand_rounding_bound, random_format, small_m_path, ulp)

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _t(a, dev=DEV):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def run_gemm(fmt, a, marlin=True, use_out=True, idx_dtype=torch.int64):
    p, s, z = _t(fmt["packed"]), _t(fmt["scales"]), _t(fmt["zeros"])
    idx = _t(fmt["outlier_idx"]).to(idx_dtype) if use_out and fmt["outlier_idx"].size else None
    ow = fmt["outlier_w_t"].to(DEV) if idx is not None else None
    c = SK.batched_w4a16_gemm(a.to(DEV), p, s, z, outlier_idx=idx, outlier_w=ow, marlin_layout=marlin)
    torch.cuda.synchronize()
    return c


def oracle_gemm(fmt, a, marlin=True, use_out=True):
    an, ad = np_of(a.reshape(-1, a.shape[-1]))
    ow, owd = np_of(fmt["outlier_w_t"])
    has = use_out and fmt["outlier_idx"].size
    return O.gemm(an, ad, fmt["packed"], fmt["scales"], fmt["zeros"],
                  outlier_idx=fmt["outlier_idx"] if has else None, outlier_w=ow if has else None,
                  ow_dtype=owd, marlin=marlin)


def takes_small_m(fmt, a, use_out=True):
    N, K = fmt["packed"].shape[0], fmt["packed"].shape[1] * 2
    n_out = int(fmt["outlier_idx"].size) if use_out else 0
    _, owd = np_of(fmt["outlier_w_t"])
    return small_m_path(a.numel() // K, N, K, n_out, np_of(a)[1], owd)


def oracle_exact_weights(fmt, a, marlin=True, use_out=True):
    an, ad = np_of(a.reshape(-1, a.shape[-1]))
    ow, owd = np_of(fmt["outlier_w_t"])
    has = use_out and fmt["outlier_idx"].size
    return gemm_exact_weights(an, ad, fmt["packed"], fmt["scales"], fmt["zeros"],
                              outlier_idx=fmt["outlier_idx"] if has else None, outlier_w=ow if has else None,
                              ow_dtype=owd, marlin=marlin)


def check(fmt, a, marlin=True, use_out=True, what=""):
    c = run_gemm(fmt, a, marlin, use_out)
    c_exact, c_round, cd = oracle_gemm(fmt, a, marlin, use_out)
    assert c.dtype == a.dtype
    assert c.shape == a.shape[:-1] + (fmt["packed"].shape[0],)
    got = out_f64(c).reshape(c_exact.shape)
    assert np.isfinite(got).all(), what
    if takes_small_m(fmt, a, use_out):
        assert np.max(np.abs(got - c_exact)) <= 1e-2 * np.max(np.abs(c_exact)), what
        c_exact, c_round, cd = oracle_exact_weights(fmt, a, marlin, use_out)
    assert_close_to_oracle(got, c_exact, c_round, cd, what)
    return c


# ---------------------------------------------------------------------------
# pins from the reference's own outputs
# ---------------------------------------------------------------------------

GEMM_CASES = [
    ("gemm_f16_marlin_m1", "f16", True, False),
    ("gemm_f16_marlin_m2", "f16", True, False),
    ("gemm_f16_marlin_m4", "f16", True, False),
    ("gemm_f16_marlin_m8", "f16", True, False),
    ("gemm_f16_marlin_m4_out", "f16", True, True),
    ("gemm_bf16_marlin_m16_out", "bf16", True, True),
    ("gemm_bf16_evenodd_m3_out", "bf16", False, True),
    ("gemm_f16_marlin_m17", "f16", True, False),
]


@pytest.mark.parametrize("name,dt,marlin,use_out", GEMM_CASES)
def test_gemm_matches_reference_outputs(golden_dir, name, dt, marlin, use_out):
    d = np.load(golden_dir / "kernel_cases.npz")
    if dt == "bf16":
        ow = torch.from_numpy(d["ow_bf16"].view(np.int16)).view(torch.bfloat16)
        a = torch.from_numpy(d[f"{name}/a"].view(np.int16)).view(torch.bfloat16)
    else:
        ow = torch.from_numpy(d["ow"].view(np.float16))
        a = torch.from_numpy(d[f"{name}/a"].view(np.float16))
    fmt = {"packed": d["packed"], "scales": d["scales"].view(np.float16), "zeros": d["zeros"],
           "outlier_idx": d["idx"].astype(np.int64), "outlier_w_t": ow}
    c = run_gemm(fmt, a, marlin=marlin, use_out=use_out)
    cb = d[f"{name}/c"]
    c_ref = (O.bf16_bits_to_f32(cb) if dt == "bf16" else cb.view(np.float16)).astype(np.float64)
    got = out_f64(c).reshape(c_ref.shape)
    # Both sides round one fp32 sum; they may differ by 1 output ulp, or by the
    # fp32 accumulation error where the sum cancels (the *_out fixtures pit
    # outlier terms against the main sum): floor 2^-16 * ||c||_inf.
    bound = np.maximum(ulp(c_ref, dt), np.exp2(-16.0) * np.max(np.abs(c_ref)))
    small = M_of(a) > 1 and takes_small_m(fmt, a, use_out)
    if small:
        # exact dequantised weights here, rounded operands there: one ulp each
        # side plus the most the operand rounding can move the result
        an, ad = np_of(a.reshape(-1, a.shape[-1]))
        ow_n, owd = np_of(fmt["outlier_w_t"])
        e = operand_rounding_bound(an, ad, fmt["packed"], fmt["scales"], fmt["zeros"],
                                   outlier_idx=fmt["outlier_idx"] if use_out else None,
                                   outlier_w=ow_n if use_out else None, ow_dtype=owd, marlin=marlin)
        bound = np.maximum(bound, 2 * ulp(c_ref, dt) + e.reshape(c_ref.shape) * 1.0001)
    d_rel = np.abs(got - c_ref) / bound
    i = np.unravel_index(int(np.argmax(d_rel)), d_rel.shape)
    assert d_rel[i] <= 1.0, (f"{name}: worst at {i}: got {got[i]!r} ref {c_ref[i]!r} "
                             f"({d_rel[i]:.2f} x max(1 ulp, 2^-16*||c||inf))")
    if dt == "f16":
        assert np.max(np.abs(got - c_ref)) <= 0.05  # tests/test_kernels.py:58
    c_exact, c_round, cd = (oracle_exact_weights if small else oracle_gemm)(fmt, a, marlin, use_out)
    assert_close_to_oracle(got, c_exact, c_round, cd, name)


def M_of(a):
    return a.numel() // a.shape[-1]


# ---------------------------------------------------------------------------
# oracle parity over shapes, dtypes and layouts
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("M", [2, 3, 16, 17, 33, 64, 100, 256])
@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_gemm_token_counts(M, dt):
    fmt = random_format(640, 1024, 21, seed=M, ow_dtype=dt)
    check(fmt, act(M, 1024, seed=M, dtype=dt), what=f"M={M} {dt}")


def test_workspace_shared_by_outlier_gather_and_split_k():
    """A call that gathers its outlier activations into the workspace (256
    tokens, 75 weight tiles: K not split) and a split-K call after it on the
    same stream share one workspace: the second call's tile counters must
    still be zero, and its result exact."""
    big = random_format(9600, 512, 21, seed=1, ow_dtype="bf16")
    check(big, act(256, 512, seed=2, dtype="bf16"), what="gathering call")
    fmt = random_format(640, 1024, 21, seed=17, ow_dtype="bf16")
    check(fmt, act(17, 1024, seed=17, dtype="bf16"), what="split-K call after it")
    check(big, act(256, 512, seed=3, dtype="bf16"), what="gathering call after it")


@pytest.mark.parametrize("M", [257, 300, 600])
def test_gemm_several_token_chunks(M):
    fmt = random_format(384, 512, 5, seed=M, ow_dtype="bf16")
    check(fmt, act(M, 512, seed=M, dtype="bf16"), what=f"M={M}")


@pytest.mark.parametrize("N,K", [(128, 64), (200, 96), (129, 160), (4160, 64), (1000, 2080), (96, 32)])
@pytest.mark.parametrize("marlin", [True, False])
def test_gemm_ragged_shapes(N, K, marlin):
    fmt = random_format(N, K, min(7, K), seed=N + K, ow_dtype="bf16")
    check(fmt, act(16, K, seed=K, dtype="bf16"), marlin=marlin, what=f"N={N} K={K}")


@pytest.mark.parametrize("n_out", [0, 1, 63, 64, 65, 130])
def test_gemm_outlier_counts(n_out):
    fmt = random_format(256, 1024, n_out, seed=n_out, ow_dtype="f16")
    check(fmt, act(24, 1024, seed=n_out, dtype="f16"), what=f"n_out={n_out}")


@pytest.mark.parametrize("ow_dtype", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("idx_dtype", [torch.int32, torch.int64])
def test_gemm_outlier_dtypes(ow_dtype, idx_dtype):
    fmt = random_format(256, 512, 9, seed=3, ow_dtype=ow_dtype)
    for M in (16, 24):  # the small-M kernel, then the tcgen05 GEMM
        a = act(M, 512, seed=3, dtype="bf16")
        c = run_gemm(fmt, a, idx_dtype=idx_dtype)
        oracle = oracle_exact_weights if takes_small_m(fmt, a) else oracle_gemm
        c_exact, c_round, cd = oracle(fmt, a)
        assert_close_to_oracle(out_f64(c), c_exact, c_round, cd, f"M={M} {ow_dtype}/{idx_dtype}")


def test_gemm_compressed_weights():
    fmt = compressed(512, 2048, seed=11, dist="t3")
    a = act(32, 2048, seed=11, dtype="bf16")
    check(fmt, a, what="compressed t3")


@pytest.mark.parametrize("N,K", [(4096, 4096), (1024, 4096), (4096, 14336)])
def test_gemm_llama3_8b_shapes(N, K):
    fmt = random_format(N, K, 40, seed=N ^ K, ow_dtype="bf16")
    check(fmt, act(16, K, seed=K, dtype="bf16"), what=f"{K}x{N}")


def test_gemm_split_k_deterministic_and_workspace_reused():
    # few weight tiles and a long K: K is split over many CTAs and the last
    # CTA of each tile sums the partials in a fixed order
    fmt = random_format(256, 16384, 12, seed=5, ow_dtype="bf16")
    assert L.lib().spectra_w4a16_gemm_workspace_bytes(16, 256, 16384, 12) > 0
    a = act(16, 16384, seed=5, dtype="bf16")
    c1 = check(fmt, a, what="split-K")
    for _ in range(3):
        c2 = run_gemm(fmt, a)
        assert torch.equal(c1, c2)


def test_gemm_fp32_activations_round_to_fp16():
    fmt = random_format(256, 512, 4, seed=8, ow_dtype="f16")
    a32 = act(8, 512, seed=8, dtype="f32")
    c32 = run_gemm(fmt, a32)
    c16 = run_gemm(fmt, a32.to(torch.float16))
    assert c32.dtype == torch.float32
    assert torch.equal(c32, c16.float())


def test_gemm_3d_input_and_strided_views():
    fmt = random_format(256, 512, 4, seed=9, ow_dtype="bf16")
    a = act(12, 512, seed=9, dtype="bf16")
    c = run_gemm(fmt, a.reshape(3, 4, 512))
    assert c.shape == (3, 4, 256)
    base = run_gemm(fmt, a)
    assert torch.equal(c.reshape(12, 256), base)
    # padded rows (row pitch 512+16) and a base that is not 16-byte aligned
    wide = torch.zeros(12, 528, dtype=torch.bfloat16)
    wide[:, :512] = a
    assert torch.equal(run_gemm(fmt, wide[:, :512]), base)
    shifted = torch.zeros(12 * 512 + 1, dtype=torch.bfloat16)
    shifted[1:] = a.reshape(-1)
    assert torch.equal(run_gemm(fmt, shifted[1:].view(12, 512)), base)


def test_gemm_errors_are_loud():
    fmt = random_format(128, 64, 0, seed=1)
    a = act(4, 64, seed=1, dtype="bf16")
    with pytest.raises(RuntimeError):
        SK.batched_w4a16_gemm(a, torch.from_numpy(fmt["packed"]), torch.from_numpy(fmt["scales"]),
                              torch.from_numpy(fmt["zeros"]))  # CPU tensors: no fallback
