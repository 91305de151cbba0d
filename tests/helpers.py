"""Shared test helpers: seeded format tensors, numpy<->torch, oracle wrappers."""
from __future__ import annotations

import numpy as np
import torch

from oracle import w4a16 as O
from spectra_b200.synthetic import draw_act, draw_weight

TORCH_DT = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def random_format(N: int, K: int, n_out: int, seed: int, ow_dtype: str = "f16"):
    """Random tensors in the reference's weight format (any values are valid
    codes), sized like a compressor output, for shapes too large to quantise
    quickly on the CPU.  Scales are fp16 in the range the compressor produces
    for N(0, 0.02) weights."""
    rng = np.random.default_rng(seed)
    G = K // 32
    packed = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    scales = (rng.uniform(0.002, 0.02, size=(N, G))).astype(np.float16)
    zeros = rng.integers(0, 16, size=(N, G), dtype=np.uint8)
    idx = np.sort(rng.choice(K, size=n_out, replace=False)).astype(np.int64) if n_out else np.zeros(0, np.int64)
    ow = rng.normal(0.0, 0.05, size=(N, n_out)).astype(np.float32)
    ow_t = torch.from_numpy(ow).to(TORCH_DT[ow_dtype])
    return {"packed": packed, "scales": scales, "zeros": zeros, "outlier_idx": idx, "outlier_w_t": ow_t}


def compressed(N: int, K: int, seed: int, dist: str = "n002"):
    """Real compressor output (oracle restatement of SpectraCompressor)."""
    w = draw_weight(N, K, seed=seed, dist=dist).numpy()
    c = O.compress_linear(w)
    c["outlier_w_t"] = torch.from_numpy(c["outlier_w"])
    return c


def np_of(t: torch.Tensor):
    """torch -> (numpy array in oracle convention, dtype tag)."""
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16), "bf16"
    if t.dtype == torch.float16:
        return t.numpy(), "f16"
    return t.float().numpy(), "f32"


def out_f64(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float64)


def ulp(v: np.ndarray, dtype: str) -> np.ndarray:
    v = np.abs(np.asarray(v, np.float64))
    e = np.floor(np.log2(np.maximum(v, 1e-30)))
    mant = {"f16": 10, "bf16": 7, "f32": 23}[dtype]
    lo = {"f16": -24.0, "bf16": -133.0, "f32": -149.0}[dtype]
    return np.exp2(np.maximum(e - mant, lo))


def assert_close_to_oracle(y_gpu: np.ndarray, y_exact: np.ndarray, y_round: np.ndarray, dtype: str, what: str = ""):
    """The path's bar: max|err| <= 1e-2*||y||_inf against the exact result, and
    (stronger) at most one output ulp from the correctly rounded exact value."""
    y_gpu = np.asarray(y_gpu, np.float64)
    tol = 1e-2 * max(np.max(np.abs(y_exact)), 1e-30)
    err = np.max(np.abs(y_gpu - y_exact)) if y_gpu.size else 0.0
    assert err <= tol, f"{what}: max|err|={err:.3e} > 1e-2*||y||inf={tol:.3e}"
    # fp32 accumulation leaves an absolute error ~1e-7*||y||; near-zero outputs
    # have ulps smaller than that, so the floor is 2^-16*||y||_inf.
    floor = np.exp2(-16.0) * np.max(np.abs(y_exact)) if y_exact.size else 0.0
    bad = np.abs(y_gpu - y_round) > np.maximum(ulp(y_round, dtype) * 1.0001, floor)
    assert not bad.any(), (f"{what}: {bad.sum()} outputs more than max(1 {dtype} ulp, 2^-16*||y||inf) "
                           f"from the rounded exact value")


def act(M: int, K: int, seed: int, dtype: str) -> torch.Tensor:
    return draw_act(M, K, seed=seed, dtype=TORCH_DT[dtype])


_DT_CODE = {"f16": 0, "bf16": 1, "f32": 2}


def small_m_path(M: int, N: int, K: int, n_out: int, a_dtype: str = "bf16", ow_dtype: str = "bf16") -> bool:
    """Whether spectra_w4a16_gemm runs its small-M kernel (M = 2..8, exact
    dequantised weights) for contiguous operands of this shape on GPU 0."""
    import ctypes
    from spectra_b200 import _lib as L
    sms = torch.cuda.get_device_properties(0).multi_processor_count if torch.cuda.is_available() else 148
    out = np.zeros(7, np.int64)
    cd = "bf16" if a_dtype == "bf16" else "f16"
    st = L.lib().spectra_gemm_small_m_plan(M, N, K, n_out, _DT_CODE[cd], _DT_CODE[ow_dtype], sms,
                                          out.ctypes.data_as(ctypes.c_void_p))
    return st == 0 and out[0] == 1


def gemm_exact_weights(a, a_dtype: str, packed, scales, zeros, outlier_idx=None, outlier_w=None,
                       ow_dtype=None, marlin: bool = True):
    """The small-M kernel's semantics: activations rounded to the compute dtype
    (as the reference GEMM's operands), the dequantised weights and outlier
    weights exact (as the reference GEMV), exact accumulation, one rounding.
    Returns (c_exact, c_rounded, compute_dtype)."""
    cd = "bf16" if a_dtype == "bf16" else "f16"
    av = O.round_to(O._as_f64(a, a_dtype), cd)
    av = av.reshape(-1, av.shape[-1])
    w = O.dequant_f32(packed, scales, zeros, marlin).astype(np.float64)
    c = av @ w.T
    if outlier_idx is not None and outlier_w is not None and np.asarray(outlier_idx).size:
        idx = np.asarray(outlier_idx, np.int64)
        c = c + av[:, idx] @ O._as_f64(outlier_w, ow_dtype).T
    return c, O.round_to(c, cd), cd


def operand_rounding_bound(a, a_dtype: str, packed, scales, zeros, outlier_idx=None, outlier_w=None,
                           ow_dtype=None, marlin: bool = True) -> np.ndarray:
    """Per output, sum_k |a_k| |w_k - R(w_k)| (+ the same over the outlier
    columns): how far the reference GEMM's operand rounding R() can move a
    result away from the exact-weights product."""
    cd = "bf16" if a_dtype == "bf16" else "f16"
    av = np.abs(O.round_to(O._as_f64(a, a_dtype), cd)).reshape(-1, np.asarray(packed).shape[1] * 2)
    w = O.dequant_f32(packed, scales, zeros, marlin).astype(np.float64)
    e = av @ np.abs(w - O.round_to(w, cd)).T
    if outlier_idx is not None and outlier_w is not None and np.asarray(outlier_idx).size:
        idx = np.asarray(outlier_idx, np.int64)
        ow = O._as_f64(outlier_w, ow_dtype)
        e = e + av[:, idx] @ np.abs(ow - O.round_to(ow, cd)).T
    return e
