"""CPU oracle for the SPECTRA W4A16 linear-layer hot path (numpy restatement).

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (``spectra_b200``)
imports this module; only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and only
as the checker or the timed CPU baseline.

Every function restates one piece of the reference (NeuraCryption/SPECTRA)
and cites the file:line it follows.  Paths are relative to the reference
project root.

Format recap (spectra/compressor.py:72-112):
  * weights are quantised per group of 32 consecutive input features with an
    asymmetric min/max affine code: ``q = clamp(round(w/s + z), 0, 15)``,
    ``s = (max-min)/15`` (fp16 on disk), ``z = clamp(round(-min/s), 0, 15)``;
  * two codes per byte.  "Marlin" order: byte j of a group holds k=j in the
    low nibble and k=j+16 in the high nibble.  "Even-odd" order: byte b holds
    k=2b (low) and k=2b+1 (high);
  * zero-points are packed two per byte on disk and unpacked to one u8 per
    group at load time (spectra/engine.py:1007-1012);
  * a few salient input columns ("outliers") are zeroed before quantisation
    and kept exactly in the source dtype (spectra/compressor.py:158-215);
    kernels add ``x[idx] @ ow.T`` on top of the dequantised product.

Numerics: bf16 has no numpy dtype, so bf16 tensors travel as their uint16
bit patterns (``bf16_bits_to_f32`` / ``f32_to_bf16_bits``).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np

GROUP = 32

# ----------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even, the rounding torch's .to(bfloat16) and
# Triton's .to(tl.bfloat16) use)
# ----------------------------------------------------------------------------


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(bits).astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even; NaN stays NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    lsb = (b >> np.uint64(16)) & np.uint64(1)
    rounded = ((b + np.uint64(0x7FFF) + lsb) >> np.uint64(16)).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded[nan] = ((b[nan] >> np.uint64(16)) | np.uint64(0x40)).astype(np.uint16)
    return rounded


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round a float array to ``dtype`` ("f16"/"bf16"/"f32") and return it as float64."""
    x32 = np.asarray(x, dtype=np.float32)
    if dtype == "f16":
        return x32.astype(np.float16).astype(np.float64)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x32)).astype(np.float64)
    if dtype == "f32":
        return x32.astype(np.float64)
    raise ValueError(dtype)


# ----------------------------------------------------------------------------
# Quantiser (input generator) -- spectra/compressor.py
# ----------------------------------------------------------------------------


def quantize_chunk_group32(w: np.ndarray) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Group-32 min/max affine INT4 quantiser.

    Follows ``SpectraCompressor._quantize_chunk_group32``
    (spectra/compressor.py:72-112) operation by operation in float32:
    constant-group rules (:81-95), half-to-even rounding (``torch.round`` ==
    ``np.round``), Marlin packing (:99-102) and two-per-byte zero packing with
    an odd-count pad (:104-110).

    Returns (packed u8 [N,K/2], scales f16 [N,K/32], packed_zeros u8 [N,ceil(G/2)]).
    """
    N, K = w.shape
    if K % GROUP:
        raise ValueError("K must be a multiple of 32")
    G = K // GROUP
    wg = np.asarray(w).reshape(N, G, GROUP).astype(np.float32)
    w_min = wg.min(axis=-1, keepdims=True)
    w_max = wg.max(axis=-1, keepdims=True)
    diff = w_max - w_min
    is_const = diff < np.float32(1e-8)
    one = np.float32(1.0)
    scales = np.where(is_const, np.where(w_min == 0, one, np.abs(w_min)), diff / np.float32(15.0))
    scales = np.maximum(scales.astype(np.float32), np.float32(1e-8))
    with np.errstate(invalid="ignore"):
        z_nc = np.clip(np.round(-w_min / scales), 0, 15).astype(np.uint8)
    zeros = np.where(is_const, np.where(w_min < 0, np.uint8(1), np.uint8(0)), z_nc).astype(np.uint8)
    zs = -(zeros.astype(np.float32) * scales)
    with np.errstate(invalid="ignore"):
        q_nc = np.clip(np.round((wg - zs) / scales), 0, 15).astype(np.uint8)
    q_const = np.broadcast_to(np.where(w_min > 0, np.uint8(1), np.uint8(0)), wg.shape)
    q = np.where(is_const, q_const, q_nc).astype(np.uint8)
    packed = (q[:, :, 0:16] | (q[:, :, 16:32] << np.uint8(4))).astype(np.uint8).reshape(N, K // 2)
    z2 = zeros[:, :, 0]
    if G % 2:
        z2 = np.concatenate([z2, np.zeros((N, 1), np.uint8)], axis=1)
    packed_zeros = (z2[:, 0::2] | (z2[:, 1::2] << np.uint8(4))).astype(np.uint8)
    return packed, scales[:, :, 0].astype(np.float16), packed_zeros


def compute_group32_quant(w: np.ndarray, outlier_idx: Optional[np.ndarray] = None):
    """``SpectraCompressor._compute_group32_quant`` (spectra/compressor.py:115-156).

    Zeroes the outlier columns, then quantises.  The reference processes rows in
    4096-row chunks when N > 4096; row chunks are independent, so one call is
    the same computation.
    """
    wd = np.array(w, copy=True)
    if outlier_idx is not None:
        wd[:, np.asarray(outlier_idx, dtype=np.int64)] = 0
    return quantize_chunk_group32(wd)


def isolate_outliers(w: np.ndarray, norm_vector: Optional[np.ndarray] = None,
                     base_outlier_ratio: float = 0.01, adaptive_kurtosis: bool = True):
    """Kurtosis-adaptive outlier-column selection.

    Follows ``SpectraCompressor._isolate_hdsq_outliers`` (spectra/compressor.py:158-215):
    fp32 column L2 norms (row-chunked sum of squares when N > 4096, :168-174),
    optional |gamma| saliency scaling (:180-183), 4th standardised moment
    (:185-188), ratio = clamp(r*(1+0.15*log1p(max(0,k-3))), 0.005, 0.03) with the
    clamp done in fp32 (:190-193), top-k then ascending sort (:197-200).
    Float reductions are restated in float32; the selected set equals the
    reference's except in exact near-ties of column norms.

    Returns (outlier_idx int32 [n_out], outlier_w [N,n_out] in w's dtype, ratio, kurtosis).
    """
    N, K = w.shape
    wf = np.asarray(w).astype(np.float32)
    if N > 4096:
        acc = np.zeros(K, np.float32)
        for r0 in range(0, N, 4096):
            c = wf[r0:r0 + 4096]
            acc += (c * c).sum(axis=0, dtype=np.float32)
        col_norms = np.sqrt(acc)
    else:
        col_norms = np.sqrt((wf * wf).sum(axis=0, dtype=np.float32))
    if norm_vector is not None and np.asarray(norm_vector).size == K:
        sal = np.asarray(norm_vector, np.float32) * col_norms
    else:
        sal = col_norms
    mu = sal.mean(dtype=np.float32)
    d = sal - mu
    sigma2 = (d * d).mean(dtype=np.float32) + np.float32(1e-8)
    m4 = (d ** 4).mean(dtype=np.float32)
    kurt = max(1.0, float(np.float32(m4 / (sigma2 * sigma2))))
    if adaptive_kurtosis:
        k_mult = 1.0 + 0.15 * math.log1p(max(0.0, kurt - 3.0))
        ratio = float(np.clip(np.float32(base_outlier_ratio * k_mult), np.float32(0.005), np.float32(0.03)))
    else:
        ratio = base_outlier_ratio
    n_out = max(1, int(round(K * ratio)))
    idx = np.argsort(-sal, kind="stable")[:n_out]
    idx = np.sort(idx).astype(np.int32)
    ow = np.asarray(w)[:, idx.astype(np.int64)].copy()
    return idx, ow, ratio, kurt


def unpack_zeros(packed_zeros: np.ndarray, K: int) -> np.ndarray:
    """Zero-point unpack done at load (spectra/engine.py:1007-1012, tests/test_kernels.py:25-29)."""
    pz = np.asarray(packed_zeros, np.uint8)
    N = pz.shape[0]
    z = np.empty((N, pz.shape[1] * 2), np.uint8)
    z[:, 0::2] = pz & 0x0F
    z[:, 1::2] = (pz >> 4) & 0x0F
    return np.ascontiguousarray(z[:, : K // GROUP])


def compress_linear(w: np.ndarray, norm_vector: Optional[np.ndarray] = None):
    """What ``SpectraCompressor.compress`` writes for one 2-D weight
    (spectra/compressor.py:475-483) and what the engine binds to
    ``SpectraFusedLinear.set_weights`` (spectra/engine.py:999-1026):
    packed u8 [N,K/2], scales f16 [N,K/32], zeros u8 [N,K/32] (unpacked),
    outlier_idx int64, outlier_w [N,n_out] (source dtype).
    """
    idx, ow, ratio, kurt = isolate_outliers(w, norm_vector)
    packed, scales, pz = compute_group32_quant(w, idx)
    zeros = unpack_zeros(pz, w.shape[1])
    return {
        "packed": packed, "scales": scales, "packed_zeros": pz, "zeros": zeros,
        "outlier_idx": idx.astype(np.int64), "outlier_w": ow,
        "ratio": ratio, "kurtosis": kurt,
    }


# ----------------------------------------------------------------------------
# Dequantisation and the two kernels (spectra/kernels.py)
# ----------------------------------------------------------------------------


def codes(packed: np.ndarray, marlin: bool) -> np.ndarray:
    """Unpack nibbles to codes q [N,K] in k order.

    Marlin order: tests/test_kernels.py:31-35 and spectra/kernels.py:78-89;
    even-odd order: spectra/kernels.py:90-98.
    """
    p = np.asarray(packed, np.uint8)
    N, Kh = p.shape
    K = Kh * 2
    lo = p & 0x0F
    hi = (p >> 4) & 0x0F
    if marlin:
        G = K // GROUP
        q = np.concatenate([lo.reshape(N, G, 16), hi.reshape(N, G, 16)], axis=-1)
        return q.reshape(N, K)
    q = np.empty((N, K), np.uint8)
    q[:, 0::2] = lo
    q[:, 1::2] = hi
    return q


def dequant_f32(packed, scales, zeros, marlin: bool) -> np.ndarray:
    """fp32 dequantised weights ``(q - z) * s`` (spectra/kernels.py:56-74).

    (q - z) is an integer in [-15, 15] and s an fp16 value, so each product is
    exact in float32: this is the bit-exact reference for every dequant path.
    """
    q = codes(packed, marlin).astype(np.float32)
    N, K = q.shape
    G = K // GROUP
    s = np.asarray(scales, np.float16).astype(np.float32)[:, :G]
    z = np.asarray(zeros, np.uint8).astype(np.float32)[:, :G]
    w = (q.reshape(N, G, GROUP) - z[:, :, None]) * s[:, :, None]
    return w.reshape(N, K).astype(np.float32)


def _as_f64(t: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16_bits_to_f32(t).astype(np.float64)
    return np.asarray(t).astype(np.float64)


def gemv(x, x_dtype: str, packed, scales, zeros, bias=None, bias_dtype: Optional[str] = None,
         outlier_idx=None, outlier_w=None, ow_dtype: Optional[str] = None, marlin: bool = False):
    """Reference M=1 GEMV semantics (``_fused_w4a16_gemv_hdsq_kernel``, spectra/kernels.py:16-129).

    y[n] = sum_k x[k]*((q-z)*s) + sum_j x[idx_j]*ow[n,j] + b[n], with the
    dequantised weights, x, ow and bias all taken exactly (fp32 in the reference,
    float64 here), and the result rounded to bf16 when x is bf16 else fp16
    (:126-129).

    Returns (y_exact float64 [N], y_rounded float64 [N], out_dtype).
    """
    xv = _as_f64(x, x_dtype).reshape(-1)
    w = dequant_f32(packed, scales, zeros, marlin).astype(np.float64)
    y = w @ xv
    if outlier_idx is not None and outlier_w is not None and np.asarray(outlier_idx).size:
        idx = np.asarray(outlier_idx, np.int64)
        y = y + _as_f64(outlier_w, ow_dtype) @ xv[idx]
    if bias is not None:
        y = y + _as_f64(bias, bias_dtype)
    out_dtype = "bf16" if x_dtype == "bf16" else "f16"
    return y, round_to(y, out_dtype), out_dtype


def gemm(a, a_dtype: str, packed, scales, zeros, outlier_idx=None, outlier_w=None,
         ow_dtype: Optional[str] = None, marlin: bool = False):
    """Reference batched GEMM semantics (``_batched_w4a16_gemm_kernel``, spectra/kernels.py:191-331).

    The dequantised weights are rounded to the compute dtype (bf16 if a is
    bf16 else fp16) before the dot (:256-261), as are the activations
    (:274-279) and the outlier weights (:315-320); products accumulate exactly
    (fp32 in the reference, float64 here) and the result is rounded to the
    compute dtype (:328-331).

    Returns (c_exact float64 [M,N], c_rounded float64 [M,N], compute_dtype).
    """
    cd = "bf16" if a_dtype == "bf16" else "f16"
    av = round_to(_as_f64(a, a_dtype), cd)
    av = av.reshape(-1, av.shape[-1])
    w = round_to(dequant_f32(packed, scales, zeros, marlin), cd)
    c = av @ w.T
    if outlier_idx is not None and outlier_w is not None and np.asarray(outlier_idx).size:
        idx = np.asarray(outlier_idx, np.int64)
        ow = round_to(_as_f64(outlier_w, ow_dtype), cd)
        c = c + av[:, idx] @ ow.T
    return c, round_to(c, cd), cd


def fwht(x: np.ndarray, normalize: bool = True) -> np.ndarray:
    """Fast Walsh-Hadamard transform over the last dimension (power of two).

    Restates ``fast_walsh_hadamard_transform`` (spectra/compressor.py:29-42):
    butterflies (u+v, u-v) with doubling span h, then optional 1/sqrt(d).
    """
    x = np.asarray(x, np.float64)
    d = x.shape[-1]
    if d & (d - 1):
        raise ValueError("last dimension must be a power of two")
    res = x.reshape(-1, d).copy()
    h = 1
    while h < d:
        r = res.reshape(-1, d // (2 * h), 2, h)
        u = r[:, :, 0, :].copy()
        v = r[:, :, 1, :].copy()
        r[:, :, 0, :] = u + v
        r[:, :, 1, :] = u - v
        res = r.reshape(-1, d)
        h *= 2
    if normalize:
        res = res / math.sqrt(d)
    return res.reshape(x.shape)


def algorithmic_bytes(M: int, N: int, K: int, n_out: int, act_bytes: int = 2, bias: bool = False) -> int:
    """Bytes one call must move at minimum: packed + fp16 scales + u8 zeros +
    outlier weights + int64 idx + activations in + outputs out (+ bias)."""
    b = N * K // 2 + 2 * N * K // GROUP + N * K // GROUP + 2 * N * n_out + 8 * n_out
    b += act_bytes * M * K + act_bytes * M * N
    if bias:
        b += 2 * N
    return b
