"""CPU oracle for the operators around the linear path: the INT4 KV-cache
quantiser, the quantised embedding gather and the greedy argmax (numpy).

TEST INFRASTRUCTURE ONLY.  Nothing in the product path imports this module;
only ``tests/`` use it, as the checker.  Each function restates one piece of
the reference (NeuraCryption/SPECTRA) and cites the file:line it follows.
bf16 tensors travel as uint16 bit patterns, as in ``oracle/w4a16.py``.
"""
from __future__ import annotations

import numpy as np

from .w4a16 import GROUP, bf16_bits_to_f32, codes, f32_to_bf16_bits

# ----------------------------------------------------------------------------
# dtype helpers
# ----------------------------------------------------------------------------


def to_f32(bits_or_vals: np.ndarray, dtype: str) -> np.ndarray:
    """Stored values (uint16 bits for bf16, float16 for f16) -> exact float32."""
    a = np.asarray(bits_or_vals)
    if dtype == "bf16":
        return bf16_bits_to_f32(a.view(np.uint16) if a.dtype != np.uint16 else a)
    if dtype == "f16":
        return (a.view(np.float16) if a.dtype == np.uint16 else a).astype(np.float32)
    return a.astype(np.float32)


def rnd(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` (nearest even) and return float32."""
    x = np.asarray(x, np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    return x


def store_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values -> stored form (uint16 bits for bf16 / f16, float32 otherwise), rounded to nearest even."""
    x = np.asarray(x, np.float32)
    if dtype == "bf16":
        return f32_to_bf16_bits(x)
    if dtype == "f16":
        return x.astype(np.float16).view(np.uint16)
    return x


# ----------------------------------------------------------------------------
# INT4 KV cache -- SpectraGroup32QuantizedLayer (spectra/engine.py:614-671)
# ----------------------------------------------------------------------------


def kv_quantize(t_vals: np.ndarray, dtype: str, scalar_div: str = "reciprocal"):
    """``SpectraGroup32QuantizedLayer._quantize`` (spectra/engine.py:625-656).

    ``t_vals``: float32 values of a [..., D] bf16/fp16 tensor.  Every step rounds
    to ``dtype`` where torch does (the method computes in the tensor's dtype):
    diff (:637), scales (:640-641), -min/scale (:645); the code step (:648-651)
    is fp32 because ``zeros.float()`` promotes it.  ``diff / 15.0`` divides a
    tensor by a Python scalar, which torch computes as a true division on the
    CPU but as a multiply by the fp32 reciprocal on a CUDA device: pick with
    ``scalar_div`` ("true" | "reciprocal").

    Returns (packed u8 [rows,G,16] even-odd, scales f16 [rows,G,1], zeros u8
    [rows,G,1], pad).
    """
    t = np.asarray(t_vals, np.float32)
    D = t.shape[-1]
    t = t.reshape(-1, D)
    pad = (GROUP - D % GROUP) % GROUP
    if pad:
        t = np.concatenate([t, np.zeros((t.shape[0], pad), np.float32)], axis=1)
    G = t.shape[1] // GROUP
    tg = t.reshape(-1, G, GROUP)
    lo = tg.min(axis=-1, keepdims=True)
    hi = tg.max(axis=-1, keepdims=True)
    diff = rnd(hi - lo, dtype)
    # torch converts the Python scalar 1e-8 to the tensor's dtype before comparing
    # and clamping (:638-641): bf16(1e-8) ~ 1.0011e-8, but fp16(1e-8) == 0, so an
    # fp16 constant group is not "constant" there and its scale becomes 0
    thr = rnd(np.float32(1e-8), dtype)
    flat = diff < thr
    if scalar_div == "true":
        live = rnd(diff / np.float32(15.0), dtype)
    else:
        live = rnd(diff * (np.float32(1.0) / np.float32(15.0)), dtype)
    s = np.where(flat, np.where(lo == 0, np.float32(1.0), np.abs(lo)), live).astype(np.float32)
    s = rnd(np.maximum(s, thr), dtype)
    # a zero scale (fp16 constant groups) divides by zero: +-inf clamps to 15 or 0,
    # NaN (0/0) converts to the code 0, as torch's float -> uint8 cast gives
    with np.errstate(invalid="ignore", divide="ignore"):
        z_live = np.nan_to_num(np.clip(np.round(rnd(-lo / s, dtype)), 0, 15), nan=0.0)
    z = np.where(flat, (lo < 0).astype(np.float32), z_live).astype(np.float32)
    zs = -(z * s)
    with np.errstate(invalid="ignore", divide="ignore"):
        q_live = np.nan_to_num(np.clip(np.round((tg - zs) / s), 0, 15), nan=0.0)
    q = np.where(flat, np.broadcast_to((lo > 0).astype(np.float32), tg.shape), q_live).astype(np.uint8)
    packed = (q[:, :, 0::2] | (q[:, :, 1::2] << np.uint8(4))).astype(np.uint8)
    return packed, s.astype(np.float16), z.astype(np.uint8), pad


def kv_dequantize(packed: np.ndarray, scales_f16: np.ndarray, zeros: np.ndarray, D: int) -> np.ndarray:
    """``SpectraGroup32QuantizedLayer._dequantize`` (spectra/engine.py:658-671):
    float32 ``(q - z) * s`` [rows, D] (exact), before the final bf16 rounding."""
    p = np.asarray(packed, np.uint8)
    rows, G, _ = p.shape
    q = np.empty((rows, G, GROUP), np.uint8)
    q[:, :, 0::2] = p & 0x0F
    q[:, :, 1::2] = (p >> 4) & 0x0F
    deq = (q.astype(np.float32) - np.asarray(zeros, np.float32).reshape(rows, G, 1)) * \
        np.asarray(scales_f16, np.float16).astype(np.float32).reshape(rows, G, 1)
    return deq.reshape(rows, G * GROUP)[:, :D]


# ----------------------------------------------------------------------------
# Quantised embedding -- SpectraFusedEmbedding.forward (spectra/engine.py:167-212)
# ----------------------------------------------------------------------------


def embedding(ids: np.ndarray, packed, scales_f16, zeros, outlier_idx=None, outlier_w_vals=None,
              marlin: bool = True, out_dtype: str = "bf16") -> np.ndarray:
    """Rows ``ids`` of the dequantised [V, K] matrix, as stored ``out_dtype``.

    Zero points unpacked [V, G] or packed [V, ceil(G/2)] (:176-183); dequant
    ``(q - z) * s`` in fp32 (:185-204), one rounding to the target dtype, then
    the outlier columns overwritten by the exact outlier weights rounded to the
    target dtype (:207-210).
    """
    ids = np.asarray(ids, np.int64).reshape(-1)
    p = np.asarray(packed)[ids]
    K = p.shape[1] * 2
    G = K // GROUP
    z = np.asarray(zeros)[ids]
    if z.shape[1] < G:
        zz = np.empty((z.shape[0], z.shape[1] * 2), np.uint8)
        zz[:, 0::2] = z & 0x0F
        zz[:, 1::2] = (z >> 4) & 0x0F
        z = zz[:, :G]
    q = codes(p, marlin).astype(np.float32).reshape(-1, G, GROUP)
    s = np.asarray(scales_f16, np.float16)[ids].astype(np.float32).reshape(-1, G, 1)
    out = ((q - z.astype(np.float32).reshape(-1, G, 1)) * s).reshape(-1, K)
    out = rnd(out, out_dtype)
    if outlier_idx is not None and outlier_w_vals is not None and np.asarray(outlier_idx).size:
        out[:, np.asarray(outlier_idx, np.int64)] = rnd(np.asarray(outlier_w_vals, np.float32)[ids], out_dtype)
    return store_bits(out, out_dtype)


# ----------------------------------------------------------------------------
# Greedy choice -- sample_token at temperature 0 (spectra/engine.py:1690-1713)
# ----------------------------------------------------------------------------


def argmax(logits: np.ndarray) -> np.ndarray:
    """torch.argmax over the last axis: first maximum, NaN counts as the maximum."""
    x = np.asarray(logits, np.float64)
    return np.argmax(x, axis=-1).astype(np.int64)  # numpy also returns the first NaN
