"""Drop-in replacement of the reference operator module ``spectra.kernels``.

Same names, signatures, argument meaning and return conventions as
spectra/kernels.py (:132-184 ``fused_w4a16_gemv_hdsq``, :333-389
``batched_w4a16_gemm``), so ``spectra/engine.py``'s ``SpectraFusedLinear``
(engine.py:90-124) runs on it unchanged.  Every call goes to the CUDA kernels
of libspectra_b200.so through the C ABI; there is no CPU, Triton or eager
PyTorch fallback -- tensors must live on a CUDA device.

Behaviour kept from the reference:
  * outputs are allocated with ``torch.empty`` on x's device (capture-safe);
  * the GEMV accumulates exactly-dequantised fp32 weights and rounds once to
    bf16 when x is bf16, else to fp16 (kernels.py:126-129), then stores into
    ``out``'s dtype;
  * the GEMM rounds dequantised weights, activations and outlier weights to
    the compute dtype (bf16 if ``a`` is bf16 else fp16) and returns
    ``c.to(a.dtype)`` (kernels.py:347-389); it adds no bias (the engine adds it);
  * strided views (offloader slots, engine.py:555-569) are accepted.
Deliberate difference: the reference GEMV computes only row 0 of a [B,K]
input and leaves rows 1.. of ``out`` unwritten; here every row is computed.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib as L

_DT = {torch.float16: L.DT_F16, torch.bfloat16: L.DT_BF16, torch.float32: L.DT_F32,
       torch.int32: L.DT_I32, torch.int64: L.DT_I64}


def _dt(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def _require_cuda(name: str, t: Optional[torch.Tensor], dev: torch.device) -> None:
    if t is None:
        return
    if not t.is_cuda:
        raise RuntimeError(f"spectra_b200: {name} must be a CUDA tensor (no CPU fallback), got {t.device}")
    if t.device != dev:
        raise RuntimeError(f"spectra_b200: {name} is on {t.device}, expected {dev}")


def _unit_cols(t: torch.Tensor) -> torch.Tensor:
    """Packed codes are read as 16-byte vectors along a row: unit column stride."""
    return t if t.stride(-1) == 1 else t.contiguous()


def _weights(packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor):
    if packed.dtype != torch.uint8 or zeros.dtype != torch.uint8:
        raise TypeError("packed weights and zero-points must be uint8")
    if scales.dtype != torch.float16:
        raise TypeError("scales must be float16")
    if packed.dim() != 2 or scales.dim() != 2 or zeros.dim() != 2:
        raise ValueError("packed, scales and zeros must be 2-D")
    return _unit_cols(packed), scales, zeros


def _outliers(outlier_idx, outlier_w, N: int):
    if outlier_idx is None or outlier_w is None or outlier_idx.numel() == 0:
        return None, None, 0
    idx = outlier_idx.reshape(-1)
    if idx.dtype not in (torch.int32, torch.int64):
        idx = idx.to(torch.int64)
    if idx.stride(0) != 1:
        idx = idx.contiguous()
    ow = outlier_w
    if ow.dim() != 2 or ow.shape[0] != N or ow.shape[1] != idx.numel():
        raise ValueError(f"outlier_w must be [N, n_out] = [{N}, {idx.numel()}], got {tuple(ow.shape)}")
    return idx, ow, idx.numel()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _gemv_row(x_row, packed, scales, zeros, bias, idx, ow, n_out, y_row, layout, N, K, stream):
    lib = L.lib()
    st = lib.spectra_w4a16_gemv(
        x_row.data_ptr(), _dt(x_row), x_row.stride(-1),
        packed.data_ptr(), packed.stride(0),
        scales.data_ptr(), scales.stride(0), scales.stride(1),
        zeros.data_ptr(), zeros.stride(0), zeros.stride(1),
        bias.data_ptr() if bias is not None else None, _dt(bias) if bias is not None else 0,
        idx.data_ptr() if idx is not None else None, _dt(idx) if idx is not None else 0, n_out,
        ow.data_ptr() if ow is not None else None, _dt(ow) if ow is not None else 0,
        ow.stride(0) if ow is not None else 0, ow.stride(1) if ow is not None else 0,
        y_row.data_ptr(), _dt(y_row), y_row.stride(-1),
        N, K, layout, stream)
    L.check("spectra_w4a16_gemv", st)


def fused_w4a16_gemv_hdsq(
    x: torch.Tensor,
    packed_w: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    outlier_idx: Optional[torch.Tensor] = None,
    outlier_w: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    marlin_layout: bool = False,
    hadamard: bool = False,
) -> torch.Tensor:
    """M=1 W4A16 GEMV with fused outlier and bias adds (spectra/kernels.py:132-184).

    ``hadamard`` (keyword, off by default, not in the reference signature):
    rotate x by the normalised Walsh-Hadamard transform first (the rotation
    prologue for weights quantised in the rotated basis; K a power of two).
    """
    orig_dim = x.ndim
    if orig_dim == 1:
        x = x.unsqueeze(0)
    if hadamard:
        x = fwht(x, normalize=True)
    B, K = x.shape
    N = packed_w.shape[0]
    dev = x.device
    for name, t in (("packed_w", packed_w), ("scales", scales), ("zeros", zeros), ("bias", bias),
                    ("outlier_idx", outlier_idx), ("outlier_w", outlier_w), ("out", out)):
        _require_cuda(name, t, dev)
    packed, scales, zeros = _weights(packed_w, scales, zeros)
    idx, ow, n_out = _outliers(outlier_idx, outlier_w, N)
    if bias is not None and bias.stride(-1) != 1:
        bias = bias.contiguous()
    if out is None:
        out = torch.empty((B, N), device=dev, dtype=x.dtype)
    # The reference rounds to bf16 for bf16 x, else fp16, then stores into out's dtype.
    compute = torch.bfloat16 if x.dtype == torch.bfloat16 else torch.float16
    y = out if out.dtype == compute else torch.empty((B, N), device=dev, dtype=compute)
    layout = L.LAYOUT_MARLIN if marlin_layout else L.LAYOUT_EVEN_ODD
    with torch.cuda.device(dev):
        stream = _stream(dev)
        for b in range(B):
            _gemv_row(x[b], packed, scales, zeros, bias, idx, ow, n_out, y[b], layout, N, K, stream)
    if y is not out:
        out.copy_(y)
    if orig_dim == 1:
        out = out.squeeze(0)
    return out


# Split-K workspace, one per (device, stream): calls that share one must not
# overlap in time, and calls on one stream never do.  Zeroed when allocated;
# every GEMM call leaves its counters zero again.  A workspace that grows is
# replaced, but the old buffer is kept alive: a CUDA graph captured earlier on
# the same stream still holds its address, and replaying that graph must not
# write into memory the caching allocator has handed to another tensor.
_WORKSPACES: dict = {}
_RETIRED_WORKSPACES: list = []


def _workspace(dev: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    key = (dev.index, stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        if ws is not None:
            _RETIRED_WORKSPACES.append(ws)
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _WORKSPACES[key] = ws
    return ws


def device_timeouts(reset: bool = False) -> int:
    """Pipeline waits that gave up (2 s limit) in this library's kernels on the
    current device since load or the last reset.  Synchronises the device.  A
    non-zero count means the outputs of the calls that timed out are undefined."""
    import ctypes
    n = ctypes.c_int64(0)
    L.check("spectra_device_timeouts", L.lib().spectra_device_timeouts(ctypes.byref(n), int(reset)))
    return int(n.value)


def batched_w4a16_gemm(
    a: torch.Tensor,
    packed_b: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    outlier_idx: Optional[torch.Tensor] = None,
    outlier_w: Optional[torch.Tensor] = None,
    marlin_layout: bool = False,
    *,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """M >= 2 W4A16 GEMM on the tcgen05 tensor cores (spectra/kernels.py:333-389).

    ``a`` is [..., K]; the result is [..., N] in a's dtype.  Operands are rounded
    to the compute dtype (bf16 if ``a`` is bf16, else fp16) exactly as the
    reference does; fp32 ``a`` is rounded to fp16 before the call, the same
    rounding the reference applies when it loads it.  No bias is added.

    ``out`` (keyword, not in the reference signature): a [M, N] tensor of the
    compute dtype with unit column stride to write into (for example a view
    into a larger buffer); it is returned, reshaped like ``a``.
    """
    orig_shape = a.shape
    K = a.shape[-1]
    M = a.numel() // K if K else 0
    N = packed_b.shape[0]
    dev = a.device
    for name, t in (("packed_b", packed_b), ("scales", scales), ("zeros", zeros),
                    ("outlier_idx", outlier_idx), ("outlier_w", outlier_w)):
        _require_cuda(name, t, dev)
    _require_cuda("a", a, dev)
    packed, scales, zeros = _weights(packed_b, scales, zeros)
    idx, ow, n_out = _outliers(outlier_idx, outlier_w, N)
    compute = torch.bfloat16 if a.dtype == torch.bfloat16 else torch.float16
    if out is not None:
        _require_cuda("out", out, dev)
        if out.dtype != compute or tuple(out.shape) != (M, N) or (N > 1 and out.stride(1) != 1):
            raise ValueError(f"out must be a [{M}, {N}] {compute} tensor with unit column stride")
        c = out
    else:
        c = torch.empty((M, N), device=dev, dtype=compute)
    if M == 0 or N == 0:
        return c.reshape(orig_shape[:-1] + (N,)).to(a.dtype)
    a2 = a.reshape(M, K)
    if a2.dtype != compute:
        a2 = a2.to(compute)
    # the activation tile is fetched by TMA: unit column stride, 16-byte
    # aligned base and row pitch
    if a2.stride(1) != 1 or (a2.stride(0) * 2) % 16 or a2.data_ptr() % 16 or a2.stride(0) < K:
        a2 = a2.clone(memory_format=torch.contiguous_format)
    if packed.data_ptr() % 16 or packed.stride(0) % 16:
        # The tensor-core GEMM streams weight rows by TMA, which needs a 16-byte
        # aligned base and row pitch.  Copying the weights here would double
        # the call's traffic, silently and on every call, so such views are
        # rejected; the M=1 GEMV accepts them.
        raise ValueError(
            "batched_w4a16_gemm: packed weights need a 16-byte aligned base address and row stride "
            f"(got address % 16 = {packed.data_ptr() % 16}, row stride {packed.stride(0)} bytes); "
            "pass a contiguous or 16-byte-aligned view")
    layout = L.LAYOUT_MARLIN if marlin_layout else L.LAYOUT_EVEN_ODD
    lib = L.lib()
    with torch.cuda.device(dev):
        stream = _stream(dev)
        nbytes = lib.spectra_w4a16_gemm_workspace_bytes(M, N, K, n_out)
        ws = _workspace(dev, stream, nbytes) if nbytes else None
        st = lib.spectra_w4a16_gemm(
            a2.data_ptr(), _dt(a2), a2.stride(0),
            packed.data_ptr(), packed.stride(0),
            scales.data_ptr(), scales.stride(0), scales.stride(1),
            zeros.data_ptr(), zeros.stride(0), zeros.stride(1),
            idx.data_ptr() if idx is not None else None, _dt(idx) if idx is not None else 0, n_out,
            ow.data_ptr() if ow is not None else None, _dt(ow) if ow is not None else 0,
            ow.stride(0) if ow is not None else 0, ow.stride(1) if ow is not None else 0,
            c.data_ptr(), _dt(c), c.stride(0),
            M, N, K, layout,
            ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0, stream)
    L.check("spectra_w4a16_gemm", st)
    if out is not None:
        return c
    return c.reshape(orig_shape[:-1] + (N,)).to(a.dtype)


def dequantize(packed_w: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
               marlin_layout: bool = False, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Dense ``(q - z) * s`` on the GPU: exact in fp32, or rounded to nearest-even
    in bf16/fp16 (the reference GEMM's operand, spectra/kernels.py:256-261)."""
    dev = packed_w.device
    for name, t in (("scales", scales), ("zeros", zeros)):
        _require_cuda(name, t, dev)
    _require_cuda("packed_w", packed_w, dev)
    packed, scales, zeros = _weights(packed_w, scales, zeros)
    N, K = packed.shape[0], packed.shape[1] * 2
    out = torch.empty((N, K), device=dev, dtype=dtype)
    with torch.cuda.device(dev):
        st = L.lib().spectra_w4a16_dequant(
            packed.data_ptr(), packed.stride(0),
            scales.data_ptr(), scales.stride(0), scales.stride(1),
            zeros.data_ptr(), zeros.stride(0), zeros.stride(1),
            out.data_ptr(), _dt(out), out.stride(0),
            N, K, L.LAYOUT_MARLIN if marlin_layout else L.LAYOUT_EVEN_ODD, _stream(dev))
    L.check("spectra_w4a16_dequant", st)
    return out


# ---------------------------------------------------------------------------
# Operators around the linear path: rotation prologue, embedding gather,
# greedy argmax (csrc/fwht.cu, csrc/embed.cu)
# ---------------------------------------------------------------------------

def fwht(x: torch.Tensor, normalize: bool = True, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Walsh-Hadamard transform of the rows of ``x`` [..., n] on the GPU (the
    reference's fast_walsh_hadamard_transform, spectra/compressor.py:29-42):
    butterflies in fp32, divided by sqrt(n) if ``normalize``, rounded once to
    ``out_dtype`` (default: x's dtype).  n must be a power of two <= 32768."""
    _require_cuda("x", x, x.device)
    n = x.shape[-1]
    x2 = x.reshape(-1, n)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    y = torch.empty(x2.shape, dtype=out_dtype or x.dtype, device=x.device)
    with torch.cuda.device(x.device):
        st = L.lib().spectra_fwht(x2.data_ptr(), _dt(x2), x2.stride(0), y.data_ptr(), _dt(y), y.stride(0),
                                  x2.shape[0], n, int(normalize), _stream(x.device))
    L.check("spectra_fwht", st)
    return y.reshape(x.shape)


def embedding(input_ids: torch.Tensor, packed_w: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
              outlier_idx: Optional[torch.Tensor] = None, outlier_w: Optional[torch.Tensor] = None,
              marlin_layout: bool = False, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Gather-dequantise the rows ``input_ids`` of a quantised [V, K] matrix
    (SpectraFusedEmbedding.forward, spectra/engine.py:167-212): exact
    ``(q - z) * s`` rounded once to ``out_dtype``, outlier columns restored from
    ``outlier_w``.  ``zeros`` may be unpacked [V, K/32] or packed two per byte."""
    dev = packed_w.device
    for name, t in (("input_ids", input_ids), ("packed_w", packed_w), ("scales", scales), ("zeros", zeros),
                    ("outlier_idx", outlier_idx), ("outlier_w", outlier_w)):
        _require_cuda(name, t, dev)
    packed, scales, zeros = _weights(packed_w, scales, zeros)
    V, K = packed.shape[0], packed.shape[1] * 2
    G = K // 32
    zeros_packed = zeros.shape[1] < G
    if scales.stride(1) != 1:
        scales = scales.contiguous()
    if zeros.stride(1) != 1:
        zeros = zeros.contiguous()
    ids = input_ids.reshape(-1)
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.to(torch.int64)
    ids = ids.contiguous()
    idx, ow, n_out = _outliers(outlier_idx, outlier_w, V)
    if ow is not None and ow.stride(1) != 1:
        ow = ow.contiguous()
    out = torch.empty(ids.numel(), K, dtype=out_dtype, device=dev)
    if ids.numel():
        with torch.cuda.device(dev):
            st = L.lib().spectra_w4a16_embedding(
                ids.data_ptr(), _dt(ids), ids.numel(),
                packed.data_ptr(), packed.stride(0), scales.data_ptr(), scales.stride(0),
                zeros.data_ptr(), zeros.stride(0), int(zeros_packed),
                idx.data_ptr() if idx is not None else None, _dt(idx) if idx is not None else 0, n_out,
                ow.data_ptr() if ow is not None else None, _dt(ow) if ow is not None else 0,
                ow.stride(0) if ow is not None else 0,
                out.data_ptr(), _dt(out), out.stride(0), V, K,
                L.LAYOUT_MARLIN if marlin_layout else L.LAYOUT_EVEN_ODD, _stream(dev))
        L.check("spectra_w4a16_embedding", st)
    return out.reshape(tuple(input_ids.shape) + (K,))


def argmax(logits: torch.Tensor, idx_offset: int = 0, with_values: bool = False):
    """Greedy choice over the last dimension of ``logits`` [..., N] (the
    engine's temperature-0 sample_token, spectra/engine.py:1690-1713): int64
    index of the first maximum (NaN counts as the maximum, as torch.argmax)
    plus ``idx_offset``; with ``with_values`` also the maxima as fp32."""
    _require_cuda("logits", logits, logits.device)
    N = logits.shape[-1]
    x2 = logits.reshape(-1, N)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    idx = torch.empty(M, dtype=torch.int64, device=logits.device)
    val = torch.empty(M, dtype=torch.float32, device=logits.device) if with_values else None
    with torch.cuda.device(logits.device):
        st = L.lib().spectra_argmax(x2.data_ptr(), _dt(x2), x2.stride(0), M, N, int(idx_offset), idx.data_ptr(),
                                    val.data_ptr() if val is not None else None, _stream(logits.device))
    L.check("spectra_argmax", st)
    shape = tuple(logits.shape[:-1])
    if with_values:
        return idx.reshape(shape), val.reshape(shape)
    return idx.reshape(shape)


def lm_head_greedy(x: torch.Tensor, packed_w: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                   bias: Optional[torch.Tensor] = None, outlier_idx: Optional[torch.Tensor] = None,
                   outlier_w: Optional[torch.Tensor] = None, marlin_layout: bool = False,
                   out: Optional[torch.Tensor] = None):
    """Greedy decode head at M=1: the lm_head GEMV (logits in x's dtype, as the
    engine's tied head computes them, spectra/engine.py:1124-1168) followed on
    the same stream by the argmax kernel.  Returns (next_token int64 [1], logits)."""
    logits = fused_w4a16_gemv_hdsq(x, packed_w, scales, zeros, bias=bias, outlier_idx=outlier_idx,
                                   outlier_w=outlier_w, out=out, marlin_layout=marlin_layout)
    return argmax(logits.reshape(1, -1)), logits
