"""INT4 KV cache on the GPU: the quantise / dequantise pair of the reference's
``SpectraGroup32QuantizedLayer`` (spectra/engine.py:614-671), as CUDA kernels
(csrc/kvcache.cu) behind the same tuple format.

``kv_quantize(t)`` returns ``(packed, scales, zeros, orig_shape, pad)`` exactly
as ``SpectraGroup32QuantizedLayer._quantize`` does (:625-656):
  packed  u8   [rows, G, 16]  even-odd nibbles (element 2i low, 2i+1 high)
  scales  fp16 [rows, G, 1]
  zeros   u8   [rows, G, 1]
  with rows = t.numel() / D, G = ceil(D / 32), pad = G*32 - D (zero padding).
``kv_dequantize(q_tuple)`` inverts it like ``_dequantize`` (:658-671): bf16
values ``(q - z) * s`` with the padding dropped, in ``orig_shape``.

``Group32KVLayer`` is the reference class with its two torch methods replaced
by these kernels, for use where the reference builds its
``SpectraQuantizedCache`` (:710-727).  There is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib as L

GROUP = 32

_DT = {torch.float16: L.DT_F16, torch.bfloat16: L.DT_BF16, torch.float32: L.DT_F32}


def kv_quantize(tensor: torch.Tensor, group_size: int = GROUP):
    """Group-32 INT4 codes of a key/value tensor [..., D] (bf16 or fp16, CUDA)."""
    if group_size != GROUP:
        raise ValueError("the KV cache kernels use groups of 32")
    if not tensor.is_cuda:
        raise RuntimeError(f"spectra_b200.kvcache: tensor must be a CUDA tensor (no CPU path), got {tensor.device}")
    if tensor.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"KV states must be bf16 or fp16, got {tensor.dtype}")
    orig_shape = tensor.shape
    D = orig_shape[-1]
    t = tensor.reshape(-1, D).contiguous()
    rows = t.shape[0]
    pad = (GROUP - D % GROUP) % GROUP
    G = (D + pad) // GROUP
    dev = t.device
    packed = torch.empty(rows, G, 16, dtype=torch.uint8, device=dev)
    scales = torch.empty(rows, G, 1, dtype=torch.float16, device=dev)
    zeros = torch.empty(rows, G, 1, dtype=torch.uint8, device=dev)
    if rows:
        with torch.cuda.device(dev):
            st = L.lib().spectra_kv_quantize(t.data_ptr(), _DT[t.dtype], rows, D, packed.data_ptr(),
                                             scales.data_ptr(), zeros.data_ptr(),
                                             torch.cuda.current_stream(dev).cuda_stream)
        L.check("spectra_kv_quantize", st)
    return packed, scales, zeros, orig_shape, pad


def kv_dequantize(q_tuple, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """bf16 (by default) values of a ``kv_quantize`` tuple in its original shape."""
    if q_tuple is None:
        return torch.tensor([], dtype=out_dtype)
    packed, scales, zeros, orig_shape, pad = q_tuple
    if not packed.is_cuda:
        raise RuntimeError("spectra_b200.kvcache: the quantised tensors must be CUDA tensors (no CPU path)")
    D = orig_shape[-1]
    rows = packed.shape[0]
    packed = packed.contiguous()
    scales = scales.contiguous()
    zeros = zeros.contiguous()
    out = torch.empty(rows, D, dtype=out_dtype, device=packed.device)
    if rows:
        with torch.cuda.device(packed.device):
            st = L.lib().spectra_kv_dequantize(packed.data_ptr(), scales.data_ptr(), zeros.data_ptr(),
                                               out.data_ptr(), _DT[out_dtype], rows, D,
                                               torch.cuda.current_stream(packed.device).cuda_stream)
        L.check("spectra_kv_dequantize", st)
    return out.reshape(orig_shape)


def _quantized_layer_base():
    try:
        from transformers.cache_utils import QuantizedLayer
        return QuantizedLayer
    except ImportError:  # transformers without quantised caches: a plain holder
        return object


class Group32KVLayer(_quantized_layer_base()):
    """The reference's ``SpectraGroup32QuantizedLayer`` (spectra/engine.py:614-671)
    with ``_quantize`` / ``_dequantize`` on the GPU kernels."""

    def __init__(self, group_size: int = GROUP, residual_length: int = 128):
        if type(self).__mro__[1] is not object:
            super().__init__(nbits=4, q_group_size=group_size, residual_length=residual_length)
        self.group_size = group_size

    def _quantize(self, tensor: torch.Tensor, axis: int = 0):
        return kv_quantize(tensor, self.group_size)

    def _dequantize(self, q_tuple):
        return kv_dequantize(q_tuple)
