"""The reference's operator modules on this package's kernels.

``SpectraFusedLinear`` and ``SpectraFusedEmbedding`` keep the constructor,
``set_weights`` and ``forward`` contracts of the reference classes
(spectra/engine.py:35-124 and :127-212): the linear routes a single token to
the M=1 GEMV with the bias fused, everything else to the tensor-core GEMM
followed by the bias add, and returns the input's dtype; the embedding
gathers and dequantises only the rows of the requested token ids.  They exist
for hosts that build their own model (the reference engine's loader binds its
own classes, which run on these kernels through ``spectra.kernels``).

``quantize_model`` replaces every ``nn.Linear`` / ``nn.Embedding`` of a model
whose input width is a multiple of 32 with these modules, compressing the
module's current weights on the GPU with the reference compressor's algorithm
(``spectra_b200.compress``), as the reference container does for every 2-D
weight (spectra/compressor.py:472-483), and ties the output head to the
embedding when the model ties them (spectra/engine.py:1124-1168).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import compress as C
from . import kernels as SK


class SpectraFusedLinear(nn.Module):
    """W4A16 linear layer (spectra/engine.py:35-124) on the CUDA kernels."""

    def __init__(self, in_features: int, out_features: int, group_size: int = 32, has_bias: bool = False,
                 enable_hdsq: bool = True, marlin_layout: bool = False):
        super().__init__()
        if group_size != 32:
            raise ValueError("SPECTRA's format uses groups of 32 input features")
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size
        self.enable_hdsq = enable_hdsq
        self.marlin_layout = marlin_layout
        self.register_buffer("packed_weight", None)
        self.register_buffer("scales", None)
        self.register_buffer("zeros", None)
        self.register_buffer("outlier_idx", None)
        self.register_buffer("outlier_weight", None)
        if has_bias:
            self.register_parameter("bias", nn.Parameter(torch.zeros(out_features, dtype=torch.bfloat16)))
        else:
            self.register_parameter("bias", None)

    def set_weights(self, packed_w, scales, zeros, bias=None, outlier_idx=None, outlier_weight=None,
                    marlin_layout: bool = False):
        self.packed_weight = packed_w
        self.scales = scales
        self.zeros = zeros
        self.marlin_layout = marlin_layout
        if bias is not None:
            self.bias = nn.Parameter(bias, requires_grad=False)
        if outlier_idx is not None and outlier_weight is not None:
            self.enable_hdsq = True
            self.outlier_idx = outlier_idx
            self.outlier_weight = outlier_weight

    @torch.compiler.disable
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        orig_shape = x.shape
        in_dtype = x.dtype
        total = x.numel() // self.in_features
        oidx = self.outlier_idx if self.enable_hdsq else None
        ow = self.outlier_weight if self.enable_hdsq else None
        if total == 1:
            y = SK.fused_w4a16_gemv_hdsq(x.reshape(1, self.in_features), self.packed_weight, self.scales,
                                         self.zeros, bias=self.bias, outlier_idx=oidx, outlier_w=ow,
                                         marlin_layout=self.marlin_layout)
            return y.view(orig_shape[:-1] + (self.out_features,)).to(in_dtype)
        y = SK.batched_w4a16_gemm(x.reshape(total, self.in_features), self.packed_weight, self.scales, self.zeros,
                                  outlier_idx=oidx, outlier_w=ow, marlin_layout=self.marlin_layout)
        if self.bias is not None:
            y = y + self.bias
        return y.reshape(orig_shape[:-1] + (self.out_features,)).to(in_dtype)


class SpectraFusedEmbedding(nn.Module):
    """Quantised token embedding (spectra/engine.py:127-212) on the gather kernel."""

    def __init__(self, num_embeddings: int, embedding_dim: int, group_size: int = 32, marlin_layout: bool = False):
        super().__init__()
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.group_size = group_size
        self.marlin_layout = marlin_layout
        self.target_dtype: Optional[torch.dtype] = None
        self.register_buffer("packed_weight", None)
        self.register_buffer("scales", None)
        self.register_buffer("zeros", None)
        self.register_buffer("outlier_idx", None)
        self.register_buffer("outlier_weight", None)
        self._dummy_param = nn.Parameter(torch.empty(0), requires_grad=False)

    @property
    def weight(self):
        return self._dummy_param

    def set_weights(self, packed_w, scales, zeros, outlier_idx=None, outlier_weight=None, marlin_layout: bool = False):
        self.packed_weight = packed_w
        self.scales = scales
        self.zeros = zeros
        self.outlier_idx = outlier_idx
        self.outlier_weight = outlier_weight
        self.marlin_layout = marlin_layout

    @torch.compiler.disable
    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        target = self.target_dtype or (self.outlier_weight.dtype if self.outlier_weight is not None
                                       else self.scales.dtype)
        return SK.embedding(input_ids, self.packed_weight, self.scales, self.zeros, outlier_idx=self.outlier_idx,
                            outlier_w=self.outlier_weight, marlin_layout=self.marlin_layout, out_dtype=target)


def _compressed(weight: torch.Tensor):
    w = weight.detach()
    c = C.compress_linear(w if w.dtype in (torch.float16, torch.bfloat16) else w.to(torch.float16))
    return c


@torch.no_grad()
def quantize_model(model: nn.Module, target_dtype: torch.dtype = torch.bfloat16, skip=()) -> nn.Module:
    """Replace the model's linears and embeddings (input width a multiple of 32)
    with SPECTRA-format modules holding GPU-compressed copies of their weights;
    the dense weights are released as each module is replaced."""
    tied = bool(getattr(getattr(model, "config", None), "tie_word_embeddings", False))
    targets = []
    for name, mod in model.named_modules():
        for cname, child in mod.named_children():
            full = f"{name}.{cname}" if name else cname
            if full in skip:
                continue
            if isinstance(child, nn.Linear) and child.in_features % 32 == 0:
                targets.append((mod, cname, child))
            elif isinstance(child, nn.Embedding) and child.embedding_dim % 32 == 0:
                targets.append((mod, cname, child))
    emb_new = None
    out_head = model.get_output_embeddings() if hasattr(model, "get_output_embeddings") else None
    for parent, cname, child in targets:
        if tied and child is out_head:
            continue  # bound to the embedding's tensors below
        c = _compressed(child.weight)
        if isinstance(child, nn.Embedding):
            new = SpectraFusedEmbedding(child.num_embeddings, child.embedding_dim, marlin_layout=True)
            new.set_weights(c.packed, c.scales, c.zeros, outlier_idx=c.outlier_idx, outlier_weight=c.outlier_w,
                            marlin_layout=True)
            new.target_dtype = target_dtype
            emb_new = new
        else:
            has_b = child.bias is not None
            new = SpectraFusedLinear(child.in_features, child.out_features, has_bias=has_b, marlin_layout=True)
            new.set_weights(c.packed, c.scales, c.zeros,
                            bias=child.bias.detach().to(target_dtype) if has_b else None,
                            outlier_idx=c.outlier_idx, outlier_weight=c.outlier_w, marlin_layout=True)
        setattr(parent, cname, new)
        del child, c
    if tied and emb_new is not None and out_head is not None:
        head = SpectraFusedLinear(emb_new.embedding_dim, emb_new.num_embeddings, marlin_layout=True)
        head.set_weights(emb_new.packed_weight, emb_new.scales, emb_new.zeros, outlier_idx=emb_new.outlier_idx,
                         outlier_weight=emb_new.outlier_weight, marlin_layout=True)
        if hasattr(model, "lm_head"):
            model.lm_head = head
    torch.cuda.empty_cache()
    return model
