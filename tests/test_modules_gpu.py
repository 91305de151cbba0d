"""The operator modules of spectra_b200.modules (mirrors of the reference's
SpectraFusedLinear / SpectraFusedEmbedding, spectra/engine.py:35-212) and the
model binder quantize_model: the routing (M=1 GEMV with bias, else GEMM +
bias), dtypes and shapes of the reference classes, and a tiny Llama bound by
quantize_model against the same model with each linear computed by the
reference formula (exact dequant, fp32 matmul, oracle/engine_kernels.py)."""
import numpy as np
import pytest
import torch

from oracle import engine_kernels as EK
from spectra_b200 import compress as C
from spectra_b200.modules import SpectraFusedEmbedding, SpectraFusedLinear, quantize_model
from tests import engine_helpers as H

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _linear(N, K, bias=True, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    c = C.compress_linear(w)
    lin = SpectraFusedLinear(K, N, has_bias=bias, marlin_layout=True).to(DEV)
    b = (torch.randn(N, generator=g, device=DEV) * 0.1).to(torch.bfloat16) if bias else None
    lin.set_weights(c.packed, c.scales, c.zeros, bias=b, outlier_idx=c.outlier_idx, outlier_weight=c.outlier_w,
                    marlin_layout=True)
    return lin, c, b


@pytest.mark.parametrize("shape", [(1, 1, 512), (1, 512), (2, 3, 512), (17, 512)])
def test_fused_linear_routes_like_the_reference(shape):
    lin, c, b = _linear(768, 512, seed=len(shape))
    x = torch.randn(*shape, device=DEV).to(torch.bfloat16)
    y = lin(x)
    assert y.shape == shape[:-1] + (768,) and y.dtype == torch.bfloat16
    M = x.numel() // 512
    x2 = x.reshape(M, 512)
    if M == 1:
        ref = EK.fused_w4a16_gemv_hdsq(x2, c.packed, c.scales, c.zeros, bias=b, outlier_idx=c.outlier_idx,
                                       outlier_w=c.outlier_w, marlin_layout=True)
    else:
        ref = EK.batched_w4a16_gemm(x2, c.packed, c.scales, c.zeros, outlier_idx=c.outlier_idx,
                                    outlier_w=c.outlier_w, marlin_layout=True) + b
    err = float((y.reshape(M, -1).float() - ref.float()).abs().max())
    assert err <= 1e-2 * float(ref.float().abs().max())


def test_fused_embedding_gathers_the_requested_rows():
    g = torch.Generator(device=DEV).manual_seed(3)
    w = (torch.randn(1000, 256, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    c = C.compress_linear(w)
    emb = SpectraFusedEmbedding(1000, 256, marlin_layout=True)
    emb.set_weights(c.packed, c.scales, c.zeros, outlier_idx=c.outlier_idx, outlier_weight=c.outlier_w,
                    marlin_layout=True)
    ids = torch.tensor([[1, 999, 5]], device=DEV)
    out = emb(ids)
    assert out.shape == (1, 3, 256) and out.dtype == torch.bfloat16  # the outlier weights' dtype
    # outlier columns carry the exact source weights
    assert torch.equal(out[0, :, c.outlier_idx], w[ids[0]][:, c.outlier_idx])
    assert float((out[0].float() - w[ids[0]].float()).abs().max()) <= 0.05


def test_quantize_model_binds_a_tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(**H.TINY_CONFIG)
    torch.manual_seed(5)
    with torch.device(DEV):
        dense = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    ids = torch.tensor([H.prompt_ids(3)], device=DEV)
    model = quantize_model(dense)
    lin = [m for m in model.modules() if isinstance(m, SpectraFusedLinear)]
    assert len(lin) == 2 * 7 + 1  # q k v o gate up down per layer, and the tied head
    assert isinstance(model.model.embed_tokens, SpectraFusedEmbedding)
    assert model.lm_head.packed_weight is model.model.embed_tokens.packed_weight  # tied
    with torch.no_grad():
        ours = model(ids).logits.float()
        # the same bound model, each linear by the reference formula instead
        import spectra_b200.modules as Mod
        keep = (Mod.SK.fused_w4a16_gemv_hdsq, Mod.SK.batched_w4a16_gemm)
        try:
            Mod.SK.fused_w4a16_gemv_hdsq, Mod.SK.batched_w4a16_gemm = (EK.fused_w4a16_gemv_hdsq,
                                                                         EK.batched_w4a16_gemm)
            ref = model(ids).logits.float()
        finally:
            Mod.SK.fused_w4a16_gemv_hdsq, Mod.SK.batched_w4a16_gemm = keep
    assert np.isfinite(ours.cpu().numpy()).all()
    assert float((ours - ref).abs().max()) <= 2e-2 * float(ref.abs().max())
