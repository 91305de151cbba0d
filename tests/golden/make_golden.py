"""Generate the golden fixtures in this directory from the REFERENCE itself.

Run once, in a container where the reference project (NeuraCryption/SPECTRA)
is importable:

    SPECTRA_REF=/path/to/SPECTRA python tests/golden/make_golden.py

It imports the reference's own ``SpectraCompressor`` (spectra/compressor.py)
and runs the reference's own Triton kernels (spectra/kernels.py) on the CPU
through ``TRITON_INTERPRET=1``.  The outputs are frozen as small .npz/.json
files so the tests (which never read the reference at run time) can pin the
numpy oracle in ``oracle/w4a16.py`` against the reference:

* quant_cases.npz   -- ``_quantize_chunk_group32`` on crafted inputs
                       (constant groups, half-way ties, odd group counts).
* outlier_cases.npz -- ``_isolate_hdsq_outliers`` + ``_compute_group32_quant``.
* kernel_cases.npz  -- reference Triton GEMV / GEMM outputs (Tier B) and the
                       reference test's torch dequant formula (Tier A) on the
                       reference unit-test setup (tests/test_kernels.py:12-41)
                       plus bf16, even-odd, bias and outlier variants.
* config1.json      -- BASELINE config 1 (K=N=2048, seed 0): sha256 of every
                       compressor output and the reference GEMV output.
* fwht_cases.npz    -- the reference's (dead-code) Walsh-Hadamard transform,
                       oracle for the optional rotation prologue.
* kv_cases.npz      -- the INT4 KV-cache quantiser / dequantiser
                       (SpectraGroup32QuantizedLayer, spectra/engine.py:625-671) run on CPU.
* embedding_cases.npz -- the quantised embedding gather (SpectraFusedEmbedding.forward,
                       spectra/engine.py:167-212).
* chunked.json      -- sha256 of the compressor outputs on an N>4096 matrix
                       (the row-chunked code path, spectra/compressor.py:143-156,168-174).

Inputs are drawn with torch's CPU generator so the tests can regenerate the
large ones from their seeds.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
REF = os.environ.get("SPECTRA_REF")
if not REF:
    sys.exit("make_golden.py: set SPECTRA_REF to the root of a NeuraCryption/SPECTRA checkout "
             "(the directory that holds spectra/compressor.py and spectra/kernels.py)")
sys.path.insert(0, REF)

from spectra.compressor import SpectraCompressor  # noqa: E402
import spectra.kernels as RK  # noqa: E402
import triton  # noqa: E402

sys.path.insert(0, str(HERE.parents[1]))
from spectra_b200.synthetic import draw_weight, draw_act  # noqa: E402


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def bits(t: torch.Tensor) -> np.ndarray:
    """fp16/bf16 tensor -> uint16 bit patterns; other dtypes -> numpy."""
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def ref_gemv(x, packed_w, scales, zeros, bias=None, outlier_idx=None, outlier_w=None, marlin=False):
    """The reference wrapper (spectra/kernels.py:132-184) with the autotuner
    bypassed (the interpreter has no driver to autotune on); config
    BLOCK_N=64, BLOCK_K=128 is one of the reference's own autotune configs."""
    if x.ndim == 1:
        x = x.unsqueeze(0)
    B, K = x.shape
    N = packed_w.shape[0]
    out = torch.empty((B, N), dtype=x.dtype)
    has_bias = bias is not None
    has_out = outlier_idx is not None and outlier_w is not None
    n_out = outlier_idx.numel() if has_out else 0
    dummy_idx = torch.empty(0, dtype=torch.int64)
    dummy_w = torch.empty((0, 0), dtype=torch.float16)
    dummy_b = torch.empty(0, dtype=x.dtype)
    RK._fused_w4a16_gemv_hdsq_kernel.fn[(triton.cdiv(N, 64),)](
        x, packed_w, scales, zeros, out,
        bias if has_bias else dummy_b,
        outlier_idx if has_out else dummy_idx,
        outlier_w if has_out else dummy_w,
        x.stride(0), x.stride(1), packed_w.stride(0), packed_w.stride(1),
        scales.stride(0), scales.stride(1), zeros.stride(0), zeros.stride(1),
        out.stride(0), out.stride(1),
        outlier_w.stride(0) if has_out else 0, outlier_w.stride(1) if has_out else 0,
        N=N, K=K, NUM_OUTLIERS=n_out, HAS_BIAS=has_bias, HAS_OUTLIERS=has_out,
        MARLIN_LAYOUT=marlin, IS_BF16=(x.dtype == torch.bfloat16),
        BLOCK_N=64, BLOCK_K=128,
    )
    return out


def unpack_zeros_t(pz: torch.Tensor, K: int) -> torch.Tensor:
    z = torch.empty((pz.shape[0], pz.shape[1] * 2), dtype=torch.uint8)
    z[:, 0::2] = pz & 0x0F
    z[:, 1::2] = (pz >> 4) & 0x0F
    return z[:, : K // 32]


def quant_cases():
    cases = {}
    torch.manual_seed(1)
    cases["randn_16x256"] = torch.randn(16, 256, dtype=torch.float16)
    torch.manual_seed(2)
    cases["small_8x96"] = (torch.randn(8, 96) * 0.02).to(torch.float16)
    cases["const"] = torch.tensor([[2.5] * 32, [-4.25] * 32, [0.0] * 32], dtype=torch.float32)
    torch.manual_seed(3)
    mixed = torch.randn(2, 64)
    mixed[0, :32] = 1.0
    mixed[1, 32:] = -0.75
    cases["mixed_const"] = mixed
    tie = [0.0, 15.0] + [i + 0.5 for i in range(15)] + [7.5, 6.5, 0.5, 1.5, 2.5, 3.5, 4.5, 5.5, 8.5, 9.5, 10.5, 11.5, 12.5, 13.5, 14.5]
    cases["ties"] = torch.tensor([tie], dtype=torch.float32)
    cases["heavy_t_32x128"] = draw_weight(32, 128, seed=3, dist="t3")
    out = {}
    for name, w in cases.items():
        p, s, z = SpectraCompressor._quantize_chunk_group32(w.clone())
        out[f"{name}/w"] = bits(w) if w.dtype != torch.float32 else w.numpy()
        out[f"{name}/w_dtype"] = np.array(str(w.dtype).replace("torch.", ""))
        out[f"{name}/packed"] = p.numpy()
        out[f"{name}/scales"] = bits(s)
        out[f"{name}/packed_zeros"] = z.numpy()
    np.savez_compressed(HERE / "quant_cases.npz", **out)


def outlier_cases():
    comp = SpectraCompressor()
    specs = [
        ("n01_128x256", 128, 256, 4, "n1", False),
        ("n002_96x512", 96, 512, 5, "n002", False),
        ("t3_64x1024", 64, 1024, 6, "t3", False),
        ("gamma_128x256", 128, 256, 7, "n002", True),
    ]
    out = {}
    for name, N, K, seed, dist, use_gamma in specs:
        w = draw_weight(N, K, seed=seed, dist=dist)
        gamma = None
        if use_gamma:
            torch.manual_seed(seed + 100)
            gamma = torch.rand(K) * 2.0
        w_dense, idx, ow, ratio, kurt = comp._isolate_hdsq_outliers(w, norm_vector=gamma)
        p, s, z = SpectraCompressor._compute_group32_quant(w_dense)
        out[f"{name}/w"] = bits(w)
        if gamma is not None:
            out[f"{name}/gamma"] = gamma.numpy()
        out[f"{name}/idx"] = idx.numpy()
        out[f"{name}/ow"] = bits(ow)
        out[f"{name}/ratio"] = np.array(ratio)
        out[f"{name}/kurtosis"] = np.array(kurt)
        out[f"{name}/packed"] = p.numpy()
        out[f"{name}/scales"] = bits(s)
        out[f"{name}/packed_zeros"] = z.numpy()
    np.savez_compressed(HERE / "outlier_cases.npz", **out)


def chunked_case():
    comp = SpectraCompressor()
    N, K, seed = 4160, 64, 8
    w = draw_weight(N, K, seed=seed, dist="n002")
    w_dense, idx, ow, ratio, kurt = comp._isolate_hdsq_outliers(w)
    assert w_dense is None
    p, s, z = SpectraCompressor._compute_group32_quant(w, outlier_idx=idx)
    rec = {"N": N, "K": K, "seed": seed, "dist": "n002", "n_out": int(idx.numel()),
           "ratio": ratio, "kurtosis": kurt, "idx": idx.tolist(),
           "sha_packed": sha(p), "sha_scales": sha(s), "sha_packed_zeros": sha(z), "sha_ow": sha(ow)}
    (HERE / "chunked.json").write_text(json.dumps(rec, indent=1))


def kernel_cases():
    """Reference unit-test setup (tests/test_kernels.py:12-41) on the CPU generator."""
    N, K, n_out = 128, 256, 16
    torch.manual_seed(42)
    w = torch.randn(N, K, dtype=torch.float16)
    idx = torch.randperm(K)[:n_out]
    ow = w[:, idx].clone()
    p, s, pz = SpectraCompressor._compute_group32_quant(w, outlier_idx=idx)
    zc = unpack_zeros_t(pz, K)
    # Tier A: the reference test's torch dequant formula (tests/test_kernels.py:31-39)
    low = (p & 0x0F).float()
    high = ((p >> 4) & 0x0F).float()
    uq = torch.cat([low.reshape(N, K // 32, 16), high.reshape(N, K // 32, 16)], dim=-1)
    w_deq32 = ((uq - zc.unsqueeze(-1).float()) * s.unsqueeze(-1).float()).reshape(N, K)
    out = {"w": bits(w), "idx": idx.numpy(), "ow": bits(ow), "packed": p.numpy(), "scales": bits(s),
           "packed_zeros": pz.numpy(), "zeros": zc.contiguous().numpy(), "w_deq_f32": w_deq32.numpy()}
    torch.manual_seed(43)
    bias_f16 = torch.randn(N, dtype=torch.float16)
    out["bias_f16"] = bits(bias_f16)
    out["bias_bf16"] = bits(bias_f16.to(torch.bfloat16))
    ow_bf16 = ow.to(torch.bfloat16)
    out["ow_bf16"] = bits(ow_bf16)

    def xs(m, dtype, seed):
        return draw_act(m, K, seed=seed, dtype=dtype)

    # GEMV cases
    gv = [
        ("gemv_f16_marlin", torch.float16, True, False, False, 100),
        ("gemv_f16_marlin_out_bias", torch.float16, True, True, True, 101),
        ("gemv_bf16_marlin_out_bias", torch.bfloat16, True, True, True, 102),
        ("gemv_bf16_evenodd_out", torch.bfloat16, False, True, False, 103),
        ("gemv_f16_evenodd", torch.float16, False, False, False, 104),
    ]
    for name, dt, marlin, use_out, use_bias, seed in gv:
        x = xs(1, dt, seed)
        bias = (bias_f16 if dt == torch.float16 else bias_f16.to(torch.bfloat16)) if use_bias else None
        o_w = (ow if dt == torch.float16 else ow_bf16) if use_out else None
        y = ref_gemv(x, p, s, zc, bias=bias, outlier_idx=idx if use_out else None,
                     outlier_w=o_w, marlin=marlin)
        out[f"{name}/x"] = bits(x)
        out[f"{name}/y"] = bits(y)
        print(name, "done", flush=True)
    # GEMM cases
    gm = [
        ("gemm_f16_marlin_m1", torch.float16, True, False, 1, 200),
        ("gemm_f16_marlin_m2", torch.float16, True, False, 2, 201),
        ("gemm_f16_marlin_m4", torch.float16, True, False, 4, 202),
        ("gemm_f16_marlin_m8", torch.float16, True, False, 8, 203),
        ("gemm_f16_marlin_m4_out", torch.float16, True, True, 4, 204),
        ("gemm_bf16_marlin_m16_out", torch.bfloat16, True, True, 16, 205),
        ("gemm_bf16_evenodd_m3_out", torch.bfloat16, False, True, 3, 206),
        ("gemm_f16_marlin_m17", torch.float16, True, False, 17, 207),
    ]
    for name, dt, marlin, use_out, m, seed in gm:
        a = xs(m, dt, seed)
        o_w = (ow if dt == torch.float16 else ow_bf16) if use_out else None
        if dt == torch.float16:
            # Tier B: the reference Triton kernel itself
            c = RK.batched_w4a16_gemm(a, p, s, zc, outlier_idx=idx if use_out else None,
                                      outlier_w=o_w, marlin_layout=marlin)
            tier = "B"
        else:
            # Triton 3.6's interpreter returns garbage for bf16 tl.dot (fp16 is
            # exact), so bf16 is pinned with Tier A: the reference test's torch
            # dequant formula (tests/test_kernels.py:31-39) with the kernel's
            # operand rounding to bf16 (spectra/kernels.py:256-258,274-276,315-317)
            # and fp32 accumulation.
            if marlin:
                wq = w_deq32
            else:
                ev = torch.stack([low, high], dim=-1).reshape(N, K // 32, 32)
                wq = ((ev - zc.unsqueeze(-1).float()) * s.unsqueeze(-1).float()).reshape(N, K)
            c = a.float() @ wq.to(torch.bfloat16).float().t()
            if use_out:
                c = c + a[:, idx].float() @ o_w.to(torch.bfloat16).float().t()
            c = c.to(torch.bfloat16)
            tier = "A"
        out[f"{name}/a"] = bits(a)
        out[f"{name}/c"] = bits(c)
        out[f"{name}/tier"] = np.array(tier)
        print(name, "done", flush=True)
    np.savez_compressed(HERE / "kernel_cases.npz", **out)


def fwht_cases():
    """The reference's (unused) ``fast_walsh_hadamard_transform`` (spectra/compressor.py:29-42)."""
    from spectra.compressor import fast_walsh_hadamard_transform
    out = {}
    for d in (1, 2, 32, 128, 1024):
        torch.manual_seed(300 + d)
        x = torch.randn(3, d, dtype=torch.float32)
        out[f"d{d}/x"] = x.numpy()
        out[f"d{d}/y"] = fast_walsh_hadamard_transform(x).numpy()
        out[f"d{d}/y_raw"] = fast_walsh_hadamard_transform(x, normalize=False).numpy()
    np.savez_compressed(HERE / "fwht_cases.npz", **out)


def config1():
    """K=N=2048, weights N(0,0.02) fp16 seed 0, x N(0,1) fp16, M=1."""
    comp = SpectraCompressor()
    N = K = 2048
    w = draw_weight(N, K, seed=0, dist="n002")
    w_dense, idx, ow, ratio, kurt = comp._isolate_hdsq_outliers(w)
    p, s, pz = SpectraCompressor._compute_group32_quant(w_dense)
    zc = unpack_zeros_t(pz, K)
    x = draw_act(1, K, seed=1, dtype=torch.float16)
    y = ref_gemv(x, p, s, zc, outlier_idx=idx.long(), outlier_w=ow, marlin=True)
    rec = {"N": N, "K": K, "seed": 0, "dist": "n002", "x_seed": 1, "n_out": int(idx.numel()),
           "ratio": ratio, "kurtosis": kurt, "idx": idx.tolist(),
           "sha_packed": sha(p), "sha_scales": sha(s), "sha_packed_zeros": sha(pz), "sha_ow": sha(ow),
           "y_bits": bits(y).reshape(-1).tolist()}
    (HERE / "config1.json").write_text(json.dumps(rec))


def kv_cases():
    """The reference's INT4 KV-cache quantiser / dequantiser
    (SpectraGroup32QuantizedLayer._quantize / _dequantize, spectra/engine.py:625-671),
    run here on the CPU, on bf16 and fp16 key-like tensors (D = 64, 128, and 80,
    which needs zero padding), including constant and all-zero rows."""
    from spectra.engine import SpectraGroup32QuantizedLayer as QL

    class _Holder:  # the two methods only read group_size
        group_size = 32

    h = _Holder()
    out = {}
    for name, shape, dt in (("bf16_d64", (2, 4, 9, 64), torch.bfloat16), ("bf16_d128", (1, 2, 5, 128), torch.bfloat16),
                            ("f16_d64", (1, 3, 7, 64), torch.float16), ("bf16_d80", (2, 2, 3, 80), torch.bfloat16)):
        torch.manual_seed(700 + shape[-1] + len(name))
        t = (torch.randn(*shape) * 1.5).to(dt)
        flat = t.reshape(-1, shape[-1])
        flat[0] = 0.0
        flat[1] = 0.75
        flat[2, :32] = -2.0
        packed, scales, zeros, orig_shape, pad = QL._quantize(h, t)
        deq = QL._dequantize(h, (packed, scales, zeros, orig_shape, pad))
        out[f"{name}/t"] = bits(t)
        out[f"{name}/dtype"] = np.array("bf16" if dt == torch.bfloat16 else "f16")
        out[f"{name}/packed"] = packed.numpy()
        out[f"{name}/scales"] = bits(scales)
        out[f"{name}/zeros"] = zeros.numpy()
        out[f"{name}/pad"] = np.array(pad)
        out[f"{name}/deq"] = bits(deq)
    np.savez_compressed(HERE / "kv_cases.npz", **out)


def embedding_cases():
    """The reference's quantised embedding gather (SpectraFusedEmbedding.forward,
    spectra/engine.py:167-212) on compressor output for a small vocabulary,
    Marlin and even-odd orders, unpacked and packed zero points, bf16 and fp16
    targets, repeated token ids."""
    from spectra.engine import SpectraFusedEmbedding
    comp = SpectraCompressor()
    V, K = 300, 256
    w = draw_weight(V, K, seed=41, dist="t3")
    w_dense, idx, ow, ratio, kurt = comp._isolate_hdsq_outliers(w)
    p, s, pz = SpectraCompressor._compute_group32_quant(w_dense)
    zc = unpack_zeros_t(pz, K)
    ids = torch.tensor([[0, 5, 5, 299], [17, 128, 3, 250]], dtype=torch.int64)
    out = {"packed": p.numpy(), "scales": bits(s), "packed_zeros": pz.numpy(), "zeros": zc.numpy(),
           "idx": idx.long().numpy(), "ow": bits(ow), "ids": ids.numpy()}
    for tag, marlin, zeros, tdt in (("marlin_unpacked_bf16", True, zc, torch.bfloat16),
                                    ("marlin_packed_f16", True, pz, torch.float16),
                                    ("evenodd_unpacked_bf16", False, zc, torch.bfloat16)):
        emb = SpectraFusedEmbedding(V, K, marlin_layout=marlin)
        emb.set_weights(p, s, zeros, outlier_idx=idx.long(), outlier_weight=ow, marlin_layout=marlin)
        emb.target_dtype = tdt
        out[f"{tag}/y"] = bits(emb(ids))
    np.savez_compressed(HERE / "embedding_cases.npz", **out)


if __name__ == "__main__":
    which = sys.argv[1:] or ["quant", "outlier", "chunked", "kernel", "config1", "fwht", "kv", "embedding"]
    if "quant" in which:
        quant_cases()
    if "outlier" in which:
        outlier_cases()
    if "chunked" in which:
        chunked_case()
    if "kernel" in which:
        kernel_cases()
    if "config1" in which:
        config1()
    if "fwht" in which:
        fwht_cases()
    if "kv" in which:
        kv_cases()
    if "embedding" in which:
        embedding_cases()
    print("golden fixtures written to", HERE)
