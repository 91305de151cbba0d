"""The package's GPU compressor (CUDA quantiser ``spectra_quantize_group32`` and
zero-point unpack ``spectra_unpack_zeros``, csrc/format.cu) against the
reference's own outputs (golden fixtures made by importing the reference
compressor) and the oracle: bit-exact codes, scales, zero points and outlier
sets."""
import hashlib
import json

import numpy as np
import pytest
import torch

from oracle import w4a16 as O
from spectra_b200 import compress as C
from spectra_b200.synthetic import draw_weight

DEV = "cuda"


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def _bits16(t: torch.Tensor) -> np.ndarray:
    return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def test_compressor_has_no_cpu_path():
    w = torch.zeros(4, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        C.quantize_group32(w)
    with pytest.raises(RuntimeError, match="CUDA"):
        C.compress_linear(w)
    with pytest.raises(RuntimeError, match="CUDA"):
        C.unpack_zeros(torch.zeros(4, 1, dtype=torch.uint8), 64)


@pytest.mark.gpu
def test_quantize_matches_reference(golden_dir):
    d = np.load(golden_dir / "quant_cases.npz")
    for name in sorted({k.split("/")[0] for k in d.files}):
        raw = d[f"{name}/w"]
        dt = str(d[f"{name}/w_dtype"])
        w = torch.from_numpy(raw.view(np.float16)) if dt == "float16" else torch.from_numpy(raw.astype(np.float32))
        p, s, z, pz = C.quantize_group32(w.to(DEV))
        np.testing.assert_array_equal(p.cpu().numpy(), d[f"{name}/packed"], err_msg=name)
        np.testing.assert_array_equal(_bits16(s), d[f"{name}/scales"], err_msg=name)
        np.testing.assert_array_equal(pz.cpu().numpy(), d[f"{name}/packed_zeros"], err_msg=name)
        np.testing.assert_array_equal(z.cpu().numpy(), O.unpack_zeros(d[f"{name}/packed_zeros"], w.shape[1]))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("marlin", [True, False])
def test_quantize_dtypes_layouts_and_outlier_columns(dtype, marlin):
    """Any source dtype, both nibble orders, outlier columns read as zero, odd
    group count (K = 5*32), ragged row count: identical to the oracle
    quantiser (spectra/compressor.py:72-156) on the same values."""
    N, K = 37, 160
    w = (torch.randn(N, K, generator=torch.Generator().manual_seed(3)) * 0.02).to(dtype)
    w[3] = 0.5            # constant positive row
    w[4] = -0.25          # constant negative row
    w[5] = 0.0            # all-zero row
    w[6, :32] = 1e-9      # group with a span below 1e-8
    idx = torch.tensor([0, 7, 33, 100, 159], dtype=torch.int64)
    p, s, z, pz = C.quantize_group32(w.to(DEV), idx.to(DEV), marlin_layout=marlin)
    wn = w.float().numpy() if dtype != torch.float16 else w.numpy()
    ep, es, epz = O.compute_group32_quant(wn, idx.numpy())
    if not marlin:  # the oracle packs Marlin order; re-pack its codes even-odd
        q = O.codes(ep, True).reshape(N, K // 32, 32)
        ep = (q[:, :, 0::2] | (q[:, :, 1::2] << 4)).astype(np.uint8).reshape(N, K // 2)
    np.testing.assert_array_equal(p.cpu().numpy(), ep)
    np.testing.assert_array_equal(_bits16(s), es.view(np.uint16))
    np.testing.assert_array_equal(pz.cpu().numpy(), epz)
    np.testing.assert_array_equal(z.cpu().numpy(), O.unpack_zeros(epz, K))


@pytest.mark.gpu
def test_compress_linear_matches_reference(golden_dir):
    d = np.load(golden_dir / "outlier_cases.npz")
    for name in sorted({k.split("/")[0] for k in d.files}):
        w = torch.from_numpy(d[f"{name}/w"].view(np.float16)).to(DEV)
        gamma = torch.from_numpy(d[f"{name}/gamma"]).to(DEV) if f"{name}/gamma" in d else None
        c = C.compress_linear(w, gamma)
        np.testing.assert_array_equal(c.outlier_idx.cpu().numpy(), d[f"{name}/idx"].astype(np.int64), err_msg=name)
        np.testing.assert_array_equal(_bits16(c.outlier_w), d[f"{name}/ow"])
        assert c.ratio == pytest.approx(float(d[f"{name}/ratio"]), rel=1e-6)
        np.testing.assert_array_equal(c.packed.cpu().numpy(), d[f"{name}/packed"], err_msg=name)
        np.testing.assert_array_equal(c.packed_zeros.cpu().numpy(), d[f"{name}/packed_zeros"], err_msg=name)


@pytest.mark.gpu
def test_config1_checksums(golden_dir):
    rec = json.loads((golden_dir / "config1.json").read_text())
    w = draw_weight(rec["N"], rec["K"], seed=rec["seed"], dist=rec["dist"]).to(DEV)
    c = C.compress_linear(w)
    assert c.outlier_idx.tolist() == rec["idx"]
    assert _sha(c.packed) == rec["sha_packed"]
    assert _sha(c.scales) == rec["sha_scales"]
    assert _sha(c.packed_zeros) == rec["sha_packed_zeros"]
    assert _sha(c.outlier_w) == rec["sha_ow"]


@pytest.mark.gpu
def test_row_chunked_norms_path(golden_dir):
    rec = json.loads((golden_dir / "chunked.json").read_text())
    w = draw_weight(rec["N"], rec["K"], seed=rec["seed"], dist=rec["dist"]).to(DEV)
    c = C.compress_linear(w)
    assert c.outlier_idx.tolist() == rec["idx"]
    assert _sha(c.packed) == rec["sha_packed"]
    assert _sha(c.scales) == rec["sha_scales"]


@pytest.mark.gpu
@pytest.mark.parametrize("G", [1, 2, 5, 64, 449])
def test_unpack_zeros_on_gpu(G):
    rng = np.random.default_rng(G)
    pz = rng.integers(0, 256, size=(33, (G + 1) // 2 + 3), dtype=np.uint8)  # wider rows: a strided view
    t = torch.from_numpy(pz).to(DEV)[:, : (G + 1) // 2]
    z = C.unpack_zeros(t, G * 32)
    np.testing.assert_array_equal(z.cpu().numpy(), O.unpack_zeros(pz[:, : (G + 1) // 2], G * 32))
