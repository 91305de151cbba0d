"""The package's device-side compressor against the reference's own outputs
(golden fixtures): bit-exact codes, scales, zero points and outlier sets."""
import hashlib
import json

import numpy as np
import pytest
import torch

from spectra_b200 import compress as C
from spectra_b200.synthetic import draw_weight


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def _dev_params():
    return [pytest.param("cpu")] + [pytest.param("cuda", marks=pytest.mark.gpu)]


@pytest.mark.parametrize("dev", _dev_params())
def test_quantize_matches_reference(golden_dir, dev):
    d = np.load(golden_dir / "quant_cases.npz")
    for name in sorted({k.split("/")[0] for k in d.files}):
        raw = d[f"{name}/w"]
        dt = str(d[f"{name}/w_dtype"])
        w = torch.from_numpy(raw.view(np.float16)) if dt == "float16" else torch.from_numpy(raw.astype(np.float32))
        p, s, z = C.quantize_group32(w.to(dev))
        np.testing.assert_array_equal(p.cpu().numpy(), d[f"{name}/packed"], err_msg=name)
        np.testing.assert_array_equal(s.cpu().view(torch.int16).numpy().view(np.uint16), d[f"{name}/scales"], err_msg=name)
        np.testing.assert_array_equal(z.cpu().numpy(), d[f"{name}/packed_zeros"], err_msg=name)


@pytest.mark.parametrize("dev", _dev_params())
def test_compress_linear_matches_reference(golden_dir, dev):
    d = np.load(golden_dir / "outlier_cases.npz")
    for name in sorted({k.split("/")[0] for k in d.files}):
        w = torch.from_numpy(d[f"{name}/w"].view(np.float16)).to(dev)
        gamma = torch.from_numpy(d[f"{name}/gamma"]).to(dev) if f"{name}/gamma" in d else None
        c = C.compress_linear(w, gamma)
        np.testing.assert_array_equal(c.outlier_idx.cpu().numpy(), d[f"{name}/idx"].astype(np.int64), err_msg=name)
        np.testing.assert_array_equal(c.outlier_w.cpu().view(torch.int16).numpy().view(np.uint16), d[f"{name}/ow"])
        assert c.ratio == pytest.approx(float(d[f"{name}/ratio"]), rel=1e-6)
        np.testing.assert_array_equal(c.packed.cpu().numpy(), d[f"{name}/packed"], err_msg=name)
        np.testing.assert_array_equal(c.packed_zeros.cpu().numpy(), d[f"{name}/packed_zeros"], err_msg=name)


def test_config1_checksums(golden_dir):
    rec = json.loads((golden_dir / "config1.json").read_text())
    w = draw_weight(rec["N"], rec["K"], seed=rec["seed"], dist=rec["dist"])
    c = C.compress_linear(w)
    assert c.outlier_idx.tolist() == rec["idx"]
    assert _sha(c.packed) == rec["sha_packed"]
    assert _sha(c.scales) == rec["sha_scales"]
    assert _sha(c.packed_zeros) == rec["sha_packed_zeros"]
    assert _sha(c.outlier_w) == rec["sha_ow"]


def test_row_chunked_norms_path(golden_dir):
    rec = json.loads((golden_dir / "chunked.json").read_text())
    w = draw_weight(rec["N"], rec["K"], seed=rec["seed"], dist=rec["dist"])
    c = C.compress_linear(w)
    assert c.outlier_idx.tolist() == rec["idx"]
    assert _sha(c.packed) == rec["sha_packed"]
    assert _sha(c.scales) == rec["sha_scales"]


def test_unpack_zeros_round_trip():
    pz = torch.tensor([[0x21, 0x43, 0x05]], dtype=torch.uint8)
    assert C.unpack_zeros(pz, 5 * 32).tolist() == [[1, 2, 3, 4, 5]]
