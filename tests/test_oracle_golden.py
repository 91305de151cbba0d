"""Pin the numpy oracle (oracle/w4a16.py) against fixtures produced by the
reference itself (tests/golden/make_golden.py).  CPU only."""
import hashlib
import json

import numpy as np
import pytest
import torch

from oracle import w4a16 as O
from spectra_b200.synthetic import draw_act, draw_weight


def _npz(golden_dir, name):
    return np.load(golden_dir / name, allow_pickle=False)


def _w_from_fixture(d, name):
    w = d[f"{name}/w"]
    dt = str(d[f"{name}/w_dtype"]) if f"{name}/w_dtype" in d else "float16"
    if dt == "float16":
        return w.view(np.float16)
    if dt == "bfloat16":
        return O.bf16_bits_to_f32(w)
    return w.astype(np.float32)


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _cases(d):
    return sorted({k.split("/")[0] for k in d.files})


# --------------------------------------------------------------------------
# quantiser: bit-exact with SpectraCompressor._quantize_chunk_group32
# --------------------------------------------------------------------------

def test_quantizer_bit_exact(golden_dir):
    d = _npz(golden_dir, "quant_cases.npz")
    names = _cases(d)
    assert {"const", "ties", "small_8x96", "mixed_const"} <= set(names)
    for name in names:
        w = _w_from_fixture(d, name)
        p, s, z = O.quantize_chunk_group32(w)
        np.testing.assert_array_equal(p, d[f"{name}/packed"], err_msg=name)
        np.testing.assert_array_equal(s.view(np.uint16), d[f"{name}/scales"], err_msg=name)
        np.testing.assert_array_equal(z, d[f"{name}/packed_zeros"], err_msg=name)


def test_constant_groups_round_trip(golden_dir):
    """Reference tests/test_quantizer.py:19-55: constant groups dequantise exactly."""
    for v in (2.5, -4.25, 0.0):
        w = np.full((1, 32), v, np.float32)
        p, s, z = O.quantize_chunk_group32(w)
        deq = O.dequant_f32(p, s, O.unpack_zeros(z, 32), marlin=True)
        assert np.max(np.abs(deq - w)) < 1e-4


def test_group_size_contract():
    with pytest.raises(ValueError):
        O.quantize_chunk_group32(np.zeros((1, 48), np.float32))


# --------------------------------------------------------------------------
# outlier isolation + full compressor output
# --------------------------------------------------------------------------

def test_outlier_isolation_matches_reference(golden_dir):
    d = _npz(golden_dir, "outlier_cases.npz")
    for name in _cases(d):
        w = d[f"{name}/w"].view(np.float16)
        gamma = d[f"{name}/gamma"] if f"{name}/gamma" in d else None
        idx, ow, ratio, kurt = O.isolate_outliers(w, gamma)
        np.testing.assert_array_equal(idx, d[f"{name}/idx"], err_msg=name)
        np.testing.assert_array_equal(ow.view(np.uint16), d[f"{name}/ow"], err_msg=name)
        assert ratio == pytest.approx(float(d[f"{name}/ratio"]), rel=1e-6)
        assert kurt == pytest.approx(float(d[f"{name}/kurtosis"]), rel=1e-4)
        p, s, z = O.compute_group32_quant(w, idx)
        np.testing.assert_array_equal(p, d[f"{name}/packed"], err_msg=name)
        np.testing.assert_array_equal(s.view(np.uint16), d[f"{name}/scales"], err_msg=name)
        np.testing.assert_array_equal(z, d[f"{name}/packed_zeros"], err_msg=name)


def test_outlier_columns_dequantise_to_zero(golden_dir):
    d = _npz(golden_dir, "outlier_cases.npz")
    name = "n01_128x256"
    w = d[f"{name}/w"].view(np.float16)
    c = O.compress_linear(w)
    deq = O.dequant_f32(c["packed"], c["scales"], c["zeros"], marlin=True)
    assert np.all(deq[:, c["outlier_idx"]] == 0.0)


def test_row_chunked_path_matches_reference(golden_dir):
    rec = json.loads((golden_dir / "chunked.json").read_text())
    w = draw_weight(rec["N"], rec["K"], seed=rec["seed"], dist=rec["dist"]).numpy()
    idx, ow, ratio, kurt = O.isolate_outliers(w)
    assert idx.tolist() == rec["idx"]
    p, s, z = O.compute_group32_quant(w, idx)
    assert _sha(p) == rec["sha_packed"]
    assert _sha(s) == rec["sha_scales"]
    assert _sha(z) == rec["sha_packed_zeros"]
    assert _sha(ow) == rec["sha_ow"]


def test_config1_compressor_and_gemv(golden_dir):
    """BASELINE config 1 (K=N=2048): every compressor output is byte-identical
    to the reference's, and the oracle GEMV agrees with the reference's own
    Triton GEMV within the path's tolerance."""
    rec = json.loads((golden_dir / "config1.json").read_text())
    N, K = rec["N"], rec["K"]
    w = draw_weight(N, K, seed=rec["seed"], dist=rec["dist"]).numpy()
    c = O.compress_linear(w)
    assert c["outlier_idx"].tolist() == rec["idx"]
    assert _sha(c["packed"]) == rec["sha_packed"]
    assert _sha(c["scales"]) == rec["sha_scales"]
    assert _sha(c["packed_zeros"]) == rec["sha_packed_zeros"]
    assert _sha(c["outlier_w"]) == rec["sha_ow"]
    x = draw_act(1, K, seed=rec["x_seed"], dtype=torch.float16).numpy()
    y_exact, y_r, od = O.gemv(x, "f16", c["packed"], c["scales"], c["zeros"],
                              outlier_idx=c["outlier_idx"], outlier_w=c["outlier_w"], ow_dtype="f16",
                              marlin=True)
    y_ref = np.array(rec["y_bits"], np.uint16).view(np.float16).astype(np.float64)
    tol = 1e-2 * np.max(np.abs(y_ref))
    assert np.max(np.abs(y_exact - y_ref)) <= tol
    # the reference's fp32 result, rounded once to fp16, is within 1 fp16 ulp of ours
    ulp = np.spacing(np.abs(y_ref).astype(np.float16)).astype(np.float64)
    assert np.all(np.abs(y_r - y_ref) <= ulp)


# --------------------------------------------------------------------------
# dequant + kernels vs the reference's Triton kernels (Tier B) and its test formula (Tier A)
# --------------------------------------------------------------------------

def _kc(golden_dir):
    return _npz(golden_dir, "kernel_cases.npz")


def test_dequant_bit_exact_vs_reference_formula(golden_dir):
    d = _kc(golden_dir)
    deq = O.dequant_f32(d["packed"], d["scales"].view(np.float16), d["zeros"], marlin=True)
    np.testing.assert_array_equal(deq.view(np.uint32), d["w_deq_f32"].view(np.uint32))


def _act(d, key, dtype):
    v = d[key]
    return v if dtype == "bf16" else v.view(np.float16)


def _ulp(v, dtype):
    """Spacing of the output dtype at |v| (fp16: 10 mantissa bits, bf16: 7)."""
    v = np.abs(np.asarray(v, np.float64))
    e = np.floor(np.log2(np.maximum(v, 1e-30)))
    mant = 10 if dtype == "f16" else 7
    lo = -24.0 if dtype == "f16" else -133.0
    return np.exp2(np.maximum(e - mant, lo))


def _out_f64(v, dtype):
    return O.bf16_bits_to_f32(v).astype(np.float64) if dtype == "bf16" else v.view(np.float16).astype(np.float64)


GEMV_CASES = [
    ("gemv_f16_marlin", "f16", True, False, False),
    ("gemv_f16_marlin_out_bias", "f16", True, True, True),
    ("gemv_bf16_marlin_out_bias", "bf16", True, True, True),
    ("gemv_bf16_evenodd_out", "bf16", False, True, False),
    ("gemv_f16_evenodd", "f16", False, False, False),
]


@pytest.mark.parametrize("name,dt,marlin,use_out,use_bias", GEMV_CASES)
def test_oracle_gemv_vs_reference_triton(golden_dir, name, dt, marlin, use_out, use_bias):
    d = _kc(golden_dir)
    x = _act(d, f"{name}/x", dt)
    bias = (d["bias_bf16"] if dt == "bf16" else d["bias_f16"].view(np.float16)) if use_bias else None
    ow = (d["ow_bf16"] if dt == "bf16" else d["ow"].view(np.float16)) if use_out else None
    y_exact, y_r, od = O.gemv(x, dt, d["packed"], d["scales"].view(np.float16), d["zeros"],
                              bias=bias, bias_dtype=dt, outlier_idx=d["idx"] if use_out else None,
                              outlier_w=ow, ow_dtype=dt, marlin=marlin)
    y_ref = _out_f64(d[f"{name}/y"], od)
    assert np.max(np.abs(y_exact - y_ref)) <= 1e-2 * np.max(np.abs(y_ref))
    # both round an (almost) exact fp32 sum once: at most one output ulp apart
    assert np.all(np.abs(y_r - y_ref) <= _ulp(y_ref, od))
    if dt == "f16":
        assert np.max(np.abs(y_exact - y_ref)) <= 0.05  # reference test tolerance (tests/test_kernels.py:49)


GEMM_CASES = [
    ("gemm_f16_marlin_m1", "f16", True, False),
    ("gemm_f16_marlin_m2", "f16", True, False),
    ("gemm_f16_marlin_m4", "f16", True, False),
    ("gemm_f16_marlin_m8", "f16", True, False),
    ("gemm_f16_marlin_m4_out", "f16", True, True),
    ("gemm_bf16_marlin_m16_out", "bf16", True, True),
    ("gemm_bf16_evenodd_m3_out", "bf16", False, True),
    ("gemm_f16_marlin_m17", "f16", True, False),
]


@pytest.mark.parametrize("name,dt,marlin,use_out", GEMM_CASES)
def test_oracle_gemm_vs_reference_triton(golden_dir, name, dt, marlin, use_out):
    d = _kc(golden_dir)
    a = _act(d, f"{name}/a", dt)
    ow = (d["ow_bf16"] if dt == "bf16" else d["ow"].view(np.float16)) if use_out else None
    c_exact, c_r, cd = O.gemm(a, dt, d["packed"], d["scales"].view(np.float16), d["zeros"],
                              outlier_idx=d["idx"] if use_out else None, outlier_w=ow, ow_dtype=dt,
                              marlin=marlin)
    c_ref = _out_f64(d[f"{name}/c"], cd).reshape(c_exact.shape)
    err = np.max(np.abs(c_exact - c_ref))
    assert err <= 1e-2 * np.max(np.abs(c_ref))
    assert np.all(np.abs(c_r - c_ref) <= _ulp(c_ref, cd))
    if dt == "f16":
        assert err <= 0.05  # reference test tolerance (tests/test_kernels.py:58)


def test_fwht_matches_reference(golden_dir):
    d = _npz(golden_dir, "fwht_cases.npz")
    for dim in (1, 2, 32, 128, 1024):
        x = d[f"d{dim}/x"]
        np.testing.assert_allclose(O.fwht(x), d[f"d{dim}/y"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(O.fwht(x, normalize=False), d[f"d{dim}/y_raw"], rtol=1e-5, atol=1e-4)


def test_bf16_rounding_helpers():
    x = np.array([1.0, 1.00390625, 1.005859375, -3.3, 65504.0, 1e-40, np.inf], np.float32)
    t = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(O.f32_to_bf16_bits(x), t)
    np.testing.assert_array_equal(O.bf16_bits_to_f32(t), torch.from_numpy(t.view(np.int16)).view(torch.bfloat16).float().numpy())
