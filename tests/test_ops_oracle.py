"""The oracle of the operators around the linear path (oracle/ops.py) pinned
to the reference's own outputs: the INT4 KV-cache quantiser / dequantiser and
the quantised embedding gather, run by tests/golden/make_golden.py with the
reference imported (CPU)."""
import numpy as np
import pytest

from oracle import ops as P
from oracle import w4a16 as O


def _kv(golden_dir):
    d = np.load(golden_dir / "kv_cases.npz")
    return d, sorted({k.split("/")[0] for k in d.files})


def test_kv_quantize_oracle_matches_reference_cpu_run(golden_dir):
    d, names = _kv(golden_dir)
    assert names
    for name in names:
        dt = str(d[f"{name}/dtype"])
        t = P.to_f32(d[f"{name}/t"], dt)
        # the fixtures were made on the CPU, where torch divides by the scalar 15.0
        packed, scales, zeros, pad = P.kv_quantize(t, dt, scalar_div="true")
        rows = int(np.prod(t.shape[:-1]))
        np.testing.assert_array_equal(packed, d[f"{name}/packed"].reshape(rows, -1, 16), err_msg=name)
        np.testing.assert_array_equal(scales.view(np.uint16).reshape(-1),
                                      d[f"{name}/scales"].reshape(-1), err_msg=name)
        np.testing.assert_array_equal(zeros.reshape(-1), d[f"{name}/zeros"].reshape(-1), err_msg=name)
        assert pad == int(d[f"{name}/pad"])


def test_kv_dequantize_oracle_matches_reference_cpu_run(golden_dir):
    d, names = _kv(golden_dir)
    for name in names:
        D = d[f"{name}/t"].shape[-1]
        rows = int(np.prod(d[f"{name}/t"].shape[:-1]))
        packed = d[f"{name}/packed"].reshape(rows, -1, 16)
        deq = P.kv_dequantize(packed, d[f"{name}/scales"].view(np.float16).reshape(rows, -1),
                              d[f"{name}/zeros"].reshape(rows, -1), D)
        np.testing.assert_array_equal(P.store_bits(deq, "bf16").reshape(-1), d[f"{name}/deq"].reshape(-1),
                                      err_msg=name)


def test_kv_scalar_division_modes_differ_only_in_rare_ties():
    # true division and the fp32-reciprocal multiply give the same codes on
    # almost every group; both are restated because torch uses one on the CPU
    # and the other on a CUDA device.
    rng = np.random.default_rng(0)
    t = P.rnd(rng.normal(size=(512, 128)).astype(np.float32), "bf16")
    a = P.kv_quantize(t, "bf16", "true")
    b = P.kv_quantize(t, "bf16", "reciprocal")
    same = (a[1] == b[1]).mean()
    assert same > 0.9


@pytest.mark.parametrize("tag,marlin,packed_z,dt", [("marlin_unpacked_bf16", True, False, "bf16"),
                                                   ("marlin_packed_f16", True, True, "f16"),
                                                   ("evenodd_unpacked_bf16", False, False, "bf16")])
def test_embedding_oracle_matches_reference(golden_dir, tag, marlin, packed_z, dt):
    d = np.load(golden_dir / "embedding_cases.npz")
    z = d["packed_zeros"] if packed_z else d["zeros"]
    ow = P.to_f32(d["ow"], "f16")
    y = P.embedding(d["ids"], d["packed"], d["scales"].view(np.float16), z, d["idx"], ow, marlin=marlin,
                    out_dtype=dt)
    np.testing.assert_array_equal(y.reshape(-1), d[f"{tag}/y"].reshape(-1))


def test_argmax_oracle_is_first_max_and_nan_first():
    x = np.array([[1.0, 3.0, 3.0, 2.0], [np.nan, 5.0, np.nan, 1.0], [-np.inf, -np.inf, -np.inf, -np.inf]])
    np.testing.assert_array_equal(P.argmax(x), [1, 0, 0])


def test_fwht_oracle_matches_reference(golden_dir):
    d = np.load(golden_dir / "fwht_cases.npz")
    for n in (1, 2, 32, 128, 1024):
        np.testing.assert_allclose(O.fwht(d[f"d{n}/x"]), d[f"d{n}/y"], rtol=1e-5, atol=1e-5)
