"""GPU parity of the operators around the linear path: the INT4 KV-cache
kernels (csrc/kvcache.cu), the quantised embedding gather and the greedy
argmax (csrc/embed.cu) and the Walsh-Hadamard rotation prologue
(csrc/fwht.cu), against the reference's own outputs (golden fixtures) and the
oracle (oracle/ops.py, oracle/w4a16.py)."""
import numpy as np
import pytest
import torch

from oracle import ops as P
from oracle import w4a16 as O
from spectra_b200 import _lib as L
from spectra_b200 import kernels as SK
from spectra_b200 import kvcache as KV
from tests.helpers import assert_close_to_oracle, compressed, np_of, out_f64

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
TDT = {"bf16": torch.bfloat16, "f16": torch.float16}


def _from_bits(bits: np.ndarray, dt: str) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(TDT[dt])


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


# ---------------------------------------------------------------------------
# INT4 KV cache
# ---------------------------------------------------------------------------

def _torch_kv_quantize(t: torch.Tensor):
    """The reference method's steps (spectra/engine.py:625-656) as torch ops on
    the CUDA device: pins which rounding torch itself uses there."""
    D = t.shape[-1]
    x = t.reshape(-1, D)
    pad = (32 - D % 32) % 32
    if pad:
        x = torch.nn.functional.pad(x, (0, pad))
    xg = x.reshape(x.shape[0], -1, 32)
    lo, hi = xg.amin(-1, keepdim=True), xg.amax(-1, keepdim=True)
    diff = hi - lo
    flat = diff < 1e-8
    s = torch.where(flat, torch.where(lo == 0, torch.ones_like(lo), lo.abs()), diff / 15.0).clamp(min=1e-8)
    z = torch.where(flat, (lo < 0).to(torch.uint8), torch.round(-lo / s).clamp(0, 15).to(torch.uint8))
    q = torch.where(flat, (lo > 0).to(torch.uint8).expand_as(xg),
                    torch.round((xg - (-z.float() * s)) / s).clamp(0, 15).to(torch.uint8))
    return (q[:, :, 0::2] | (q[:, :, 1::2] << 4)).to(torch.uint8), s.to(torch.float16), z


def test_kv_kernels_match_reference_fixtures(golden_dir):
    d = np.load(golden_dir / "kv_cases.npz")
    for name in sorted({k.split("/")[0] for k in d.files}):
        dt = str(d[f"{name}/dtype"])
        t = _from_bits(d[f"{name}/t"], dt).to(DEV)
        packed, scales, zeros, shape, pad = KV.kv_quantize(t)
        assert tuple(shape) == t.shape and pad == int(d[f"{name}/pad"])
        # the kernel follows torch-on-CUDA rounding; the fixtures are a CPU run,
        # so compare with the oracle in each mode and the fixtures where they agree
        tv = P.to_f32(d[f"{name}/t"], dt)
        ep, es, ez, _ = P.kv_quantize(tv, dt, scalar_div="reciprocal")
        np.testing.assert_array_equal(packed.cpu().numpy(), ep, err_msg=name)
        np.testing.assert_array_equal(_bits(scales).reshape(-1), es.view(np.uint16).reshape(-1), err_msg=name)
        np.testing.assert_array_equal(zeros.cpu().numpy().reshape(-1), ez.reshape(-1), err_msg=name)
        cp, cs, _, _ = P.kv_quantize(tv, dt, scalar_div="true")
        same = (cs == es).reshape(-1)
        fx = d[f"{name}/scales"].reshape(-1)
        np.testing.assert_array_equal(_bits(scales).reshape(-1)[same], fx[same], err_msg=name)
        # dequantisation is exact: the reference's own output bits
        deq = KV.kv_dequantize((torch.from_numpy(d[f"{name}/packed"]).to(DEV).reshape(packed.shape),
                                _from_bits(d[f"{name}/scales"], "f16").to(DEV).reshape(scales.shape),
                                torch.from_numpy(d[f"{name}/zeros"]).to(DEV).reshape(zeros.shape), shape, pad))
        assert deq.dtype == torch.bfloat16 and deq.shape == t.shape
        np.testing.assert_array_equal(_bits(deq).reshape(-1), d[f"{name}/deq"].reshape(-1), err_msg=name)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("D", [64, 128, 96, 80])
def test_kv_kernels_match_torch_on_cuda(dt, D):
    g = torch.Generator(device=DEV).manual_seed(D)
    t = (torch.randn(3, 8, 37, D, generator=g, device=DEV) * 2.0).to(TDT[dt])
    t.view(-1, D)[0] = 0.0
    t.view(-1, D)[1] = 1.25
    packed, scales, zeros, shape, pad = KV.kv_quantize(t)
    rp, rs, rz = _torch_kv_quantize(t)
    assert torch.equal(packed, rp)
    assert torch.equal(scales, rs)
    assert torch.equal(zeros, rz)
    deq = KV.kv_dequantize((packed, scales, zeros, shape, pad))
    ref = P.kv_dequantize(packed.cpu().numpy(), scales.cpu().numpy().reshape(packed.shape[0], -1),
                          zeros.cpu().numpy().reshape(packed.shape[0], -1), D)
    np.testing.assert_array_equal(_bits(deq).reshape(-1), P.store_bits(ref, "bf16").reshape(-1))


def test_kv_layer_class_uses_the_kernels():
    layer = KV.Group32KVLayer()
    t = torch.randn(1, 2, 4, 64, device=DEV).to(torch.bfloat16)
    q = layer._quantize(t)
    back = layer._dequantize(q)
    assert back.shape == t.shape and back.dtype == torch.bfloat16
    assert float((back.float() - t.float()).abs().max()) <= float(t.float().abs().max()) / 7.0


# ---------------------------------------------------------------------------
# quantised embedding gather
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("tag,marlin,packed_z,dt", [("marlin_unpacked_bf16", True, False, "bf16"),
                                                   ("marlin_packed_f16", True, True, "f16"),
                                                   ("evenodd_unpacked_bf16", False, False, "bf16")])
def test_embedding_matches_reference(golden_dir, tag, marlin, packed_z, dt):
    d = np.load(golden_dir / "embedding_cases.npz")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    z = d["packed_zeros"] if packed_z else d["zeros"]
    y = SK.embedding(t(d["ids"]), t(d["packed"]), _from_bits(d["scales"], "f16").to(DEV), t(z),
                     outlier_idx=t(d["idx"]), outlier_w=_from_bits(d["ow"], "f16").to(DEV),
                     marlin_layout=marlin, out_dtype=TDT[dt])
    assert y.shape == tuple(d["ids"].shape) + (d["packed"].shape[1] * 2,)
    np.testing.assert_array_equal(_bits(y).reshape(-1), d[f"{tag}/y"].reshape(-1))


def test_embedding_large_vocab_and_bad_ids():
    c = compressed(2048, 512, seed=21, dist="t3")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    ids = np.array([0, 2047, 1000, 1000, 5], np.int64)
    y = SK.embedding(t(ids), t(c["packed"]), t(c["scales"]), t(c["zeros"]), outlier_idx=t(c["outlier_idx"]),
                     outlier_w=c["outlier_w_t"].to(DEV), marlin_layout=True)
    ref = P.embedding(ids, c["packed"], c["scales"], c["zeros"], c["outlier_idx"],
                      c["outlier_w"].astype(np.float32), marlin=True, out_dtype="bf16")
    np.testing.assert_array_equal(_bits(y).reshape(-1), ref.reshape(-1))
    # an id outside the vocabulary gives a zero row instead of an out-of-bounds read
    y2 = SK.embedding(t(np.array([3, 2048, -1], np.int64)), t(c["packed"]), t(c["scales"]), t(c["zeros"]),
                      marlin_layout=True)
    assert torch.count_nonzero(y2[1:]) == 0 and torch.count_nonzero(y2[0]) > 0


# ---------------------------------------------------------------------------
# greedy argmax
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("N", [1, 7, 1024, 128256])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
def test_argmax_matches_torch(N, dt):
    g = torch.Generator(device=DEV).manual_seed(N)
    x = torch.randn(5, N, generator=g, device=DEV).to(dt)
    if N > 10:
        x[1, 3] = x[1].max() + 1
        x[1, N - 2] = x[1, 3]          # tie: the first index wins
        x[2, 9] = float("nan")          # NaN counts as the maximum
        x[3] = -float("inf")
    idx, val = SK.argmax(x, with_values=True)
    assert torch.equal(idx, torch.argmax(x, dim=-1))
    np.testing.assert_array_equal(idx.cpu().numpy(), P.argmax(x.float().cpu().numpy()))
    ok = ~torch.isnan(val)
    assert torch.equal(val[ok], x.float().gather(1, idx.view(-1, 1)).view(-1)[ok])
    assert torch.equal(SK.argmax(x, idx_offset=1000), idx + 1000)


def test_lm_head_greedy_matches_gemv_then_argmax():
    c = compressed(4096, 1024, seed=22)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    x = torch.randn(1, 1024, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).to(DEV)
    tok, logits = SK.lm_head_greedy(x, t(c["packed"]), t(c["scales"]), t(c["zeros"]),
                                    outlier_idx=t(c["outlier_idx"]), outlier_w=c["outlier_w_t"].to(DEV),
                                    marlin_layout=True)
    assert int(tok) == int(torch.argmax(logits))
    xb, xd = np_of(x)
    y_exact, y_round, od = O.gemv(xb, xd, c["packed"], c["scales"], c["zeros"], outlier_idx=c["outlier_idx"],
                                  outlier_w=c["outlier_w"], ow_dtype="f16", marlin=True)
    assert_close_to_oracle(out_f64(logits).reshape(-1), y_exact, y_round, od, "lm_head logits")


# ---------------------------------------------------------------------------
# Walsh-Hadamard rotation prologue
# ---------------------------------------------------------------------------

def test_fwht_matches_reference(golden_dir):
    d = np.load(golden_dir / "fwht_cases.npz")
    for n in (1, 2, 32, 128, 1024):
        x = torch.from_numpy(d[f"d{n}/x"]).to(DEV)
        np.testing.assert_array_equal(SK.fwht(x).cpu().numpy(), d[f"d{n}/y"], err_msg=f"n={n}")
        np.testing.assert_array_equal(SK.fwht(x, normalize=False).cpu().numpy(), d[f"d{n}/y_raw"])


@pytest.mark.parametrize("n", [2048, 4096, 8192, 16384, 32768])
def test_fwht_large_against_oracle(n):
    x = torch.randn(3, n, generator=torch.Generator().manual_seed(n))
    y = SK.fwht(x.to(DEV)).cpu().numpy().astype(np.float64)
    ref = O.fwht(x.numpy())
    assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref))
    # orthonormal: applying it twice gives x back
    back = SK.fwht(SK.fwht(x.to(DEV))).cpu()
    assert float((back - x).abs().max()) <= 1e-4


@pytest.mark.parametrize("K,N", [(2048, 512), (4096, 1024), (8192, 256)])
def test_gemv_hadamard_prologue(K, N):
    c = compressed(N, K, seed=K + N)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    x = torch.randn(1, K, generator=torch.Generator().manual_seed(K)).to(torch.bfloat16)
    y = SK.fused_w4a16_gemv_hdsq(x.to(DEV), t(c["packed"]), t(c["scales"]), t(c["zeros"]),
                                 outlier_idx=t(c["outlier_idx"]), outlier_w=c["outlier_w_t"].to(DEV),
                                 marlin_layout=True, hadamard=True)
    # oracle: the rotated activations (fp64 transform, rounded to bf16 as the
    # prologue stores them), then the reference GEMV semantics
    xr = torch.from_numpy(O.fwht(x.float().numpy())).to(torch.bfloat16)
    xb, xd = np_of(xr)
    y_exact, y_round, od = O.gemv(xb, xd, c["packed"], c["scales"], c["zeros"], outlier_idx=c["outlier_idx"],
                                  outlier_w=c["outlier_w"], ow_dtype="f16", marlin=True)
    got = out_f64(y).reshape(-1)
    assert np.max(np.abs(got - y_exact)) <= 1e-2 * np.max(np.abs(y_exact))


def test_fwht_rejects_non_power_of_two():
    x = torch.zeros(1, 14336, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(L.SpectraError):
        SK.fwht(x)
