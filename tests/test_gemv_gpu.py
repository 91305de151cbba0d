"""GPU parity of the M=1 GEMV and the dequant kernel against the oracle and the
reference's own kernel outputs.  Bar: dequantised weights bit-exact; outputs
within 1e-2*||y||_inf of the exact result and within 1 output ulp of its
correctly rounded value."""
import json

import numpy as np
import pytest
import torch

from oracle import w4a16 as O
from spectra_b200 import kernels as SK
from spectra_b200.synthetic import draw_act, draw_weight
from tests.helpers import (TORCH_DT, act, assert_close_to_oracle, compressed, np_of, out_f64,
                           random_format, ulp)

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _t(a, dev=DEV):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def run_gemv(fmt, x, marlin=True, bias=None, use_out=True, idx_dtype=torch.int64, out=None):
    p, s, z = _t(fmt["packed"]), _t(fmt["scales"]), _t(fmt["zeros"])
    idx = _t(fmt["outlier_idx"]).to(idx_dtype) if use_out and fmt["outlier_idx"].size else None
    ow = fmt["outlier_w_t"].to(DEV) if idx is not None else None
    y = SK.fused_w4a16_gemv_hdsq(x.to(DEV), p, s, z, bias=None if bias is None else bias.to(DEV),
                                 outlier_idx=idx, outlier_w=ow, out=out, marlin_layout=marlin)
    torch.cuda.synchronize()
    return y


def oracle_gemv(fmt, x, marlin=True, bias=None, use_out=True):
    xn, xd = np_of(x)
    ow, owd = np_of(fmt["outlier_w_t"])
    bn, bd = np_of(bias) if bias is not None else (None, None)
    has = use_out and fmt["outlier_idx"].size
    return O.gemv(xn, xd, fmt["packed"], fmt["scales"], fmt["zeros"], bias=bn, bias_dtype=bd,
                  outlier_idx=fmt["outlier_idx"] if has else None, outlier_w=ow if has else None,
                  ow_dtype=owd, marlin=marlin)


# ---------------------------------------------------------------------------
# pins from the reference's own outputs
# ---------------------------------------------------------------------------

def _kc(golden_dir):
    return np.load(golden_dir / "kernel_cases.npz")


def _fmt_from_kc(d, ow_key="ow", ow_dtype=torch.float16):
    ow = torch.from_numpy(d[ow_key].view(np.int16)).view(ow_dtype) if ow_dtype == torch.bfloat16 \
        else torch.from_numpy(d[ow_key].view(np.float16))
    return {"packed": d["packed"], "scales": d["scales"].view(np.float16), "zeros": d["zeros"],
            "outlier_idx": d["idx"].astype(np.int64), "outlier_w_t": ow}


@pytest.mark.parametrize("name,dt,marlin,use_out,use_bias", [
    ("gemv_f16_marlin", "f16", True, False, False),
    ("gemv_f16_marlin_out_bias", "f16", True, True, True),
    ("gemv_bf16_marlin_out_bias", "bf16", True, True, True),
    ("gemv_bf16_evenodd_out", "bf16", False, True, False),
    ("gemv_f16_evenodd", "f16", False, False, False),
])
def test_gemv_matches_reference_triton_outputs(golden_dir, name, dt, marlin, use_out, use_bias):
    d = _kc(golden_dir)
    fmt = _fmt_from_kc(d, "ow_bf16" if dt == "bf16" else "ow", TORCH_DT[dt])
    xb = d[f"{name}/x"]
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16) if dt == "bf16" else torch.from_numpy(xb.view(np.float16))
    bias = None
    if use_bias:
        bias = torch.from_numpy(d["bias_bf16"].view(np.int16)).view(torch.bfloat16) if dt == "bf16" \
            else torch.from_numpy(d["bias_f16"].view(np.float16))
    y = run_gemv(fmt, x, marlin=marlin, bias=bias, use_out=use_out)
    yb = d[f"{name}/y"]
    y_ref = (O.bf16_bits_to_f32(yb) if dt == "bf16" else yb.view(np.float16)).astype(np.float64).reshape(-1)
    got = out_f64(y).reshape(-1)
    # the reference's own Triton result and ours: both round an fp32 sum once
    d_ulp = np.abs(got - y_ref) / ulp(y_ref, dt)
    i = int(np.argmax(d_ulp))
    assert d_ulp[i] <= 1.0, f"{name}: worst at {i}: got {got[i]!r} ref {y_ref[i]!r} ({d_ulp[i]:.2f} ulp)"
    if dt == "f16":
        assert np.max(np.abs(got - y_ref)) <= 0.05  # tests/test_kernels.py:49
    y_exact, y_round, od = oracle_gemv(fmt, x, marlin, bias, use_out)
    assert_close_to_oracle(got, y_exact, y_round, od, name)


def test_gemv_config1_matches_reference(golden_dir):
    """BASELINE config 1 (K=N=2048, compressor defaults, fp16 x)."""
    rec = json.loads((golden_dir / "config1.json").read_text())
    fmt = compressed(rec["N"], rec["K"], seed=rec["seed"], dist=rec["dist"])
    x = draw_act(1, rec["K"], seed=rec["x_seed"], dtype=torch.float16)
    y = out_f64(run_gemv(fmt, x, marlin=True)).reshape(-1)
    y_ref = np.array(rec["y_bits"], np.uint16).view(np.float16).astype(np.float64)
    assert np.all(np.abs(y - y_ref) <= ulp(y_ref, "f16"))
    y_exact, y_round, od = oracle_gemv(fmt, x)
    assert_close_to_oracle(y, y_exact, y_round, od, "config1")


# ---------------------------------------------------------------------------
# BASELINE shapes (configs 2, 3, 5 at M=1) against the oracle
# ---------------------------------------------------------------------------

BASELINE_SHAPES = [  # (K, N, n_out)
    (2048, 2048, 21), (2048, 512, 21), (2048, 8192, 21), (8192, 2048, 82),
    (4096, 4096, 41), (4096, 1024, 41), (4096, 14336, 41), (14336, 4096, 143),
    (8192, 8192, 146), (28672, 8192, 651),
]


@pytest.mark.parametrize("K,N,n_out", BASELINE_SHAPES)
@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_gemv_baseline_shapes(K, N, n_out, dt):
    fmt = random_format(N, K, n_out, seed=K * 7 + N, ow_dtype=dt)
    x = act(1, K, seed=K + N, dtype=dt)
    y = out_f64(run_gemv(fmt, x)).reshape(-1)
    y_exact, y_round, od = oracle_gemv(fmt, x)
    assert_close_to_oracle(y, y_exact, y_round, od, f"{K}x{N}")


def test_gemv_compressed_llama_layer_shapes():
    """Config 2 shapes with real compressor output (q,k/v,gate/up,down)."""
    for K, N, seed in ((2048, 512, 11), (2048, 8192, 12), (8192, 2048, 13)):
        fmt = compressed(N, K, seed=seed)
        x = act(1, K, seed=seed + 1, dtype="bf16")
        y = out_f64(run_gemv(fmt, x)).reshape(-1)
        y_exact, y_round, od = oracle_gemv(fmt, x)
        assert_close_to_oracle(y, y_exact, y_round, od, f"compressed {K}x{N}")


# ---------------------------------------------------------------------------
# edge cases
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("N", [1, 3, 17, 100, 257])
@pytest.mark.parametrize("K", [32, 96, 1056, 2080])
def test_gemv_ragged_shapes(N, K):
    fmt = random_format(N, K, min(5, K // 32), seed=N * 131 + K)
    x = act(1, K, seed=N + K, dtype="bf16")
    y = out_f64(run_gemv(fmt, x)).reshape(-1)
    y_exact, y_round, od = oracle_gemv(fmt, x)
    assert_close_to_oracle(y, y_exact, y_round, od, f"N={N} K={K}")


@pytest.mark.parametrize("K", [28672, 40960, 57344])
def test_gemv_multi_window_k(K):
    """K beyond one staged window (14336 features) exercises the K-window loop."""
    fmt = random_format(256, K, 40, seed=K)
    x = act(1, K, seed=K + 1, dtype="bf16")
    y = out_f64(run_gemv(fmt, x)).reshape(-1)
    y_exact, y_round, od = oracle_gemv(fmt, x)
    assert_close_to_oracle(y, y_exact, y_round, od, f"K={K}")


@pytest.mark.parametrize("marlin", [True, False])
@pytest.mark.parametrize("xdt", ["f16", "bf16", "f32"])
def test_gemv_dtypes_and_layouts(marlin, xdt):
    fmt = random_format(300, 1024, 9, seed=5, ow_dtype="f16")
    x = act(1, 1024, seed=6, dtype=xdt)
    y = run_gemv(fmt, x, marlin=marlin)
    assert y.dtype == x.dtype
    # the reference rounds to fp16 for any non-bf16 input (spectra/kernels.py:126-129)
    od = "bf16" if xdt == "bf16" else "f16"
    y_exact, y_round, _ = oracle_gemv(fmt, x, marlin)
    assert_close_to_oracle(out_f64(y).reshape(-1), y_exact, y_round, od, f"{xdt} marlin={marlin}")


def test_gemv_bias_and_bf16_outliers_and_int32_unsorted_idx():
    K, N = 2048, 777
    fmt = random_format(N, K, 33, seed=9, ow_dtype="bf16")
    perm = np.random.default_rng(1).permutation(fmt["outlier_idx"].size)
    fmt["outlier_idx"] = fmt["outlier_idx"][perm]
    fmt["outlier_w_t"] = fmt["outlier_w_t"][:, torch.from_numpy(perm)]
    bias = torch.randn(N, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    x = act(1, K, seed=10, dtype="bf16")
    y = run_gemv(fmt, x, bias=bias, idx_dtype=torch.int32)
    y_exact, y_round, od = oracle_gemv(fmt, x, bias=bias)
    assert_close_to_oracle(out_f64(y).reshape(-1), y_exact, y_round, od, "bias+idx32")


def test_gemv_duplicate_and_out_of_range_outlier_indices():
    """Duplicates add twice (as the reference's loop does); indices outside
    [0, K) are skipped by the kernel's bounds check and contribute nothing."""
    K, N = 1024, 64
    fmt = random_format(N, K, 6, seed=12)
    fmt["outlier_idx"] = np.array([5, 5, 100, K + 3, -2, 1023], np.int64)
    x = act(1, K, seed=13, dtype="bf16")
    y = out_f64(run_gemv(fmt, x)).reshape(-1)
    keep = np.array([1, 1, 1, 0, 0, 1], bool)
    ref_fmt = dict(fmt, outlier_idx=fmt["outlier_idx"][keep],
                   outlier_w_t=fmt["outlier_w_t"][:, torch.from_numpy(np.nonzero(keep)[0])])
    y_exact, y_round, od = oracle_gemv(ref_fmt, x)
    assert_close_to_oracle(y, y_exact, y_round, od, "dup/oob idx")


def test_gemv_no_outliers_and_empty_outliers():
    fmt = random_format(128, 512, 0, seed=14)
    x = act(1, 512, seed=15, dtype="f16")
    y = out_f64(run_gemv(fmt, x)).reshape(-1)
    y_exact, y_round, od = oracle_gemv(fmt, x, use_out=False)
    assert_close_to_oracle(y, y_exact, y_round, od, "n_out=0")


def test_gemv_strided_views_like_offloader_slots():
    """Weights bound as [:N, :K/2] views of wider slots (spectra/engine.py:555-569),
    zeros as the engine's [:, :K//32] unpack view, strided x and out."""
    K, N = 1536, 200
    fmt = random_format(N, K, 12, seed=16)
    for pad in (16, 3):  # aligned and misaligned row strides
        slot_p = torch.zeros(N + 5, K // 2 + pad, dtype=torch.uint8)
        slot_p[:N, :K // 2] = torch.from_numpy(fmt["packed"])
        slot_s = torch.zeros(N + 5, K // 32 + 7, dtype=torch.float16)
        slot_s[:N, :K // 32] = torch.from_numpy(fmt["scales"])
        pz_width = (K // 32 + 1) // 2
        slot_z = torch.zeros(N, pz_width * 2, dtype=torch.uint8)
        slot_z[:, :K // 32] = torch.from_numpy(fmt["zeros"])
        p = slot_p.to(DEV)[:N, :K // 2]
        s = slot_s.to(DEV)[:N, :K // 32]
        z = slot_z.to(DEV)[:, :K // 32]
        xw = act(1, 2 * K, seed=17, dtype="bf16").to(DEV)
        x = xw[:, ::2]
        out_full = torch.zeros(1, 2 * N, dtype=torch.bfloat16, device=DEV)
        out = out_full[:, ::2]
        idx = _t(fmt["outlier_idx"])
        ow = fmt["outlier_w_t"].to(DEV)
        y = SK.fused_w4a16_gemv_hdsq(x, p, s, z, outlier_idx=idx, outlier_w=ow, out=out, marlin_layout=True)
        torch.cuda.synchronize()
        assert y.data_ptr() == out.data_ptr()
        assert torch.all(out_full[:, 1::2] == 0)
        y_exact, y_round, od = oracle_gemv(fmt, x.cpu())
        assert_close_to_oracle(out_f64(y).reshape(-1), y_exact, y_round, od, f"strided pad={pad}")


def test_gemv_1d_input_and_multirow_input():
    K, N = 512, 96
    fmt = random_format(N, K, 4, seed=18)
    x = act(3, K, seed=19, dtype="bf16")
    y1 = run_gemv(fmt, x[0])
    assert y1.shape == (N,)
    y3 = run_gemv(fmt, x)
    assert y3.shape == (3, N)
    for b in range(3):
        y_exact, y_round, od = oracle_gemv(fmt, x[b:b + 1])
        assert_close_to_oracle(out_f64(y3[b]), y_exact, y_round, od, f"row {b}")
    assert torch.equal(y1, y3[0])


def test_gemv_deterministic():
    fmt = random_format(4096, 4096, 41, seed=20)
    x = act(1, 4096, seed=21, dtype="bf16")
    a = run_gemv(fmt, x)
    b = run_gemv(fmt, x)
    assert torch.equal(a, b)


def test_gemv_reference_unit_test_port():
    """tests/test_kernels.py:43-49 on our own generator: N=128, K=256, fp16, Marlin."""
    torch.manual_seed(42)
    w = torch.randn(128, 256, dtype=torch.float16)
    c = O.compress_linear(w.numpy())
    deq = O.dequant_f32(c["packed"], c["scales"], c["zeros"], True).astype(np.float16)
    x = torch.randn(1, 256, dtype=torch.float16)
    fmt = dict(c, outlier_w_t=torch.from_numpy(c["outlier_w"]))
    y = run_gemv(fmt, x, use_out=False)
    ref = torch.matmul(x.cuda(), torch.from_numpy(deq).cuda().t())
    assert torch.max(torch.abs(ref - y)).item() <= 0.05


# ---------------------------------------------------------------------------
# dequant: bit-exact
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("marlin", [True, False])
def test_dequant_bit_exact(marlin, golden_dir):
    d = _kc(golden_dir)
    fmt = random_format(333, 2048, 0, seed=22)
    for f in (fmt, {"packed": d["packed"], "scales": d["scales"].view(np.float16), "zeros": d["zeros"]}):
        ref = O.dequant_f32(f["packed"], f["scales"], f["zeros"], marlin)
        p, s, z = _t(f["packed"]), _t(f["scales"]), _t(f["zeros"])
        w32 = SK.dequantize(p, s, z, marlin_layout=marlin, dtype=torch.float32).cpu().numpy()
        np.testing.assert_array_equal(w32.view(np.uint32), ref.view(np.uint32))
        wb = SK.dequantize(p, s, z, marlin_layout=marlin, dtype=torch.bfloat16).cpu()
        np.testing.assert_array_equal(wb.view(torch.int16).numpy().view(np.uint16), O.f32_to_bf16_bits(ref))
        wh = SK.dequantize(p, s, z, marlin_layout=marlin, dtype=torch.float16).cpu().numpy()
        np.testing.assert_array_equal(wh.view(np.uint16), ref.astype(np.float16).view(np.uint16))
    # the reference test's own dequant (tests/test_kernels.py:31-36)
    w32 = SK.dequantize(_t(d["packed"]), _t(d["scales"].view(np.float16)), _t(d["zeros"]), marlin_layout=True)
    np.testing.assert_array_equal(w32.cpu().numpy().view(np.uint32), d["w_deq_f32"].view(np.uint32))


# ---------------------------------------------------------------------------
# weight-prefetching kernel (K % 512 == 0, 16-byte aligned unit-stride weights)
# ---------------------------------------------------------------------------

def _padded_weights(fmt, N, K, pad_rows=3, pad_p=32, pad_s=8, pad_z=16):
    """Weights as [:N, :width] views of wider, 16-byte-aligned slots."""
    slot_p = torch.zeros(N + pad_rows, K // 2 + pad_p, dtype=torch.uint8)
    slot_p[:N, :K // 2] = torch.from_numpy(fmt["packed"])
    slot_s = torch.zeros(N + pad_rows, K // 32 + pad_s, dtype=torch.float16)
    slot_s[:N, :K // 32] = torch.from_numpy(fmt["scales"])
    slot_z = torch.zeros(N + pad_rows, K // 32 + pad_z, dtype=torch.uint8)
    slot_z[:N, :K // 32] = torch.from_numpy(fmt["zeros"])
    return (slot_p.to(DEV)[:N, :K // 2], slot_s.to(DEV)[:N, :K // 32], slot_z.to(DEV)[:N, :K // 32])


@pytest.mark.parametrize("padded", [False, True])
@pytest.mark.parametrize("xdt", ["bf16", "f16"])
@pytest.mark.parametrize("marlin", [True, False])
def test_gemv_prefetch_strided_x(padded, xdt, marlin):
    """Strided x with contiguous weights (the prefetching kernel's scalar x
    staging) and with weights bound as views of wider slots (the other kernel)."""
    K, N = 3072, 1000
    fmt = random_format(N, K, 31, seed=40, ow_dtype=xdt)
    if padded:
        p, s, z = _padded_weights(fmt, N, K)
    else:
        p, s, z = _t(fmt["packed"]), _t(fmt["scales"]), _t(fmt["zeros"])
    xw = act(1, 2 * K, seed=41, dtype=xdt).to(DEV)
    x = xw[:, 1::2]
    idx = _t(fmt["outlier_idx"])
    ow = fmt["outlier_w_t"].to(DEV)
    y = SK.fused_w4a16_gemv_hdsq(x, p, s, z, outlier_idx=idx, outlier_w=ow, marlin_layout=marlin)
    torch.cuda.synchronize()
    y_exact, y_round, od = oracle_gemv(fmt, x.cpu(), marlin)
    assert_close_to_oracle(out_f64(y).reshape(-1), y_exact, y_round, od, f"padded={padded} {xdt} marlin={marlin}")


@pytest.mark.parametrize("N", [1, 16, 31, 148 * 16 * 2 + 5, 148 * 16 * 7 - 9])
def test_gemv_prefetch_row_splits(N):
    """One row, one block, a ragged block, CTAs with 2-3 and 7 row blocks
    (the last refills the stage ring at K=4096)."""
    K = 4096 if N > 5000 else 1024
    fmt = random_format(N, K, 7, seed=N + 3)
    x = act(1, K, seed=N + 4, dtype="bf16")
    y = out_f64(run_gemv(fmt, x)).reshape(-1)
    y_exact, y_round, od = oracle_gemv(fmt, x)
    assert_close_to_oracle(y, y_exact, y_round, od, f"N={N}")


@pytest.mark.parametrize("K,N,strided", [(8192, 148 * 16 * 5 + 7, False), (10240, 148 * 16 * 2 + 1, False),
                                          (5120, 148 * 16 * 5 + 3, False), (3584, 148 * 16 * 5 + 9, True),
                                          (28672, 1024, False)])
def test_gemv_prefetch_two_groups(K, N, strided):
    """Two compute groups on alternate stages: chunked stages for CTAs with
    >= 5 row blocks of a large K (ragged last block), an odd number of chunks
    per row block, whole-row-block stages whose ring depth (3) is rounded
    down to an even number, strided x (scalar staging whose trip count
    differs between warps: K / 2 is not a multiple of the 512 threads), and
    one row block per CTA at K = 28672 (the CTA owns its SM)."""
    fmt = random_format(N, K, 9, seed=K + N)
    x = act(1, K, seed=K + N + 1, dtype="bf16")
    if strided:  # a strided view on the device (a host copy would come back contiguous)
        x = act(1, 2 * K, seed=K + N + 2, dtype="bf16").to(DEV)[:, ::2]
    y = out_f64(run_gemv(fmt, x)).reshape(-1)
    y_exact, y_round, od = oracle_gemv(fmt, x.cpu() if strided else x)
    assert_close_to_oracle(y, y_exact, y_round, od, f"{K}x{N} strided={strided}")


@pytest.mark.parametrize("n_out,ow_dt", [(601, "f32"), (700, "bf16")])
def test_gemv_prefetch_outliers_streamed_through_ring(n_out, ow_dt):
    """Outlier weights too large to stage beside the ring (144 rows per CTA)
    stream through the freed ring after the main loop: 64 rows per piece,
    2-3 pieces, the last CTA's rows ending off a 16-byte boundary."""
    K, N = 2048, 148 * 16 * 8 + 5
    fmt = random_format(N, K, n_out, seed=n_out, ow_dtype=ow_dt)
    x = act(1, K, seed=n_out + 1, dtype="bf16")
    y = out_f64(run_gemv(fmt, x)).reshape(-1)
    y_exact, y_round, od = oracle_gemv(fmt, x)
    assert_close_to_oracle(y, y_exact, y_round, od, f"n_out={n_out} {ow_dt}")


def test_gemv_prefetch_f32_outliers_and_bias_f32_out():
    K, N = 2048, 600
    fmt = random_format(N, K, 40, seed=42, ow_dtype="f32")
    bias = torch.randn(N, generator=torch.Generator().manual_seed(43)).to(torch.bfloat16)
    x = act(1, K, seed=44, dtype="bf16")
    out = torch.empty(1, N, dtype=torch.float32, device=DEV)
    y = run_gemv(fmt, x, bias=bias, out=out)
    assert y.dtype == torch.float32
    # the reference rounds to x's dtype (bf16) before storing into out
    y_exact, y_round, od = oracle_gemv(fmt, x, bias=bias)
    assert_close_to_oracle(out_f64(y).reshape(-1), y_exact, y_round, od, "f32 ow / out")


@pytest.mark.parametrize("graph", [False, True])
def test_gemv_chained_launches_respect_stream_order(graph):
    """Each GEMV reads the previous one's output and writes the buffer the one
    before it read: the dependency wait must order both the read of x and the
    write of y, eagerly and inside a CUDA graph."""
    D, steps = 2048, 12
    fmts = [random_format(D, D, 5, seed=50 + i) for i in range(3)]
    ws = [(_t(f["packed"]), _t(f["scales"]), _t(f["zeros"]), _t(f["outlier_idx"]), f["outlier_w_t"].to(DEV))
          for f in fmts]
    x0 = act(1, D, seed=60, dtype="bf16").to(DEV) * 0.05
    bufs = [torch.empty(1, D, dtype=torch.bfloat16, device=DEV) for _ in range(2)]

    def chain():
        bufs[0].copy_(x0)
        for i in range(steps):
            p, s, z, idx, ow = ws[i % 3]
            SK.fused_w4a16_gemv_hdsq(bufs[i % 2], p, s, z, outlier_idx=idx, outlier_w=ow,
                                     out=bufs[(i + 1) % 2], marlin_layout=True)
            # keep magnitudes bounded without leaving the GEMV chain
            SK.fused_w4a16_gemv_hdsq(bufs[(i + 1) % 2], p, s, z, outlier_idx=idx, outlier_w=ow,
                                     out=bufs[i % 2], marlin_layout=True)

    if graph:
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            chain()
        torch.cuda.current_stream().wait_stream(st)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            chain()
        g.replay()
    else:
        chain()
    torch.cuda.synchronize()
    got = bufs[0].clone()

    # replay step by step with a full synchronisation between launches
    ref = [torch.empty_like(b) for b in bufs]
    ref[0].copy_(x0)
    for i in range(steps):
        p, s, z, idx, ow = ws[i % 3]
        for src, dst in ((i % 2, (i + 1) % 2), ((i + 1) % 2, i % 2)):
            SK.fused_w4a16_gemv_hdsq(ref[src], p, s, z, outlier_idx=idx, outlier_w=ow, out=ref[dst],
                                     marlin_layout=True)
            torch.cuda.synchronize()
    assert torch.equal(got, ref[0])
