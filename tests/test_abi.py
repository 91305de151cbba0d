"""The C ABI library: loads without a GPU, exports exactly what
include/spectra_b200.h declares, and rejects bad arguments on the host before
any CUDA call (so these run on a CPU-only machine)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from spectra_b200 import _lib as L
from spectra_b200 import kernels as SK

HEADER = Path(__file__).resolve().parents[1] / "include" / "spectra_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(spectra_\w+)\s*\(", text)))


def test_library_loads_and_version():
    lib = L.lib()
    assert lib.spectra_abi_version() == L.ABI_VERSION == 1
    assert lib.spectra_status_string(0) == b"ok"
    assert lib.spectra_last_cuda_error() == 0


def test_every_declared_symbol_is_exported_and_bound():
    names = declared_functions()
    assert names, "no declarations parsed"
    raw = ctypes.CDLL(str(L.LIB_PATH))
    for n in names:
        assert hasattr(raw, n), f"{n} declared in the header but not exported"
    assert set(names) == set(L.PROTOTYPES), "ctypes prototypes out of sync with the header"


def test_header_constants_match_binding():
    text = HEADER.read_text()
    consts = dict(re.findall(r"#define\s+(SPECTRA_\w+)\s+(\d+)", text))
    assert int(consts["SPECTRA_DT_F16"]) == L.DT_F16
    assert int(consts["SPECTRA_DT_BF16"]) == L.DT_BF16
    assert int(consts["SPECTRA_DT_I64"]) == L.DT_I64
    assert int(consts["SPECTRA_LAYOUT_MARLIN"]) == L.LAYOUT_MARLIN
    assert int(consts["SPECTRA_ERR_CUDA"]) == L.ERR_CUDA
    assert int(consts["SPECTRA_ERR_UNSUPPORTED"]) == L.ERR_UNSUPPORTED
    assert int(consts["SPECTRA_P2P_STATE_INTS"]) == L.P2P_STATE_INTS


# Fake, never-dereferenced device addresses: every call below fails its host
# checks before reaching CUDA.
P = 0x10000


def _gemv(**kw):
    args = dict(x=P, x_dtype=L.DT_BF16, x_stride=1, packed=P, w_rs=64, scales=P, s_rs=4, s_cs=1,
                zeros=P, z_rs=4, z_cs=1, bias=None, bias_dtype=0, idx=None, idx_dtype=0, n_out=0,
                ow=None, ow_dtype=0, ow_rs=0, ow_cs=0, y=P, y_dtype=L.DT_BF16, y_stride=1,
                N=16, K=128, layout=L.LAYOUT_MARLIN, stream=None)
    args.update(kw)
    return L.lib().spectra_w4a16_gemv(*args.values())


@pytest.mark.parametrize("kw,code", [
    (dict(K=48), L.ERR_SHAPE),
    (dict(K=0), L.ERR_SHAPE),
    (dict(N=0), L.ERR_SHAPE),
    (dict(N=-5), L.ERR_SHAPE),
    (dict(K=1 << 33), L.ERR_SHAPE),
    (dict(packed=None), L.ERR_NULL_POINTER),
    (dict(x=None), L.ERR_NULL_POINTER),
    (dict(y=None), L.ERR_NULL_POINTER),
    (dict(n_out=4), L.ERR_NULL_POINTER),
    (dict(n_out=-1), L.ERR_SHAPE),
    (dict(x_dtype=7), L.ERR_DTYPE),
    (dict(y_dtype=L.DT_I32), L.ERR_DTYPE),
    (dict(bias=P, bias_dtype=9), L.ERR_DTYPE),
    (dict(n_out=2, idx=P, idx_dtype=L.DT_F16, ow=P, ow_dtype=L.DT_F16), L.ERR_DTYPE),
    (dict(layout=5), L.ERR_UNSUPPORTED),
    (dict(scales=P + 1), L.ERR_ALIGNMENT),
    (dict(x=P + 1), L.ERR_ALIGNMENT),
    (dict(y=P + 1, y_dtype=L.DT_F32), L.ERR_ALIGNMENT),
    (dict(n_out=2, idx=P + 4, idx_dtype=L.DT_I64, ow=P, ow_dtype=L.DT_F16), L.ERR_ALIGNMENT),
    (dict(y_stride=0), L.ERR_STRIDE),
])
def test_gemv_rejects_bad_arguments_on_host(kw, code):
    assert _gemv(**kw) == code


def test_dequant_rejects_bad_arguments_on_host():
    f = L.lib().spectra_w4a16_dequant
    ok = dict(packed=P, w_rs=64, scales=P, s_rs=4, s_cs=1, zeros=P, z_rs=4, z_cs=1,
              out=P, out_dtype=L.DT_F32, out_rs=128, N=16, K=128, layout=1, stream=None)
    assert f(*{**ok, "K": 100}.values()) == L.ERR_SHAPE
    assert f(*{**ok, "out": None}.values()) == L.ERR_NULL_POINTER
    assert f(*{**ok, "out_dtype": L.DT_I64}.values()) == L.ERR_DTYPE
    assert f(*{**ok, "out_rs": 64}.values()) == L.ERR_STRIDE
    assert f(*{**ok, "out": P + 2}.values()) == L.ERR_ALIGNMENT


def _gemm(**kw):
    args = dict(a=P, a_dtype=L.DT_BF16, a_rs=128, packed=P, w_rs=64, scales=P, s_rs=4, s_cs=1,
                zeros=P, z_rs=4, z_cs=1, idx=None, idx_dtype=0, n_out=0,
                ow=None, ow_dtype=0, ow_rs=0, ow_cs=0, c=P, c_dtype=L.DT_BF16, c_rs=4096,
                M=16, N=4096, K=128, layout=L.LAYOUT_MARLIN, ws=None, ws_bytes=0, stream=None)
    args.update(kw)
    return L.lib().spectra_w4a16_gemm(*args.values())


@pytest.mark.parametrize("kw,code", [
    (dict(K=48), L.ERR_SHAPE),
    (dict(M=0), L.ERR_SHAPE),
    (dict(M=-3), L.ERR_SHAPE),
    (dict(a=None), L.ERR_NULL_POINTER),
    (dict(c=None), L.ERR_NULL_POINTER),
    (dict(n_out=3), L.ERR_NULL_POINTER),
    (dict(a_dtype=L.DT_F32, c_dtype=L.DT_F32), L.ERR_DTYPE),
    (dict(c_dtype=L.DT_F16), L.ERR_DTYPE),
    (dict(n_out=2, idx=P, idx_dtype=L.DT_BF16, ow=P, ow_dtype=L.DT_F16), L.ERR_DTYPE),
    (dict(a=P + 8), L.ERR_ALIGNMENT),           # TMA needs a 16-byte aligned base
    (dict(a_rs=132), L.ERR_ALIGNMENT),          # ... and a 16-byte row pitch
    (dict(a_rs=64), L.ERR_ALIGNMENT),           # row pitch below K
    (dict(packed=P + 4), L.ERR_ALIGNMENT),
    (dict(w_rs=72), L.ERR_ALIGNMENT),
    (dict(c_rs=100), L.ERR_STRIDE),
    (dict(layout=3), L.ERR_UNSUPPORTED),
])
def test_gemm_rejects_bad_arguments_on_host(kw, code):
    assert _gemm(**kw) == code


def test_gemm_workspace_size_and_check():
    lib = L.lib()
    # 2 weight tiles, long K: split-K, needs counters + fp32 partials
    need = lib.spectra_w4a16_gemm_workspace_bytes(16, 256, 16384, 0)
    assert need >= 2 * 16 * 256 * 4
    # enough tiles to fill the GPU: no split, no workspace
    assert lib.spectra_w4a16_gemm_workspace_bytes(256, 65536, 4096, 0) == 0
    assert lib.spectra_w4a16_gemm_workspace_bytes(0, 256, 128, 0) == 0
    assert _gemm(N=256, c_rs=256, K=16384, a_rs=16384, w_rs=8192, s_rs=512, z_rs=512) == L.ERR_WORKSPACE
    assert _gemm(N=256, c_rs=256, K=16384, a_rs=16384, w_rs=8192, s_rs=512, z_rs=512,
                 ws=P, ws_bytes=need - 1) == L.ERR_WORKSPACE


def test_status_strings_cover_all_codes():
    lib = L.lib()
    for code in range(0, 9):
        assert lib.spectra_status_string(code) != b"unknown status"
    assert lib.spectra_status_string(99) == b"unknown status"


def test_python_api_has_no_cpu_fallback():
    x = torch.zeros(1, 64, dtype=torch.bfloat16)
    p = torch.zeros(8, 32, dtype=torch.uint8)
    s = torch.ones(8, 2, dtype=torch.float16)
    z = torch.zeros(8, 2, dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="CUDA"):
        SK.fused_w4a16_gemv_hdsq(x, p, s, z, marlin_layout=True)
    with pytest.raises(RuntimeError, match="CUDA"):
        SK.dequantize(p, s, z)
    with pytest.raises(RuntimeError, match="CUDA"):
        SK.batched_w4a16_gemm(x.repeat(4, 1), p, s, z, marlin_layout=True)
