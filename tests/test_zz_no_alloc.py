"""spectra_w4a16_gemm_noalloc, the allocation-free GEMM entry point: split-K
scratch in a static device array instead of a caller workspace.

Collected last on purpose (file name): it must pass both alone in a fresh
process and after every other test has run in the same process.  The entry
point is compared with spectra_w4a16_gemm (through batched_w4a16_gemm) on two
calls in a row, the second of which relies on the first having left the
scratch counters at zero."""
import re
from pathlib import Path

import pytest
import torch

from spectra_b200 import _lib as L
from spectra_b200 import kernels as SK
from tests.helpers import act, random_format

HEADER = Path(__file__).resolve().parents[1] / "include" / "spectra_b200.h"
SCRATCH_BYTES = int(re.search(r"#define\s+SPECTRA_GEMM_NOALLOC_SCRATCH_BYTES\s+(\d+)", HEADER.read_text()).group(1))


def _noalloc(a, p, s, z, idx, ow, c, marlin=True):
    M, K = a.shape
    N = p.shape[0]
    n_out = idx.numel() if idx is not None else 0
    return L.lib().spectra_w4a16_gemm_noalloc(
        a.data_ptr(), L.DT_BF16 if a.dtype == torch.bfloat16 else L.DT_F16, a.stride(0),
        p.data_ptr(), p.stride(0),
        s.data_ptr(), s.stride(0), s.stride(1),
        z.data_ptr(), z.stride(0), z.stride(1),
        idx.data_ptr() if n_out else None, L.DT_I64 if n_out else 0, n_out,
        ow.data_ptr() if n_out else None, L.DT_BF16 if n_out else 0,
        ow.stride(0) if n_out else 0, ow.stride(1) if n_out else 0,
        c.data_ptr(), L.DT_BF16 if c.dtype == torch.bfloat16 else L.DT_F16, c.stride(0),
        M, N, K, L.LAYOUT_MARLIN if marlin else L.LAYOUT_EVEN_ODD,
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_rejects_problems_beyond_the_scratch_on_host():
    # 8 weight tiles, 256 tokens: 16-way split-K needs 16 MiB of partials
    M, N, K = 256, 1024, 4096
    assert L.lib().spectra_w4a16_gemm_workspace_bytes(M, N, K, 0) > SCRATCH_BYTES
    P = 0x10000  # never dereferenced: the size check runs before any CUDA call
    st = L.lib().spectra_w4a16_gemm_noalloc(P, L.DT_BF16, K, P, K // 2, P, K // 32, 1, P, K // 32, 1,
                                            None, 0, 0, None, 0, 0, 0, P, L.DT_BF16, N,
                                            M, N, K, L.LAYOUT_MARLIN, None)
    assert st == L.ERR_WORKSPACE


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,n_out", [(16, 256, 16384, 12), (32, 1024, 4096, 40), (64, 4096, 4096, 0)])
def test_noalloc_matches_gemm_on_two_calls_in_a_row(M, N, K, n_out):
    need = L.lib().spectra_w4a16_gemm_workspace_bytes(M, N, K, n_out)
    assert 0 < need <= SCRATCH_BYTES  # split-K: the static scratch is used
    fmt = random_format(N, K, n_out, seed=M + N, ow_dtype="bf16")
    dev = torch.device("cuda")
    p = torch.from_numpy(fmt["packed"]).to(dev)
    s = torch.from_numpy(fmt["scales"]).to(dev)
    z = torch.from_numpy(fmt["zeros"]).to(dev)
    idx = torch.from_numpy(fmt["outlier_idx"]).to(dev) if n_out else None
    ow = fmt["outlier_w_t"].to(dev) if n_out else None
    a = act(M, K, seed=M, dtype="bf16").to(dev)
    ref = SK.batched_w4a16_gemm(a, p, s, z, outlier_idx=idx, outlier_w=ow, marlin_layout=True).float()
    outs = [torch.empty(M, N, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    for c in outs:  # back to back on one stream
        assert _noalloc(a, p, s, z, idx, ow, c) == L.OK
    torch.cuda.synchronize()
    tol = 1e-2 * float(ref.abs().max())
    for i, c in enumerate(outs):
        err = float((c.float() - ref).abs().max())
        assert err <= tol, f"call {i}: max|err| {err:.3e} > {tol:.3e}"
