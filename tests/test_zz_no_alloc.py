"""spectra_w4a16_gemm_noalloc, the allocation-free GEMM entry point: split-K
scratch in a static device array instead of a caller workspace.

Collected last on purpose (file name): it must pass both alone in a fresh
process and after every other test has run in the same process.  The entry
point is compared with spectra_w4a16_gemm (through batched_w4a16_gemm) on two
calls in a row, the second of which relies on the first having left the
scratch counters at zero; it must give the same bits (same kernel, same
split-K summation order), stay within the oracle's bar, and allocate nothing
through torch's caching allocator."""
import re
from pathlib import Path

import pytest
import torch

from oracle import w4a16 as O
from spectra_b200 import _lib as L
from spectra_b200 import kernels as SK
from tests.helpers import act, assert_close_to_oracle, np_of, out_f64, random_format

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


def _case(M, N, K, n_out, seed):
    fmt = random_format(N, K, n_out, seed=seed, ow_dtype="bf16")
    dev = torch.device("cuda")
    t = {"p": torch.from_numpy(fmt["packed"]).to(dev), "s": torch.from_numpy(fmt["scales"]).to(dev),
         "z": torch.from_numpy(fmt["zeros"]).to(dev),
         "idx": torch.from_numpy(fmt["outlier_idx"]).to(dev) if n_out else None,
         "ow": fmt["outlier_w_t"].to(dev) if n_out else None,
         "a": act(M, K, seed=seed + 1, dtype="bf16").to(dev)}
    return fmt, t


def _oracle(fmt, a, n_out):
    an, ad = np_of(a)
    ow, owd = np_of(fmt["outlier_w_t"])
    return O.gemm(an, ad, fmt["packed"], fmt["scales"], fmt["zeros"],
                  outlier_idx=fmt["outlier_idx"] if n_out else None, outlier_w=ow if n_out else None,
                  ow_dtype=owd, marlin=True)


CASES = [(16, 256, 16384, 12), (32, 1024, 4096, 40), (64, 4096, 4096, 0)]


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,n_out", CASES)
def test_noalloc_matches_gemm_on_two_calls_in_a_row(M, N, K, n_out):
    need = L.lib().spectra_w4a16_gemm_workspace_bytes(M, N, K, n_out)
    assert 0 < need <= SCRATCH_BYTES  # split-K: the static scratch is used
    fmt, t = _case(M, N, K, n_out, seed=M + N)
    dev = t["a"].device
    # the entry point for workspace-owning callers, through the drop-in module
    ref = SK.batched_w4a16_gemm(t["a"], t["p"], t["s"], t["z"], outlier_idx=t["idx"], outlier_w=t["ow"],
                                marlin_layout=True)
    outs = [torch.empty(M, N, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated(dev)
    for c in outs:  # back to back on one stream
        assert _noalloc(t["a"], t["p"], t["s"], t["z"], t["idx"], t["ow"], c) == L.OK
    torch.cuda.synchronize()
    # nothing allocated through the caching allocator by the two calls
    assert torch.cuda.memory_allocated(dev) == before
    # same kernel, same deterministic split-K summation order: identical bits
    for i, c in enumerate(outs):
        assert torch.equal(c, ref), f"call {i} differs from spectra_w4a16_gemm"
    # and the oracle's bar: within 1e-2*||c||_inf and one output ulp of exact
    c_exact, c_round, cd = _oracle(fmt, t["a"].cpu(), n_out)
    assert_close_to_oracle(out_f64(outs[1]), c_exact, c_round, cd, "noalloc vs oracle")


@pytest.mark.gpu
def test_noalloc_smaller_tile_layout_after_a_larger_one():
    """The scratch keeps the last call's contents.  A call with many (tile,
    m-chunk) counters is followed by one with fewer, differently placed ones:
    the second call only works if the first left every counter it used at
    zero.  Both results must equal spectra_w4a16_gemm's, bit for bit."""
    big = (260, 1024, 1024, 8)    # 8 weight tiles x 2 token chunks of 256: 16 counters
    small = (16, 512, 8192, 4)    # 4 weight tiles x 1 token chunk: 4 counters, deeper split
    need_big = L.lib().spectra_w4a16_gemm_workspace_bytes(*big)
    need_small = L.lib().spectra_w4a16_gemm_workspace_bytes(*small)
    assert 0 < need_small <= SCRATCH_BYTES and 0 < need_big <= SCRATCH_BYTES
    results = []
    for (M, N, K, n_out), seed in ((big, 11), (small, 12), (big, 13)):
        fmt, t = _case(M, N, K, n_out, seed=seed)
        ref = SK.batched_w4a16_gemm(t["a"], t["p"], t["s"], t["z"], outlier_idx=t["idx"], outlier_w=t["ow"],
                                    marlin_layout=True)
        c = torch.empty(M, N, dtype=torch.bfloat16, device=t["a"].device)
        assert _noalloc(t["a"], t["p"], t["s"], t["z"], t["idx"], t["ow"], c) == L.OK
        torch.cuda.synchronize()
        results.append((c, ref))
    for i, (c, ref) in enumerate(results):
        assert torch.equal(c, ref), f"call {i} differs from spectra_w4a16_gemm"
