"""ctypes binding of libspectra_b200.so (the C ABI in include/spectra_b200.h).

The library is built in-tree (``python -m spectra_b200.build``).  There is no
fallback: if it is missing, every kernel call raises.
"""
from __future__ import annotations

import ctypes
from ctypes import c_char_p, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libspectra_b200.so")

# dtype / layout / status codes (mirror include/spectra_b200.h)
DT_F16, DT_BF16, DT_F32, DT_I32, DT_I64 = 0, 1, 2, 3, 4
LAYOUT_EVEN_ODD, LAYOUT_MARLIN = 0, 1
OK = 0
ERR_NULL_POINTER, ERR_SHAPE, ERR_STRIDE, ERR_ALIGNMENT, ERR_DTYPE, ERR_WORKSPACE, ERR_CUDA, ERR_UNSUPPORTED = range(1, 9)
ABI_VERSION = 1
P2P_STATE_INTS = 128  # SPECTRA_P2P_STATE_INTS
P2P_SIGNAL_BYTES = 8 * 128 * 4  # epoch flags [rank][cta] at the start of an exchange buffer

# name -> (restype, argtypes)
PROTOTYPES = {
    "spectra_abi_version": (c_int, []),
    "spectra_status_string": (c_char_p, [c_int]),
    "spectra_last_cuda_error": (c_int, []),
    "spectra_w4a16_gemv": (c_int, [
        c_void_p, c_int, c_int64,                      # x, x_dtype, x_stride
        c_void_p, c_int64,                             # packed, w_row_stride
        c_void_p, c_int64, c_int64,                    # scales, s_row_stride, s_col_stride
        c_void_p, c_int64, c_int64,                    # zeros, z_row_stride, z_col_stride
        c_void_p, c_int,                               # bias, bias_dtype
        c_void_p, c_int, c_int64,                      # outlier_idx, idx_dtype, n_out
        c_void_p, c_int, c_int64, c_int64,             # outlier_w, ow_dtype, ow_row_stride, ow_col_stride
        c_void_p, c_int, c_int64,                      # y, y_dtype, y_stride
        c_int64, c_int64, c_int, c_void_p]),           # N, K, layout, stream
    "spectra_w4a16_gemm": (c_int, [
        c_void_p, c_int, c_int64,                      # a, a_dtype, a_row_stride
        c_void_p, c_int64,                             # packed, w_row_stride
        c_void_p, c_int64, c_int64,                    # scales
        c_void_p, c_int64, c_int64,                    # zeros
        c_void_p, c_int, c_int64,                      # outlier_idx, idx_dtype, n_out
        c_void_p, c_int, c_int64, c_int64,             # outlier_w
        c_void_p, c_int, c_int64,                      # c, c_dtype, c_row_stride
        c_int64, c_int64, c_int64, c_int,              # M, N, K, layout
        c_void_p, c_size_t, c_void_p]),                # workspace, workspace_bytes, stream
    "spectra_w4a16_gemm_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64]),
    # diagnostic: the M=1 GEMV's configuration for a shape (host only)
    "spectra_gemv_pf_plan": (c_int, [c_int64, c_int64, c_int64, c_int, c_int, c_int, c_void_p]),
    "spectra_gemm_small_m_plan": (c_int, [c_int64, c_int64, c_int64, c_int64, c_int, c_int, c_int, c_void_p]),
    "spectra_gemm_plan": (c_int, [c_int64, c_int64, c_int64, c_int64, c_void_p]),
    "spectra_gemm_pair_capacity": (c_int, [c_void_p]),
    "spectra_w4a16_gemm_noalloc": (c_int, [
        c_void_p, c_int, c_int64,                      # a, a_dtype, a_row_stride
        c_void_p, c_int64,                             # packed, w_row_stride
        c_void_p, c_int64, c_int64,                    # scales
        c_void_p, c_int64, c_int64,                    # zeros
        c_void_p, c_int, c_int64,                      # outlier_idx, idx_dtype, n_out
        c_void_p, c_int, c_int64, c_int64,             # outlier_w
        c_void_p, c_int, c_int64,                      # c, c_dtype, c_row_stride
        c_int64, c_int64, c_int64, c_int,              # M, N, K, layout
        c_void_p]),                                    # stream
    "spectra_quantize_group32": (c_int, [
        c_void_p, c_int, c_int64,                      # w, w_dtype, w_row_stride
        c_void_p, c_int, c_int64,                      # outlier_idx, idx_dtype, n_out
        c_void_p, c_int64, c_void_p, c_int64,          # packed, scales
        c_void_p, c_int64, c_void_p, c_int64,          # zeros, packed_zeros
        c_int64, c_int64, c_int, c_void_p]),           # N, K, layout, stream
    "spectra_unpack_zeros": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_void_p]),
    "spectra_kv_quantize": (c_int, [c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p]),
    "spectra_kv_dequantize": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64, c_void_p]),
    "spectra_w4a16_embedding": (c_int, [
        c_void_p, c_int, c_int64,                      # ids, ids_dtype, T
        c_void_p, c_int64, c_void_p, c_int64,          # packed, scales
        c_void_p, c_int64, c_int,                      # zeros, z_row_stride, zeros_packed
        c_void_p, c_int, c_int64,                      # outlier_idx, idx_dtype, n_out
        c_void_p, c_int, c_int64,                      # outlier_w, ow_dtype, ow_row_stride
        c_void_p, c_int, c_int64,                      # out, out_dtype, out_row_stride
        c_int64, c_int64, c_int, c_void_p]),           # V, K, layout, stream
    "spectra_argmax": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "spectra_fwht": (c_int, [c_void_p, c_int, c_int64, c_void_p, c_int, c_int64, c_int64, c_int64, c_int, c_void_p]),
    "spectra_p2p_buffer_bytes": (c_int64, [c_int64, c_int64, c_int64, c_int]),
    "spectra_p2p_alloc": (c_int, [c_int64, c_void_p, c_void_p]),
    "spectra_p2p_open": (c_int, [c_void_p, c_void_p]),
    "spectra_p2p_close": (c_int, [c_void_p]),
    "spectra_p2p_free": (c_int, [c_void_p]),
    "spectra_p2p_allgather": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int64,
                                      c_int64, c_void_p, c_int, c_int, c_int64, c_void_p]),
    "spectra_device_timeouts": (c_int, [c_void_p, c_int]),
    "spectra_selftest_wait_timeout": (c_int, [c_void_p]),
    "spectra_w4a16_dequant": (c_int, [
        c_void_p, c_int64,
        c_void_p, c_int64, c_int64,
        c_void_p, c_int64, c_int64,
        c_void_p, c_int, c_int64,
        c_int64, c_int64, c_int, c_void_p]),
}

_lib = None


class SpectraError(RuntimeError):
    def __init__(self, fn: str, status: int):
        self.status = status
        msg = _status_string(status)
        if status == ERR_CUDA and _lib is not None:
            msg += f" (cudaError {_lib.spectra_last_cuda_error()})"
        super().__init__(f"{fn} failed with status {status}: {msg}")


def _status_string(status: int) -> str:
    if _lib is None:
        return "library not loaded"
    return _lib.spectra_status_string(status).decode()


def lib():
    """Load (once) and return the ctypes handle; raises if the library is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python -m spectra_b200.build` "
                "(spectra_b200 has no CPU or Python fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in PROTOTYPES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        if L.spectra_abi_version() != ABI_VERSION:
            raise RuntimeError(f"ABI version mismatch: library {L.spectra_abi_version()}, binding {ABI_VERSION}")
        _lib = L
    return _lib


def check(fn: str, status: int) -> None:
    if status != OK:
        raise SpectraError(fn, status)
