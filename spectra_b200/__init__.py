"""spectra_b200 -- B200-native (sm_100a) W4A16 linear-layer hot path for SPECTRA.

Drop-in replacement for the reference's ``spectra.kernels`` operator API:
``fused_w4a16_gemv_hdsq`` (M=1 decode GEMV) and ``batched_w4a16_gemm``
(M>=2 GEMM), backed by hand-written CUDA kernels in ``libspectra_b200.so``
reached through a plain C ABI (``include/spectra_b200.h``).
"""
__version__ = "0.1.0"
