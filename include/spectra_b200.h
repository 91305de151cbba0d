/*
 * spectra_b200.h -- C ABI of libspectra_b200.so, the B200 (sm_100a) W4A16
 * linear-layer hot path of SPECTRA.
 *
 * Weight format (produced by the reference's SpectraCompressor,
 * spectra/compressor.py:72-112, and bound by spectra/engine.py:999-1026):
 *   packed   u8   [N, K/2]   two 4-bit codes per byte, unit column stride
 *   scales   fp16 [N, K/32]  one per group of 32 input features
 *   zeros    u8   [N, K/32]  one zero-point (0..15) per group, unpacked
 *   outlier_idx  int64|int32 [n_out]     input columns kept exactly
 *   outlier_w    fp16|bf16  [N, n_out]   their exact weights
 * dequantised weight:  w[n,k] = (q[n,k] - z[n,k/32]) * s[n,k/32]
 * Nibble order inside a 32-code group (16 bytes):
 *   SPECTRA_LAYOUT_MARLIN   byte j: k=j in the low nibble, k=j+16 in the high nibble
 *   SPECTRA_LAYOUT_EVEN_ODD byte b: k=2b low, k=2b+1 high
 *
 * Conventions: every pointer is a device pointer; strides are in ELEMENTS of
 * the pointed-to type; `stream` is a cudaStream_t (NULL = legacy default
 * stream).  Calls never allocate device memory and never synchronise the
 * host.  All argument checks run on the host before any CUDA call, so a bad
 * call returns an error code and launches nothing.  Return value: SPECTRA_OK
 * or one of the SPECTRA_ERR_* codes below.
 */
#ifndef SPECTRA_B200_H
#define SPECTRA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SPECTRA_API __attribute__((visibility("default")))
#else
#define SPECTRA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SPECTRA_B200_ABI_VERSION 1

/* element types */
#define SPECTRA_DT_F16  0
#define SPECTRA_DT_BF16 1
#define SPECTRA_DT_F32  2
#define SPECTRA_DT_I32  3
#define SPECTRA_DT_I64  4

/* nibble order */
#define SPECTRA_LAYOUT_EVEN_ODD 0
#define SPECTRA_LAYOUT_MARLIN   1

/* status codes */
#define SPECTRA_OK               0
#define SPECTRA_ERR_NULL_POINTER 1
#define SPECTRA_ERR_SHAPE        2
#define SPECTRA_ERR_STRIDE       3
#define SPECTRA_ERR_ALIGNMENT    4
#define SPECTRA_ERR_DTYPE        5
#define SPECTRA_ERR_WORKSPACE    6
#define SPECTRA_ERR_CUDA         7
#define SPECTRA_ERR_UNSUPPORTED  8

/* Version of this ABI (SPECTRA_B200_ABI_VERSION of the built library). */
SPECTRA_API int spectra_abi_version(void);

/* Static, NUL-terminated description of a status code. */
SPECTRA_API const char* spectra_status_string(int status);

/* cudaError_t of the last CUDA call that failed on the calling thread
 * (0 if none); read it after a call returned SPECTRA_ERR_CUDA. */
SPECTRA_API int spectra_last_cuda_error(void);

/*
 * M=1 decode GEMV with fused outlier-column and bias adds.
 * Replaces spectra/kernels.py:132-184 (fused_w4a16_gemv_hdsq, the wrapper)
 * and spectra/kernels.py:16-129 (_fused_w4a16_gemv_hdsq_kernel).
 *   y[n] = sum_k x[k]*w[n,k] + sum_j x[idx_j]*ow[n,j] + bias[n]
 * accumulated in fp32 and rounded once to y_dtype.
 *   x      [K]  at x + k*x_stride, x_dtype F16|BF16|F32
 *   packed row n at packed + n*w_row_stride (bytes); column stride is 1
 *   scales[n,g] at scales + n*s_row_stride + g*s_col_stride (fp16 bits)
 *   zeros [n,g] at zeros  + n*z_row_stride + g*z_col_stride
 *   bias   [N] or NULL (bias_dtype F16|BF16|F32)
 *   outlier_idx NULL or [n_out] (idx_dtype I32|I64); outlier_w [n,j] at
 *          outlier_w + n*ow_row_stride + j*ow_col_stride (ow_dtype F16|BF16|F32)
 *   y      [N]  at y + n*y_stride, y_dtype F16|BF16|F32
 * K must be a positive multiple of 32 and N positive.
 */
SPECTRA_API int spectra_w4a16_gemv(
    const void* x, int x_dtype, int64_t x_stride,
    const uint8_t* packed, int64_t w_row_stride,
    const uint16_t* scales, int64_t s_row_stride, int64_t s_col_stride,
    const uint8_t* zeros, int64_t z_row_stride, int64_t z_col_stride,
    const void* bias, int bias_dtype,
    const void* outlier_idx, int idx_dtype, int64_t n_out,
    const void* outlier_w, int ow_dtype, int64_t ow_row_stride, int64_t ow_col_stride,
    void* y, int y_dtype, int64_t y_stride,
    int64_t N, int64_t K, int layout, void* stream);

/*
 * Dequantise to a dense matrix.  out_dtype F32 gives (q-z)*s exactly (the
 * fp32 value the reference GEMV multiplies by, spectra/kernels.py:73-74);
 * BF16 / F16 give that value rounded to nearest-even, the operand the
 * reference GEMM feeds its tensor-core dot (spectra/kernels.py:256-261).
 * Outlier columns are left as dequantised (the reference test overwrites
 * them with outlier_w, tests/test_kernels.py:38-39; that is the caller's job).
 *   out[n,k] at out + n*out_row_stride + k
 */
SPECTRA_API int spectra_w4a16_dequant(
    const uint8_t* packed, int64_t w_row_stride,
    const uint16_t* scales, int64_t s_row_stride, int64_t s_col_stride,
    const uint8_t* zeros, int64_t z_row_stride, int64_t z_col_stride,
    void* out, int out_dtype, int64_t out_row_stride,
    int64_t N, int64_t K, int layout, void* stream);

/*
 * M >= 2 GEMM on the tensor cores.
 * Replaces spectra/kernels.py:333-389 (batched_w4a16_gemm, the wrapper) and
 * spectra/kernels.py:191-331 (_batched_w4a16_gemm_kernel).
 *   c[m,n] = sum_k a[m,k] * R((q-z)*s) + sum_j a[m,idx_j] * R(ow[n,j])
 * where R() rounds to a's dtype (the reference's tensor-core operands),
 * accumulated in fp32 and rounded once to c (same dtype as a).  No bias
 * (the engine adds it, spectra/engine.py:122-123).  For M <= 16 with the
 * layout spectra_gemm_small_m_plan accepts, a small-M kernel computes the same
 * product with the exact dequantised weights instead of R((q-z)*s) (as the
 * M=1 GEMV does; within the path's tolerance of the rounded form) and uses no
 * workspace.
 *   a      [M, K] at a + m*a_row_stride + k; a_dtype F16|BF16; 16-byte aligned
 *          base, row stride a multiple of 8 elements (TMA tensor map)
 *   packed row n at packed + n*w_row_stride; base and row stride 16-byte aligned
 *   c      [M, N] at c + m*c_row_stride + n, c_dtype == a_dtype
 *   workspace: caller-owned device memory of at least
 *          spectra_w4a16_gemm_workspace_bytes(M, N, K, n_out) bytes (split-K
 *          counters and partials; from 17 tokens on with outlier columns, the
 *          activations at those columns gathered once per call), zeroed once
 *          before its first use; every call leaves its counter region zero
 *          again.  Calls that share a workspace must not overlap in time.
 */
SPECTRA_API int spectra_w4a16_gemm(
    const void* a, int a_dtype, int64_t a_row_stride,
    const uint8_t* packed, int64_t w_row_stride,
    const uint16_t* scales, int64_t s_row_stride, int64_t s_col_stride,
    const uint8_t* zeros, int64_t z_row_stride, int64_t z_col_stride,
    const void* outlier_idx, int idx_dtype, int64_t n_out,
    const void* outlier_w, int ow_dtype, int64_t ow_row_stride, int64_t ow_col_stride,
    void* c, int c_dtype, int64_t c_row_stride,
    int64_t M, int64_t N, int64_t K, int layout,
    void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes spectra_w4a16_gemm needs for this problem (0: none). */
SPECTRA_API size_t spectra_w4a16_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t n_out);

/*
 * Allocation-free variant of spectra_w4a16_gemm.  It has no counterpart in the
 * reference (spectra/kernels.py allocates its output and scratch through
 * torch).  It is for callers that cannot allocate device memory or hand the
 * GEMM a workspace: a host whose own arena already owns the device memory
 * (a cudaMalloc there fails or synchronises the whole device in the middle
 * of a forward pass), or a plugin interface that passes only the operands,
 * like the reference's batched_w4a16_gemm signature (no workspace argument).
 *
 * Same arguments and results as spectra_w4a16_gemm, without the workspace:
 * its scratch (split-K counters and partials, the gathered activations at the
 * outlier columns) lives in one file-scope device array of
 * SPECTRA_GEMM_NOALLOC_SCRATCH_BYTES per device, and the call makes no
 * cudaMalloc/cudaFree or other allocating call.
 *   - Limit: a problem whose spectra_w4a16_gemm_workspace_bytes(M, N, K, n_out)
 *     exceeds SPECTRA_GEMM_NOALLOC_SCRATCH_BYTES is rejected with
 *     SPECTRA_ERR_WORKSPACE before anything launches.
 *   - Zero state: the scratch's counters must be zero when a call starts.  The
 *     array is zero when the module loads and every call leaves its counters
 *     zero again, so the caller never clears anything.
 *   - Setup: the first call on each device looks the array's address up with
 *     cudaGetSymbolAddress (with that device current), which may load the
 *     module; make that first call before any stream capture begins.  The
 *     address is looked up again when the device's context has been recreated
 *     since (cudaDeviceReset), so make the first call after a reset outside a
 *     capture too.
 *   - Races: all calls on one device (all streams and host threads of the
 *     process) share the one array, so calls that overlap in time race and
 *     give wrong results.  Issue them one after another, e.g. on one stream.
 */
#define SPECTRA_GEMM_NOALLOC_SCRATCH_BYTES 8388608  /* 8 MiB */

SPECTRA_API int spectra_w4a16_gemm_noalloc(
    const void* a, int a_dtype, int64_t a_row_stride,
    const uint8_t* packed, int64_t w_row_stride,
    const uint16_t* scales, int64_t s_row_stride, int64_t s_col_stride,
    const uint8_t* zeros, int64_t z_row_stride, int64_t z_col_stride,
    const void* outlier_idx, int idx_dtype, int64_t n_out,
    const void* outlier_w, int ow_dtype, int64_t ow_row_stride, int64_t ow_col_stride,
    void* c, int c_dtype, int64_t c_row_stride,
    int64_t M, int64_t N, int64_t K, int layout, void* stream);

/*
 * Group-32 INT4 quantiser on the GPU: the tensors SpectraCompressor writes
 * for one weight (replaces SpectraCompressor._quantize_chunk_group32 and
 * _compute_group32_quant, spectra/compressor.py:72-156).  Input columns listed
 * in outlier_idx (may be NULL with n_out = 0) are read as zero, as the
 * reference zeroes them before quantising (:137-140).  Per group of 32: fp32
 * min/max, s = (max-min)/15 (constant groups: |min|, or 1 when min == 0),
 * clamped to >= 1e-8, z = clamp(round(-min/s), 0, 15), q = clamp(round((w +
 * z*s)/s), 0, 15), round half to even, correctly rounded divisions: the codes
 * are bit-identical to the reference run on a CPU.
 *   w       [N, K] at w + n*w_row_stride + k, w_dtype F16|BF16|F32
 *   packed  [N, K/2] (layout MARLIN as the compressor writes, or EVEN_ODD)
 *   scales  [N, K/32] fp16 bits
 *   zeros   [N, K/32] one byte per group (as the engine binds them) or NULL
 *   packed_zeros [N, ceil(K/64)] two per byte, low nibble = even group (the
 *           container form, spectra/compressor.py:104-110) or NULL
 */
SPECTRA_API int spectra_quantize_group32(
    const void* w, int w_dtype, int64_t w_row_stride,
    const void* outlier_idx, int idx_dtype, int64_t n_out,
    uint8_t* packed, int64_t p_row_stride,
    uint16_t* scales, int64_t s_row_stride,
    uint8_t* zeros, int64_t z_row_stride,
    uint8_t* packed_zeros, int64_t pz_row_stride,
    int64_t N, int64_t K, int layout, void* stream);

/*
 * Load-time zero-point unpack on the GPU (replaces the torch code at
 * spectra/engine.py:1007-1012): packed_zeros [N, ceil(G/2)] (low nibble =
 * group 2j, high nibble = group 2j+1) -> zeros [N, G], one byte per group.
 */
SPECTRA_API int spectra_unpack_zeros(const uint8_t* packed_zeros, int64_t pz_row_stride, uint8_t* zeros,
                                     int64_t z_row_stride, int64_t N, int64_t G, void* stream);

/*
 * INT4 KV-cache quantiser (replaces SpectraGroup32QuantizedLayer._quantize,
 * spectra/engine.py:625-656).  t: contiguous [rows, D] F16|BF16; groups of 32
 * along D (zero-padded to a multiple of 32, G = ceil(D/32)); computed in t's
 * dtype with the reference's rounding steps as torch runs them on a CUDA
 * device.  Outputs (contiguous): packed [rows, G, 16] even-odd nibbles
 * (16-byte aligned), scales [rows, G] fp16 bits, zeros [rows, G] bytes.
 */
SPECTRA_API int spectra_kv_quantize(const void* t, int t_dtype, int64_t rows, int64_t D, uint8_t* packed,
                                    uint16_t* scales, uint8_t* zeros, void* stream);

/*
 * INT4 KV-cache dequantiser (replaces SpectraGroup32QuantizedLayer._dequantize,
 * spectra/engine.py:658-671): out [rows, D] = (q - z) * s, exact in fp32,
 * rounded once to out_dtype (the reference returns bf16); padding dropped.
 */
SPECTRA_API int spectra_kv_dequantize(const uint8_t* packed, const uint16_t* scales, const uint8_t* zeros,
                                      void* out, int out_dtype, int64_t rows, int64_t D, void* stream);

/*
 * Quantised token-embedding gather (replaces SpectraFusedEmbedding.forward,
 * spectra/engine.py:167-212): out[t, :] = dequantised row ids[t] of the
 * [V, K] vocabulary matrix ((q - z) * s in fp32, rounded once to out_dtype),
 * then the outlier columns set to outlier_w[ids[t], j] rounded to out_dtype.
 * zeros_packed != 0: zeros are [V, ceil(G/2)] two per byte.  An id outside
 * [0, V) yields a zero row.
 *   ids    [T] I32|I64;  packed [V, K/2];  scales [V, K/32] fp16 bits
 *   outlier_w [v, j] at outlier_w + v*ow_row_stride + j
 *   out    [T, K] at out + t*out_row_stride + k, out_dtype F16|BF16|F32
 */
SPECTRA_API int spectra_w4a16_embedding(
    const void* ids, int ids_dtype, int64_t T,
    const uint8_t* packed, int64_t w_row_stride,
    const uint16_t* scales, int64_t s_row_stride,
    const uint8_t* zeros, int64_t z_row_stride, int zeros_packed,
    const void* outlier_idx, int idx_dtype, int64_t n_out,
    const void* outlier_w, int ow_dtype, int64_t ow_row_stride,
    void* out, int out_dtype, int64_t out_row_stride,
    int64_t V, int64_t K, int layout, void* stream);

/*
 * Greedy next-token choice (the argmax of the engine's temperature-0
 * sample_token, spectra/engine.py:1690-1713): idx[m] = idx_offset + the first
 * index of the maximum of row m of x [M, N] (a NaN counts as the maximum, as
 * in torch.argmax); val[m] (optional) = that maximum as fp32.  idx_offset lets
 * an N-sharded lm_head report the layer's row index, so the shards reduce
 * (value, index) pairs instead of gathering every logit.  M <= 65535.
 */
SPECTRA_API int spectra_argmax(const void* x, int x_dtype, int64_t x_row_stride, int64_t M, int64_t N,
                               int64_t idx_offset, int64_t* idx, float* val, void* stream);

/*
 * Walsh-Hadamard rotation of activation rows, the optional GEMV prologue
 * (the reference's fast_walsh_hadamard_transform, spectra/compressor.py:29-42,
 * which its compressor cannot yet apply to weights: off by default in the
 * drop-in).  y[m] = H x[m] (/ sqrt(n) if normalize), butterflies in fp32, one
 * rounding to y_dtype; n a power of two, <= 32768.
 */
SPECTRA_API int spectra_fwht(const void* x, int x_dtype, int64_t x_row_stride, void* y, int y_dtype,
                             int64_t y_row_stride, int64_t M, int64_t n, int normalize, void* stream);

/*
 * All-gather of an N-sharded layer's output over NVLink peer memory (the
 * reference has no multi-GPU path: this is the exchange step of its large
 * layers column-sharded over the GPUs of one node, in place of an NCCL
 * all-gather).  Setup, once per layer shape on every rank:
 *   bytes = spectra_p2p_buffer_bytes(M, ns, elem_bytes, world);
 *   spectra_p2p_alloc(bytes, &mine, handle);     -- cudaMalloc'd, zeroed (synchronises the device);
 *                                                   64-byte CUDA IPC handle
 *   (exchange the handles between the ranks, e.g. over the host's process group)
 *   spectra_p2p_open(handle_of_r, &peer[r]);     -- for every r != rank; peer[rank] = mine
 * and an int32[SPECTRA_P2P_STATE_INTS] device `state`, zeroed.  Per call, with this rank's slice
 * [M][ns] (elem_bytes each, 16-byte aligned, spectra_p2p_buffer_bytes' slice
 * rounded up to 16 bytes readable) in `src`: the launched kernel pushes it into
 * every peer's buffer, exchanges an epoch flag with every peer and writes the
 * gathered [M][N] output (row stride out_row_stride elements; rank r's columns
 * start at r*ns, N <= world*ns: the last ranks' may be ragged or empty).
 * All ranks must make the same calls in the same order; one call may be
 * replayed from a CUDA graph.  A peer that does not signal within
 * wait_limit_ns ends the wait: the event is counted by
 * spectra_device_timeouts and the output is undefined.  Teardown:
 * spectra_p2p_close(peer[r]) for r != rank, then spectra_p2p_free(mine).
 * spectra_p2p_buffer_bytes returns -1 for an unsupported shape
 * (elem_bytes 2, 4 or 8; world 1..8).
 */
#define SPECTRA_P2P_STATE_INTS 128
SPECTRA_API int64_t spectra_p2p_buffer_bytes(int64_t M, int64_t ns, int64_t elem_bytes, int world);
SPECTRA_API int spectra_p2p_alloc(int64_t bytes, void** ptr, void* ipc_handle);
SPECTRA_API int spectra_p2p_open(const void* ipc_handle, void** ptr);
SPECTRA_API int spectra_p2p_close(void* ptr);
SPECTRA_API int spectra_p2p_free(void* ptr);
SPECTRA_API int spectra_p2p_allgather(const void* src, void* const* peer_buffers, int64_t buffer_bytes, void* out,
                                      int64_t out_row_stride, int64_t M, int64_t ns, int64_t N, int64_t elem_bytes,
                                      int* state, int rank, int world, int64_t wait_limit_ns, void* stream);

/*
 * Diagnostic, not a reference interface (the reference's Triton kernels have
 * no bounded waits).  Every pipeline wait in this library's kernels gives up
 * after 2 s instead of hanging; the kernel then abandons its work, leaves the
 * output of that call undefined and counts the event in a device counter.
 * This returns in *count the number of such timed-out waits on the current
 * device since the library loaded (or since the last reset), and zeroes the
 * counters if `reset` is non-zero.  It reads device memory, so it waits for
 * all work queued on the device: call it between steps, not inside a CUDA
 * graph capture.  A non-zero count means the results of some earlier call
 * must be discarded.
 */
SPECTRA_API int spectra_device_timeouts(int64_t* count, int reset);

/*
 * Self-test of the bounded wait (not a reference interface): launches one
 * thread that waits on a pipeline barrier nothing ever arrives on.  The wait
 * gives up after the library's 2 s limit, the kernel returns and
 * spectra_device_timeouts() counts one more timeout.  Nothing is copied and
 * nothing is written besides the counter.
 */
SPECTRA_API int spectra_selftest_wait_timeout(void* stream);

/*
 * Diagnostic, not a reference interface: the configuration the M=1 GEMV
 * (spectra_w4a16_gemv) picks for contiguous, 16-byte-aligned weights of
 * shape [N, K], contiguous x of x_dtype and n_out outlier columns of ow_dtype
 * stored [N, n_out], on a GPU with `sms` SMs.  Computed on the host without a
 * GPU.  out[10]: 1 if the weight-prefetching kernel takes the call (else all
 * zero: the other kernel does), compute groups, chunked stages (1/0), ring
 * stages, bytes per stage, outlier rows staged before the wait (1/0), outlier
 * rows per piece streamed through the ring (0: none), dynamic shared memory
 * bytes, grid, row blocks per CTA.
 */
SPECTRA_API int spectra_gemv_pf_plan(int64_t N, int64_t K, int64_t n_out, int x_dtype, int ow_dtype, int sms,
                                     int64_t* out);

/*
 * Diagnostic, not a reference interface: whether spectra_w4a16_gemm takes its
 * small-M kernel for an [M, K] x [N, K] product with contiguous, 16-byte
 * aligned operands and n_out outlier columns of ow_dtype stored [N, n_out],
 * on a GPU with `sms` SMs (host only, no GPU).  out[7]: 1 if it does (else all
 * zero: the tcgen05 GEMM runs), grid, dynamic shared memory bytes, ring
 * stages, outlier rows staged before the wait (1/0), compute groups, token
 * tiles of 8.  The kernel takes
 * 2 <= M <= 16, K a multiple of 512, bf16/fp16 activations, when the staged
 * activations of all M rows and two weight stages fit in shared memory.
 * SPECTRA_B200_GEMM_SMALL_M=0 in the environment turns it off.
 */
SPECTRA_API int spectra_gemm_small_m_plan(int64_t M, int64_t N, int64_t K, int64_t n_out, int a_dtype, int ow_dtype,
                                          int sms, int64_t* out);

/*
 * Diagnostic, not a reference interface: the tcgen05 GEMM's plan for an
 * [M, K] x [N, K] product with n_out outlier columns (host only, no GPU).
 * out[8]: token tile MT, token chunks, weight tiles, K splits, SM pairs
 * (1/0: tiles of >= 128 tokens on two-CTA clusters, cta_group::2), CTAs per
 * chunk, activation stages, workspace bytes.  The SM pairs are off unless
 * SPECTRA_B200_GEMM_PAIR=1 is in the environment (read once per process).
 */
SPECTRA_API int spectra_gemm_plan(int64_t M, int64_t N, int64_t K, int64_t n_out, int64_t* out);

/*
 * Diagnostic: how many two-CTA clusters of the SM-pair GEMM kernel the current
 * device holds at once (cudaOccupancyMaxActiveClusters at the kernel's largest
 * shared-memory size).  The plan assumes all SMs pair up: 74 on a B200.
 */
SPECTRA_API int spectra_gemm_pair_capacity(int* clusters);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* SPECTRA_B200_H */
