// Internal interface of the tensor-core GEMM launcher (not part of the public C ABI).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>

namespace spectra {

struct GemmArgs {
  const void* a; int a_dtype; int64_t a_rs;           // [M, K], unit column stride
  const uint8_t* packed; int64_t w_rs;
  const __half* scales; int64_t s_rs, s_cs;
  const uint8_t* zeros; int64_t z_rs, z_cs;
  const void* idx; int idx_dtype; int n_out;
  const void* ow; int ow_dtype; int64_t ow_rs, ow_cs;
  void* c; int c_dtype; int64_t c_rs;                 // [M, N], unit column stride, a's dtype
  int M, N, K, layout;
};

struct GemmPlan {
  int MT, m_chunks, tiles_n;
  bool pair;                  // tiles on SM pairs (cta_group::2): MT >= 128
  int tiles_pad;              // tiles_n, rounded up to even in pair mode (the last pair's odd CTA has no rows)
  int nk, ncs, n_os;          // 64-k MMA steps, 256-k code stages, 64-column outlier steps
  int S;                      // K splits per tile
  int act_stages, code_stages, act_stage_bytes;
  int issuers;                // warps issuing MMAs (each with its own accumulator)
  int a_slots;                // TMEM A slots of one 256-k unit (2 or 3)
  uint32_t tmem_cols;
  bool pregather;             // outlier activations gathered once per call (token tiles >= 32)
  size_t partials_off;        // workspace offset of the split-K partials (after the counters)
  size_t gather_off;          // workspace offset of the gathered tile [M][n_os * 64]
  size_t smem, workspace;
};

GemmPlan plan_gemm(int64_t M, int64_t N, int64_t K, int64_t n_out);
int launch_gemm(const GemmArgs& a, void* ws, size_t ws_bytes, cudaStream_t st);
// Two-CTA clusters of the SM-pair kernel resident at once on the current device.
int gemm_pair_capacity(int* clusters);

// Small-M GEMM (M = 2..16) on the raw-code tensor-core step (gemv_mt.cu);
// SPECTRA_ERR_UNSUPPORTED (nothing launched) when the arguments do not meet
// its conditions, and the tcgen05 GEMM takes the call.
int launch_gemv_mt(const GemmArgs& a, cudaStream_t st);
int gemv_mt_timeouts(long long* out, bool reset);

// Address and size of the static split-K scratch of the current device
// (looked up once per device with cudaGetSymbolAddress).
int gemm_noalloc_scratch(void** ptr, size_t* bytes);

}  // namespace spectra
