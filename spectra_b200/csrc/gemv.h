// Internal interface of the GEMV launcher (not part of the public C ABI).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <algorithm>

namespace spectra {

// Staged activation window (groups) and dynamic shared-memory ceiling.
constexpr int kGemvMaxWindowGroups = 448;   // 14336 input features per window
constexpr size_t kGemvMaxSmem = 200 * 1024;

struct GemvArgs {
  const void* x; int x_dtype; int64_t x_stride;
  const uint8_t* packed; int64_t w_rs;
  const __half* scales; int64_t s_rs, s_cs;
  const uint8_t* zeros; int64_t z_rs, z_cs;
  const void* bias; int bias_dtype;
  const void* idx; int idx_dtype; int n_out;
  const void* ow; int ow_dtype; int64_t ow_rs, ow_cs;
  void* y; int y_dtype; int64_t y_stride;
  int N, K, layout;
};

struct GemvPlan {
  int S, RG, R, threads, win_groups;
  int64_t grid;
  size_t smem;
};

GemvPlan plan_gemv(int64_t N, int64_t K, int64_t n_out);
int launch_gemv(const GemvArgs& a, cudaStream_t st);

// Weight-prefetching tensor-core GEMV (gemv_pf.cu); SPECTRA_ERR_UNSUPPORTED
// (nothing launched) when the arguments do not meet its layout conditions.
int launch_gemv_pf(const GemvArgs& a, cudaStream_t st);

struct DequantArgs {
  const uint8_t* packed; int64_t w_rs;
  const __half* scales; int64_t s_rs, s_cs;
  const uint8_t* zeros; int64_t z_rs, z_cs;
  void* out; int out_dtype; int64_t out_rs;
  int64_t N; int K; int layout;
};

int launch_dequant(const DequantArgs& a, cudaStream_t st);

}  // namespace spectra
