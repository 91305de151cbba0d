// Internal interface of the format, KV-cache, embedding and rotation kernels
// (not part of the public C ABI; the extern "C" wrappers live in abi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace spectra {

// Group-32 INT4 quantiser (format.cu).
struct QuantArgs {
  const void* w; int w_dtype; int64_t w_rs;  // [N, K] source weights
  int w_vec;                                  // 16-byte aligned rows (set by the launcher)
  const void* idx; int idx_dtype; int n_out;  // outlier columns (read as 0), may be empty
  uint8_t* packed; int64_t p_rs; int packed_vec;  // [N, K/2]; packed_vec: 16-byte aligned rows
  uint16_t* scales; int64_t s_rs;             // [N, K/32] fp16
  uint8_t* zeros; int64_t z_rs;               // [N, K/32] or NULL
  uint8_t* packed_zeros; int64_t pz_rs;       // [N, ceil(K/64)] or NULL
  int N, K, layout;
};
int launch_quantize_group32(QuantArgs a, cudaStream_t st);

struct UnpackZerosArgs {
  const uint8_t* packed_zeros; int64_t pz_rs;  // [N, ceil(G/2)]
  uint8_t* zeros; int64_t z_rs;                // [N, G]
  int64_t N; int G;
};
int launch_unpack_zeros(const UnpackZerosArgs& a, cudaStream_t st);

// INT4 KV-cache group quantiser / dequantiser (kvcache.cu).
struct KvQuantArgs {
  const void* t; int t_dtype; int64_t rows; int D;  // [rows, D] contiguous, F16|BF16
  uint8_t* packed;                                   // [rows, G, 16]
  uint16_t* scales;                                  // [rows, G] fp16
  uint8_t* zeros;                                    // [rows, G]
};
struct KvDequantArgs {
  const uint8_t* packed; const uint16_t* scales; const uint8_t* zeros;  // as above
  void* out; int out_dtype; int64_t rows; int D;                        // [rows, D]
};
int launch_kv_quantize(const KvQuantArgs& a, cudaStream_t st);
int launch_kv_dequantize(const KvDequantArgs& a, cudaStream_t st);

// Embedding gather-dequantise and greedy argmax (embed.cu).
struct EmbedArgs {
  const void* ids; int ids_dtype; int64_t T;          // token ids [T]
  const uint8_t* packed; int64_t w_rs;                // [V, K/2]
  const uint16_t* scales; int64_t s_rs;               // [V, G] fp16
  const uint8_t* zeros; int64_t z_rs; int zeros_packed;  // [V, G] or packed [V, ceil(G/2)]
  const void* idx; int idx_dtype; int n_out;          // outlier columns
  const void* ow; int ow_dtype; int64_t ow_rs;        // [V, n_out]
  void* out; int out_dtype; int64_t out_rs;           // [T, K]
  int64_t V; int K; int layout;
  bool vec_out;                                       // 16-byte stores (set by the launcher)
};
int launch_embedding(EmbedArgs a, cudaStream_t st);

struct ArgmaxArgs {
  const void* x; int x_dtype; int64_t x_rs;  // [M, N]
  int64_t* idx;                              // [M]
  float* val;                                // [M] or NULL
  int64_t M; int64_t N; int64_t idx_offset;  // idx_offset added to every index (a shard's first row)
  int64_t span;                              // elements per CTA of a row's cluster (set by the launcher)
  bool vec;                                  // 16-byte loads (set by the launcher)
};
int launch_argmax(ArgmaxArgs a, cudaStream_t st);

// Walsh-Hadamard rotation of activation rows (fwht.cu).
struct FwhtArgs {
  const void* x; int x_dtype; int64_t x_rs;  // [M, n]
  void* y; int y_dtype; int64_t y_rs;        // [M, n]
  int64_t M; int n; float inv_norm;          // inv_norm: sqrt(n) (divisor) or 1 (no normalisation)
  int normalize;
};
int launch_fwht(const FwhtArgs& a, cudaStream_t st);

}  // namespace spectra
