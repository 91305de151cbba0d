// Dense dequantisation (q - z) * s: the bit-exact check of the weight decode
// and a load-time utility.  Follows spectra/kernels.py:56-74 (fp32 value) and
// :256-261 (rounded to the GEMM operand dtype).
#include "common.cuh"
#include "gemv.h"

namespace spectra {

namespace {

__global__ void dequant_kernel(const DequantArgs a) {
  const int G = a.K / kGroup;
  const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= a.N * G) return;
  const int64_t row = t / G;
  const int g = int(t % G);
  const uint8_t* src = a.packed + row * a.w_rs + int64_t(g) * kGroupBytes;
  const float s = __half2float(a.scales[row * a.s_rs + int64_t(g) * a.s_cs]);
  const float z = float(a.zeros[row * a.z_rs + int64_t(g) * a.z_cs]);
  const int64_t o = row * a.out_rs + int64_t(g) * kGroup;
#pragma unroll 4
  for (int b = 0; b < kGroupBytes; ++b) {
    const uint32_t byte = src[b];
    const float lo = (float(byte & 0xFu) - z) * s;   // exact: |q-z| <= 15, s fp16
    const float hi = (float(byte >> 4) - z) * s;
    store_from_float(a.out, o + code_k(b, 0, a.layout), a.out_dtype, lo);
    store_from_float(a.out, o + code_k(b, 1, a.layout), a.out_dtype, hi);
  }
}

}  // namespace

int launch_dequant(const DequantArgs& a, cudaStream_t st) {
  const int64_t total = a.N * (a.K / kGroup);
  const int threads = 256;
  const int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 0x7fffffff) return SPECTRA_ERR_SHAPE;
  dequant_kernel<<<unsigned(blocks), threads, 0, st>>>(a);
  return cuda_status(cudaGetLastError());
}

}  // namespace spectra
