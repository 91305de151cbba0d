// Weight-format kernels: the group-32 INT4 quantiser that produces SPECTRA's
// weight tensors (restating spectra/compressor.py:72-156 on the GPU) and the
// load-time zero-point unpack (spectra/engine.py:1007-1012).
//
// Quantiser, per group of 32 input features (outlier columns read as 0,
// spectra/compressor.py:137-140), all in IEEE fp32 with the reference's
// operation order -- that order is what makes the codes bit-identical:
//   lo, hi = min, max;  diff = hi - lo;  constant = diff < 1e-8f
//   s = constant ? (lo == 0 ? 1 : |lo|) : diff / 15;   s = max(s, 1e-8f)
//   z = constant ? (lo < 0) : clamp(rint(-lo / s), 0, 15)
//   q = constant ? (lo > 0) : clamp(rint((w - (-(z * s))) / s), 0, 15)
// rint is round-half-to-even (torch.round); divisions are correctly rounded
// (__fdiv_rn: never a multiply by a reciprocal).  Scales are stored as fp16
// (round to nearest even), zero points both unpacked (one byte per group, what
// the engine binds) and packed two per byte (the container form, odd group
// counts padded with 0).
//
// Work decomposition: one thread per pair of groups of one row (64 features:
// 32 code bytes, one packed zero-point byte), so the packed zero point needs
// no exchange between threads.  The outlier columns are a bitmask in shared
// memory, built by each CTA from the index list.  HBM-bound: ~2 B read (fp16)
// and ~0.6 B written per weight.
#include <algorithm>

#include "common.cuh"
#include "format.h"
#include "gemv_mma.cuh"

namespace spectra {

namespace {

constexpr int kQuantThreads = 256;

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }

template <typename T>
__global__ void __launch_bounds__(kQuantThreads) quantize_group32_kernel(QuantArgs a) {
  extern __shared__ uint32_t out_mask[];  // one bit per input feature: outlier column
  const int words = (a.K + 31) / 32;
  for (int i = threadIdx.x; i < words; i += blockDim.x) out_mask[i] = 0u;
  __syncthreads();
  for (int j = threadIdx.x; j < a.n_out; j += blockDim.x) {
    const int64_t k = load_index(a.idx, j, a.idx_dtype);
    if (k >= 0 && k < a.K) atomicOr(&out_mask[k >> 5], 1u << (k & 31));
  }
  __syncthreads();

  const int G = a.K / kGroup;
  const int pairs = (G + 1) / 2;
  const int64_t total = int64_t(a.N) * pairs;
  const T* w = reinterpret_cast<const T*>(a.w);
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t n = t / pairs;
    const int pr = int(t - n * pairs);
    const T* row = w + n * a.w_rs;
    uint32_t zpair = 0;
    for (int h = 0; h < 2; ++h) {
      const int g = 2 * pr + h;
      if (g >= G) break;
      float v[kGroup];
      const uint32_t m = out_mask[g];  // group g covers features 32g..32g+31: one mask word
      if (a.w_vec) {
        // the group's 32 values by 16-byte loads
        constexpr int kWords = kGroup * int(sizeof(T)) / 4;
        uint32_t wd[kWords];
        const uint4* src = reinterpret_cast<const uint4*>(row + int64_t(g) * kGroup);
#pragma unroll
        for (int q4 = 0; q4 < kWords / 4; ++q4) {
          const uint4 u4 = __ldg(src + q4);
          wd[4 * q4] = u4.x; wd[4 * q4 + 1] = u4.y; wd[4 * q4 + 2] = u4.z; wd[4 * q4 + 3] = u4.w;
        }
        const T* vals = reinterpret_cast<const T*>(wd);
#pragma unroll
        for (int i = 0; i < kGroup; ++i) v[i] = ((m >> i) & 1u) ? 0.f : to_f32(vals[i]);
      } else {
#pragma unroll
        for (int i = 0; i < kGroup; ++i) {
          const float x = to_f32(row[int64_t(g) * kGroup + i]);
          v[i] = ((m >> i) & 1u) ? 0.f : x;
        }
      }
      float lo = v[0], hi = v[0];
#pragma unroll
      for (int i = 1; i < kGroup; ++i) {
        lo = fminf(lo, v[i]);
        hi = fmaxf(hi, v[i]);
      }
      const float diff = __fsub_rn(hi, lo);
      const bool flat = diff < 1e-8f;
      float s = flat ? (lo == 0.f ? 1.f : fabsf(lo)) : __fdiv_rn(diff, 15.f);
      s = fmaxf(s, 1e-8f);
      float z;
      if (flat) {
        z = lo < 0.f ? 1.f : 0.f;
      } else {
        z = fminf(fmaxf(rintf(__fdiv_rn(-lo, s)), 0.f), 15.f);
      }
      const float zs = -__fmul_rn(z, s);
      uint8_t q[kGroup];
#pragma unroll
      for (int i = 0; i < kGroup; ++i) {
        float c;
        if (flat) {
          c = lo > 0.f ? 1.f : 0.f;
        } else {
          c = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(v[i], zs), s)), 0.f), 15.f);
        }
        q[i] = uint8_t(c);
      }
      uint32_t words4[4];
#pragma unroll
      for (int wd = 0; wd < 4; ++wd) {
        uint32_t acc = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int byte = 4 * wd + b;
          const int k_lo = a.layout == SPECTRA_LAYOUT_MARLIN ? byte : 2 * byte;
          const int k_hi = a.layout == SPECTRA_LAYOUT_MARLIN ? byte + 16 : 2 * byte + 1;
          acc |= uint32_t(q[k_lo] | (q[k_hi] << 4)) << (8 * b);
        }
        words4[wd] = acc;
      }
      uint8_t* dst = a.packed + n * a.p_rs + int64_t(g) * kGroupBytes;
      if (a.packed_vec) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(words4[0], words4[1], words4[2], words4[3]);
      } else {
#pragma unroll
        for (int b = 0; b < 16; ++b) dst[b] = uint8_t(words4[b >> 2] >> (8 * (b & 3)));
      }
      reinterpret_cast<__half*>(a.scales)[n * a.s_rs + g] = __float2half_rn(s);
      const uint32_t zb = uint32_t(z);
      if (a.zeros) a.zeros[n * a.z_rs + g] = uint8_t(zb);
      zpair |= zb << (4 * h);
    }
    if (a.packed_zeros) a.packed_zeros[n * a.pz_rs + pr] = uint8_t(zpair);
  }
}

// Zero points packed two per byte -> one byte per group (low nibble: even group).
// Vector path: 8 packed bytes -> 16 zero points per item (rows padded to
// whole 16-group blocks, 8/16-byte aligned).
__global__ void unpack_zeros_vec_kernel(UnpackZerosArgs a) {
  const int blocks = a.G / 16;
  const int64_t total = a.N * int64_t(blocks);
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t n = t / blocks;
    const int b = int(t - n * blocks);
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(a.packed_zeros + n * a.pz_rs) + b);
    uint32_t o[4];
    const uint32_t in[2] = {w.x, w.y};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t lo = in[i] & 0x0F0F0F0Fu, hi = (in[i] >> 4) & 0x0F0F0F0Fu;
      uint32_t r0, r1;  // {b0.lo, b0.hi, b1.lo, b1.hi}, {b2.lo, b2.hi, b3.lo, b3.hi}
      asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(r0) : "r"(lo), "r"(hi));
      asm("prmt.b32 %0, %1, %2, 0x7362;" : "=r"(r1) : "r"(lo), "r"(hi));
      o[2 * i] = r0;
      o[2 * i + 1] = r1;
    }
    reinterpret_cast<uint4*>(a.zeros + n * a.z_rs)[b] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void unpack_zeros_kernel(UnpackZerosArgs a) {
  const int64_t total = a.N * int64_t(a.G);
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t n = t / a.G;
    const int g = int(t - n * a.G);
    const uint8_t b = a.packed_zeros[n * a.pz_rs + (g >> 1)];
    a.zeros[n * a.z_rs + g] = (g & 1) ? uint8_t(b >> 4) : uint8_t(b & 0x0F);
  }
}

int grid_for(int64_t work, int threads, int dev) {
  const int64_t want = (work + threads - 1) / threads;
  const int64_t cap = int64_t(device_sms(dev)) * 8;
  return int(std::max<int64_t>(1, std::min(want, cap)));
}

}  // namespace

int launch_quantize_group32(QuantArgs a, cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  const int64_t es = a.w_dtype == SPECTRA_DT_F32 ? 4 : 2;
  a.w_vec = reinterpret_cast<uintptr_t>(a.w) % 16 == 0 && (a.w_rs * es) % 16 == 0 ? 1 : 0;
  const size_t smem = size_t((a.K + 31) / 32) * 4;
  if (smem > 48 * 1024) return SPECTRA_ERR_SHAPE;  // K <= 393216
  const int64_t pairs = (int64_t(a.K / kGroup) + 1) / 2;
  const int grid = grid_for(int64_t(a.N) * pairs, kQuantThreads, dev);
  if (a.w_dtype == SPECTRA_DT_F16)
    quantize_group32_kernel<__half><<<grid, kQuantThreads, smem, st>>>(a);
  else if (a.w_dtype == SPECTRA_DT_BF16)
    quantize_group32_kernel<__nv_bfloat16><<<grid, kQuantThreads, smem, st>>>(a);
  else
    quantize_group32_kernel<float><<<grid, kQuantThreads, smem, st>>>(a);
  return cuda_status(cudaGetLastError());
}

int launch_unpack_zeros(const UnpackZerosArgs& a, cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  const bool vec = a.G % 16 == 0 && a.pz_rs % 8 == 0 && a.z_rs % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(a.packed_zeros) % 8 == 0 && reinterpret_cast<uintptr_t>(a.zeros) % 16 == 0;
  if (vec) {
    unpack_zeros_vec_kernel<<<grid_for(a.N * int64_t(a.G / 16), 256, dev), 256, 0, st>>>(a);
    return cuda_status(cudaGetLastError());
  }
  const int grid = grid_for(a.N * int64_t(a.G), 256, dev);
  unpack_zeros_kernel<<<grid, 256, 0, st>>>(a);
  return cuda_status(cudaGetLastError());
}

}  // namespace spectra
