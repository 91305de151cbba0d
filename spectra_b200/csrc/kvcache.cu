// INT4 KV-cache quantiser and dequantiser for sm_100a, replacing the torch
// code of SpectraGroup32QuantizedLayer (spectra/engine.py:625-671): key/value
// rows [rows, D] in groups of 32 along D (zero-padded to a multiple of 32),
// asymmetric min/max codes, even-odd nibble packing (byte i of a group holds
// element 2i in the low and 2i+1 in the high nibble), fp16 scales and one
// zero point per group.
//
// The reference computes in the cache's own dtype T (bf16 or fp16) on the
// device the cache lives on; each step below rounds where torch does, so the
// codes match the reference run on a CUDA device bit for bit:
//   lo, hi        min / max of the group (exact)
//   diff        = T(hi - lo)
//   constant    = diff < T(1e-8)
//   s           = constant ? (lo == 0 ? 1 : |lo|) : T(diff * fp32(1/15))
//                 (torch on CUDA divides a tensor by a Python scalar as a
//                 multiply by the fp32 reciprocal)
//   s           = T(max(s, T(1e-8)))
//   z           = constant ? (lo < 0) : clamp(rint(T(-lo / s)), 0, 15)
//   q           = constant ? (lo > 0) : clamp(rint((t - (-(z * s))) / s), 0, 15)
//                 (this line in fp32: the zero point is promoted to float)
//   scale       stored as fp16(s)
// Dequantisation (:658-671): T_out((q - z) * fp32(scale_fp16)), exact in fp32
// before the final rounding, padding columns dropped.
//
// One thread per (row, group): 64 bytes in (bf16), 19 bytes out.  HBM-bound.
#include "common.cuh"
#include "format.h"
#include "gemv_mma.cuh"

namespace spectra {

namespace {

constexpr int kKvThreads = 256;

template <typename T>
struct Num;
template <>
struct Num<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};
template <>
struct Num<__half> {
  static __device__ __forceinline__ float f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
};

template <typename T>
__device__ __forceinline__ T bits_lo(uint32_t w) {
  const uint16_t b = uint16_t(w & 0xFFFFu);
  return *reinterpret_cast<const T*>(&b);
}
template <typename T>
__device__ __forceinline__ T bits_hi(uint32_t w) {
  const uint16_t b = uint16_t(w >> 16);
  return *reinterpret_cast<const T*>(&b);
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(kKvThreads) kv_quantize_kernel(KvQuantArgs a) {
  const int G = (a.D + kGroup - 1) / kGroup;
  const int64_t total = a.rows * G;
  const T* t = reinterpret_cast<const T*>(a.t);
  const float inv15 = 1.0f / 15.0f;  // fp32 reciprocal, as torch computes it on the device
  for (int64_t u = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; u < total; u += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = u / G;
    const int g = int(u - r * G);
    const T* row = t + r * a.D;
    float v[kGroup];
    if (VEC) {
      // whole groups, 16-byte aligned: four 16-byte loads
      const uint4* src = reinterpret_cast<const uint4*>(row + g * kGroup);
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const uint4 w = __ldg(src + q4);
        const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          v[8 * q4 + 2 * i] = Num<T>::f(bits_lo<T>(wv[i]));
          v[8 * q4 + 2 * i + 1] = Num<T>::f(bits_hi<T>(wv[i]));
        }
      }
    }
    if (!VEC) {
#pragma unroll
      for (int i = 0; i < kGroup; ++i) {
        const int d = g * kGroup + i;
        v[i] = d < a.D ? Num<T>::f(row[d]) : 0.f;  // zero padding (torch.nn.functional.pad)
      }
    }
    float lo = v[0], hi = v[0];
#pragma unroll
    for (int i = 1; i < kGroup; ++i) {
      lo = fminf(lo, v[i]);
      hi = fmaxf(hi, v[i]);
    }
    const float diff = Num<T>::round(__fsub_rn(hi, lo));
    // torch converts the Python scalar 1e-8 to T before comparing and clamping:
    // bf16(1e-8) ~ 1.0011e-8, fp16(1e-8) == 0 (an fp16 constant group is then not
    // "constant" and its scale is 0; the divisions below give +-inf or NaN,
    // which the clamps turn into the codes torch's conversion gives: 15, 0, 0)
    const float thr = Num<T>::round(1e-8f);
    const bool flat = diff < thr;
    float s = flat ? (lo == 0.f ? 1.f : fabsf(lo)) : Num<T>::round(__fmul_rn(diff, inv15));
    s = Num<T>::round(fmaxf(s, thr));
    float z;
    if (flat)
      z = lo < 0.f ? 1.f : 0.f;
    else
      z = fminf(fmaxf(rintf(Num<T>::round(__fdiv_rn(-lo, s))), 0.f), 15.f);
    const float zs = -__fmul_rn(z, s);
    uint32_t w4[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < kGroup; ++i) {
      float c;
      if (flat)
        c = lo > 0.f ? 1.f : 0.f;
      else
        c = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(v[i], zs), s)), 0.f), 15.f);
      // even-odd order: element i -> byte i/2, low nibble for even i
      w4[i >> 3] |= uint32_t(c) << (4 * (i & 7));
    }
    uint8_t* dst = a.packed + u * kGroupBytes;
    *reinterpret_cast<uint4*>(dst) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    reinterpret_cast<__half*>(a.scales)[u] = __float2half_rn(s);
    a.zeros[u] = uint8_t(z);
  }
}

template <typename T>
__device__ __forceinline__ void store_t(void* out, int64_t i, float v);
template <>
__device__ __forceinline__ void store_t<__nv_bfloat16>(void* out, int64_t i, float v) {
  reinterpret_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ void store_t<__half>(void* out, int64_t i, float v) {
  reinterpret_cast<__half*>(out)[i] = __float2half_rn(v);
}
template <>
__device__ __forceinline__ void store_t<float>(void* out, int64_t i, float v) {
  reinterpret_cast<float*>(out)[i] = v;
}

// Vector path (D a multiple of 8): four threads per group, eight values each
// (bytes 4qq..4qq+3 of the group's codes: elements 8qq..8qq+7), one or two
// 16-byte stores -- the four threads of a group write 64 contiguous bytes.
template <typename T>
__global__ void __launch_bounds__(kKvThreads) kv_dequantize_vec_kernel(KvDequantArgs a) {
  const int G = (a.D + kGroup - 1) / kGroup;
  const int64_t total = a.rows * G * 4;
  for (int64_t it = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; it < total; it += int64_t(gridDim.x) * blockDim.x) {
    const int64_t u = it >> 2;
    const int qq = int(it & 3);
    const int64_t r = u / G;
    const int g = int(u - r * G);
    const int d0 = g * kGroup + qq * 8;
    if (d0 >= a.D) continue;
    const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(a.packed + u * kGroupBytes) + qq);
    const float s = __half2float(__ushort_as_half(__ldg(a.scales + u)));
    const float z = float(__ldg(a.zeros + u));
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(float((w >> (4 * j)) & 0xFu) - z, s);  // element 2b: low nibble of byte b
    T* dst = reinterpret_cast<T*>(a.out) + r * a.D + d0;
    if constexpr (sizeof(T) == 4) {
      reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        T lo, hi;
        store_t<T>(&lo, 0, v[2 * j]);
        store_t<T>(&hi, 0, v[2 * j + 1]);
        o[j] = uint32_t(*reinterpret_cast<const uint16_t*>(&lo)) | (uint32_t(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
      }
      *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kKvThreads) kv_dequantize_kernel(KvDequantArgs a) {
  const int G = (a.D + kGroup - 1) / kGroup;
  const int64_t total = a.rows * G;
  for (int64_t u = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; u < total; u += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = u / G;
    const int g = int(u - r * G);
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(a.packed + u * kGroupBytes));
    const float s = __half2float(__ushort_as_half(a.scales[u]));
    const float z = float(a.zeros[u]);
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
    const int64_t base = r * a.D + int64_t(g) * kGroup;
#pragma unroll
    for (int i = 0; i < kGroup; ++i) {
      const int d = g * kGroup + i;
      if (d >= a.D) break;
      const float q = float((wv[i >> 3] >> (4 * (i & 7))) & 0xFu);
      store_t<T>(a.out, base + i, __fmul_rn(q - z, s));
    }
  }
}

int kv_grid(int64_t work, int dev) {
  const int64_t want = (work + kKvThreads - 1) / kKvThreads;
  return int(std::max<int64_t>(1, std::min<int64_t>(want, int64_t(device_sms(dev)) * 8)));
}

}  // namespace

int launch_kv_quantize(const KvQuantArgs& a, cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  const int G = (a.D + kGroup - 1) / kGroup;
  const int grid = kv_grid(a.rows * G, dev);
  // whole groups on 16-byte boundaries: 16-byte loads
  const bool vec = a.D % kGroup == 0 && reinterpret_cast<uintptr_t>(a.t) % 16 == 0;
  if (a.t_dtype == SPECTRA_DT_BF16) {
    if (vec)
      kv_quantize_kernel<__nv_bfloat16, true><<<grid, kKvThreads, 0, st>>>(a);
    else
      kv_quantize_kernel<__nv_bfloat16, false><<<grid, kKvThreads, 0, st>>>(a);
  } else {
    if (vec)
      kv_quantize_kernel<__half, true><<<grid, kKvThreads, 0, st>>>(a);
    else
      kv_quantize_kernel<__half, false><<<grid, kKvThreads, 0, st>>>(a);
  }
  return cuda_status(cudaGetLastError());
}

int launch_kv_dequantize(const KvDequantArgs& a, cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  const int G = (a.D + kGroup - 1) / kGroup;
  const bool vec = a.D % 8 == 0 && reinterpret_cast<uintptr_t>(a.out) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(a.packed) % 4 == 0;
  if (vec) {
    const int gv = kv_grid(a.rows * G * 4, dev);
    if (a.out_dtype == SPECTRA_DT_BF16)
      kv_dequantize_vec_kernel<__nv_bfloat16><<<gv, kKvThreads, 0, st>>>(a);
    else if (a.out_dtype == SPECTRA_DT_F16)
      kv_dequantize_vec_kernel<__half><<<gv, kKvThreads, 0, st>>>(a);
    else
      kv_dequantize_vec_kernel<float><<<gv, kKvThreads, 0, st>>>(a);
    return cuda_status(cudaGetLastError());
  }
  const int grid = kv_grid(a.rows * G, dev);
  if (a.out_dtype == SPECTRA_DT_BF16)
    kv_dequantize_kernel<__nv_bfloat16><<<grid, kKvThreads, 0, st>>>(a);
  else if (a.out_dtype == SPECTRA_DT_F16)
    kv_dequantize_kernel<__half><<<grid, kKvThreads, 0, st>>>(a);
  else
    kv_dequantize_kernel<float><<<grid, kKvThreads, 0, st>>>(a);
  return cuda_status(cudaGetLastError());
}

}  // namespace spectra
