// Building blocks shared by the M=1 GEMV kernels: the raw-code tensor-core
// step (mma.sync m16n8k16), bulk copies, warp reductions, SM count.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace spectra {

template <bool BF16>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// Pair type t of a 32-bit code word (bytes b0..b3): t=0 {b0.lo, b2.lo},
// t=1 {b0.hi, b2.hi}, t=2 {b1.lo, b3.lo}, t=3 {b1.hi, b3.hi}.  One shift
// brings the pair's nibbles to the top four mantissa bits of each 16-bit
// half, one LOP3 masks them and ORs in the exponent of 16.0: each half is
// then exactly 16 + q (bf16: nibble at bits 3-6; fp16: bits 6-9).  The small
// offset keeps the fp32 accumulation of (16 + q) * x as accurate as q * x.
template <bool BF16, int T>
__device__ __forceinline__ uint32_t pair_code(uint32_t w, uint32_t magic_reg) {
  constexpr int kShift = BF16 ? 3 - 4 * T : 6 - 4 * T;  // > 0: left shift
  constexpr uint32_t kMask = BF16 ? 0x00780078u : 0x03C003C0u;
  const uint32_t v = kShift >= 0 ? (w << (kShift >= 0 ? kShift : 0)) : (w >> (kShift < 0 ? -kShift : 0));
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(v), "n"(kMask), "r"(magic_reg));
  return r;
}

// k (0..31, within the group) of the low / high code of pair kk = 4j + t.
__host__ __device__ __forceinline__ int pair_k(int kk, int high, int layout) {
  const int j = kk >> 2, t = kk & 3;
  const int byte = 4 * j + 2 * high + (t >> 1);
  return code_k(byte, t & 1, layout);
}

template <int R>
__device__ __forceinline__ void warp_transpose_reduce(float (&v)[R], int lane) {
  // Each stage halves the rows a lane holds: the lower half-warp keeps the
  // first half of its rows, the upper half keeps the second half.
  int off = 16;
#pragma unroll
  for (int half = R / 2; half >= 1; half /= 2) {
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = up ? v[i] : v[i + half];
      const float keep = up ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
    off >>= 1;
  }
  for (; off >= 1; off >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
}

template <int R>
__device__ __forceinline__ int reduced_row(int lane) {
  int row = 0, off = 16;
#pragma unroll
  for (int half = R / 2; half >= 1; half /= 2) {
    if (lane & off) row += half;
    off >>= 1;
  }
  return row;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(bytes), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
               : "memory");
}

// Same copy with an L2 cache-policy hint (from createpolicy).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
      "l"(src), "r"(bytes), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar))), "l"(policy)
      : "memory");
}

inline int device_sms(int dev) {
  static int sms[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (sms[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    sms[dev] = v;
  }
  return sms[dev];
}

}  // namespace spectra
