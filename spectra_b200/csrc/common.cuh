// Shared device/host helpers for the W4A16 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "spectra_b200.h"

namespace spectra {

constexpr int kGroup = 32;          // quantisation group (input features)
constexpr int kGroupBytes = 16;     // packed bytes per group
constexpr uint32_t kMagic = 0x4B000000u;  // bit pattern of 2^23 in fp32
constexpr int kMaxDevices = 64;           // per-device launch-attribute caches

// Per-thread record of the last failed CUDA call (exported by
// spectra_last_cuda_error()).
void set_last_cuda_error(cudaError_t e);

// Programmatic dependent launch (kernels overlap their weight prefetch with
// the previous kernel's tail).  On unless SPECTRA_B200_PDL=0 in the environment.
bool pdl_enabled();


// M=1 GEMV tensor-core path for bf16/fp16 activations (on unless
// SPECTRA_B200_GEMV_MMA=0, which selects the exact CUDA-core kernel).
bool mma_path_enabled();

// M=1 GEMV weight-prefetching kernel for layouts that allow it (on unless
// SPECTRA_B200_GEMV_PF=0).
bool pf_path_enabled();

// GEMM scales / zero points fetched by tensor map when their layout allows
// (on unless SPECTRA_B200_GEMM_SZ_TMA=0, which forces the plain-load path).
bool sz_tma_enabled();

// GEMM token tiles of >= 128 on SM pairs (cta_group::2, one M=256 MMA over
// two CTAs' TMEM, each CTA loading half of the tokens): off unless
// SPECTRA_B200_GEMM_PAIR=1 (bit-identical results; on B200 it measured within
// a few percent of the one-SM kernel either way).
bool pair_enabled();

inline int cuda_status(cudaError_t e) {
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return SPECTRA_ERR_CUDA;
  }
  return SPECTRA_OK;
}

// Unique id of the CUDA context current on the calling thread (0: none yet).
// A device's primary context gets a new id when it is torn down and created
// again (cudaDeviceReset), which invalidates everything cached per device:
// kernel attributes and module symbol addresses.
unsigned long long current_context_id();

// One-time initialisation per (device, CUDA context): `init` runs on the first
// call on each device and again after that device's context was recreated.
// Two host threads making their first call at once may both run `init`, so it
// must be idempotent (setting a kernel attribute, looking an address up).
class PerContextOnce {
 public:
  template <class F>
  cudaError_t run(int dev, F&& init) {
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    const unsigned long long id = current_context_id();
    if (id != 0 && ctx_[dev].load(std::memory_order_acquire) == id) return cudaSuccess;
    const cudaError_t e = init();  // a runtime call: makes the primary context current
    if (e == cudaSuccess) ctx_[dev].store(current_context_id(), std::memory_order_release);
    return e;
  }

 private:
  std::atomic<unsigned long long> ctx_[kMaxDevices] = {};
};

// Reads a device-side counter of waits that gave up (a `__device__ int` of the
// calling translation unit) on the current device, and zeroes it if `reset`.
// Synchronous: it waits for the device's queued work.
template <class T>
int read_timeout_counter(const T& symbol, long long* out, bool reset) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, symbol, sizeof(int));
  if (e == cudaSuccess && reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(symbol, &zero, sizeof(int));
  }
  if (e != cudaSuccess) return cuda_status(e);
  *out = v;
  return SPECTRA_OK;
}

// Timed-out waits counted by each kernel family (per translation unit).
int gemv_timeouts(long long* out, bool reset);
int gemv_pf_timeouts(long long* out, bool reset);
int gemm_timeouts(long long* out, bool reset);
// Launches the bounded-wait self-test kernel (gemv_pf.cu).
int launch_selftest_wait(cudaStream_t st);

// ---------------------------------------------------------------------------
// typed scalar loads/stores selected by a runtime dtype code
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_as_float(const void* base, int64_t i, int dt) {
  if (dt == SPECTRA_DT_BF16) {
    uint16_t b = __ldg(reinterpret_cast<const unsigned short*>(base) + i);
    return __uint_as_float(uint32_t(b) << 16);
  }
  if (dt == SPECTRA_DT_F16) {
    return __half2float(__ldg(reinterpret_cast<const __half*>(base) + i));
  }
  return __ldg(reinterpret_cast<const float*>(base) + i);
}

// Same, through L2 only (ld.global.cg): for data another kernel may have
// written while this one was already resident.
__device__ __forceinline__ float load_as_float_cg(const void* base, int64_t i, int dt) {
  if (dt == SPECTRA_DT_BF16) {
    uint16_t b = __ldcg(reinterpret_cast<const unsigned short*>(base) + i);
    return __uint_as_float(uint32_t(b) << 16);
  }
  if (dt == SPECTRA_DT_F16) {
    return __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short*>(base) + i)));
  }
  return __ldcg(reinterpret_cast<const float*>(base) + i);
}

// Raw bits of one element (through L2 only) and their later conversion.
__device__ __forceinline__ uint32_t load_bits_cg(const void* base, int64_t i, int dt) {
  if (dt == SPECTRA_DT_BF16 || dt == SPECTRA_DT_F16) return __ldcg(reinterpret_cast<const unsigned short*>(base) + i);
  return __ldcg(reinterpret_cast<const unsigned int*>(base) + i);
}
__device__ __forceinline__ float bits_to_float(uint32_t b, int dt) {
  if (dt == SPECTRA_DT_BF16) return __uint_as_float(b << 16);
  if (dt == SPECTRA_DT_F16) return __half2float(__ushort_as_half(uint16_t(b)));
  return __uint_as_float(b);
}

__device__ __forceinline__ int64_t load_index(const void* base, int64_t i, int dt) {
  if (dt == SPECTRA_DT_I32) return __ldg(reinterpret_cast<const int*>(base) + i);
  return __ldg(reinterpret_cast<const long long*>(base) + i);
}

__device__ __forceinline__ void store_from_float(void* base, int64_t i, int dt, float v) {
  if (dt == SPECTRA_DT_BF16) {
    reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
  } else if (dt == SPECTRA_DT_F16) {
    reinterpret_cast<__half*>(base)[i] = __float2half_rn(v);
  } else {
    reinterpret_cast<float*>(base)[i] = v;
  }
}

// 16 packed bytes (one 32-code group of one row), read once, not kept in L1.
template <int ALIGN>
__device__ __forceinline__ uint4 load_group16(const uint8_t* p) {
  uint4 v;
  if constexpr (ALIGN >= 16) {
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
  } else if constexpr (ALIGN >= 4) {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p);
    v.x = __ldg(q + 0); v.y = __ldg(q + 1); v.z = __ldg(q + 2); v.w = __ldg(q + 3);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      w[j] = uint32_t(__ldg(p + 4 * j)) | (uint32_t(__ldg(p + 4 * j + 1)) << 8) |
             (uint32_t(__ldg(p + 4 * j + 2)) << 16) | (uint32_t(__ldg(p + 4 * j + 3)) << 24);
    }
    v = make_uint4(w[0], w[1], w[2], w[3]);
  }
  return v;
}

// k offset (0..31) inside its group of the code stored at byte `byte`
// (0..15), high nibble if `hi`.
__host__ __device__ __forceinline__ int code_k(int byte, int hi, int layout) {
  return layout == SPECTRA_LAYOUT_MARLIN ? byte + 16 * hi : 2 * byte + hi;
}

}  // namespace spectra
