// Walsh-Hadamard rotation of activation rows for sm_100a: the optional
// rotation prologue of the M=1 GEMV (off by default: the reference's
// compressor cannot produce rotated weights -- hadamard_incoherence raises,
// spectra/compressor.py:55-56 -- so only callers that rotated their weights
// themselves turn it on).
//
// Semantics: the reference's fast_walsh_hadamard_transform
// (spectra/compressor.py:29-42): butterflies (u + v, u - v) over spans
// h = 1, 2, 4, ..., n/2, then an optional division by sqrt(n); n must be a
// power of two.  Here every butterfly runs in fp32 (the rows are rounded once,
// to the output dtype, at the end).
//
// One CTA of 1024 threads per row, E = n / 1024 consecutive elements per
// thread (at least one):
//   spans h <  E        inside a thread's registers,
//   spans E <= h < 32E  across the lanes of a warp (shuffle xor h / E),
//   spans h >= 32E      through shared memory, one barrier per span.
#include "common.cuh"
#include "format.h"

namespace spectra {

namespace {

constexpr int kFwhtThreads = 1024;
constexpr int kFwhtMaxE = 32;  // n <= 32768

template <int E>
__global__ void __launch_bounds__(kFwhtThreads) fwht_kernel(FwhtArgs a) {
  extern __shared__ float buf[];  // [n] when n > 32 E (spans beyond one warp)
  const int64_t m = blockIdx.x;
  const int n = a.n;
  const int tid = threadIdx.x, lane = tid & 31;
  const int active = n / E < kFwhtThreads ? n / E : kFwhtThreads;  // threads holding elements
  float v[E];
  const bool has = tid < active;
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = has ? load_as_float_cg(a.x, m * a.x_rs + int64_t(tid) * E + e, a.x_dtype) : 0.f;
  // spans inside the thread
#pragma unroll
  for (int h = 1; h < E; h <<= 1) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      if ((e & h) == 0) {
        const float u = v[e], w = v[e + h];
        v[e] = u + w;
        v[e + h] = u - w;
      }
    }
  }
  // spans across the lanes of a warp: element index bit h lives in lane bit h / E
  for (int hl = 1; hl < 32 && hl * E < n; hl <<= 1) {
    const bool upper = (lane & hl) != 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float o = __shfl_xor_sync(0xffffffffu, v[e], hl);
      v[e] = upper ? o - v[e] : v[e] + o;
    }
  }
  // spans beyond a warp: shared memory
  if (n > 32 * E) {
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (has) buf[tid * E + e] = v[e];
    __syncthreads();
    for (int h = 32 * E; h < n; h <<= 1) {
      for (int p = tid; p < n / 2; p += blockDim.x) {
        const int i = (p / h) * 2 * h + (p % h);
        const float u = buf[i], w = buf[i + h];
        buf[i] = u + w;
        buf[i + h] = u - w;
      }
      __syncthreads();
    }
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (has) v[e] = buf[tid * E + e];
  }
  if (has) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float r = a.normalize ? __fdiv_rn(v[e], a.inv_norm) : v[e];
      store_from_float(a.y, m * a.y_rs + int64_t(tid) * E + e, a.y_dtype, r);
    }
  }
}

template <int E>
int launch_e(const FwhtArgs& a, cudaStream_t st) {
  const size_t smem = a.n > 32 * E ? size_t(a.n) * 4 : 0;
  auto kern = fwht_kernel<E>;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return cuda_status(e);
  }
  kern<<<unsigned(a.M), kFwhtThreads, smem, st>>>(a);
  return cuda_status(cudaGetLastError());
}

}  // namespace

int launch_fwht(const FwhtArgs& a, cudaStream_t st) {
  if (a.M == 0) return SPECTRA_OK;
  if (a.M > int64_t(INT32_MAX)) return SPECTRA_ERR_SHAPE;
  const int E = a.n <= kFwhtThreads ? 1 : a.n / kFwhtThreads;
  switch (E) {
    case 1: return launch_e<1>(a, st);
    case 2: return launch_e<2>(a, st);
    case 4: return launch_e<4>(a, st);
    case 8: return launch_e<8>(a, st);
    case 16: return launch_e<16>(a, st);
    case 32: return launch_e<32>(a, st);
    default: return SPECTRA_ERR_SHAPE;
  }
}

}  // namespace spectra
