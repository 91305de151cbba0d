// Token-embedding gather-dequantise and greedy argmax for sm_100a.
//
// Embedding: replaces SpectraFusedEmbedding.forward (spectra/engine.py:167-212).
// For every token id, the packed row of the quantised vocabulary matrix is
// dequantised -- ((q - z) * s) in fp32, exact, then rounded once to the output
// dtype -- and the outlier columns are overwritten with the exact outlier
// weights rounded to the output dtype (:207-210).  Zero points may be given
// unpacked (one byte per group) or packed two per byte (:176-183).  A token id
// outside [0, V) writes a row of zeros instead of reading out of bounds (the
// reference's torch indexing would raise).  One CTA per token: thread i
// dequantises group i (16 bytes -> 32 outputs), then the outlier columns.
//
// Argmax: the greedy next-token choice over logits [M, N] (the engine's
// sample_token at temperature 0, spectra/engine.py:1690-1713, is
// torch.argmax): first index of the maximum, a NaN counts as the maximum (as
// in torch).  One cluster of 8 CTAs per row; `idx_offset` turns a shard's local index into
// the layer's row index, so the N-sharded lm_head reduces (value, index)
// pairs across ranks instead of gathering every logit.
#include <algorithm>
#include <cooperative_groups.h>

#include "common.cuh"
#include "format.h"
#include "gemv_mma.cuh"
#include "sm100_ptx.cuh"

namespace spectra {

namespace {

constexpr int kEmbedThreads = 256;
constexpr int kArgmaxThreads = 512;
constexpr int kArgmaxCluster = 8;  // CTAs per row (a portable cluster size)

__global__ void __launch_bounds__(kEmbedThreads) embedding_kernel(EmbedArgs a) {
  const int64_t t = blockIdx.x;
  const int64_t id = load_index(a.ids, t, a.ids_dtype);
  const bool valid = id >= 0 && id < a.V;
  const int G = a.K / kGroup;
  for (int g = threadIdx.x; g < G; g += blockDim.x) {
    float v[kGroup];
    if (valid) {
      const uint4 w = load_group16<1>(a.packed + id * a.w_rs + int64_t(g) * kGroupBytes);
      const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
      const float s = __half2float(__ushort_as_half(a.scales[id * a.s_rs + g]));
      uint32_t zb;
      if (a.zeros_packed) {
        const uint8_t b = a.zeros[id * a.z_rs + (g >> 1)];
        zb = (g & 1) ? (b >> 4) & 0xFu : b & 0xFu;
      } else {
        zb = a.zeros[id * a.z_rs + g];
      }
      const float z = float(zb);
#pragma unroll
      for (int byte = 0; byte < 16; ++byte) {
        const uint32_t bv = (wv[byte >> 2] >> (8 * (byte & 3))) & 0xFFu;
        v[code_k(byte, 0, a.layout)] = __fmul_rn(float(bv & 0xFu) - z, s);
        v[code_k(byte, 1, a.layout)] = __fmul_rn(float(bv >> 4) - z, s);
      }
    } else {
#pragma unroll
      for (int i = 0; i < kGroup; ++i) v[i] = 0.f;
    }
    const int64_t base = t * a.out_rs + int64_t(g) * kGroup;
    if (a.vec_out) {
      // 16-bit output, 16-byte aligned rows: four 16-byte stores
      uint32_t o[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float lo = v[2 * i], hi = v[2 * i + 1];
        uint32_t bl, bh;
        if (a.out_dtype == SPECTRA_DT_BF16) {
          bl = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
          bh = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
        } else {
          bl = __half_as_ushort(__float2half_rn(lo));
          bh = __half_as_ushort(__float2half_rn(hi));
        }
        o[i] = bl | (bh << 16);
      }
      uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + base);
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) dst[q4] = make_uint4(o[4 * q4], o[4 * q4 + 1], o[4 * q4 + 2], o[4 * q4 + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < kGroup; ++i) store_from_float(a.out, base + i, a.out_dtype, v[i]);
    }
  }
  if (a.n_out > 0 && valid) {
    __syncthreads();  // the outlier columns overwrite what the loop above stored
    for (int j = threadIdx.x; j < a.n_out; j += blockDim.x) {
      const int64_t k = load_index(a.idx, j, a.idx_dtype);
      if (k < 0 || k >= a.K) continue;
      const float w = load_as_float(a.ow, id * a.ow_rs + j, a.ow_dtype);
      store_from_float(a.out, t * a.out_rs + k, a.out_dtype, w);
    }
  }
}

// (value, index) order of torch.argmax: larger value first; NaN above every
// number; on ties (and between NaNs) the smaller index.
__device__ __forceinline__ bool better(float v, int64_t i, float bv, int64_t bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn || bn) return vn && (!bn || i < bi);
  return v > bv || (v == bv && i < bi);
}

// One row per cluster of kArgmaxCluster CTAs: CTA c scans the c-th slice of
// the row with 16-byte loads where the row allows them, reduces it to one
// (value, index) pair, and CTA 0 combines the cluster's pairs from the other
// CTAs' shared memory (distributed shared memory; the cluster barriers are
// hardware barriers over co-scheduled CTAs, nothing spins).
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(ArgmaxArgs a) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  sm100::pdl_wait();  // the logits are the previous kernel's output
  const int64_t m = blockIdx.y;
  const int c = int(cluster.block_rank());
  const int64_t lo = min(a.N, c * a.span), hi = min(a.N, lo + a.span);
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  if (a.vec) {
    // 16-byte units of the row (the row start is 16-byte aligned, the span a multiple of the unit)
    const int per = a.x_dtype == SPECTRA_DT_F32 ? 4 : 8;
    const uint4* row = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.x) +
                                                      m * a.x_rs * (a.x_dtype == SPECTRA_DT_F32 ? 4 : 2));
    const int64_t u_lo = lo / per, u_hi = (hi + per - 1) / per;
    for (int64_t u = u_lo + threadIdx.x; u < u_hi; u += kArgmaxThreads) {
      const uint4 w = __ldcg(row + u);
      const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (e >= per) break;
        const int64_t n = u * per + e;
        if (n >= hi) break;
        float v;
        if (a.x_dtype == SPECTRA_DT_F32) {
          v = __uint_as_float(wv[e]);
        } else {
          const uint32_t h = (wv[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
          v = a.x_dtype == SPECTRA_DT_BF16 ? __uint_as_float(h << 16) : __half2float(__ushort_as_half(uint16_t(h)));
        }
        if (better(v, n, bv, bi)) {
          bv = v;
          bi = n;
        }
      }
    }
  } else {
    for (int64_t n = lo + threadIdx.x; n < hi; n += kArgmaxThreads) {
      const float v = load_as_float_cg(a.x, m * a.x_rs + n, a.x_dtype);
      if (better(v, n, bv, bi)) {
        bv = v;
        bi = n;
      }
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  __shared__ float sv[kArgmaxThreads / 32];
  __shared__ int64_t si[kArgmaxThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    constexpr int nw = kArgmaxThreads / 32;
    bv = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : INT64_MAX;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
  }
  __syncthreads();  // every warp has read sv / si
  if (threadIdx.x == 0) {
    sv[0] = bv;  // this CTA's pair, for CTA 0 of the cluster
    si[0] = bi;
  }
  cluster.sync();
  if (c == 0 && warp == 0) {
    bv = -INFINITY;
    bi = INT64_MAX;
    if (lane < kArgmaxCluster) {
      bv = *cluster.map_shared_rank(&sv[0], lane);
      bi = *cluster.map_shared_rank(&si[0], lane);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      a.idx[m] = (bi == INT64_MAX ? 0 : bi) + a.idx_offset;
      if (a.val) a.val[m] = bv;
    }
  }
  cluster.sync();  // no CTA leaves while CTA 0 may still read its shared memory
}

}  // namespace

int launch_embedding(EmbedArgs a, cudaStream_t st) {
  if (a.T == 0) return SPECTRA_OK;
  if (a.T > int64_t(INT32_MAX)) return SPECTRA_ERR_SHAPE;
  // 16-byte stores when the output rows allow them; one thread per group
  // (CTAs no wider than the row's groups)
  a.vec_out = (a.out_dtype == SPECTRA_DT_BF16 || a.out_dtype == SPECTRA_DT_F16) &&
              reinterpret_cast<uintptr_t>(a.out) % 16 == 0 && (a.out_rs * 2) % 16 == 0;
  const int G = int(a.K / kGroup);
  const int threads = std::max(32, std::min(kEmbedThreads, (G + 31) / 32 * 32));
  embedding_kernel<<<unsigned(a.T), threads, 0, st>>>(a);
  return cuda_status(cudaGetLastError());
}

int launch_argmax(ArgmaxArgs a, cudaStream_t st) {
  if (a.M == 0) return SPECTRA_OK;
  if (a.M > 65535) return SPECTRA_ERR_SHAPE;  // grid y
  // 16-byte loads when every row starts on a 16-byte boundary and each CTA's
  // slice is a whole number of 16-byte units
  const int64_t esz = a.x_dtype == SPECTRA_DT_F32 ? 4 : 2;
  const int64_t per = 16 / esz;
  a.span = ((a.N + kArgmaxCluster - 1) / kArgmaxCluster + per - 1) / per * per;  // whole 16-byte units
  a.vec = reinterpret_cast<uintptr_t>(a.x) % 16 == 0 && (a.M == 1 || (a.x_rs * esz) % 16 == 0);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kArgmaxCluster, unsigned(a.M));
  cfg.blockDim = dim3(kArgmaxThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kArgmaxCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cuda_status(cudaLaunchKernelEx(&cfg, argmax_kernel, a));
}

}  // namespace spectra
