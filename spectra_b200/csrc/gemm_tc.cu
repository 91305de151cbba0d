// M >= 2 W4A16 GEMM on the sm_100a tensor cores (tcgen05 + TMEM).
// Replaces spectra/kernels.py:191-389 (_batched_w4a16_gemm_kernel / batched_w4a16_gemm).
//
//   C[m, n] = sum_k a[m, k] * bf16((q[n,k] - z[n,k/32]) * s[n,k/32])
//           + sum_j a[m, idx_j] * bf16(ow[n, j])            (fp16 when a is fp16)
// accumulated in fp32 and rounded once to a's dtype -- the reference's operand
// rounding (spectra/kernels.py:256-261, 315-320) and output cast (:328-331).
//
// Swap-AB: the MMA's M dimension is 128 weight rows, its N dimension the
// tokens (a multiple of 16, <= 256), so M = 16 wastes nothing.
//
// CTA = 10 warps: warp 0 issues TMA loads (packed codes, activations), warp 1
// owns TMEM and issues the MMAs, warps 2..9 dequantise and run the epilogue.
// Per 64-k stage:
//   producer : packed codes [128 rows x 32 B] and activations [MT x 128 B,
//              128B-swizzled, K-major] land in shared memory (mbarrier tx).
//   dequant  : thread (row r = its TMEM lane, half h) turns one 32-code group
//              into 16 bf16x2 words of exact (q - z) * s rounded to nearest
//              even, tcgen05.st into the stage's A columns of TMEM.
//   MMA      : tcgen05.mma kind::f16, A from TMEM, B from shared memory,
//              D (fp32, 128 lanes x MT columns) in TMEM; tcgen05.commit frees
//              the stage.
// Outlier columns become extra stages: the dequant warps gather a[:, idx]
// into the B stage (same swizzled layout) and convert ow rows into the A
// stage.  K is split across CTAs when there are too few weight tiles to fill
// the GPU; the last CTA of a tile sums the fp32 partials in split order
// (deterministic) and resets the tile's counter for the next call.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemm.h"
#include "sm100_ptx.cuh"

// Split-K scratch of spectra_w4a16_gemm_noalloc, laid out like a caller
// workspace (tile counters, then fp32 partials).  Zero when the module loads;
// every GEMM leaves its counters zero again.
static __device__ __align__(256) unsigned char g_gemm_noalloc_scratch[SPECTRA_GEMM_NOALLOC_SCRATCH_BYTES];

namespace spectra {

namespace {

using namespace sm100;

constexpr int kRows = 128;     // weight rows per tile (MMA M)
constexpr int kBK = 64;        // k per stage (4 MMAs of K=16)
constexpr int kWarps = 10;
constexpr int kDeqWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxMT = 256;
constexpr size_t kMaxDynSmem = 200 * 1024;

__device__ int g_gemm_timeouts;  // stuck pipeline waits since load (diagnostic)

struct GemmKParams {
  const __half* scales; int64_t s_rs, s_cs;
  const uint8_t* zeros; int64_t z_rs, z_cs;
  const void* a; int64_t a_rs;  // activations (outlier gather)
  const void* idx; int idx_dtype; int n_out;
  const void* ow; int ow_dtype; int64_t ow_rs, ow_cs;
  void* c; int c_dtype; int64_t c_rs;
  float* partials;  // [S][M][N] when S > 1
  int* counters;    // [tiles_n * m_chunks]
  int M, N, K, layout;
  int MT, stages, S, nk, n_os, tiles_n;
  uint32_t idesc;
  uint32_t tmem_cols;
  int off_act, act_stage_bytes, off_w, off_bar;
};

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// 32 codes of one group -> 16 words of two 16-bit floats each, (q-z)*s exact
// in fp32 then rounded to nearest even.  Column c of the group holds k = 2c
// (low half) and 2c+1 (high half).
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}

template <bool BF16>
__device__ __forceinline__ void dequant_group(const uint4 w, float s, float z, int layout, uint32_t (&out)[16]) {
  // nibble at position p (bits 4p..4p+3) of a 16-bit half -> 2^23 + q*16^p;
  // subtract 2^23 + z*16^p, multiply by s*16^-p: exact (q - z) * s.
  const float c0 = -(8388608.0f + z), c1 = -(8388608.0f + 16.f * z), c2 = -(8388608.0f + 256.f * z),
              c3 = -(8388608.0f + 4096.f * z);
  const float s0 = s, s1 = s * 0.0625f, s2 = s * 0.00390625f, s3 = s * 0.000244140625f;
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int hw = 0; hw < 2; ++hw) {
      const uint32_t v = hw ? (words[j] >> 16) : words[j];
      const float q0 = __uint_as_float((v & 0x000Fu) | kMagic);
      const float q1 = __uint_as_float((v & 0x00F0u) | kMagic);
      const float q2 = __uint_as_float((v & 0x0F00u) | kMagic);
      const float q3 = __uint_as_float((v & 0xF000u) | kMagic);
      if (layout == SPECTRA_LAYOUT_MARLIN) {
        // low nibbles of the half's two bytes -> column 2j+hw; high -> 8+2j+hw
        float2 lo = __fmul2_rn(__fadd2_rn(f2(q0, q2), f2(c0, c2)), f2(s0, s2));
        float2 hi = __fmul2_rn(__fadd2_rn(f2(q1, q3), f2(c1, c3)), f2(s1, s3));
        out[2 * j + hw] = pack2<BF16>(lo.x, lo.y);
        out[8 + 2 * j + hw] = pack2<BF16>(hi.x, hi.y);
      } else {
        // byte b holds k = 2b (low) and 2b+1 (high) -> column b
        float2 b0 = __fmul2_rn(__fadd2_rn(f2(q0, q1), f2(c0, c1)), f2(s0, s1));
        float2 b1 = __fmul2_rn(__fadd2_rn(f2(q2, q3), f2(c2, c3)), f2(s2, s3));
        out[4 * j + 2 * hw] = pack2<BF16>(b0.x, b0.y);
        out[4 * j + 2 * hw + 1] = pack2<BF16>(b1.x, b1.y);
      }
    }
  }
}

__device__ __forceinline__ uint16_t to16(float v, bool bf16) {
  if (bf16) {
    const __nv_bfloat16 b = __float2bfloat16_rn(v);
    return *reinterpret_cast<const uint16_t*>(&b);
  }
  const __half h = __float2half_rn(v);
  return *reinterpret_cast<const uint16_t*>(&h);
}

__device__ __forceinline__ uint16_t load_act16(const void* a, int64_t i) {
  return __ldg(reinterpret_cast<const unsigned short*>(a) + i);
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_w4a16_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_a,
                         const __grid_constant__ GemmKParams kp) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* act_st = smem + kp.off_act;   // [stages][MT x 128 B], 1024-aligned
  uint8_t* w_st = smem + kp.off_w;       // [stages][128 x 32 B]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kp.off_bar);
  uint64_t* aready = full + kp.stages;
  uint64_t* mdone = aready + kp.stages;
  uint64_t* accf = mdone + kp.stages;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tile = blockIdx.x % kp.tiles_n;
  const int split = blockIdx.x / kp.tiles_n;
  const int mchunk = blockIdx.y;
  const int n0 = tile * kRows;
  const int m0 = mchunk * kp.MT;
  // main k-stages of this split (balanced, never empty since S <= nk), then
  // (last split only) the outlier stages
  const int it0 = int(int64_t(split) * kp.nk / kp.S);
  const int it1 = int(int64_t(split + 1) * kp.nk / kp.S);
  const int n_main = it1 - it0;
  const int n_out_st = (split == kp.S - 1) ? kp.n_os : 0;
  const int n_it = n_main + n_out_st;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < kp.stages; ++i) {
      mbar_init(full + i, 1);
      mbar_init(aready + i, kDeqWarps);
      mbar_init(mdone + i, 1);
    }
    mbar_init(accf, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, kp.tmem_cols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&map_w);
    prefetch_tensormap(&map_a);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const uint32_t a_col0 = uint32_t(kp.MT);  // A stages follow the accumulator's MT columns
  const uint32_t act_bytes = uint32_t(kp.act_stage_bytes);
  const bool bf16 = BF16;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int issued = 0;
      for (int it = 0; it < n_it; ++it) {
        const int s = it % kp.stages;
        const int r = it / kp.stages;
        if (r > 0 && !mbar_wait(mdone + s, uint32_t((r - 1) & 1), &s_abort)) { s_abort = 1; atomicAdd(&g_gemm_timeouts, 1); break; }
        issued = it + 1;
        if (it < n_main) {
          const int kk = (it0 + it) * kBK;
          mbar_arrive_expect_tx(full + s, 4096u + act_bytes);
          tma_load_2d(w_st + s * 4096, &map_w, kk / 2, n0, full + s);
          tma_load_2d(act_st + s * act_bytes, &map_a, kk, m0, full + s);
        } else {
          mbar_arrive(full + s);  // outlier stage: the dequant warps fill B themselves
        }
      }
      // Before the CTA may exit, every TMA copy it issued must have landed: wait
      // (bounded, ignoring the abort flag) for the last use of each stage.
      // On the normal path these phases completed long ago.
      const int zero = 0;
      for (int it = max(0, issued - kp.stages); it < issued; ++it)
        mbar_wait(full + it % kp.stages, uint32_t((it / kp.stages) & 1), &zero);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issue
    if (lane == 0) {
      for (int it = 0; it < n_it; ++it) {
        const int s = it % kp.stages;
        const uint32_t par = uint32_t((it / kp.stages) & 1);
        if (!mbar_wait(aready + s, par, &s_abort) || !mbar_wait(full + s, par, &s_abort)) {
          s_abort = 1;
          atomicAdd(&g_gemm_timeouts, 1);
          break;
        }
        tc_fence_after();
        const uint32_t b_base = smem_u32(act_st + s * act_bytes);
#pragma unroll
        for (int k16 = 0; k16 < kBK / 16; ++k16) {
          const uint64_t bdesc = smem_desc_k_sw128(b_base + k16 * 32);
          mma_ts(tmem, tmem + a_col0 + uint32_t(s * 32 + k16 * 8), bdesc, kp.idesc, (it > 0 || k16 > 0) ? 1u : 0u);
        }
        mma_commit(mdone + s);
      }
      mma_commit(accf);
    }
  } else {
    // ---------------------------------------------------------------- dequant + epilogue
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int h = (warp - 2) >> 2;     // which half of the 64-k stage (one group)
    const int row = q * 32 + lane;     // weight row within the tile
    const int64_t n = int64_t(n0) + row;
    const bool nv = n < kp.N;
    const uint32_t lane_base = uint32_t(q * 32) << 16;
    const int G = kp.K / kGroup;
    // scale / zero of the next main stage, loaded one stage ahead
    auto sz = [&](int it, float& sv, float& zv) {
      const int g = (it0 + it) * 2 + h;
      if (nv && it < n_main && g < G) {
        sv = __half2float(__ldg(kp.scales + n * kp.s_rs + int64_t(g) * kp.s_cs));
        zv = float(__ldg(kp.zeros + n * kp.z_rs + int64_t(g) * kp.z_cs));
      } else {
        sv = 0.f;
        zv = 0.f;
      }
    };
    float s_next, z_next;
    sz(0, s_next, z_next);
    for (int it = 0; it < n_it; ++it) {
      const int s = it % kp.stages;
      const int r = it / kp.stages;
      float sv = s_next, zv = z_next;
      sz(it + 1, s_next, z_next);
      // the wait result is made warp-uniform: tcgen05.st below is .aligned
      bool got = mbar_wait(full + s, uint32_t(r & 1), &s_abort);
      if (got && r > 0) got = mbar_wait(mdone + s, uint32_t((r - 1) & 1), &s_abort);
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) { s_abort = 1; atomicAdd(&g_gemm_timeouts, 1); }
        break;
      }
      tc_fence_after();
      uint32_t vals[16];
      if (it < n_main) {
        const uint4 wv = *reinterpret_cast<const uint4*>(w_st + s * 4096 + row * 32 + h * 16);
        dequant_group<BF16>(wv, sv, zv, kp.layout, vals);
      } else {
        // outlier stage o: columns j0 .. j0+63 of ow / of a[:, idx]
        const int j0 = (it - n_main) * kBK;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          float lo = 0.f, hi = 0.f;
          const int j = j0 + h * 32 + 2 * c;
          if (nv && j < kp.n_out) lo = load_as_float(kp.ow, n * kp.ow_rs + int64_t(j) * kp.ow_cs, kp.ow_dtype);
          if (nv && j + 1 < kp.n_out) hi = load_as_float(kp.ow, n * kp.ow_rs + int64_t(j + 1) * kp.ow_cs, kp.ow_dtype);
          vals[c] = pack2<BF16>(lo, hi);
        }
        // gather a[m0+m, idx[j0+jj]] into the B stage, 128B-swizzled K-major
        uint8_t* bst = act_st + s * act_bytes;
        const int tid_d = (warp - 2) * 32 + lane;
        for (int e = tid_d; e < kp.MT * kBK; e += kDeqWarps * 32) {
          const int m = e / kBK, jj = e % kBK;
          uint16_t v = 0;
          const int j = j0 + jj;
          if (m0 + m < kp.M && j < kp.n_out) {
            const int64_t k = load_index(kp.idx, j, kp.idx_dtype);
            if (k >= 0 && k < kp.K) v = load_act16(kp.a, int64_t(m0 + m) * kp.a_rs + k);
          }
          const int chunk = (jj >> 3) ^ (m & 7);
          *reinterpret_cast<uint16_t*>(bst + m * 128 + chunk * 16 + (jj & 7) * 2) = v;
        }
        fence_proxy_async_smem();
      }
      tmem_st_x16(tmem + lane_base + a_col0 + uint32_t(s * 32 + h * 16), vals);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(aready + s);
    }

    // ---------------------------------------------------------------- epilogue
    // n_it == 0 cannot happen (S <= nk), but an empty split would leave the
    // accumulator unwritten: treat it as zero.
    const bool ok = mbar_wait(accf, 0u, &s_abort) && n_it > 0;
    tc_fence_after();
    const int half_cols = kp.MT / 2;
    const int64_t nrow = int64_t(n0) + row;
    if (kp.S == 1) {
      for (int c0 = h * half_cols; c0 < (h + 1) * half_cols; c0 += 8) {
        float v[8];
        tmem_ld_x8(tmem + lane_base + uint32_t(c0), v);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int m = m0 + c0 + i;
          if (nv && m < kp.M)
            reinterpret_cast<uint16_t*>(kp.c)[int64_t(m) * kp.c_rs + nrow] = to16(ok ? v[i] : 0.f, bf16);
        }
      }
    } else {
      float* part = kp.partials + int64_t(split) * kp.M * kp.N;
      for (int c0 = h * half_cols; c0 < (h + 1) * half_cols; c0 += 8) {
        float v[8];
        tmem_ld_x8(tmem + lane_base + uint32_t(c0), v);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int m = m0 + c0 + i;
          if (nv && m < kp.M) part[int64_t(m) * kp.N + nrow] = ok ? v[i] : 0.f;
        }
      }
    }
  }

  // split-K: the last CTA of this (tile, m-chunk) sums the partials in order
  if (kp.S > 1) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      int* cnt = kp.counters + (mchunk * kp.tiles_n + tile);
      const int ticket = atomicAdd(cnt, 1);
      s_last = (ticket == kp.S - 1);
      if (s_last) *cnt = 0;  // ready for the next call on this workspace
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      const int rows_here = min(kRows, kp.N - n0);
      const int toks = min(kp.MT, kp.M - m0);
      for (int e = threadIdx.x; e < rows_here * toks; e += blockDim.x) {
        const int m = m0 + e / rows_here;
        const int64_t nn = n0 + (e % rows_here);
        float acc = 0.f;
        for (int sp = 0; sp < kp.S; ++sp) acc += __ldcg(kp.partials + (int64_t(sp) * kp.M + m) * kp.N + nn);
        reinterpret_cast<uint16_t*>(kp.c)[int64_t(m) * kp.c_rs + nn] = to16(acc, bf16);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kp.tmem_cols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

}  // namespace

GemmPlan plan_gemm(int64_t M, int64_t N, int64_t K, int64_t n_out) {
  GemmPlan p{};
  const int mt_needed = int(((std::min<int64_t>(M, kMaxMT) + 15) / 16) * 16);
  p.MT = std::max(16, mt_needed);
  p.m_chunks = int((M + kMaxMT - 1) / kMaxMT);
  if (p.m_chunks > 1) p.MT = kMaxMT;
  p.tiles_n = int((N + kRows - 1) / kRows);
  p.nk = int((K + kBK - 1) / kBK);
  p.n_os = int((n_out + kBK - 1) / kBK);
  const int sms = 148;
  const int64_t ctas = int64_t(p.tiles_n) * p.m_chunks;
  int S = int(std::max<int64_t>(1, (sms + ctas / 2) / ctas));
  S = std::min(S, std::max(1, p.nk / 4));  // at least 4 stages of work per split
  p.S = S;
  const int act_stage = p.MT * 128;
  p.stages = p.MT >= 192 ? 4 : 6;
  p.act_stage_bytes = act_stage;
  p.smem = 1024 + size_t(p.stages) * (act_stage + 4096) + size_t(3 * p.stages + 1) * 8 + 64;
  p.tmem_cols = 32;
  while (p.tmem_cols < uint32_t(p.MT + p.stages * 32)) p.tmem_cols <<= 1;
  p.workspace = p.S > 1 ? (256 * ((size_t(p.tiles_n) * p.m_chunks * 4 + 255) / 256) + size_t(p.S) * M * N * 4) : 0;
  return p;
}

int launch_gemm(const GemmArgs& a, void* ws, size_t ws_bytes, cudaStream_t st) {
  const GemmPlan pl = plan_gemm(a.M, a.N, a.K, a.n_out);
  if (pl.tmem_cols > 512 || pl.smem > kMaxDynSmem) return SPECTRA_ERR_UNSUPPORTED;
  if (pl.S > 1 && (ws == nullptr || ws_bytes < pl.workspace)) return SPECTRA_ERR_WORKSPACE;
  auto enc = encode_fn();
  if (!enc) return SPECTRA_ERR_UNSUPPORTED;
  const bool bf16 = a.a_dtype == SPECTRA_DT_BF16;

  CUtensorMap mw, ma;
  {
    cuuint64_t dims[2] = {cuuint64_t(a.K / 2), cuuint64_t(a.N)};
    cuuint64_t strides[1] = {cuuint64_t(a.w_rs)};
    cuuint32_t box[2] = {32, 128}, es[2] = {1, 1};
    if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.packed), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return SPECTRA_ERR_ALIGNMENT;
  }
  {
    cuuint64_t dims[2] = {cuuint64_t(a.K), cuuint64_t(a.M)};
    cuuint64_t strides[1] = {cuuint64_t(a.a_rs) * 2};
    cuuint32_t box[2] = {64, cuuint32_t(pl.MT)}, es[2] = {1, 1};
    if (enc(&ma, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.a),
            dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return SPECTRA_ERR_ALIGNMENT;
  }

  GemmKParams kp{};
  kp.scales = a.scales; kp.s_rs = a.s_rs; kp.s_cs = a.s_cs;
  kp.zeros = a.zeros; kp.z_rs = a.z_rs; kp.z_cs = a.z_cs;
  kp.a = a.a; kp.a_rs = a.a_rs;
  kp.idx = a.idx; kp.idx_dtype = a.idx_dtype; kp.n_out = a.n_out;
  kp.ow = a.ow; kp.ow_dtype = a.ow_dtype; kp.ow_rs = a.ow_rs; kp.ow_cs = a.ow_cs;
  kp.c = a.c; kp.c_dtype = a.c_dtype; kp.c_rs = a.c_rs;
  kp.M = a.M; kp.N = a.N; kp.K = a.K; kp.layout = a.layout;
  kp.MT = pl.MT; kp.stages = pl.stages; kp.S = pl.S; kp.nk = pl.nk; kp.n_os = pl.n_os; kp.tiles_n = pl.tiles_n;
  kp.idesc = idesc_f16(bf16, kRows, pl.MT);
  kp.tmem_cols = pl.tmem_cols;
  kp.act_stage_bytes = pl.act_stage_bytes;
  kp.off_act = 0;
  kp.off_w = pl.stages * pl.act_stage_bytes;
  kp.off_bar = kp.off_w + pl.stages * 4096;
  if (pl.S > 1) {
    const size_t cnt_bytes = 256 * ((size_t(pl.tiles_n) * pl.m_chunks * 4 + 255) / 256);
    kp.counters = reinterpret_cast<int*>(ws);
    kp.partials = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + cnt_bytes);
  }

  auto kern = bf16 ? gemm_w4a16_tc_kernel<true> : gemm_w4a16_tc_kernel<false>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev >= kMaxDevices) return SPECTRA_ERR_UNSUPPORTED;
  static bool attr_set[2][kMaxDevices] = {};
  if (!attr_set[bf16][dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMaxDynSmem));
    if (e != cudaSuccess) return cuda_status(e);
    attr_set[bf16][dev] = true;
  }
  kern<<<dim3(unsigned(pl.tiles_n * pl.S), unsigned(pl.m_chunks)), kThreads, pl.smem, st>>>(mw, ma, kp);
  return cuda_status(cudaGetLastError());
}

int gemm_noalloc_scratch(void** ptr, size_t* bytes) {
  static std::atomic<void*> addr[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return SPECTRA_ERR_UNSUPPORTED;
  void* p = addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    e = cudaGetSymbolAddress((void**)&p, g_gemm_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e);
    addr[dev].store(p, std::memory_order_release);
  }
  *ptr = p;
  *bytes = sizeof(g_gemm_noalloc_scratch);
  return SPECTRA_OK;
}

}  // namespace spectra
