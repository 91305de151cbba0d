// Small-M W4A16 GEMM (M = 2..16 token rows) for sm_100a: the decode batch
// sizes of the M >= 2 branch (spectra/kernels.py:191-389, batched_w4a16_gemm,
// which the engine's batched generation reaches with M = 2..4), computed with
// the M=1 GEMV's raw-code tensor-core step instead of the dequantising tcgen05
// GEMM.  The tcgen05 GEMM turns every weight into a 16-bit operand before its
// MMA (~3 instructions per code), so below a full token tile it costs the same
// as at M = 16; here the codes enter the MMA as they are and the tokens share
// every conversion.
//
// Math
//   A unit is 16 weight rows x 8 groups (256 k).  For one group, lane (g, c) of
//   a warp holds word c (bytes 4c..4c+3: 8 codes) of rows g and g+8; one shift
//   + LOP3 turns a pair of codes into two bf16/fp16 (16 + q) (pair_code), so two
//   m16n8k16 MMAs cover the group's 32 k.  B (16 k x 8) is dense: column n is
//   token n's activations at the same k (staged once per call in exactly this
//   fragment order; M > 8 takes a second tile of 8 tokens on the same A
//   registers), so D[row][token] = sum_k (16 + q_k) x_k over the group and
//   y[row][token] += s (D - (16 + z) X_g[token]), X_g the group's activation
//   sum, in fp32 -- the exact dequantised weights, like the M=1 GEMV (the
//   reference GEMM rounds them to the compute dtype first; both are within the
//   path's tolerance of each other).
//
// Bank-conflict-free stages
//   All lanes of a row quad read the same group, so 8 lanes read 8 rows at the
//   same column: with a power-of-two row pitch that is an 8-way conflict.  The
//   weight stages are therefore [16 rows x 2048 k] tensor-map boxes 16 bytes
//   wider than the data (codes as 64-bit elements, 130 per row; scales 72;
//   zero points 80): the row pitches become 1040, 144 and 80 bytes, every row
//   starts in a different 16-byte bank group, and `ldmatrix.x4` fetches the
//   words of two groups for rows g and g+8 in one conflict-free instruction.
//   The extra 16 bytes per row are the next chunk's first bytes (or zeros past
//   K): they are never used.
//
// Pipeline (as in the weight-prefetching GEMV): one producer warp fills a ring
// of stages by TMA before and after the dependency wait (programmatic
// dependent launch), eight compute warps take one unit each per stage; the
// activations of all M tokens are staged once after the wait.  A CTA owns a
// contiguous range of 16-row blocks; row partials are summed per warp in fixed
// order (deterministic), then the outlier columns in fp32, one rounding to the
// output dtype.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "gemm.h"
#include "gemv_mma.cuh"
#include "sm100_ptx.cuh"
#include "tmap.h"

namespace spectra {

namespace {

constexpr int kMtGroupWarps = 8;             // warps of a compute group: one 256-k unit each per stage
constexpr int kMtMaxStages = 8;
constexpr int kMtChunk = 2048;               // k per stage
constexpr int kMtCodePitch = kMtChunk / 2 + 16;        // bytes per staged code row (130 x 8 B)
constexpr int kMtScalePitch = 2 * (kMtChunk / 32) + 16;  // 144
constexpr int kMtZeroPitch = kMtChunk / 32 + 16;       // 80
constexpr int kMtTok = 8;                    // token columns of the MMA
constexpr size_t kMtSmem = 220 * 1024;

struct MtParams {
  GemmArgs a;
  int nkc;                  // stages per row block
  int ns;                   // ring depth
  int off_sc, off_z, stage_bytes;
  int off_xb, xb_tok;       // x fragments [M][G][4] x 16 B, token pitch in bytes
  int off_xsum;             // [G][8 nt] fp32
  int off_xos;              // [n_out][8 nt] fp32
  int off_red;              // [warps][rows_max][8 nt] fp32
  int off_ow;               // staged outlier weight rows (or -1)
  int off_stage;
  int rows_max;
  int vec_a;                // 16-byte activation loads
  int ng;                   // compute groups (alternate stages)
  int nt;                   // token tiles of 8
};

struct MtMaps {
  CUtensorMap c, s, z;
};

__device__ int g_gemv_mt_timeouts;

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
}

// 16-byte shared load when `pred` (B fragments of tokens past M stay zero).
__device__ __forceinline__ void lds128_if(uint32_t (&v)[4], const void* p, bool pred) {
  asm volatile(
      "{\n\t.reg .pred q;\n\t"
      "setp.ne.b32 q, %5, 0;\n\t"
      "@q ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n\t}"
      : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3])
      : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))), "r"(int(pred)));
}

__device__ __forceinline__ bool mt_wait(uint64_t* bar, uint32_t parity, const volatile int* abort) {
  using namespace sm100;
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    if (i == 0 ? mbar_test(bar, parity) : mbar_try_wait(bar, parity)) return true;
    if ((i & 31) == 31) {
      if (*abort) return false;
      const uint64_t now = global_ns();
      if (i == 31)
        t0 = now;
      else if (now - t0 > kWaitLimitNs)
        return false;
    }
  }
}

template <int NT>
__device__ __forceinline__ void mt_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
}

// NG compute groups of 8 warps (group i takes stages i, i + NG, ...) and one
// producer warp; NT token tiles of 8 (M <= 8 NT), which share every A operand.
template <bool BF16, int NG, int NT>
__global__ void __launch_bounds__((NG * kMtGroupWarps + 1) * 32, 1)
    gemv_mt_kernel(const __grid_constant__ MtMaps maps, const __grid_constant__ MtParams kp) {
  using namespace sm100;
  constexpr int kMtWarps = NG * kMtGroupWarps;  // compute warps
  constexpr int TOK = kMtTok * NT;              // token stride of the per-token shared arrays
  const GemmArgs& p = kp.a;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full_bar[kMtMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMtMaxStages];
  __shared__ __align__(8) uint64_t ow_bar;
  __shared__ int s_abort;

  pdl_trigger();

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t nblk = (int64_t(p.N) + 15) / 16;
  const int64_t b0 = (nblk * blockIdx.x) / gridDim.x;
  const int64_t b1 = (nblk * (blockIdx.x + 1)) / gridDim.x;
  const int nrb = int(b1 - b0);
  const int64_t r_begin = b0 * 16;
  const int64_t r_end = int64_t(p.N) < b1 * 16 ? int64_t(p.N) : b1 * 16;
  const int nrows = int(r_end - r_begin);
  const int G = p.K / kGroup;
  const int M = p.M;

  const int ow_es = p.ow_dtype == SPECTRA_DT_F32 ? 4 : 2;
  const bool ow_staged = kp.off_ow >= 0 && p.n_out > 0;
  const int64_t ow_b0 = r_begin * p.n_out * ow_es, ow_b1 = r_end * p.n_out * ow_es;
  const int64_t ow_a0 = ow_b0 & ~int64_t(15), ow_a1 = ow_b1 & ~int64_t(15);

  if (tid == 0) {
    s_abort = 0;
    for (int s = 0; s < kp.ns; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kMtGroupWarps);  // a stage is consumed by one group
    }
    mbar_init(&ow_bar, ow_staged ? 2 : 1);
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kMtWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint64_t policy;
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
      if (ow_staged) {
        const uint8_t* ow_src = reinterpret_cast<const uint8_t*>(p.ow);
        mbar_arrive_expect_tx(&ow_bar, uint32_t(ow_a1 - ow_a0));
        if (ow_a1 > ow_a0) bulk_g2s_hint(smem + kp.off_ow, ow_src + ow_a0, uint32_t(ow_a1 - ow_a0), &ow_bar, policy);
        for (int64_t bt = ow_a1; bt < ow_b1; ++bt) smem[kp.off_ow + (bt - ow_a0)] = ow_src[bt];
        mbar_arrive(&ow_bar);
      }
      const uint32_t tx = 16u * uint32_t(kMtCodePitch + kMtScalePitch + kMtZeroPitch);  // whole boxes
      int s = 0, issued = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int rb = 0; rb < nrb && ok; ++rb) {
        const int row0 = int(r_begin) + rb * 16;
        for (int ch = 0; ch < kp.nkc; ++ch) {
          if (issued >= kp.ns && !mt_wait(&empty_bar[s], ph ^ 1u, &s_abort)) {
            s_abort = 1;
            atomicAdd(&g_gemv_mt_timeouts, 1);
            ok = false;
            break;
          }
          uint8_t* st = smem + kp.off_stage + s * kp.stage_bytes;
          mbar_arrive_expect_tx(&full_bar[s], tx);
          tma_load_2d_hint(st, &maps.c, ch * (kMtChunk / 16), row0, &full_bar[s], policy);
          tma_load_2d_hint(st + kp.off_sc, &maps.s, ch * (kMtChunk / 32), row0, &full_bar[s], policy);
          tma_load_2d_hint(st + kp.off_z, &maps.z, ch * (kMtChunk / 32), row0, &full_bar[s], policy);
          ++issued;
          if (++s == kp.ns) { s = 0; ph ^= 1u; }
        }
      }
      // leave no copy in flight: wait (bounded) for the last stages issued
      const int tail = issued < kp.ns ? issued : kp.ns;
      for (int i = 0; i < tail; ++i) {
        if (s == 0) { s = kp.ns; ph ^= 1u; }
        --s;
        (void)mt_wait(&full_bar[s], ph, &s_abort);
      }
      if (ow_staged) (void)mt_wait(&ow_bar, 0, &s_abort);
    }
    return;
  }

  // -------------------------------------------------------------- compute
  uint8_t* xb = smem + kp.off_xb;
  float* xsum = reinterpret_cast<float*>(smem + kp.off_xsum);
  float* xos = reinterpret_cast<float*>(smem + kp.off_xos);
  float* red = reinterpret_cast<float*>(smem + kp.off_red);
  constexpr int kCT = kMtWarps * 32;
  const int rows_max = kp.rows_max;

  // the row partials start at zero (shared memory only: before the wait)
  for (int i = tid; i < kMtWarps * rows_max * TOK; i += kCT) red[i] = 0.f;

  pdl_wait();  // the activations may be the previous kernel's output

  // x at the outlier features, [j][token]
  for (int i = tid; i < p.n_out * TOK; i += kCT) {
    const int j = i / TOK, t = i % TOK;
    float v = 0.f;
    if (t < M) {
      const int64_t k = load_index(p.idx, j, p.idx_dtype);
      if (k >= 0 && k < p.K) v = load_as_float_cg(p.a, int64_t(t) * p.a_rs + k, p.a_dtype);
    }
    xos[i] = v;
  }
  // Activations -> B fragments, one item per (token, group): its 32 values,
  // the group sum X_g, and the four 16-byte fragments of lanes c = 0..3 (k of
  // word c of the codes: Marlin bytes 4c..4c+3 hold k 4c+i (low nibble) and
  // 4c+16+i (high); even-odd bytes hold k 2b and 2b+1).
  const bool marlin = p.layout == SPECTRA_LAYOUT_MARLIN;
  for (int i = tid; i < M * G; i += kCT) {
    const int t = i / G, grp = i - t * G;
    uint32_t w[16];
    const int64_t e0 = int64_t(t) * p.a_rs + int64_t(grp) * kGroup;
    if (kp.vec_a) {
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.a) + e0);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 v = __ldcg(src + q);
        w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
      }
    } else {
      const uint16_t* src = static_cast<const uint16_t*>(p.a) + e0;
#pragma unroll
      for (int q = 0; q < 16; ++q) w[q] = uint32_t(__ldcg(src + 2 * q)) | (uint32_t(__ldcg(src + 2 * q + 1)) << 16);
    }
    float X = 0.f;
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      if constexpr (BF16) {
        X += __uint_as_float(w[q] << 16) + __uint_as_float(w[q] & 0xFFFF0000u);
      } else {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[q]));
        X += f.x + f.y;
      }
    }
    xsum[grp * TOK + t] = X;
    uint4* dst = reinterpret_cast<uint4*>(xb + t * kp.xb_tok + grp * 64);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint4 f;
      if (marlin) {
        f.x = prmt(w[2 * c], w[2 * c + 1], 0x5410u);      // k 4c, 4c+2
        f.y = prmt(w[2 * c], w[2 * c + 1], 0x7632u);      // k 4c+1, 4c+3
        f.z = prmt(w[8 + 2 * c], w[9 + 2 * c], 0x5410u);  // k 4c+16, 4c+18
        f.w = prmt(w[8 + 2 * c], w[9 + 2 * c], 0x7632u);  // k 4c+17, 4c+19
      } else {
        f.x = prmt(w[4 * c], w[4 * c + 2], 0x5410u);      // k 8c, 8c+4
        f.y = prmt(w[4 * c + 1], w[4 * c + 3], 0x5410u);  // k 8c+2, 8c+6
        f.z = prmt(w[4 * c], w[4 * c + 2], 0x7632u);      // k 8c+1, 8c+5
        f.w = prmt(w[4 * c + 1], w[4 * c + 3], 0x7632u);  // k 8c+3, 8c+7
      }
      dst[c] = f;
    }
  }
  for (int i = tid; i < G * TOK; i += kCT)
    if (i % TOK >= M) xsum[i] = 0.f;
  mt_bar<kCT>();

  // ------------------------------------------------------------ main loop
  uint32_t magic_reg;
  asm volatile("mov.b32 %0, %1;" : "=r"(magic_reg) : "n"(BF16 ? 0x41804180u : 0x4C004C00u));  // 16.0 x2
  const int g = lane >> 2, c = lane & 3;
  // this lane's B column of tile tt is token g + 8 tt
  // ldmatrix row addresses: lanes 0-7 rows 0-7 / 8-15 rows 8-15 of group gl,
  // 16-31 the same rows of group gl + 1
  const int lm_row = (lane & 7) + 8 * ((lane >> 3) & 1);
  const int lm_grp = lane >> 4;
  const int KB = p.K >> 8;  // 256-feature units per row
  const int grp_id = NG == 1 ? 0 : warp / kMtGroupWarps;  // compute group, and warp inside it
  const int w8 = NG == 1 ? warp : warp % kMtGroupWarps;
  // Stages are consumed in issue order: stage si by group si % NG.  With two
  // groups the ring depth is even, so a group's previous use of a ring slot
  // was its own and was waited for.
  int s = 0, si = 0;
  uint32_t ph = 0;
  for (int rb = 0; rb < nrb; ++rb) {
    float acc[NT][4] = {};
    for (int ch = 0; ch < kp.nkc; ++ch, ++si) {
      if (NG > 1 && si % NG != grp_id) {
        if (++s == kp.ns) { s = 0; ph ^= 1u; }
        continue;
      }
      bool ready = mt_wait(&full_bar[s], ph, &s_abort);
      ready = __all_sync(0xffffffffu, ready);
      if (!ready) {
        if (lane == 0) { s_abort = 1; atomicAdd(&g_gemv_mt_timeouts, 1); }
      } else {
        const int kb = ch * (kMtChunk / 256) + w8;  // this warp's unit along K
        if (kb < KB) {
          const uint8_t* st = smem + kp.off_stage + s * kp.stage_bytes;
          const uint8_t* cst = st + w8 * 128;  // the unit's first group: 8 groups x 16 B
          // scales / zero points of the unit's 8 groups, rows g and g+8
          const uint4 sa4 = *reinterpret_cast<const uint4*>(st + kp.off_sc + g * kMtScalePitch + w8 * 16);
          const uint4 sb4 = *reinterpret_cast<const uint4*>(st + kp.off_sc + (g + 8) * kMtScalePitch + w8 * 16);
          const uint2 za2 = *reinterpret_cast<const uint2*>(st + kp.off_z + g * kMtZeroPitch + w8 * 8);
          const uint2 zb2 = *reinterpret_cast<const uint2*>(st + kp.off_z + (g + 8) * kMtZeroPitch + w8 * 8);
          const uint32_t sa[4] = {sa4.x, sa4.y, sa4.z, sa4.w}, sb[4] = {sb4.x, sb4.y, sb4.z, sb4.w};
          const uint32_t za[2] = {za2.x, za2.y}, zb[2] = {zb2.x, zb2.y};
#pragma unroll
          for (int gp = 0; gp < 4; ++gp) {  // pairs of groups
            uint32_t wv[4];
            ldsm_x4(wv, cst + lm_row * kMtCodePitch + (2 * gp + lm_grp) * 16);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int gi = 2 * gp + h;
              const int grp = kb * 8 + gi;
              const uint32_t wg = wv[2 * h], wg8 = wv[2 * h + 1];
              const uint32_t a0 = pair_code<BF16, 0>(wg, magic_reg), a1 = pair_code<BF16, 0>(wg8, magic_reg);
              const uint32_t a2 = pair_code<BF16, 2>(wg, magic_reg), a3 = pair_code<BF16, 2>(wg8, magic_reg);
              const uint32_t a4 = pair_code<BF16, 1>(wg, magic_reg), a5 = pair_code<BF16, 1>(wg8, magic_reg);
              const uint32_t a6 = pair_code<BF16, 3>(wg, magic_reg), a7 = pair_code<BF16, 3>(wg8, magic_reg);
              const float s_a = __half2float(__ushort_as_half(uint16_t(sa[gi >> 1] >> (16 * (gi & 1)))));
              const float s_b = __half2float(__ushort_as_half(uint16_t(sb[gi >> 1] >> (16 * (gi & 1)))));
              const float z_a = 16.f + float((za[gi >> 2] >> (8 * (gi & 3))) & 0xFFu);
              const float z_b = 16.f + float((zb[gi >> 2] >> (8 * (gi & 3))) & 0xFFu);
#pragma unroll
              for (int tt = 0; tt < NT; ++tt) {
                uint32_t bf[4] = {0u, 0u, 0u, 0u};
                lds128_if(bf, xb + (g + 8 * tt) * kp.xb_tok + grp * 64 + c * 16, g + 8 * tt < M);
                float d[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816<BF16>(d, a0, a1, a2, a3, bf[0], bf[1]);
                mma16816<BF16>(d, a4, a5, a6, a7, bf[2], bf[3]);
                // d = {D[g][2c], D[g][2c+1], D[g+8][2c], D[g+8][2c+1]} of tile tt
                const float2 X = *reinterpret_cast<const float2*>(xsum + grp * TOK + 8 * tt + 2 * c);
                acc[tt][0] += s_a * fmaf(-z_a, X.x, d[0]);
                acc[tt][1] += s_a * fmaf(-z_a, X.y, d[1]);
                acc[tt][2] += s_b * fmaf(-z_b, X.x, d[2]);
                acc[tt][3] += s_b * fmaf(-z_b, X.y, d[3]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[s]);
      if (++s == kp.ns) { s = 0; ph ^= 1u; }
    }
    // this warp's partials of the row block: rows g, g+8, tokens 8 tt + 2c, + 1
    float* rw = red + (int64_t(warp) * rows_max + rb * 16) * TOK;
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) {
      *reinterpret_cast<float2*>(rw + g * TOK + 8 * tt + 2 * c) = make_float2(acc[tt][0], acc[tt][1]);
      *reinterpret_cast<float2*>(rw + (g + 8) * TOK + 8 * tt + 2 * c) = make_float2(acc[tt][2], acc[tt][3]);
    }
  }

  // ---------------------------- outlier columns, the partials in order, store
  bool ow_ok = true;
  if (ow_staged) {
    ow_ok = mt_wait(&ow_bar, 0, &s_abort);
    ow_ok = __all_sync(0xffffffffu, ow_ok);
    if (!ow_ok && lane == 0) { s_abort = 1; atomicAdd(&g_gemv_mt_timeouts, 1); }
  }
  mt_bar<kCT>();
  // eight threads per row: outlier features j = sub, sub + 8, ... for all
  // tokens, then a transposing reduction leaves token reduced_row<8>(lane) of
  // the row in each thread
  constexpr int tpr = 8;
  const int sub = tid & (tpr - 1);
  const int64_t row_bytes = int64_t(p.n_out) * ow_es;
  const uint8_t* ow_rows = smem + (kp.off_ow >= 0 ? kp.off_ow : 0) + (ow_b0 - ow_a0);
  for (int i0 = 0; i0 < nrows; i0 += kCT / tpr) {  // CTA-uniform trips
    const int i = i0 + tid / tpr;
#pragma unroll 1
    for (int tt = 0; tt < NT; ++tt) {  // 8 tokens at a time
      float v[kMtTok];
#pragma unroll
      for (int t = 0; t < kMtTok; ++t) v[t] = 0.f;
      if (i < nrows && ow_ok) {
        for (int j = sub; j < p.n_out; j += tpr) {
          float w;
          if (ow_staged) {
            const uint8_t* orow = ow_rows + int64_t(i) * row_bytes;
            w = ow_es == 4 ? reinterpret_cast<const float*>(orow)[j]
                : p.ow_dtype == SPECTRA_DT_BF16
                    ? __uint_as_float(uint32_t(reinterpret_cast<const uint16_t*>(orow)[j]) << 16)
                    : __half2float(reinterpret_cast<const __half*>(orow)[j]);
          } else {
            w = load_as_float(p.ow, (r_begin + i) * p.ow_rs + int64_t(j) * p.ow_cs, p.ow_dtype);
          }
          const float4 x0 = *reinterpret_cast<const float4*>(xos + j * TOK + 8 * tt);
          const float4 x1 = *reinterpret_cast<const float4*>(xos + j * TOK + 8 * tt + 4);
          v[0] = fmaf(x0.x, w, v[0]); v[1] = fmaf(x0.y, w, v[1]); v[2] = fmaf(x0.z, w, v[2]); v[3] = fmaf(x0.w, w, v[3]);
          v[4] = fmaf(x1.x, w, v[4]); v[5] = fmaf(x1.y, w, v[5]); v[6] = fmaf(x1.z, w, v[6]); v[7] = fmaf(x1.w, w, v[7]);
        }
      }
      // sum over the row's 8 lanes, transposing: afterwards v[0] of lane
      // (sub) is the total of token 8 tt + sub
#pragma unroll
      for (int half = 4; half >= 1; half >>= 1) {
        const bool up = (lane & half) != 0;
#pragma unroll
        for (int q = 0; q < half; ++q) {
          const float send = up ? v[q] : v[q + half];
          const float keep = up ? v[q + half] : v[q];
          v[q] = keep + __shfl_xor_sync(0xffffffffu, send, half);
        }
      }
      const int t = 8 * tt + sub;
      if (i < nrows && t < M) {
        float y = 0.f;
#pragma unroll
        for (int ww = 0; ww < kMtWarps; ++ww) y += red[(int64_t(ww) * rows_max + i) * TOK + t];
        y += v[0];
        store_from_float(p.c, int64_t(t) * p.c_rs + r_begin + i, p.c_dtype, y);
      }
    }
  }
}

inline size_t r16(size_t v) { return (v + 15) & ~size_t(15); }
inline size_t r128(size_t v) { return (v + 127) & ~size_t(127); }
inline bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

bool small_m_enabled() {
  static const bool on = [] {
    const char* e = getenv("SPECTRA_B200_GEMM_SMALL_M");
    return !(e && e[0] == '0');
  }();
  return on;
}

// The configuration of the small-M kernel for `a` (no CUDA call); false when
// it does not take the call (the tcgen05 GEMM does).
bool plan_gemv_mt(const GemmArgs& a, int sms, MtParams& kp, int64_t& grid, size_t& smem) {
  if (a.M < 2 || a.M > 2 * kMtTok || a.K % 512 != 0 || a.N <= 0 || sms <= 0) return false;
  if (a.a_dtype != SPECTRA_DT_BF16 && a.a_dtype != SPECTRA_DT_F16) return false;
  if (!al16(a.packed) || !al16(a.scales) || !al16(a.zeros) || a.s_cs != 1 || a.z_cs != 1) return false;
  if (a.w_rs % 16 != 0 || (a.s_rs * 2) % 16 != 0 || a.z_rs % 16 != 0) return false;  // tensor-map pitches
  const int G = a.K / kGroup;
  kp = MtParams{};
  kp.a = a;
  const int64_t nblk = (int64_t(a.N) + 15) / 16;
  grid = std::min<int64_t>(nblk, sms);
  const int64_t rb_max = (nblk + grid - 1) / grid;
  kp.rows_max = int(rb_max * 16);
  kp.nkc = (a.K + kMtChunk - 1) / kMtChunk;
  kp.vec_a = (al16(a.a) && (a.a_rs * 2) % 16 == 0) ? 1 : 0;
  size_t off = 0;
  kp.off_xb = 0;
  kp.xb_tok = G * 64 + 64;  // + 64: tokens start in different bank groups
  off = r16(size_t(a.M) * kp.xb_tok);
  kp.off_xsum = int(off);
  kp.nt = a.M > kMtTok ? 2 : 1;  // token tiles
  const int tok = kMtTok * kp.nt;
  off = r16(off + size_t(G) * tok * 4);
  kp.off_xos = int(off);
  off = r16(off + size_t(a.n_out) * tok * 4);
  kp.off_red = int(off);
  const size_t red_base = off;
  const int64_t units = rb_max * kp.nkc;
  kp.off_sc = 16 * kMtCodePitch;
  kp.off_z = kp.off_sc + 16 * kMtScalePitch;
  kp.stage_bytes = int(r128(size_t(kp.off_z) + 16 * kMtZeroPitch));
  const int ow_es = a.ow_dtype == SPECTRA_DT_F32 ? 4 : 2;
  const bool ow_contig = a.n_out > 0 && a.ow_cs == 1 && a.ow_rs == a.n_out && al16(a.ow);
  // Two compute groups on alternate stages (16 warps hide the shared-memory
  // and MMA latencies better than 8) while the ring stays >= 4 stages deep;
  // otherwise one group with the deeper ring.
  for (int ng = units >= 4 ? 2 : 1; ng >= 1; --ng) {
    kp.ng = ng;
    const size_t ow_base = r16(red_base + size_t(ng * kMtGroupWarps) * kp.rows_max * tok * 4);
    for (int try_ow = ow_contig ? 1 : 0; try_ow >= 0; --try_ow) {
      size_t o = ow_base;
      kp.off_ow = -1;
      if (try_ow) {
        kp.off_ow = int(o);
        o = r16(o + size_t(kp.rows_max) * a.n_out * ow_es + 32);
      }
      kp.off_stage = int(r128(o));
      if (size_t(kp.off_stage) >= kMtSmem) continue;
      int64_t ns = std::min<int64_t>({int64_t(kMtMaxStages), int64_t((kMtSmem - kp.off_stage) / kp.stage_bytes),
                                      units});
      if (ng == 2) {
        ns &= ~int64_t(1);  // a ring slot's consecutive stages belong to one group
        if (ns < 4) continue;
      }
      if (ns < std::min<int64_t>(2, units)) continue;
      kp.ns = int(ns);
      smem = size_t(kp.off_stage) + size_t(ns) * kp.stage_bytes;
      return true;
    }
  }
  return false;
}

bool encode_mt_maps(const GemmArgs& a, MtMaps& maps) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const int G = a.K / kGroup;
  cuuint32_t es[2] = {1, 1};
  // boxes 16 bytes wider than a chunk's data: staged row pitches 1040 / 144 / 80 bytes
  cuuint64_t dc[2] = {cuuint64_t(a.K / 16), cuuint64_t(a.N)}, sc[1] = {cuuint64_t(a.w_rs)};
  cuuint32_t bc[2] = {cuuint32_t(kMtCodePitch / 8), 16};
  cuuint64_t dg[2] = {cuuint64_t(G), cuuint64_t(a.N)};
  cuuint64_t ss[1] = {cuuint64_t(a.s_rs) * 2}, zs[1] = {cuuint64_t(a.z_rs)};
  cuuint32_t bs[2] = {cuuint32_t(kMtScalePitch / 2), 16}, bz[2] = {cuuint32_t(kMtZeroPitch), 16};
  return enc(&maps.c, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(a.packed), dc, sc, bc, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS &&
         enc(&maps.s, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<__half*>(a.scales), dg, ss, bs, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS &&
         enc(&maps.z, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.zeros), dg, zs, bz, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool BF16, int NG, int NT>
int launch_mt(const MtMaps& maps, const MtParams& kp, int64_t grid, size_t smem, int dev, cudaStream_t st) {
  auto kern = gemv_mt_kernel<BF16, NG, NT>;
  static PerContextOnce attrs;
  cudaError_t e = attrs.run(dev, [&] {
    cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMtSmem));
    if (r == cudaSuccess)
      r = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
    return r;
  });
  if (e != cudaSuccess) return cuda_status(e);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3((NG * kMtGroupWarps + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, maps, kp));
}

}  // namespace

int gemv_mt_timeouts(long long* out, bool reset) { return read_timeout_counter(g_gemv_mt_timeouts, out, reset); }

int launch_gemv_mt(const GemmArgs& a, cudaStream_t st) {
  if (!small_m_enabled()) return SPECTRA_ERR_UNSUPPORTED;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev >= kMaxDevices) return SPECTRA_ERR_UNSUPPORTED;
  MtParams kp;
  int64_t grid = 0;
  size_t smem = 0;
  if (!plan_gemv_mt(a, device_sms(dev), kp, grid, smem)) return SPECTRA_ERR_UNSUPPORTED;
  MtMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (!encode_mt_maps(a, maps)) return SPECTRA_ERR_UNSUPPORTED;
  const bool bf = a.a_dtype == SPECTRA_DT_BF16;
  if (kp.nt == 2) {
    if (kp.ng == 2)
      return bf ? launch_mt<true, 2, 2>(maps, kp, grid, smem, dev, st) : launch_mt<false, 2, 2>(maps, kp, grid, smem, dev, st);
    return bf ? launch_mt<true, 1, 2>(maps, kp, grid, smem, dev, st) : launch_mt<false, 1, 2>(maps, kp, grid, smem, dev, st);
  }
  if (kp.ng == 2)
    return bf ? launch_mt<true, 2, 1>(maps, kp, grid, smem, dev, st) : launch_mt<false, 2, 1>(maps, kp, grid, smem, dev, st);
  return bf ? launch_mt<true, 1, 1>(maps, kp, grid, smem, dev, st) : launch_mt<false, 1, 1>(maps, kp, grid, smem, dev, st);
}

}  // namespace spectra

// Diagnostic (declared in include/spectra_b200.h): whether the small-M kernel
// takes a GEMM of this shape with contiguous, 16-byte-aligned operands, and
// its configuration, without a GPU.
extern "C" SPECTRA_API int spectra_gemm_small_m_plan(int64_t M, int64_t N, int64_t K, int64_t n_out, int a_dtype,
                                                     int ow_dtype, int sms, int64_t* out) {
  if (!out) return SPECTRA_ERR_NULL_POINTER;
  if (M <= 0 || N <= 0 || K <= 0 || K % 32 != 0 || n_out < 0 || n_out > K || N > 2147483647LL ||
      K > 2147483647LL || M > 2147483647LL)
    return SPECTRA_ERR_SHAPE;
  auto float_dt = [](int dt) { return dt == SPECTRA_DT_F16 || dt == SPECTRA_DT_BF16 || dt == SPECTRA_DT_F32; };
  if ((a_dtype != SPECTRA_DT_F16 && a_dtype != SPECTRA_DT_BF16) || (n_out > 0 && !float_dt(ow_dtype)))
    return SPECTRA_ERR_DTYPE;
  spectra::GemmArgs a{};
  const uintptr_t aligned = 4096;  // stand-in 16-byte-aligned addresses (never dereferenced)
  a.a = reinterpret_cast<const void*>(aligned);
  a.a_dtype = a_dtype;
  a.a_rs = K;
  a.packed = reinterpret_cast<const uint8_t*>(aligned);
  a.w_rs = K / 2;
  a.scales = reinterpret_cast<const __half*>(aligned);
  a.s_rs = K / 32;
  a.s_cs = 1;
  a.zeros = reinterpret_cast<const uint8_t*>(aligned);
  a.z_rs = K / 32;
  a.z_cs = 1;
  a.n_out = int(n_out);
  a.ow = n_out > 0 ? reinterpret_cast<const void*>(aligned) : nullptr;
  a.ow_dtype = ow_dtype;
  a.ow_rs = n_out;
  a.ow_cs = 1;
  a.c_dtype = a_dtype;
  a.c_rs = N;
  a.M = int(M);
  a.N = int(N);
  a.K = int(K);
  a.layout = SPECTRA_LAYOUT_MARLIN;
  spectra::MtParams kp;
  int64_t grid = 0;
  size_t smem = 0;
  const bool ok = spectra::plan_gemv_mt(a, sms, kp, grid, smem);
  out[0] = ok ? 1 : 0;
  out[1] = ok ? grid : 0;
  out[2] = ok ? int64_t(smem) : 0;
  out[3] = ok ? kp.ns : 0;
  out[4] = ok ? (kp.off_ow >= 0 ? 1 : 0) : 0;
  out[5] = ok ? kp.ng : 0;
  out[6] = ok ? kp.nt : 0;
  return SPECTRA_OK;
}
