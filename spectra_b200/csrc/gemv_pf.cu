// M=1 W4A16 decode GEMV, weight-prefetching variant for sm_100a (replaces
// spectra/kernels.py:16-184 for contiguous, 16-byte-aligned weights with K a
// multiple of 512; other layouts take gemv.cu).
//
// Why a second kernel
//   A decoder layer at M=1 is a chain of small GEMVs (0.5-10 MB of weights
//   each), so per-launch latency (the previous kernel's completion, then the
//   activation load, then the first weight loads) outweighs the streaming
//   time.  This kernel moves every weight byte of a CTA into shared memory
//   BEFORE it waits on the previous kernel (programmatic dependent launch):
//   weights, scales, zero points and outlier weights are never written by the
//   kernels of this library that release their dependents early, so reading
//   them ahead of the dependency wait is safe.  Only the copies run early:
//   compute there would take issue slots from the previous kernel.
//
// Residency
//   A CTA that owns one row block uses at most ~110 KB of shared memory and
//   <= 96 registers per thread, so two CTAs -- this launch's and the next
//   one's -- fit on one SM: while one computes, the next one's bulk copies
//   already stream its weights.  A CTA that owns several row blocks takes its
//   SM alone (>= 116 KB): sharing the SM with the next launch's prefetch was
//   measured slower on a decoder layer (the co-resident copies delay this
//   kernel's post-wait loads); the next launch's CTAs start on SMs as they free.
//
// Work decomposition
//   Grid = min(16-row blocks, SMs); CTA c owns 16-row blocks [b0, b1) (an even
//   split).  With contiguous weights a row block's codes, scales and zero
//   points are three contiguous ranges: a "stage" is one row block, fetched by
//   three bulk copies (a copy costs ~70-100 cycles to issue plus ~1 cycle per
//   60 bytes, so few large copies keep the issue time far below the streaming
//   time), with an L2 evict-first hint.  When two such stages do not fit
//   (K = 14336, 28672) or the rows are padded views, a stage is [16 rows x 2048
//   features] instead, fetched by three 2D tensor-map copies (codes as 32-bit
//   words, scales, zero points; rows past N read as zeros).  The last warp
//   fills a ring of `ns` stages (every stage of the CTA up front when they fit)
//   and refills it as stages free; the other warps compute: one group of 8,
//   or two groups on alternate stages (whole-row-block stages: CTAs with >= 5
//   row blocks; chunked stages: every CTA that owns its SM).  The CTA's
//   outlier-weight rows arrive by one bulk copy before the wait when they
//   fit beside a ring of >= 4 stages; otherwise (two groups only) they
//   stream through the ring in pieces once its last stage is consumed, or
//   (one group) are read from global memory in the final pass.
//
// Math (same as gemv.cu's tensor-core kernel)
//   A unit is 16 rows x 8 groups (256 k).  Lane (g, c) of a warp holds rows g
//   and g+8, groups 2c and 2c+1 of the unit; codes become bf16/fp16 16+q by
//   one shift + LOP3, x sits block-diagonally in the B operand, so the 16
//   m16n8k16 MMAs give D[row][group] = sum_k (16+q_k) x_k.  Per group:
//   sum_k (q_k - z) s x_k = s (D - (16 + z) X_g), X_g = sum of the group's x.
//   Warp w of a group takes units w, w+8, ... of the group's stages and keeps
//   one fp32 partial per row; the 8 (16) partials of a row are summed in warp
//   order at the end (deterministic), then the outlier columns
//   (kernels.py:102-120), the bias (:122-124) and one rounding to y's dtype.
#include "common.cuh"
#include "gemv.h"
#include "gemv_mma.cuh"
#include "sm100_ptx.cuh"
#include "tmap.h"

namespace spectra {

namespace {

constexpr int kPfGroupWarps = 8;  // warps of one compute group: the 8 units of 256 features of a row block
constexpr int kPfMaxStages = 8;
constexpr size_t kPfSmemPair = 110 * 1024;    // two CTAs per SM (228 KB per SM)
constexpr size_t kPfSmemSolo = 200 * 1024;    // one CTA per SM
constexpr size_t kPfSoloFloor = 116 * 1024;   // more than half an SM's shared memory: one CTA per SM
constexpr int kPfKQuantum = 512;
constexpr int kPfChunk = 2048;      // features per tensor-map stage (codes box: 256 32-bit words)
constexpr int kPfMinWholeStages = 3;  // ring depth below which whole-row-block stages give way to chunks
constexpr int kPfMinStagedRing = 4;   // ring depth below which staged outlier rows give way to streaming
constexpr int kXpWords = 20;  // staged x pairs per group: 16 + 4 pad (conflict-free B-fragment loads)

struct PfParams {
  GemvArgs a;
  int ns;                          // ring stages
  int kc, nkc;                     // input features per stage (a multiple of 512), stages per row block
  int off_sc, off_z, stage_bytes;  // offsets inside one stage (codes at 0)
  int cs, ss, zs;                  // staged row pitches (bytes) of codes, scales, zero points
  int off_x, off_xsum, off_xos, off_red, off_ow, off_stage;
  int rows_max;
  int vec_x;                       // x contiguous and 16-byte aligned
  int ow_ring_rows;                // > 0: outlier rows stream through the freed ring, this many per piece
};

// Tensor maps of the chunked mode; the contiguous mode passes an empty struct
// (no 384 bytes of unused kernel parameters per launch).
template <bool CHUNKED>
struct PfMaps {
  CUtensorMap c, s, z;  // codes, scales, zero points
};
template <>
struct PfMaps<false> {};

__device__ int g_gemv_pf_timeouts;  // stuck pipeline waits since load (diagnostic)

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// 16-byte shared load into v when `pred`; v keeps its value otherwise (no
// request for the lanes that are off).  The B fragments of the lanes that
// never load stay at their initial zeros.
__device__ __forceinline__ void lds128_keep(uint32_t& v0, uint32_t& v1, uint32_t& v2, uint32_t& v3, const uint4* p,
                                            bool pred) {
  asm volatile(
      "{\n\t.reg .pred q;\n\t"
      "setp.ne.b32 q, %5, 0;\n\t"
      "@q ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n\t}"
      : "+r"(v0), "+r"(v1), "+r"(v2), "+r"(v3)
      : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))), "r"(int(pred)));
}

// The bounded wait of sm100_ptx.cuh, inlined: at a call site with many live
// registers the out-of-line slow path costs a stack frame and spills.
__device__ __forceinline__ bool mbar_wait_inl(uint64_t* bar, uint32_t parity, const volatile int* abort) {
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
__device__ __forceinline__ void compute_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
}

// NG compute groups of 8 warps plus one copy warp.  NG = 1: <= 96 registers,
// so two CTAs fit on an SM; NG = 2 (CTAs that own their SM): group i takes
// stages i, i+2, ... of the ring.
template <bool BF16, int NG, bool CHUNKED>
__global__ void __launch_bounds__((NG * kPfGroupWarps + 1) * 32, NG == 1 ? 2 : 1)
    gemv_pf_kernel(const __grid_constant__ PfMaps<CHUNKED> maps, const __grid_constant__ PfParams kp) {
  constexpr int kPfComputeWarps = NG * kPfGroupWarps;
  using namespace sm100;
  const GemvArgs& p = kp.a;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full_bar[kPfMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kPfMaxStages];
  __shared__ __align__(8) uint64_t ow_bar;
  __shared__ int s_abort;
  __shared__ int s_zero;

  pdl_trigger();

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t nblk = (int64_t(p.N) + 15) / 16;
  const int64_t b0 = (nblk * blockIdx.x) / gridDim.x;
  const int64_t b1 = (nblk * (blockIdx.x + 1)) / gridDim.x;
  const int nrb = int(b1 - b0);
  const int64_t r_begin = b0 * 16;
  const int64_t r_end = (int64_t(p.N) < b1 * 16) ? int64_t(p.N) : b1 * 16;
  const int nrows = int(r_end - r_begin);
  const int G = p.K / kGroup;

  // Outlier weights of this CTA's rows: the 16-byte-aligned middle by one bulk
  // copy, the ragged tail (< 16 B) by plain loads, both before the wait.
  const int ow_es = p.ow_dtype == SPECTRA_DT_F32 ? 4 : 2;
  const bool ow_staged = kp.off_ow >= 0 && p.n_out > 0;
  const int64_t ow_b0 = r_begin * p.n_out * ow_es;
  const int64_t ow_b1 = r_end * p.n_out * ow_es;
  const int64_t ow_a0 = ow_b0 & ~int64_t(15);
  const int64_t ow_a1 = ow_b1 & ~int64_t(15);

  if (tid == 0) {
    s_abort = 0;
    s_zero = 0;
    for (int s = 0; s < kp.ns; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kPfGroupWarps);  // a stage is consumed by one group
    }
    // Staged outlier weights: the bulk copy's arrival + the tail writer's;
    // streamed through the ring: one arrival per piece.
    mbar_init(&ow_bar, ow_staged ? 2 : 1);
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kPfComputeWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint64_t policy;  // streamed once: first out of L2
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
      const int G = p.K / kGroup;
      const uint32_t code_row = uint32_t(p.K / 2), sc_row = uint32_t(G * 2), z_row = uint32_t(G);
      if (ow_staged) {
        const uint8_t* ow_src = reinterpret_cast<const uint8_t*>(p.ow);
        mbar_arrive_expect_tx(&ow_bar, uint32_t(ow_a1 - ow_a0));
        if (ow_a1 > ow_a0) bulk_g2s_hint(smem + kp.off_ow, ow_src + ow_a0, uint32_t(ow_a1 - ow_a0), &ow_bar, policy);
        for (int64_t bt = ow_a1; bt < ow_b1; ++bt) smem[kp.off_ow + (bt - ow_a0)] = ow_src[bt];
        mbar_arrive(&ow_bar);
      }
      int s = 0;
      uint32_t ph = 0;
      int issued = 0;
      bool ok = true;
      const uint32_t tma_tx = 16u * uint32_t(kp.cs + kp.ss + kp.zs);  // full boxes (OOB rows and columns: zeros)
      const int nkc = CHUNKED ? kp.nkc : 1;
      for (int rb = 0; rb < nrb && ok; ++rb) {
        const int64_t row0 = r_begin + int64_t(rb) * 16;
        const uint32_t rv = uint32_t(r_end - row0 < 16 ? r_end - row0 : 16);
        for (int ch = 0; ch < nkc; ++ch) {
          if (issued >= kp.ns && !mbar_wait(&empty_bar[s], ph ^ 1u, &s_abort)) {
            s_abort = 1;
            atomicAdd(&g_gemv_pf_timeouts, 1);
            ok = false;
            break;
          }
          uint8_t* st = smem + kp.off_stage + s * kp.stage_bytes;
          if constexpr (CHUNKED) {
            mbar_arrive_expect_tx(&full_bar[s], tma_tx);
            tma_load_2d_hint(st, &maps.c, ch * (kp.kc / 16), int(row0), &full_bar[s], policy);
            tma_load_2d_hint(st + kp.off_sc, &maps.s, ch * (kp.kc / 32), int(row0), &full_bar[s], policy);
            tma_load_2d_hint(st + kp.off_z, &maps.z, ch * (kp.kc / 32), int(row0), &full_bar[s], policy);
          } else {
            mbar_arrive_expect_tx(&full_bar[s], rv * (code_row + sc_row + z_row));
            bulk_g2s_hint(st, p.packed + row0 * code_row, rv * code_row, &full_bar[s], policy);
            bulk_g2s_hint(st + kp.off_sc, reinterpret_cast<const uint8_t*>(p.scales) + row0 * sc_row, rv * sc_row,
                          &full_bar[s], policy);
            bulk_g2s_hint(st + kp.off_z, p.zeros + row0 * z_row, rv * z_row, &full_bar[s], policy);
          }
          ++issued;
          if (++s == kp.ns) { s = 0; ph ^= 1u; }
        }
      }
      // Leave no copy in flight: wait (bounded) for the last stages issued.
      const int tail = issued < kp.ns ? issued : kp.ns;
      for (int i = 0; i < tail; ++i) {
        if (s == 0) { s = kp.ns; ph ^= 1u; }
        --s;
        (void)mbar_wait(&full_bar[s], ph, &s_zero);
      }
      if (ow_staged) (void)mbar_wait(&ow_bar, 0, &s_zero);
    }
    return;
  }

  // -------------------------------------------------------------- compute
  uint32_t* xp = reinterpret_cast<uint32_t*>(smem + kp.off_x);  // [G][kXpWords] x pairs, MMA order
  float* xsum = reinterpret_cast<float*>(smem + kp.off_xsum);   // [G]
  float* xos = reinterpret_cast<float*>(smem + kp.off_xos);     // [n_out]
  float* red = reinterpret_cast<float*>(smem + kp.off_red);     // [rows_max][8]
  constexpr int kCT = kPfComputeWarps * 32;

  constexpr int kOutPerThread = 2;
  int64_t oidx[kOutPerThread];
#pragma unroll
  for (int m = 0; m < kOutPerThread; ++m) {
    const int j = tid + m * kCT;
    oidx[m] = (j < p.n_out) ? load_index(p.idx, j, p.idx_dtype) : -1;
  }

  pdl_wait();  // x (and y) may belong to the previous kernel

  // Stage x: 16 pairs per group in the MMA's k order (bit-exact copies of x)
  // and the per-group sums X_g.  x is read through L2 only (ld.global.cg):
  // it may have been written by the kernel this one waited for.
  // x at the outlier features: loaded now, stored to shared memory only
  // before the final pass, so their latency overlaps everything below (a
  // gather after the x staging measured 1.5 % slower on a 1B decoder layer).
  uint32_t xo_raw[kOutPerThread];
#pragma unroll
  for (int m = 0; m < kOutPerThread; ++m)
    xo_raw[m] = (oidx[m] >= 0 && oidx[m] < p.K) ? load_bits_cg(p.x, oidx[m] * p.x_stride, p.x_dtype) : 0u;
  const bool marlin = p.layout == SPECTRA_LAYOUT_MARLIN;
  if (kp.vec_x) {
    // Thread t stages 8 consecutive features (one 16-byte load): quarter
    // q = t & 3 of a group, 4 pairs.  Marlin pairs (k, k+2), even-odd (k, k+4).
    const int q = tid & 3;
    const int sbase = marlin ? 8 * (q & 1) + (q >> 1) : 4 * q;
    const int sstep = marlin ? 2 : 1;
    const int nchunk = p.K / 8;  // a multiple of 64: every warp's 32 chunks are all valid or all not
    const uint4* xv = reinterpret_cast<const uint4*>(p.x);
    constexpr int kB = 4;
    for (int c0 = tid; c0 < nchunk; c0 += kB * kCT) {
      uint4 raw[kB];
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        const int c = c0 + b * kCT;
        raw[b] = c < nchunk ? __ldcg(xv + c) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        const int c = c0 + b * kCT;
        if (c >= nchunk) break;  // warp-uniform: the shuffles below see the whole warp
        const uint32_t w0 = raw[b].x, w1 = raw[b].y, w2 = raw[b].z, w3 = raw[b].w;
        uint32_t pr[4];
        if (marlin) {
          pr[0] = prmt(w0, w1, 0x5410u); pr[1] = prmt(w0, w1, 0x7632u);
          pr[2] = prmt(w2, w3, 0x5410u); pr[3] = prmt(w2, w3, 0x7632u);
        } else {
          pr[0] = prmt(w0, w2, 0x5410u); pr[1] = prmt(w0, w2, 0x7632u);
          pr[2] = prmt(w1, w3, 0x5410u); pr[3] = prmt(w1, w3, 0x7632u);
        }
        float t = 0.f;
        const uint32_t wv[4] = {w0, w1, w2, w3};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if constexpr (BF16) {
            t += __uint_as_float(wv[i] << 16) + __uint_as_float(wv[i] & 0xFFFF0000u);
          } else {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv[i]));
            t += f.x + f.y;
          }
        }
        const int gl = c >> 2;
#pragma unroll
        for (int i = 0; i < 4; ++i) xp[gl * kXpWords + sbase + i * sstep] = pr[i];
        t += __shfl_xor_sync(0xffffffffu, t, 1);
        t += __shfl_xor_sync(0xffffffffu, t, 2);
        if (q == 0) xsum[gl] = t;
      }
    }
  } else {
    // Strided x: one pair per lane, 16 lanes per group.
    const int nstage = G * 16;
    const unsigned short* xh = reinterpret_cast<const unsigned short*>(p.x);
    // nstage = 16 G = K / 2, a multiple of 256: the trip count is uniform
    // within each warp (the shuffles below), not always across the CTA.
    for (int e = tid; e < nstage; e += kCT) {
      const int gl = e >> 4, kk = e & 15;
      const int64_t kb = int64_t(gl) * kGroup;
      const uint32_t lo = __ldcg(xh + (kb + pair_k(kk, 0, p.layout)) * p.x_stride);
      const uint32_t hi = __ldcg(xh + (kb + pair_k(kk, 1, p.layout)) * p.x_stride);
      xp[gl * kXpWords + kk] = lo | (hi << 16);
      float t = BF16 ? (__uint_as_float(lo << 16) + __uint_as_float(hi << 16))
                     : (__half2float(__ushort_as_half(uint16_t(lo))) + __half2float(__ushort_as_half(uint16_t(hi))));
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if ((lane & 15) == 0) xsum[gl] = t;
    }
  }
  compute_bar<kCT>();

  // ------------------------------------------------------------ main loop
  uint32_t magic_reg;
  asm volatile("mov.b32 %0, %1;" : "=r"(magic_reg) : "n"(BF16 ? 0x41804180u : 0x4C004C00u));  // 16.0 x2
  const int g = lane >> 2, c = lane & 3;
  // Block-diagonal B: only lanes (g = 2c) and (g = 2c + 1) hold x (columns 2c
  // and 2c + 1 of the unit); the loads of the other lanes are predicated off.
  const bool lane_a = (lane % 9) == 0;  // lanes 0, 9, 18, 27
  const bool lane_b = (lane % 9) == 4;  // lanes 4, 13, 22, 31
  uint32_t bA[16] = {}, bB[16] = {};
  int cached_kb = -1;
  const int KB = p.K >> 8;                               // 256-feature units per row
  const int kc = CHUNKED ? kp.kc : p.K;                 // features per stage
  const int KBc = kc >> 8;                               // 256-feature units per stage
  const int cs = kp.cs, ss = kp.ss, zs = kp.zs;          // stage row pitches (bytes)
  const int nkc = CHUNKED ? kp.nkc : 1;
  const int grp = NG == 1 ? 0 : warp / kPfGroupWarps;  // compute group, and warp inside it
  const int w8 = NG == 1 ? warp : warp % kPfGroupWarps;
  constexpr int RW = kPfComputeWarps;  // partials per row: one per compute warp
  // Stages are consumed in issue order: stage si (row block si / nkc, chunk
  // si % nkc) by group si % NG.  ns is even when NG == 2, so a group's previous
  // use of a ring slot (stage si - ns) was its own and was waited for: the
  // parity wait cannot complete on an older phase of the slot.
  int s = 0;  // ring slot of stage si
  uint32_t ph = 0;
  int si = 0;
  for (int rb = 0; rb < nrb; ++rb) {
    float acc0 = 0.f, acc1 = 0.f;
    for (int ch = 0; ch < nkc; ++ch, ++si) {
    if (NG > 1 && si % NG != grp) {
      if (++s == kp.ns) { s = 0; ph ^= 1u; }
      continue;
    }
    bool ready = mbar_wait(&full_bar[s], ph, &s_abort);
    ready = __all_sync(0xffffffffu, ready);
    if (!ready) {
      if (lane == 0) { s_abort = 1; atomicAdd(&g_gemv_pf_timeouts, 1); }
    } else {
      const uint8_t* st = smem + kp.off_stage + s * kp.stage_bytes;
      const int kb0 = ch * KBc;                         // first unit of this stage along K
      const int kbn = KB - kb0 < KBc ? KB - kb0 : KBc;  // units in this stage
      for (int kl = w8; kl < kbn; kl += kPfGroupWarps) {
        const int kb = kb0 + kl;
        const int gl = kl * 8 + 2 * c;  // this lane's first group inside the stage
        const int gg = kb * 8 + 2 * c;  // ... inside the row
        if (kb != cached_kb) {          // warp-uniform
          cached_kb = kb;
          const uint4* srcA = reinterpret_cast<const uint4*>(xp + gg * kXpWords);
          const uint4* srcB = reinterpret_cast<const uint4*>(xp + (gg + 1) * kXpWords);
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            lds128_keep(bA[4 * qq], bA[4 * qq + 1], bA[4 * qq + 2], bA[4 * qq + 3], srcA + qq, lane_a);
            lds128_keep(bB[4 * qq], bB[4 * qq + 1], bB[4 * qq + 2], bB[4 * qq + 3], srcB + qq, lane_b);
          }
        }
        const uint8_t* c0p = st + g * cs + gl * kGroupBytes;
        const uint8_t* c1p = c0p + 8 * cs;
        const uint4 w0 = *reinterpret_cast<const uint4*>(c0p);
        const uint4 w1 = *reinterpret_cast<const uint4*>(c1p);
        const uint4 w2 = *reinterpret_cast<const uint4*>(c0p + kGroupBytes);
        const uint4 w3 = *reinterpret_cast<const uint4*>(c1p + kGroupBytes);
        const uint8_t* sp = st + kp.off_sc + g * ss + gl * 2;
        const uint32_t sc0 = *reinterpret_cast<const uint32_t*>(sp);
        const uint32_t sc1 = *reinterpret_cast<const uint32_t*>(sp + 8 * ss);
        const uint8_t* zp = st + kp.off_z + g * zs + gl;
        const uint32_t zr0 = *reinterpret_cast<const uint16_t*>(zp);
        const uint32_t zr1 = *reinterpret_cast<const uint16_t*>(zp + 8 * zs);
        const uint32_t wa[4][4] = {{w0.x, w0.y, w0.z, w0.w},
                                   {w1.x, w1.y, w1.z, w1.w},
                                   {w2.x, w2.y, w2.z, w2.w},
                                   {w3.x, w3.y, w3.z, w3.w}};
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        float e[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#define SPECTRA_PF_MMA(ACC, T)                                                                                  \
  mma16816<BF16>(ACC, pair_code<BF16, T>(wa[0][j], magic_reg), pair_code<BF16, T>(wa[1][j], magic_reg),           \
                 pair_code<BF16, T>(wa[2][j], magic_reg), pair_code<BF16, T>(wa[3][j], magic_reg),                \
                 bA[4 * j + T], bB[4 * j + T]);
          SPECTRA_PF_MMA(d, 0) SPECTRA_PF_MMA(e, 1) SPECTRA_PF_MMA(d, 2) SPECTRA_PF_MMA(e, 3)
#undef SPECTRA_PF_MMA
        }
        // d + e = {D[g][gA], D[g][gA+1], D[g+8][gA], D[g+8][gA+1]}
        const float XA = xsum[gg], XB = xsum[gg + 1];
        const uint32_t scs[2] = {sc0, sc1};
        const uint32_t zrs[2] = {zr0, zr1};
        float rs[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float sa = __half2float(__ushort_as_half(uint16_t(scs[h] & 0xFFFFu)));
          const float sb = __half2float(__ushort_as_half(uint16_t(scs[h] >> 16)));
          // 2^23 + z (the zero-point byte under the exponent of 2^23) - (2^23 - 16) = 16 + z, exact
          const float za = __uint_as_float(prmt(zrs[h], kMagic, 0x7540u)) - 8388592.0f;
          const float zb = __uint_as_float(prmt(zrs[h], kMagic, 0x7541u)) - 8388592.0f;
          rs[h] = sa * fmaf(-za, XA, d[2 * h] + e[2 * h]) + sb * fmaf(-zb, XB, d[2 * h + 1] + e[2 * h + 1]);
        }
        acc0 += rs[0];
        acc1 += rs[1];
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);
    if (++s == kp.ns) { s = 0; ph ^= 1u; }
    }  // stages of the row block
    // rows g, g+8 of this row block: sum the 4 lanes of a quad
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    if (c == 0) {
      red[(rb * 16 + g) * RW + warp] = acc0;  // zero for a row block of the other group
      red[(rb * 16 + g + 8) * RW + warp] = acc1;
    }
  }

  // --------------------------------------- outlier columns, bias, one store
  // Eight threads per row: the outlier dot product split over them, then the
  // 8 warp partials in warp order.
#pragma unroll
  for (int m = 0; m < kOutPerThread; ++m) {
    const int j = tid + m * kCT;
    if (j < p.n_out) xos[j] = bits_to_float(xo_raw[m], p.x_dtype);
  }
  for (int j = tid + kOutPerThread * kCT; j < p.n_out; j += kCT) {
    const int64_t k = load_index(p.idx, j, p.idx_dtype);
    xos[j] = (k >= 0 && k < p.K) ? load_as_float_cg(p.x, k * p.x_stride, p.x_dtype) : 0.f;
  }
  bool ow_ok = true;
  if (ow_staged) {
    ow_ok = mbar_wait(&ow_bar, 0, &s_abort);
    ow_ok = __all_sync(0xffffffffu, ow_ok);
    if (!ow_ok && lane == 0) { s_abort = 1; atomicAdd(&g_gemv_pf_timeouts, 1); }
  }
  compute_bar<kCT>();
  constexpr int tpr = 8;
  const int sub = tid & (tpr - 1);
  // Outlier weights too large to stage beside the ring stream through the
  // ring itself once every stage is consumed (all its copies have landed:
  // each was waited for), `ow_ring_rows` rows per piece by one bulk copy of
  // the 16-byte-aligned middle plus plain loads of the ragged end.
  const int64_t row_bytes = int64_t(p.n_out) * ow_es;
  // Rows [pr0, pr1) of the CTA: outlier dot products (staged rows: row i at
  // ow_rows + (i - ow_row0) * row_bytes), the partials in order, bias, store.
  auto final_rows = [&](int pr0, int pr1, bool ow_in_smem, const uint8_t* ow_rows, int ow_row0, bool ow_ok) {
    for (int i0 = pr0; i0 < pr1; i0 += kCT / tpr) {  // CTA-uniform trips
      const int i = i0 + tid / tpr;
      float v = 0.f;
      if (i < pr1 && p.n_out > 0 && ow_ok) {
        if (ow_in_smem) {
          const uint8_t* orow = ow_rows + int64_t(i - ow_row0) * row_bytes;
          if (ow_es == 4) {
            for (int j = sub; j < p.n_out; j += tpr) v = fmaf(xos[j], reinterpret_cast<const float*>(orow)[j], v);
          } else if (p.ow_dtype == SPECTRA_DT_BF16) {
            for (int j = sub; j < p.n_out; j += tpr)
              v = fmaf(xos[j], __uint_as_float(uint32_t(reinterpret_cast<const uint16_t*>(orow)[j]) << 16), v);
          } else {
            for (int j = sub; j < p.n_out; j += tpr)
              v = fmaf(xos[j], __half2float(reinterpret_cast<const __half*>(orow)[j]), v);
          }
        } else {
          for (int j = sub; j < p.n_out; j += tpr)
            v = fmaf(xos[j], load_as_float(p.ow, (r_begin + i) * p.ow_rs + int64_t(j) * p.ow_cs, p.ow_dtype), v);
        }
      }
#pragma unroll
      for (int o = tpr >> 1; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (sub == 0 && i < pr1) {
        const float4* rr = reinterpret_cast<const float4*>(red + i * RW);
        float y = rr[0].x;
        y += rr[0].y; y += rr[0].z; y += rr[0].w;
#pragma unroll
        for (int q = 1; q < RW / 4; ++q) { y += rr[q].x; y += rr[q].y; y += rr[q].z; y += rr[q].w; }
        y += v;
        const int64_t row = r_begin + i;
        if (p.bias) y += load_as_float_cg(p.bias, row, p.bias_dtype);
        store_from_float(p.y, row * p.y_stride, p.y_dtype, y);
      }
    }
  };
  const uint8_t* ow_staged_rows = smem + (kp.off_ow >= 0 ? kp.off_ow : 0) + (ow_b0 - ow_a0);
  if constexpr (NG == 1) {
    final_rows(0, nrows, ow_staged, ow_staged_rows, 0, ow_ok);
  } else if (!(kp.ow_ring_rows > 0 && p.n_out > 0)) {
    final_rows(0, nrows, ow_staged, ow_staged_rows, 0, ow_ok);
  } else {
    // Two groups, outlier rows too large to stage: they stream through the
    // ring once every stage is consumed (all its copies have landed: each was
    // waited for), ow_ring_rows rows per piece by one bulk copy of the
    // 16-byte-aligned middle plus plain loads of the ragged end.
    const uint8_t* ow_src = reinterpret_cast<const uint8_t*>(p.ow);
    uint8_t* ring = smem + kp.off_stage;
    uint32_t ow_phase = 0;
    for (int pr0 = 0; pr0 < nrows; pr0 += kp.ow_ring_rows) {  // CTA-uniform
      const int pr1 = nrows - pr0 < kp.ow_ring_rows ? nrows : pr0 + kp.ow_ring_rows;
      const int64_t pb0 = (r_begin + pr0) * row_bytes, pb1 = (r_begin + pr1) * row_bytes;
      const int64_t pa0 = pb0 & ~int64_t(15);
      const int64_t pa1 = (pb1 & ~int64_t(15)) > pa0 ? (pb1 & ~int64_t(15)) : pa0;
      if (tid == 0) {
        fence_proxy_async_smem();  // the ring's last reads were generic loads
        mbar_arrive_expect_tx(&ow_bar, uint32_t(pa1 - pa0));
        if (pa1 > pa0) bulk_g2s(ring, ow_src + pa0, uint32_t(pa1 - pa0), &ow_bar);
      }
      for (int64_t bt = pa1 + tid; bt < pb1; bt += kCT) ring[bt - pa0] = ow_src[bt];  // < 16 bytes
      bool ok = mbar_wait_inl(&ow_bar, ow_phase, &s_abort);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok && lane == 0) { s_abort = 1; atomicAdd(&g_gemv_pf_timeouts, 1); }
      ow_phase ^= 1u;
      compute_bar<kCT>();  // the plain tail stores
      final_rows(pr0, pr1, true, ring + (pb0 - pa0), pr0, ow_ok && ok);
      if (pr1 < nrows) compute_bar<kCT>();  // the next piece overwrites the ring
    }
  }
}

// Self-test of the bounded wait: one thread waits on an mbarrier phase that
// never completes (nothing arrives on it), with the production limit of
// sm100::kWaitLimitNs.  The wait gives up, the timeout is counted exactly as
// the pipeline kernels count theirs, and the kernel returns; no copy is in
// flight at any point.
__global__ void selftest_wait_kernel() {
  using namespace sm100;
  __shared__ __align__(8) uint64_t bar;
  __shared__ int s_abort;
  if (threadIdx.x == 0) {
    s_abort = 0;
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait(&bar, 0u, &s_abort)) atomicAdd(&g_gemv_pf_timeouts, 1);
}

inline size_t r16(size_t v) { return (v + 15) & ~size_t(15); }
inline size_t r128(size_t v) { return (v + 127) & ~size_t(127); }
inline bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

template <bool BF16, int NG, bool CHUNKED>
int launch_pf(const PfMaps<true>& all_maps, const PfParams& kp, int64_t grid, size_t smem, int dev, cudaStream_t st) {
  auto kern = gemv_pf_kernel<BF16, NG, CHUNKED>;
  static PerContextOnce attrs;
  cudaError_t e = attrs.run(dev, [&] {
    cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kPfSmemSolo));
    if (r == cudaSuccess)
      r = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
    return r;
  });
  if (e != cudaSuccess) return cuda_status(e);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3((NG * kPfGroupWarps + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PfMaps<CHUNKED> maps;
  if constexpr (CHUNKED) maps = all_maps;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, maps, kp));
}

// Tensor maps of the three weight tensors for [16 rows x kc features] boxes:
// codes as 32-bit words, scales as 16-bit, zero points as bytes.
bool encode_stage_maps(const GemvArgs& a, const PfParams& kp, PfMaps<true>& maps) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const int G = a.K / kGroup;
  cuuint32_t es[2] = {1, 1};
  // codes as 64-bit elements: a box row of cs bytes (the chunk's kc/2 plus the pad)
  cuuint64_t dc[2] = {cuuint64_t(a.K / 16), cuuint64_t(a.N)}, sc[1] = {cuuint64_t(a.w_rs)};
  cuuint32_t bc[2] = {cuuint32_t(kp.cs / 8), 16};
  cuuint64_t dg[2] = {cuuint64_t(G), cuuint64_t(a.N)};
  cuuint64_t ss[1] = {cuuint64_t(a.s_rs) * 2}, zs[1] = {cuuint64_t(a.z_rs)};
  cuuint32_t bs[2] = {cuuint32_t(kp.ss / 2), 16}, bz[2] = {cuuint32_t(kp.zs), 16};
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

}  // namespace

// Kernel configuration of one call (with the PfParams it fills).
struct PfPlan {
  int ng = 0;            // compute groups
  bool chunked = false;  // [16 x 2048] tensor-map stages (else whole row blocks)
  int64_t grid = 0;
  size_t smem = 0;       // dynamic shared memory bytes
};

// The configuration for `a` on a GPU with `sms` SMs, decided on the host
// without any CUDA call (the caller encodes a chunked plan's tensor maps).
// False: the prefetching kernel does not take this call.
bool plan_gemv_pf(const GemvArgs& a, int sms, PfParams& kp, PfPlan& pl) {
  if (a.x_dtype != SPECTRA_DT_BF16 && a.x_dtype != SPECTRA_DT_F16) return false;
  if (a.K % kPfKQuantum != 0 || a.N <= 0 || sms <= 0) return false;
  const int G = a.K / kGroup;
  if (!al16(a.packed) || !al16(a.scales) || !al16(a.zeros) || a.s_cs != 1 || a.z_cs != 1) return false;
  // Contiguous weights: a stage is a whole row block, three contiguous bulk
  // copies, when two such stages fit.  Otherwise stages of [16 rows x 2048
  // features] by tensor maps (row pitches must be multiples of 16 bytes).
  const bool contiguous = a.w_rs == a.K / 2 && a.s_rs == G && a.z_rs == G;
  const bool pitches16 = a.w_rs % 16 == 0 && (a.s_rs * 2) % 16 == 0 && a.z_rs % 16 == 0;

  kp = PfParams{};
  kp.a = a;
  const int64_t nblk = (int64_t(a.N) + 15) / 16;
  const int64_t grid = std::min<int64_t>(nblk, sms);
  const int64_t rb_max = (nblk + grid - 1) / grid;
  kp.rows_max = int(rb_max * 16);
  kp.vec_x = (a.x_stride == 1 && al16(a.x)) ? 1 : 0;
  size_t off = 0;
  kp.off_x = 0;
  off = r16(size_t(G) * kXpWords * 4);
  kp.off_xsum = int(off);
  off = r16(off + size_t(G) * 4);
  kp.off_xos = int(off);
  off = r16(off + size_t(a.n_out) * 4);
  kp.off_red = int(off);

  const int ow_es = a.ow_dtype == SPECTRA_DT_F32 ? 4 : 2;
  const bool ow_contig = a.n_out > 0 && a.ow_cs == 1 && a.ow_rs == a.n_out && al16(a.ow);
  // CTAs that own several row blocks run alone on their SM: sharing it with
  // the next launch's prefetching CTA slowed a decoder layer by ~12 % (the
  // co-resident copies delay this kernel's post-wait loads); CTAs with one
  // row block finish quickly and keep the two-per-SM footprint -- unless that
  // footprint cannot hold two stages (K = 28672: the staged x alone is 72 KB),
  // then they own their SM too.
  auto try_plan = [&](bool solo) -> bool {
  const size_t budget = solo ? kPfSmemSolo : kPfSmemPair;
  // Whole-row-block stages unless a CTA owns >= 5 row blocks and the ring
  // holds fewer than kPfMinWholeStages of them: then the chunked mode's small
  // stages keep more copies in flight and feed two compute groups (8192 x
  // 28672: 48.8 -> 40.6 us; with 4 row blocks, 8192 x 8192, whole stages
  // stayed 3 % faster).
  bool prefer_chunked = false;
  if (contiguous && pitches16 && rb_max >= 5) {
    const size_t sb_whole = r128(16 * (size_t(a.K) / 2 + size_t(a.K) / 16 + size_t(a.K) / 32));
    const size_t base = r16(off + size_t(kp.rows_max) * kPfGroupWarps * 4);
    const int64_t ns_whole = base < budget ? int64_t((budget - base) / sb_whole) : 0;
    prefer_chunked = ns_whole < std::min<int64_t>(rb_max, kPfMinWholeStages);
  }
  for (int chunked = (contiguous && !prefer_chunked) ? 0 : 1; chunked <= 1; ++chunked) {
    if (chunked && !pitches16) break;
    kp.kc = chunked ? std::min(a.K, kPfChunk) : a.K;
    kp.nkc = (a.K + kp.kc - 1) / kp.kc;
    // Chunked stages are tensor-map boxes 16 bytes wider than the chunk's data
    // (the extra bytes are never read): row pitches kc/2 + 16, kc/16 + 16 and
    // kc/32 + 16 put the 16 rows of a stage in different shared-memory bank
    // groups, so the lanes of a warp, which read 8 rows at one column, do not
    // conflict (with power-of-two pitches scales conflicted 8-way, zero points
    // 4-way, codes 2-way).  Whole-row-block stages keep the tensors' own pitches.
    const int pad = chunked ? 16 : 0;
    kp.cs = kp.kc / 2 + pad;
    kp.ss = kp.kc / 16 + pad;
    kp.zs = kp.kc / 32 + pad;
    kp.off_sc = 16 * kp.cs;                          // codes [16][cs B]
    kp.off_z = kp.off_sc + 16 * kp.ss;               // scales [16][ss B]
    const size_t sb = r128(size_t(kp.off_z) + 16 * size_t(kp.zs));  // zero points [16][zs B]
    kp.stage_bytes = int(sb);
    const int64_t units = rb_max * kp.nkc;
    // Two compute groups (16 warps) on alternate stages when the CTA owns its
    // SM: a stage's consumption (one 256-feature unit per warp) is latency
    // bound at two warps per scheduler, and a ring of 19-39 KB stages is
    // drained only as fast as it is consumed.  Contiguous stages (a whole row
    // block each) keep one group below 5 row blocks: two were slower on a 1B
    // decoder layer, where the CTA's SM is soon wanted by the next launch.
    const int ng_pref = chunked ? (solo ? 2 : 1) : (rb_max >= 5 ? 2 : 1);
    for (int ng = ng_pref; ng >= 1; --ng) {
      const size_t off_ow = r16(off + size_t(kp.rows_max) * kPfGroupWarps * ng * 4);  // red: [rows][8 ng]
      // Ring depth with the outlier rows staged beside the ring (o = its end)
      // or not (they then stream through the ring after the main loop, two
      // groups only): staging gives way when it leaves fewer than
      // kPfMinStagedRing stages and streaming would leave more.
      auto ring_depth = [&](size_t o) -> int64_t {
        const size_t st_off = r128(o);
        if (st_off >= budget) return 0;
        int64_t n = std::min<int64_t>({int64_t(kPfMaxStages), int64_t((budget - st_off) / sb), units});
        if (ng == 2) n &= ~int64_t(1);  // a ring slot's consecutive stages belong to one group
        return n;
      };
      const int64_t ns_unstaged = ring_depth(off_ow);
      for (int try_ow = ow_contig ? 1 : 0; try_ow >= 0; --try_ow) {
        size_t o = off_ow;
        kp.off_ow = -1;
        if (try_ow) {
          kp.off_ow = int(o);
          o = r16(o + size_t(kp.rows_max) * a.n_out * ow_es + 32);
        }
        kp.off_stage = int(r128(o));
        const int64_t ns = ring_depth(o);
        if (ns < std::min<int64_t>(2, units)) continue;  // no overlap of copies and compute: gemv.cu does better
        if (try_ow && ng == 2 && ns < std::min<int64_t>(kPfMinStagedRing, ns_unstaged)) continue;
        kp.ns = int(ns);
        kp.ow_ring_rows = 0;
        if (!try_ow && ow_contig && ng == 2) {  // stream the outlier rows through the ring at the end
          const int64_t row_bytes = int64_t(a.n_out) * ow_es, rpp = 32 * ng;
          const int64_t rows = (ns * int64_t(sb) - 16) / row_bytes;
          if (rows >= rpp) kp.ow_ring_rows = int(std::min<int64_t>(kp.rows_max, rows - rows % rpp));
        }
        pl.ng = ng;
        pl.chunked = chunked != 0;
        pl.grid = grid;
        pl.smem = size_t(kp.off_stage) + size_t(kp.ns) * sb;
        if (solo) pl.smem = std::max(pl.smem, kPfSoloFloor);
        return true;
      }
    }
  }
  return false;
  };
  return try_plan(rb_max > 1) || (rb_max == 1 && try_plan(true));
}

int gemv_pf_timeouts(long long* out, bool reset) { return read_timeout_counter(g_gemv_pf_timeouts, out, reset); }

int launch_selftest_wait(cudaStream_t st) {
  selftest_wait_kernel<<<1, 32, 0, st>>>();
  return cuda_status(cudaGetLastError());
}

int launch_gemv_pf(const GemvArgs& a, cudaStream_t st) {
  if (!pf_path_enabled()) return SPECTRA_ERR_UNSUPPORTED;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev >= kMaxDevices) return SPECTRA_ERR_UNSUPPORTED;
  PfParams kp{};
  PfPlan pl;
  if (!plan_gemv_pf(a, device_sms(dev), kp, pl)) return SPECTRA_ERR_UNSUPPORTED;
  PfMaps<true> maps;
  memset(&maps, 0, sizeof(maps));
  if (pl.chunked && !encode_stage_maps(a, kp, maps)) return SPECTRA_ERR_UNSUPPORTED;
  const bool bf = a.x_dtype == SPECTRA_DT_BF16;
  if (pl.chunked) {
    if (pl.ng == 2)
      return bf ? launch_pf<true, 2, true>(maps, kp, pl.grid, pl.smem, dev, st)
                : launch_pf<false, 2, true>(maps, kp, pl.grid, pl.smem, dev, st);
    return bf ? launch_pf<true, 1, true>(maps, kp, pl.grid, pl.smem, dev, st)
              : launch_pf<false, 1, true>(maps, kp, pl.grid, pl.smem, dev, st);
  }
  if (pl.ng == 2)
    return bf ? launch_pf<true, 2, false>(maps, kp, pl.grid, pl.smem, dev, st)
              : launch_pf<false, 2, false>(maps, kp, pl.grid, pl.smem, dev, st);
  return bf ? launch_pf<true, 1, false>(maps, kp, pl.grid, pl.smem, dev, st)
            : launch_pf<false, 1, false>(maps, kp, pl.grid, pl.smem, dev, st);
}

}  // namespace spectra

// Diagnostic (declared in include/spectra_b200.h): the plan above for
// contiguous, 16-byte-aligned weights, contiguous x and [N, n_out] outlier
// weights, without a GPU.
extern "C" SPECTRA_API int spectra_gemv_pf_plan(int64_t N, int64_t K, int64_t n_out, int x_dtype, int ow_dtype,
                                                int sms, int64_t* out) {
  if (!out) return SPECTRA_ERR_NULL_POINTER;
  if (N <= 0 || K <= 0 || K % 32 != 0 || n_out < 0 || n_out > K || N > 2147483647LL || K > 2147483647LL)
    return SPECTRA_ERR_SHAPE;
  // the dtype codes spectra_w4a16_gemv accepts (x: F16|BF16|F32; outlier weights: F16|BF16|F32)
  auto float_dt = [](int dt) { return dt == SPECTRA_DT_F16 || dt == SPECTRA_DT_BF16 || dt == SPECTRA_DT_F32; };
  if (!float_dt(x_dtype) || (n_out > 0 && !float_dt(ow_dtype))) return SPECTRA_ERR_DTYPE;
  spectra::GemvArgs a{};
  const uintptr_t aligned = 4096;  // stand-in 16-byte-aligned addresses (never dereferenced)
  a.x = reinterpret_cast<const void*>(aligned);
  a.x_dtype = x_dtype;
  a.x_stride = 1;
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
  a.N = int(N);
  a.K = int(K);
  a.layout = SPECTRA_LAYOUT_MARLIN;
  spectra::PfParams kp{};
  spectra::PfPlan pl;
  const bool taken = spectra::plan_gemv_pf(a, sms, kp, pl);
  for (int i = 0; i < 10; ++i) out[i] = 0;
  if (!taken) return SPECTRA_OK;
  out[0] = 1;
  out[1] = pl.ng;
  out[2] = pl.chunked ? 1 : 0;
  out[3] = kp.ns;
  out[4] = kp.stage_bytes;
  out[5] = kp.off_ow >= 0 ? 1 : 0;
  out[6] = kp.ow_ring_rows;
  out[7] = int64_t(pl.smem);
  out[8] = pl.grid;
  out[9] = kp.rows_max / 16;
  return SPECTRA_OK;
}
