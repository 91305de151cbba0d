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
// CTA = 14 warps: warp 0 streams weights, warp 10 streams activations, warp 1
// owns TMEM, warps 1 and 11..13 issue the MMAs (as many as the token tile
// needs), warps 2..9 dequantise and run the epilogue.
// Every copy engine here is limited by requests (row segments), not bytes, so
// each stream is fetched in the widest rows it has:
//   code ring  : packed codes [128 rows x 128 B = 256 k] per stage, one TMA
//                box, 128B-swizzled.
//   sz ring    : scales [128 rows x 64 groups = 128 B] and zero points
//                [128 rows x 64 B] per 2048 k, TMA boxes swizzled 128B / 64B
//                (when their strides allow a tensor map; else the dequant
//                warps read them from global memory one code stage ahead).
//   act ring   : activations [MT x 64 k, 128B-swizzled, K-major] per MMA step
//                by TMA.
//   dequant    : thread (row r = its TMEM lane, half h) turns one 32-code
//                group per 64-k step into 16 bf16x2 words of exact
//                (q - z) * s rounded to nearest even, tcgen05.st into one of
//                four A slots of TMEM.
//   MMA        : tcgen05.mma kind::f16, A from TMEM, B from shared memory,
//                D (fp32, 128 lanes x MT columns) in TMEM; tcgen05.commit
//                frees the act slot and the A slot.
// Outlier columns become extra 64-column steps: the dequant warps convert ow
// rows into the A slot; the activations a[:, idx] come from the tile that
// gather_outlier_acts_kernel gathered once per call (token tiles >= 32, by
// TMA like any step), or at 16 tokens the dequant warps gather them into the
// act slot themselves (same swizzled layout).  K is split across CTAs (in 256-k code stages) when there are too
// few weight tiles to fill the GPU; the last CTA of a tile sums the fp32
// partials in split order (deterministic) and resets the tile's counter for
// the next call.
// Optionally (SPECTRA_B200_GEMM_PAIR=1), token tiles of >= 128 run on SM pairs
// (a cluster of two CTAs, cta_group::2): each CTA still dequantises its own
// 128-row tile into its own TMEM but loads only half of the token tile, and
// the even CTA issues one M = 256 MMA per K=16 slice for both.  Per SM this
// halves the activation bytes fetched and the MMA instructions issued.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <type_traits>

#include "common.cuh"
#include "gemm.h"
#include "sm100_ptx.cuh"
#include "tmap.h"

// Split-K scratch of spectra_w4a16_gemm_noalloc, laid out like a caller
// workspace (tile counters, then fp32 partials).  Zero when the module loads;
// every GEMM leaves its counters zero again.
static __device__ __align__(256) unsigned char g_gemm_noalloc_scratch[SPECTRA_GEMM_NOALLOC_SCRATCH_BYTES];

namespace spectra {

namespace {

using namespace sm100;

constexpr int kRows = 128;                           // weight rows per tile (MMA M)
constexpr int kStep = 64;                            // k per MMA step (4 MMAs of K=16)
constexpr int kCodeK = 256;                          // k per code stage
constexpr int kStepsPerCode = kCodeK / kStep;        // 4
constexpr int kCodeBytes = kRows * kCodeK / 2;       // 16 KB of packed codes
constexpr int kSzGroups = 64;                        // groups per sz chunk (2048 k)
constexpr int kCodesPerSz = kSzGroups * kGroup / kCodeK;  // 8 code stages
constexpr int kSzScaleBytes = kRows * kSzGroups * 2; // 16 KB
constexpr int kSzZeroBytes = kRows * kSzGroups;      // 8 KB
constexpr int kSzSlot = kSzScaleBytes + kSzZeroBytes;
constexpr int kSzSlots = 2;
constexpr int kWarps = 14;       // 0 weights, 1 + 11..13 MMA issuers, 2..9 dequant, 10 activations
constexpr int kDeqWarps = 8;
constexpr int kActWarp = 10;
constexpr int kMaxIssuers = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxMT = 256;
constexpr int kDone = 8;                             // units tracked by the MMA-done barrier ring
constexpr int kMaxActStages = 16;
constexpr size_t kMaxDynSmem = 200 * 1024;
// Workspace layout: split-K tile counters in the first kCounterBytes (K is
// split only when a wave holds >= 2 CTAs per tile, i.e. <= 74 tiles), the
// fp32 partials after them, the gathered outlier activations after those.
// The counter region is the same for every call, so no call's other regions
// overwrite counters another call sharing the workspace relies on being zero.
constexpr size_t kCounterBytes = 1024;

__device__ int g_gemm_timeouts;  // stuck pipeline waits since load (diagnostic)

// Position in a ring of `size` slots: slot index and the parity of the pass
// (the mbarrier phase a consumer of that slot waits for).  Advanced by one per
// use instead of dividing a running counter by a runtime ring size, which
// costs a single-thread producer or MMA issuer tens of cycles per division.
struct Ring {
  int idx = 0;
  uint32_t phase = 0;
  int size;
  __device__ explicit Ring(int n) : size(n) {}
  __device__ void next() {
    if (++idx == size) {
      idx = 0;
      phase ^= 1u;
    }
  }
};

struct GemmKParams {
  const __half* scales; int64_t s_rs, s_cs;
  const uint8_t* zeros; int64_t z_rs, z_cs;
  const void* a; int64_t a_rs;
  const void* idx; int idx_dtype; int n_out;
  const void* ow; int ow_dtype; int64_t ow_rs, ow_cs;
  void* c; int c_dtype; int64_t c_rs;
  float* partials;  // [S][M][N] when S > 1
  int* counters;    // [tiles_n * m_chunks]
  int M, N, K, layout;
  int MT, S, nk, ncs, n_os, tiles_n, tiles_pad;
  int act_stages, code_stages, issuers, a_slots;
  uint32_t idesc, tmem_cols;
  int off_act, act_stage_bytes, off_code, off_sz, off_oidx, off_bar;
  int pregather;  // outlier steps' activations come from the gathered tile (map_g) by TMA
};

// a[:, idx] for every token, gathered once per call into the compact tile
// g[M][cols] (cols = 64 per outlier step; zero where an outlier column is
// padding or out of range), which the GEMM then loads by tensor map like any
// activation step.  Each CTA of the GEMM gathering it for itself would repeat
// the same scattered loads once per weight tile (~8 us at 256 tokens).
// Thread = 8 consecutive columns of one token: eight 2-byte loads, one
// 16-byte store.  The indices are constants of the weights (loaded before the
// dependency wait); a may be the previous kernel's output (loaded after it).
__global__ void gather_outlier_acts_kernel(const uint16_t* __restrict__ a, int64_t a_rs, const void* idx, int idx_dtype,
                                           int n_out, int K, int M, int cols, uint16_t* __restrict__ g) {
  pdl_trigger();  // the GEMM may start its weight prefetch now
  const int per_row = cols / 8;
  const int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= int64_t(M) * per_row) return;
  const int m = int(e / per_row), j0 = int(e % per_row) * 8;
  int k[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t kk = j0 + i < n_out ? load_index(idx, j0 + i, idx_dtype) : -1;
    k[i] = (kk >= 0 && kk < K) ? int(kk) : -1;
  }
  pdl_wait();
  uint32_t v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = k[i] >= 0 ? __ldg(a + int64_t(m) * a_rs + k[i]) : 0u;
  uint4 o;
  o.x = v[0] | (v[1] << 16);
  o.y = v[2] | (v[3] << 16);
  o.z = v[4] | (v[5] << 16);
  o.w = v[6] | (v[7] << 16);
  *reinterpret_cast<uint4*>(g + int64_t(m) * cols + j0) = o;
}

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

__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t m, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(m), "r"(c));  // (a & m) | c
  return r;
}

// Marlin group (byte j: k = j low nibble, k = j + 16 high nibble) -> 16 words
// of two 16-bit floats, done in packed 16-bit arithmetic.  Bytes j, j+1 are
// spread to the two halves of a word (PRMT); a low nibble then becomes the
// 16-bit float 128 + q (bf16) / 1024 + q (fp16) by one AND-OR, a high nibble
// (shifted) 16 + q / 1024 + q.  Subtracting the same offset plus z is exact.
//   fp16: (q - z) * s is one multiply, rounded once.
//   bf16: s (fp16, 11 significant bits) = s_hi + s_lo with s_hi = bf16(s) and
//         s_lo exact in bf16 (at most 3 significant bits); (q - z) * s_lo is
//         exact (at most 7 bits) and fma(q - z, s_hi, (q - z) * s_lo) rounds
//         the exact (q - z) * s once.
// Both give the same bits as rounding the exact fp32 (q - z) * s.
template <bool BF16>
__device__ __forceinline__ void dequant_marlin(const uint4 w, float s, float z, uint32_t (&out)[16]) {
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
  if constexpr (BF16) {
    const __nv_bfloat16 shi = __float2bfloat16_rn(s);
    const __nv_bfloat16 slo = __float2bfloat16_rn(s - __bfloat162float(shi));
    const __nv_bfloat162 S_hi = __bfloat162bfloat162(shi), S_lo = __bfloat162bfloat162(slo);
    const __nv_bfloat162 Z_lo = __bfloat162bfloat162(__float2bfloat16_rn(128.f + z));
    const __nv_bfloat162 Z_hi = __bfloat162bfloat162(__float2bfloat16_rn(16.f + z));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t A = __byte_perm(words[j], 0, 0x4140), B = __byte_perm(words[j], 0, 0x4342);
      const uint32_t p[4] = {and_or(A, 0x000F000Fu, 0x43004300u), and_or(B, 0x000F000Fu, 0x43004300u),
                             and_or(A >> 1, 0x00780078u, 0x41804180u), and_or(B >> 1, 0x00780078u, 0x41804180u)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 P = *reinterpret_cast<const __nv_bfloat162*>(&p[i]);
        const __nv_bfloat162 qz = __hsub2(P, i < 2 ? Z_lo : Z_hi);
        const __nv_bfloat162 r = __hfma2(qz, S_hi, __hmul2(qz, S_lo));
        out[(i < 2 ? 0 : 8) + 2 * j + (i & 1)] = *reinterpret_cast<const uint32_t*>(&r);
      }
    }
  } else {
    const __half2 S = __half2half2(__float2half_rn(s));
    const __half2 Z = __half2half2(__float2half_rn(1024.f + z));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t A = __byte_perm(words[j], 0, 0x4140), B = __byte_perm(words[j], 0, 0x4342);
      const uint32_t p[4] = {and_or(A, 0x000F000Fu, 0x64006400u), and_or(B, 0x000F000Fu, 0x64006400u),
                             and_or(A >> 4, 0x000F000Fu, 0x64006400u), and_or(B >> 4, 0x000F000Fu, 0x64006400u)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __half2 P = *reinterpret_cast<const __half2*>(&p[i]);
        const __half2 r = __hmul2(__hsub2(P, Z), S);
        out[(i < 2 ? 0 : 8) + 2 * j + (i & 1)] = *reinterpret_cast<const uint32_t*>(&r);
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

template <bool BF16, bool SZ_TMA, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_w4a16_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_s,
                         const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_a,
                         const __grid_constant__ CUtensorMap map_g,
                         const __grid_constant__ GemmKParams kp) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int AS = kp.act_stages, CS = kp.code_stages, NI = kp.issuers, NAS = kp.a_slots;
  uint8_t* act_st = smem + kp.off_act;     // [AS][MT x 128 B]
  uint8_t* code_st = smem + kp.off_code;   // [CS][128 x 128 B]
  uint8_t* sz_st = smem + kp.off_sz;       // [2][scales 128 x 128 B | zeros 128 x 64 B]
  int* oidx = reinterpret_cast<int*>(smem + kp.off_oidx);  // [n_os * 64] outlier columns (-1: none)
  uint64_t* cfull = reinterpret_cast<uint64_t*>(smem + kp.off_bar);  // [CS] code stage landed
  uint64_t* cfree = cfull + CS;                                       // [CS] code stage read (8 warps)
  uint64_t* szfull = cfree + CS;                                      // [2] sz chunk landed
  uint64_t* szfree = szfull + kSzSlots;                               // [2] sz chunk read (8 warps)
  uint64_t* afull = szfree + kSzSlots;                                // [AS] act slot landed / filled
  uint64_t* afree = afull + AS;                                       // [AS] act slot consumed by MMAs
  uint64_t* aready = afree + AS;                                      // [NAS] A slot written (8 warps)
  uint64_t* mdone = aready + NAS;                                     // [kDone] unit's MMAs complete (NI)
  uint64_t* accf = mdone + kDone;                                     // accumulators final (NI)
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tile = blockIdx.x % kp.tiles_pad;
  const int split = blockIdx.x / kp.tiles_pad;
  const int mchunk = blockIdx.y;
  const int n0 = tile * kRows;
  const int m0 = mchunk * kp.MT;
  // Pair mode: clusters of two CTAs (consecutive blockIdx.x: tiles 2i and
  // 2i+1 of the same split).  Each CTA dequantises its own 128 weight rows
  // into its own TMEM and loads half of the token tile (tokens m_own ..
  // m_own + mt_local - 1) into its own act ring; rank 0 issues one M = 256
  // MMA per K=16 slice for both and commits to the barriers of both.
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const bool issuer_cta = rank == 0;
  const int mt_local = PAIR ? kp.MT / 2 : kp.MT;
  const int m_own = m0 + int(rank) * mt_local;
  // This split's code stages [cs0, cs1) (balanced, never empty since S <= ncs)
  // and its main 64-k steps, then (last split only) the outlier steps.  The
  // unit of work between the dequant warps and the MMA issuers is one code
  // stage (up to 4 steps; fewer at the K tail), then units of up to 4 outlier
  // steps.
  const int cs0 = int(int64_t(split) * kp.ncs / kp.S);
  const int cs1 = int(int64_t(split + 1) * kp.ncs / kp.S);
  const int n_code = cs1 - cs0;
  const int st0 = cs0 * kStepsPerCode;
  const int n_main = min(kp.nk, cs1 * kStepsPerCode) - st0;
  // outlier steps dealt round-robin over the K splits (split s: steps s, s+S, ...)
  const int n_out_st = kp.n_os > split ? (kp.n_os - split + kp.S - 1) / kp.S : 0;
  auto ostep = [&](int local) { return split + kp.S * local; };  // global outlier step
  const int n_it = n_main + n_out_st;
  // Outlier units come first: their loads (outlier weights, gathered
  // activations) then overlap the arrival of the first code stages instead of
  // extending the end of the pipeline.  Units [0, n_ou) are outlier steps,
  // units [n_ou, n_units) the code stages.
  const int n_ou = (n_out_st + kStepsPerCode - 1) / kStepsPerCode;
  const int n_units = n_ou + n_code;
  auto steps_of = [&](int u) {
    return u < n_ou ? min(kStepsPerCode, n_out_st - u * kStepsPerCode)
                    : min(kStepsPerCode, n_main - (u - n_ou) * kStepsPerCode);
  };
  // steps in unit order: n_out_st outlier steps (last outlier unit may be
  // short), then the main steps
  auto step_of = [&](int u, int j) {
    return u < n_ou ? u * kStepsPerCode + j : n_out_st + (u - n_ou) * kStepsPerCode + j;
  };
  const uint32_t act_bytes = uint32_t(kp.act_stage_bytes);
  auto act_slot = [&](int u, int j) -> uint8_t* { return act_st + (step_of(u, j) % AS) * act_bytes; };
  // sz chunk (local index) of local code stage lc
  const int sz0 = cs0 / kCodesPerSz;
  auto sz_of = [&](int lc) { return (cs0 + lc) / kCodesPerSz - sz0; };

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < CS; ++i) {
      mbar_init(cfull + i, 1);
      mbar_init(cfree + i, kDeqWarps);
    }
    for (int i = 0; i < kSzSlots; ++i) {
      mbar_init(szfull + i, 1);
      mbar_init(szfree + i, kDeqWarps);
    }
    for (int i = 0; i < AS; ++i) {
      mbar_init(afull + i, 1);
      mbar_init(afree + i, NI);  // one commit per MMA issuer
    }
    // pair mode: the dequant warps of both CTAs arrive on rank 0's barrier
    for (int i = 0; i < NAS; ++i) mbar_init(aready + i, PAIR ? 2 * kDeqWarps : kDeqWarps);
    for (int i = 0; i < kDone; ++i) mbar_init(mdone + i, NI);  // one commit per MMA issuer
    mbar_init(accf, NI);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&map_w);
    if constexpr (SZ_TMA) {
      prefetch_tensormap(&map_s);
      prefetch_tensormap(&map_z);
    }
    prefetch_tensormap(&map_a);
    if (kp.pregather) prefetch_tensormap(&map_g);
  }
  __syncthreads();
  // the peer arrives on (and its copies complete on) this CTA's barriers:
  // both CTAs' barriers are initialised before either goes on
  if constexpr (PAIR) cluster_sync_all();

  // weight producer (warp 0, lane 0): code stage lc -> slot ring.idx, preceded
  // by its sz chunk when lc starts one.  Returns false if a wait gave up.
  Ring wring(CS);
  auto issue_weights = [&](int lc, bool may_wait) -> bool {
    if constexpr (SZ_TMA) {
      const int ch = sz_of(lc);
      if (lc == 0 || ch != sz_of(lc - 1)) {
        if (ch >= kSzSlots && !(may_wait && mbar_wait(szfree + ch % kSzSlots, uint32_t((ch / kSzSlots - 1) & 1), &s_abort)))
          return false;
        uint8_t* slot = sz_st + (ch % kSzSlots) * kSzSlot;
        uint64_t* bar = szfull + ch % kSzSlots;
        mbar_arrive_expect_tx(bar, uint32_t(kSzSlot));
        tma_load_2d(slot, &map_s, (sz0 + ch) * kSzGroups, n0, bar);
        tma_load_2d(slot + kSzScaleBytes, &map_z, (sz0 + ch) * kSzGroups, n0, bar);
      }
    }
    const int c = wring.idx;
    if (lc >= CS && !(may_wait && mbar_wait(cfree + c, wring.phase ^ 1u, &s_abort))) return false;
    mbar_arrive_expect_tx(cfull + c, uint32_t(kCodeBytes));
    tma_load_2d(code_st + c * kCodeBytes, &map_w, (cs0 + lc) * (kCodeK / 2), n0, cfull + c);
    wring.next();
    return true;
  };
  // The packed codes, scales and zero points are constant weights, never
  // written by a kernel this one depends on: their first stages are requested
  // before the dependency wait (the first CS code stages span at most two sz
  // chunks, so nothing here waits).
  const int pre = min(CS, n_code);
  if (warp == 0 && lane == 0)
    for (int lc = 0; lc < pre; ++lc) issue_weights(lc, false);
  pdl_wait();
  // TMEM is taken only after the wait, so a CTA waiting on the previous grid
  // never holds tensor memory that grid's CTAs could need.
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(&s_tmem, kp.tmem_cols);  // the same columns in both SMs
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&s_tmem, kp.tmem_cols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem = s_tmem;
  // TMEM columns: one fp32 accumulator [128 x MT] per MMA issuer, then NAS
  // (2 or 3) A slots of 128 columns (one unit = 4 steps x 32 columns each)
  const uint32_t a_col0 = uint32_t(NI * kp.MT);
  const bool bf16 = BF16;
  const int zero_flag = 0;
  auto done_parity = [](int u) { return uint32_t((u / kDone) & 1); };

  if (warp == 0) {
    // ---------------------------------------------------------------- weight producer
    if (lane == 0) {
      int issued = pre;
      for (int lc = pre; lc < n_code; ++lc) {
        if (!issue_weights(lc, true)) {
          s_abort = 1;
          atomicAdd(&g_gemm_timeouts, 1);
          break;
        }
        issued = lc + 1;
      }
      // every TMA copy issued must land before the CTA may exit (bounded wait,
      // ignoring the abort flag); on the normal path these completed long ago
      for (int lc = max(0, issued - CS); lc < issued; ++lc)
        mbar_wait(cfull + lc % CS, uint32_t((lc / CS) & 1), &zero_flag);  // once, at exit
      if constexpr (SZ_TMA) {
        if (issued > 0) {
          const int last = sz_of(issued - 1);
          for (int ch = max(0, last - kSzSlots + 1); ch <= last; ++ch)
            mbar_wait(szfull + ch % kSzSlots, uint32_t((ch / kSzSlots) & 1), &zero_flag);
        }
      }
    }
  } else if (warp == kActWarp) {
    // ---------------------------------------------------------------- activation producer
    // activations [MT x 64 k] per step by TMA; slots recycle per step (a unit
    // may have more steps than there are slots)
    if (lane == 0) {
      int issued = 0;
      Ring ar(AS);
      for (int st = 0; st < n_it; ++st, ar.next()) {
        const int sa = ar.idx;
        if (st >= AS && !mbar_wait(afree + sa, ar.phase ^ 1u, &s_abort)) {
          s_abort = 1;
          atomicAdd(&g_gemm_timeouts, 1);
          break;
        }
        if (st >= n_out_st || kp.pregather) {
          // a main step: activations at k; an outlier step with the gathered
          // tile: its 64 columns of that tile
          const bool main_step = st >= n_out_st;
          const CUtensorMap* map = main_step ? &map_a : &map_g;
          const int kx = main_step ? (st0 + st - n_out_st) * kStep : ostep(st) * kStep;
          if constexpr (PAIR) {
            // both halves complete on rank 0's barrier; rank 1's own barrier
            // is only stepped, so that its phases keep counting steps (its
            // dequant warps wait on it for the outlier steps)
            if (issuer_cta)
              mbar_arrive_expect_tx(afull + sa, 2u * act_bytes);
            else
              mbar_arrive(afull + sa);
            tma_load_2d_pair(act_st + sa * act_bytes, map, kx, m_own, cluster_addr(afull + sa, 0));
          } else {
            mbar_arrive_expect_tx(afull + sa, act_bytes);
            tma_load_2d(act_st + sa * act_bytes, map, kx, m0, afull + sa);
          }
        } else {
          mbar_arrive(afull + sa);  // outlier step: the dequant warps gather into the slot
        }
        issued = st + 1;
      }
      for (int st = max(0, issued - AS); st < issued; ++st)
        mbar_wait(afull + st % AS, uint32_t((st / AS) & 1), &zero_flag);  // once, at exit
    }
  } else if (warp == 1 || warp > kActWarp) {
    // ---------------------------------------------------------------- MMA issue
    // One elected thread can start a tcgen05.mma only every ~50 cycles and
    // each commit / wait costs tens of cycles more, so the MMAs of a whole
    // unit (16) are issued between one wait and one commit, and for small MT
    // they are spread over several warps, each accumulating its own K-slice
    // (k16 = issuer, issuer + NI, ...) into its own accumulator.
    const int issuer = warp == 1 ? 0 : warp - kActWarp;
    if (issuer < NI && lane == 0 && issuer_cta) {
      const uint32_t d_tmem = tmem + uint32_t(issuer * kp.MT);
      // pair mode: every completion is signalled to the same barrier in both CTAs
      auto commit = [&](uint64_t* bar) {
        if constexpr (PAIR) {
          mma_commit_pair(cluster_addr(bar, 0));
          mma_commit_pair(cluster_addr(bar, 1));
        } else {
          mma_commit(bar);
        }
      };
      auto mma = [&](uint32_t d, uint32_t a_t, uint64_t b, uint32_t acc) {
        if constexpr (PAIR)
          mma_ts_pair(d, a_t, b, kp.idesc, acc);
        else
          mma_ts(d, a_t, b, kp.idesc, acc);
      };
      bool live = true;
      Ring ar(AS), asl(NAS);
      for (int u = 0; u < n_units && live; ++u, asl.next()) {
        const int ns = steps_of(u);
        // (rank 1's dequant warps arrive on it from the other SM: cluster-scope acquire)
        const bool a_ok = PAIR ? mbar_wait_cluster(aready + asl.idx, asl.phase, &s_abort)
                               : mbar_wait(aready + asl.idx, asl.phase, &s_abort);
        if (!a_ok) {
          s_abort = 1;
          atomicAdd(&g_gemm_timeouts, 1);
          live = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_unit = tmem + a_col0 + uint32_t(asl.idx * 128);
        if (AS > kStepsPerCode) {
          // The act ring holds more than a unit: wait for all its steps, issue
          // the unit's MMAs back to back, then free the slots (one wait-MMA-
          // commit round per step cost ~600 cycles a step at small MT).
          int slot[kStepsPerCode];
          for (int j = 0; j < ns; ++j, ar.next()) {
            slot[j] = ar.idx;
            if (!mbar_wait(afull + ar.idx, ar.phase, &s_abort)) {
              s_abort = 1;
              atomicAdd(&g_gemm_timeouts, 1);
              live = false;
              break;
            }
          }
          if (!live) break;
          tc_fence_after();
          for (int j = 0; j < ns; ++j) {
            const uint32_t b_base = smem_u32(act_st + slot[j] * act_bytes);
            for (int k16 = issuer; k16 < kStep / 16; k16 += NI) {
              const uint64_t bdesc = smem_desc_k_sw128(b_base + k16 * 32);
              mma(d_tmem, a_unit + uint32_t(j * 32 + k16 * 8), bdesc, (u > 0 || j > 0 || k16 > issuer) ? 1u : 0u);
            }
          }
          for (int j = 0; j < ns; ++j) commit(afree + slot[j]);
        } else {
          // fewer act slots than steps in a unit: release each slot after its
          // own step, or the producer could never fill the unit's last step
          for (int j = 0; j < ns && live; ++j, ar.next()) {
            if (!mbar_wait(afull + ar.idx, ar.phase, &s_abort)) {
              s_abort = 1;
              atomicAdd(&g_gemm_timeouts, 1);
              live = false;
              break;
            }
            tc_fence_after();
            const uint32_t b_base = smem_u32(act_st + ar.idx * act_bytes);
            for (int k16 = issuer; k16 < kStep / 16; k16 += NI) {
              const uint64_t bdesc = smem_desc_k_sw128(b_base + k16 * 32);
              mma(d_tmem, a_unit + uint32_t(j * 32 + k16 * 8), bdesc, (u > 0 || j > 0 || k16 > issuer) ? 1u : 0u);
            }
            commit(afree + ar.idx);
          }
        }
        if (!live) break;
        commit(mdone + u % kDone);
      }
      commit(accf);
    }
  } else {
    // ---------------------------------------------------------------- dequant + epilogue
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int h = (warp - 2) >> 2;     // which group of each 64-k step
    const int row = q * 32 + lane;     // weight row within the tile
    const int64_t n = int64_t(n0) + row;
    const bool nv = n < kp.N;
    const uint32_t lane_base = uint32_t(q * 32) << 16;
    const int G = kp.K / kGroup;

    // the warp leaves the pipeline (warp-uniformly) when a wait gave up; only
    // lane 0 polls, the vote hands the result (and the ordering) to the warp
    auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
      const bool ok = __all_sync(0xffffffffu, lane == 0 ? mbar_wait(bar, parity, &s_abort) : true);
      if (!ok && lane == 0) {
        s_abort = 1;
        atomicAdd(&g_gemm_timeouts, 1);
      }
      return ok;
    };
    // this unit's A slot written: hand it to the MMA issuers
    Ring asl(NAS);
    auto publish = [&]() {
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(cluster_addr(aready + asl.idx, 0));  // the issuing CTA's barrier
        else
          mbar_arrive(aready + asl.idx);
      }
      asl.next();
    };

    // scale / zero point of this row for the four groups 2j+h of code stage lc
    // (global-memory path, used when they cannot be fetched by tensor map)
    auto load_sz = [&](int lc, float (&sv)[4], float (&zv)[4]) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int g = (cs0 + lc) * 8 + 2 * j + h;
        if (nv && lc < n_code && g < G) {
          sv[j] = __half2float(__ldg(kp.scales + n * kp.s_rs + int64_t(g) * kp.s_cs));
          zv[j] = float(__ldg(kp.zeros + n * kp.z_rs + int64_t(g) * kp.z_cs));
        } else {
          sv[j] = 0.f;
          zv[j] = 0.f;
        }
      }
    };
    float s_next[4], z_next[4];
    if constexpr (!SZ_TMA) load_sz(0, s_next, z_next);

    // outlier column indices of this CTA's outlier steps, once (the gather of
    // a[:, idx] then needs a single dependent load per element)
    if (n_out_st > 0 && !kp.pregather) {
      const int tid_d = (warp - 2) * 32 + lane;
      for (int j = tid_d; j < n_out_st * kStep; j += kDeqWarps * 32) {
        const int jg = ostep(j / kStep) * kStep + j % kStep;  // outlier column
        int64_t k = jg < kp.n_out ? load_index(kp.idx, jg, kp.idx_dtype) : -1;
        oidx[j] = (k >= 0 && k < kp.K) ? int(k) : -1;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kDeqWarps * 32) : "memory");  // dequant warps only
    }

    bool alive = true;
    // outlier units: columns j0 .. j0+63 of ow / of a[:, idx] per step
    for (int u = 0; u < n_ou && alive; ++u) {
      bool ok = u < NAS || wait_all(mdone + (u - NAS) % kDone, done_parity(u - NAS));
      const int ns = steps_of(u);
      // the act slots: free for the gather (or filled by the producer's copy
      // of the gathered tile, which only the MMA issuer waits for)
      for (int j = 0; j < ns && ok && !kp.pregather; ++j) {
        const int st = step_of(u, j);
        ok = wait_all(afull + st % AS, uint32_t((st / AS) & 1));
      }
      if (!ok) {
        alive = false;
        break;
      }
      tc_fence_after();
      const uint32_t a_unit = tmem + lane_base + a_col0 + uint32_t(asl.idx * 128);
      for (int j = 0; j < ns; ++j) {
        const int jl = step_of(u, j);       // local outlier step
        const int j0 = ostep(jl) * kStep;   // its first outlier column
        // this row's 32 outlier weights of the step, 16 at a time: the dtype is
        // resolved once, then the loads go out back to back (predicated)
        uint32_t vals[16];
        const int64_t obase = n * kp.ow_rs;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int jb = j0 + h * 32 + half * 16;
          float ov[16];
          if (kp.ow_dtype == SPECTRA_DT_F32) {
            const float* o32 = reinterpret_cast<const float*>(kp.ow);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              ov[i] = (nv && jb + i < kp.n_out) ? __ldg(o32 + obase + int64_t(jb + i) * kp.ow_cs) : 0.f;
          } else {
            const unsigned short* o16 = reinterpret_cast<const unsigned short*>(kp.ow);
            unsigned short raw[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              raw[i] = (nv && jb + i < kp.n_out) ? __ldg(o16 + obase + int64_t(jb + i) * kp.ow_cs) : (unsigned short)0;
            const bool obf = kp.ow_dtype == SPECTRA_DT_BF16;
#pragma unroll
            for (int i = 0; i < 16; ++i)
              ov[i] = obf ? __uint_as_float(uint32_t(raw[i]) << 16) : __half2float(__ushort_as_half(raw[i]));
          }
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) vals[half * 8 + cc] = pack2<BF16>(ov[2 * cc], ov[2 * cc + 1]);
        }
        // gather a[m_own+m, idx[j0+jj]] into the act slot (this CTA's tokens),
        // 128B-swizzled K-major; 8 independent loads in flight per thread
        uint8_t* bst = act_slot(u, j);
        const int tid_d = (warp - 2) * 32 + lane;
        constexpr int kBatch = 8;
        const int n_el = mt_local * kStep;
        for (int e0 = tid_d; e0 < (kp.pregather ? 0 : n_el); e0 += kDeqWarps * 32 * kBatch) {
          uint16_t v[kBatch];
#pragma unroll
          for (int i = 0; i < kBatch; ++i) {
            const int e = e0 + i * kDeqWarps * 32;
            const int m = e / kStep, jj = e % kStep;
            const int k = e < n_el ? oidx[jl * kStep + jj] : -1;
            v[i] = (k >= 0 && m_own + m < kp.M) ? load_act16(kp.a, int64_t(m_own + m) * kp.a_rs + k) : uint16_t(0);
          }
#pragma unroll
          for (int i = 0; i < kBatch; ++i) {
            const int e = e0 + i * kDeqWarps * 32;
            if (e < n_el) {
              const int m = e / kStep, jj = e % kStep;
              const int chunk = (jj >> 3) ^ (m & 7);
              *reinterpret_cast<uint16_t*>(bst + m * 128 + chunk * 16 + (jj & 7) * 2) = v[i];
            }
          }
        }
        tmem_st_x16(a_unit + uint32_t(j * 32 + h * 16), vals);
      }
      fence_proxy_async_smem();
      publish();
    }

    auto main_units = [&](auto marlin_tag) {
      constexpr bool kMarlin = decltype(marlin_tag)::value;
      Ring cr(CS);
      for (int lc = 0; lc < n_code && alive; ++lc, cr.next()) {
        const int c = cr.idx;
        const uint8_t* slot = code_st + c * kCodeBytes;
        const int ch = sz_of(lc);
        const bool first_of_sz = (lc == 0 || ch != sz_of(lc - 1));
        const bool last_of_sz = (lc == n_code - 1 || ch != sz_of(lc + 1));
        // A slot free (MMAs of unit u - NAS done), codes and sz landed
        const int u = n_ou + lc;
        if ((u >= NAS && !wait_all(mdone + (u - NAS) % kDone, done_parity(u - NAS))) ||
            !wait_all(cfull + c, cr.phase) ||
            (SZ_TMA && first_of_sz && !wait_all(szfull + ch % kSzSlots, uint32_t((ch / kSzSlots) & 1)))) {
          alive = false;
          break;
        }
        tc_fence_after();
        float sv[4], zv[4];
        if constexpr (SZ_TMA) {
          // this code stage's 8 groups: one 16-byte chunk of the row's 128-byte
          // scale line (128B swizzle) and 8 bytes of its 64-byte zero line (64B
          // swizzle: 16-byte chunk c of row r at c ^ ((r >> 1) & 3))
          const uint8_t* sslot = sz_st + (ch % kSzSlots) * kSzSlot;
          const int gi = (cs0 + lc) % kCodesPerSz;  // 8-group block within the chunk
          const uint4 s8 = *reinterpret_cast<const uint4*>(sslot + row * 128 + ((gi ^ (row & 7)) << 4));
          const uint2 z8 = *reinterpret_cast<const uint2*>(sslot + kSzScaleBytes + row * 64 +
                                                           (((gi >> 1) ^ ((row >> 1) & 3)) << 4) + (gi & 1) * 8);
          const uint32_t sw[4] = {s8.x, s8.y, s8.z, s8.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t hw = h ? (sw[j] >> 16) : (sw[j] & 0xFFFFu);
            sv[j] = __half2float(__ushort_as_half(static_cast<unsigned short>(hw)));
            const int b = 2 * j + h;
            zv[j] = float(((b < 4 ? z8.x : z8.y) >> ((b & 3) * 8)) & 0xFFu);
          }
          if (last_of_sz) {
            __syncwarp();
            if (lane == 0) mbar_arrive(szfree + ch % kSzSlots);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            sv[j] = s_next[j];
            zv[j] = z_next[j];
          }
          load_sz(lc + 1, s_next, z_next);
        }
        const uint32_t a_unit = tmem + lane_base + a_col0 + uint32_t(asl.idx * 128);
        const int ns = steps_of(u);
#pragma unroll
        for (int j = 0; j < kStepsPerCode; ++j) {
          if (j < ns) {  // K tail (warp-uniform)
            const int chunk = (2 * j + h) ^ (row & 7);  // 128B swizzle of the code tile
            const uint4 wv = *reinterpret_cast<const uint4*>(slot + row * 128 + chunk * 16);
            uint32_t vals[16];
            if constexpr (kMarlin)
              dequant_marlin<BF16>(wv, sv[j], zv[j], vals);
            else
              dequant_group<BF16>(wv, sv[j], zv[j], SPECTRA_LAYOUT_EVEN_ODD, vals);
            tmem_st_x16(a_unit + uint32_t(j * 32 + h * 16), vals);
          }
        }
        publish();
        // this code stage has been read: hand the slot back to the producer
        if (lane == 0) mbar_arrive(cfree + c);
      }
    };
    if (kp.layout == SPECTRA_LAYOUT_MARLIN)
      main_units(std::true_type{});
    else
      main_units(std::false_type{});

    // ---------------------------------------------------------------- epilogue
    // n_it == 0 cannot happen (S <= ncs), but an empty split would leave the
    // accumulators unwritten: treat them as zero.
    const bool ok = mbar_wait(accf, 0u, &s_abort) && n_it > 0;
    tc_fence_after();
    const int half_cols = kp.MT / 2;
    // accumulator columns c0..c0+7, summed over the issuers in order
    // (the issuers' loads all in flight before one wait)
    auto acc8 = [&](int c0, float (&v)[8]) {
      uint32_t r[kMaxIssuers][8];
#pragma unroll
      for (int i = 0; i < kMaxIssuers; ++i)
        if (i < NI) tmem_ld_x8_nowait(tmem + lane_base + uint32_t(i * kp.MT + c0), r[i]);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[0][e]);
#pragma unroll
      for (int i = 1; i < kMaxIssuers; ++i)
        if (i < NI) {
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] += __uint_as_float(r[i][e]);
        }
    };
    // one issuer: 32 columns per TMEM load and one wait per load (a wait per 8
    // columns made the epilogue ~6 us of a 55 us launch at MT = 256)
    int c_fast = h * half_cols;
    if (NI == 1) {
      for (; c_fast + 32 <= (h + 1) * half_cols; c_fast += 32) {
        uint32_t r[32];
        tmem_ld_x32_nowait(tmem + lane_base + uint32_t(c_fast), r);
        tmem_ld_wait();
        if (kp.S == 1) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int m = m0 + c_fast + i;
            if (nv && m < kp.M)
              reinterpret_cast<uint16_t*>(kp.c)[int64_t(m) * kp.c_rs + n] = to16(ok ? __uint_as_float(r[i]) : 0.f, bf16);
          }
        } else {
          float* part = kp.partials + int64_t(split) * kp.M * kp.N;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int m = m0 + c_fast + i;
            if (nv && m < kp.M) part[int64_t(m) * kp.N + n] = ok ? __uint_as_float(r[i]) : 0.f;
          }
        }
      }
    }
    if (kp.S == 1) {
      for (int c0 = c_fast; c0 < (h + 1) * half_cols; c0 += 8) {
        float v[8];
        acc8(c0, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int m = m0 + c0 + i;
          if (nv && m < kp.M) reinterpret_cast<uint16_t*>(kp.c)[int64_t(m) * kp.c_rs + n] = to16(ok ? v[i] : 0.f, bf16);
        }
      }
    } else {
      float* part = kp.partials + int64_t(split) * kp.M * kp.N;
      for (int c0 = c_fast; c0 < (h + 1) * half_cols; c0 += 8) {
        float v[8];
        acc8(c0, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int m = m0 + c0 + i;
          if (nv && m < kp.M) part[int64_t(m) * kp.N + n] = ok ? v[i] : 0.f;
        }
      }
    }
  }

  // split-K: the last CTA of this (tile, m-chunk) sums the partials in split
  // order (deterministic).  (The rowless CTA that pads an odd tile count in
  // pair mode has no partials and no counter.)
  if (kp.S > 1 && n0 < kp.N) {
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
      const int64_t plane = int64_t(kp.M) * kp.N;
      uint16_t* c16 = reinterpret_cast<uint16_t*>(kp.c);
      if ((kp.N & 3) == 0) {
        // 4 consecutive rows per element, 4 elements per thread in flight
        const int r4 = rows_here >> 2;
        const int total = r4 * toks;
        for (int e0 = threadIdx.x; e0 < total; e0 += kThreads * 4) {
          float4 acc[4];
          int64_t off[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int e = min(e0 + j * kThreads, total - 1);
            acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            off[j] = int64_t(m0 + e / r4) * kp.N + n0 + 4 * (e % r4);
          }
          for (int sp = 0; sp < kp.S; ++sp) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 v = __ldcg(reinterpret_cast<const float4*>(kp.partials + sp * plane + off[j]));
              acc[j].x += v.x;
              acc[j].y += v.y;
              acc[j].z += v.z;
              acc[j].w += v.w;
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int e = e0 + j * kThreads;
            if (e < total) {
              const int m = m0 + e / r4;
              uint16_t* dst = c16 + int64_t(m) * kp.c_rs + n0 + 4 * (e % r4);
              dst[0] = to16(acc[j].x, bf16);
              dst[1] = to16(acc[j].y, bf16);
              dst[2] = to16(acc[j].z, bf16);
              dst[3] = to16(acc[j].w, bf16);
            }
          }
        }
      } else {
        const int total = rows_here * toks;
        for (int e0 = threadIdx.x; e0 < total; e0 += kThreads * 4) {
          float acc[4];
          int64_t off[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int e = min(e0 + j * kThreads, total - 1);
            acc[j] = 0.f;
            off[j] = int64_t(m0 + e / rows_here) * kp.N + n0 + (e % rows_here);
          }
          for (int sp = 0; sp < kp.S; ++sp) {
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[j] += __ldcg(kp.partials + sp * plane + off[j]);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int e = e0 + j * kThreads;
            if (e < total) c16[int64_t(m0 + e / rows_here) * kp.c_rs + n0 + (e % rows_here)] = to16(acc[j], bf16);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) {
    // Neither CTA frees its TMEM or leaves before both are done: rank 0's
    // MMAs read rank 1's shared memory and TMEM, and rank 1's copies and
    // arrivals land on rank 0's barriers.
    cluster_sync_all();
    if (warp == 1) {
      __syncwarp();
      tc_fence_after();
      tmem_dealloc_pair(tmem, kp.tmem_cols);
    }
    cluster_sync_all();
  } else if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kp.tmem_cols);
  }
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

GemmPlan plan_gemm(int64_t M, int64_t N, int64_t K, int64_t n_out) {
  GemmPlan p{};
  const int mt_needed = int(((std::min<int64_t>(M, kMaxMT) + 15) / 16) * 16);
  p.MT = std::max(16, mt_needed);
  p.m_chunks = int((M + kMaxMT - 1) / kMaxMT);
  if (p.m_chunks > 1) p.MT = kMaxMT;
  p.tiles_n = int((N + kRows - 1) / kRows);
  // SM pairs for token tiles of >= 128: the pair MMA's N (the whole token
  // tile) is a multiple of 32, each CTA loads half of it
  p.pair = pair_enabled() && p.MT >= 128;
  if (p.pair) p.MT = (p.MT + 31) / 32 * 32;
  p.tiles_pad = p.pair ? (p.tiles_n + 1) & ~1 : p.tiles_n;
  const int mt_local = p.pair ? p.MT / 2 : p.MT;
  p.nk = int((K + kStep - 1) / kStep);
  p.ncs = int((K + kCodeK - 1) / kCodeK);
  p.n_os = int((n_out + kStep - 1) / kStep);
  const int sms = 148;  // B200; one CTA per SM (~200 KB of shared memory)
  const int64_t ctas = int64_t(p.tiles_pad) * p.m_chunks;
  // split K so that all CTAs fit in ONE wave: rounding up (e.g. 32 tiles x 5 =
  // 160 CTAs) leaves a second wave of a few CTAs that doubles the time
  p.S = int(std::min<int64_t>(std::max<int64_t>(1, sms / ctas), p.ncs));
  p.act_stage_bytes = mt_local * 128;
  p.code_stages = mt_local <= 32 ? 6 : mt_local <= 64 ? 5 : mt_local <= 128 ? 4 : 3;
  const size_t fixed = 1024 + 64 + size_t(2 * kSzSlots + 3 + kDone + 1) * 8 + size_t(kSzSlots) * kSzSlot +
                       size_t(p.n_os) * kStep * 4;  // + outlier column indices
  const size_t code = size_t(p.code_stages) * (kCodeBytes + 16);
  p.act_stages = int(std::min<size_t>(kMaxActStages, (kMaxDynSmem - fixed - code) / (p.act_stage_bytes + 16)));
  p.smem = fixed + code + size_t(p.act_stages) * (p.act_stage_bytes + 16);
  p.issuers = p.MT <= 32 ? kMaxIssuers : p.MT <= 64 ? 2 : 1;
  // a third A slot (128 columns) where the accumulators leave room for it
  p.a_slots = p.issuers * p.MT + 3 * 128 <= 512 ? 3 : 2;
  p.tmem_cols = 32;
  while (p.tmem_cols < uint32_t(p.issuers * p.MT + p.a_slots * 128)) p.tmem_cols <<= 1;
  p.partials_off = kCounterBytes;
  p.workspace = p.S > 1 ? kCounterBytes + size_t(p.S) * M * N * 4 : 0;
  // Token tiles of >= 32: the outlier columns' activations are gathered once
  // per call into the workspace (after the split-K region, never over the
  // counters) instead of once per weight tile (measured equal at 32 tokens,
  // faster from 64 on and with many outlier columns; at 16 tokens each CTA's
  // share is too small to pay for the extra launch).
  p.pregather = n_out > 0 && p.MT >= 32;
  p.gather_off = 256 * ((std::max(p.workspace, kCounterBytes) + 255) / 256);
  if (p.pregather) p.workspace = p.gather_off + 256 * ((size_t(M) * p.n_os * kStep * 2 + 255) / 256);
  return p;
}

namespace {

template <bool BF16, bool SZ_TMA, bool PAIR>
int launch_variant(const GemmPlan& pl, const CUtensorMap (&maps)[5], const GemmKParams& kp, cudaStream_t st) {
  auto kern = gemm_w4a16_tc_kernel<BF16, SZ_TMA, PAIR>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return SPECTRA_ERR_UNSUPPORTED;
  static PerContextOnce attrs;
  e = attrs.run(dev, [&] { return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMaxDynSmem)); });
  if (e != cudaSuccess) return cuda_status(e);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(pl.tiles_pad * pl.S), unsigned(pl.m_chunks));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if constexpr (PAIR) {  // consecutive blockIdx.x in clusters of two
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], maps[2], maps[3], maps[4], kp));
}

}  // namespace

int launch_gemm(const GemmArgs& a, void* ws, size_t ws_bytes, cudaStream_t st) {
  const GemmPlan pl = plan_gemm(a.M, a.N, a.K, a.n_out);
  if (pl.tmem_cols > 512 || pl.smem > kMaxDynSmem || pl.act_stages < 3) return SPECTRA_ERR_UNSUPPORTED;
  if (pl.workspace > 0 && (ws == nullptr || ws_bytes < pl.workspace)) return SPECTRA_ERR_WORKSPACE;
  if (pl.S > 1 && size_t(pl.tiles_n) * pl.m_chunks * 4 > kCounterBytes) return SPECTRA_ERR_UNSUPPORTED;
  auto enc = tensor_map_encoder();
  if (!enc) return SPECTRA_ERR_UNSUPPORTED;
  const bool bf16 = a.a_dtype == SPECTRA_DT_BF16;
  const int G = a.K / kGroup;

  CUtensorMap maps[5];  // codes, scales, zero points, activations, gathered outlier activations
  memset(maps, 0, sizeof(maps));
  {
    cuuint64_t dims[2] = {cuuint64_t(a.K / 2), cuuint64_t(a.N)};
    cuuint64_t strides[1] = {cuuint64_t(a.w_rs)};
    cuuint32_t box[2] = {kCodeK / 2, kRows}, es[2] = {1, 1};
    if (enc(&maps[0], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.packed), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return SPECTRA_ERR_ALIGNMENT;
  }
  // scales / zero points by tensor map when their layout allows one (unit
  // column stride, 16-byte aligned base and row pitch); else by plain loads
  bool sz_tma = a.s_cs == 1 && a.z_cs == 1 && (a.s_rs * 2) % 16 == 0 && a.z_rs % 16 == 0 &&
                reinterpret_cast<uintptr_t>(a.scales) % 16 == 0 && reinterpret_cast<uintptr_t>(a.zeros) % 16 == 0 &&
                sz_tma_enabled();
  if (sz_tma) {
    cuuint64_t dims[2] = {cuuint64_t(G), cuuint64_t(a.N)};
    cuuint64_t s_strides[1] = {cuuint64_t(a.s_rs) * 2};
    cuuint64_t z_strides[1] = {cuuint64_t(a.z_rs)};
    cuuint32_t box[2] = {kSzGroups, kRows}, es[2] = {1, 1};
    sz_tma = enc(&maps[1], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<__half*>(a.scales), dims, s_strides, box,
                 es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS &&
             enc(&maps[2], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.zeros), dims, z_strides, box, es,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  {
    cuuint64_t dims[2] = {cuuint64_t(a.K), cuuint64_t(a.M)};
    cuuint64_t strides[1] = {cuuint64_t(a.a_rs) * 2};
    // pair mode: each CTA of a pair fetches half of the token tile
    cuuint32_t box[2] = {kStep, cuuint32_t(pl.pair ? pl.MT / 2 : pl.MT)}, es[2] = {1, 1};
    if (enc(&maps[3], bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
            const_cast<void*>(a.a), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return SPECTRA_ERR_ALIGNMENT;
  }

  uint16_t* gathered = pl.pregather ? reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(ws) + pl.gather_off) : nullptr;
  if (pl.pregather) {
    const int cols = pl.n_os * kStep;
    cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(a.M)};
    cuuint64_t strides[1] = {cuuint64_t(cols) * 2};
    cuuint32_t box[2] = {kStep, cuuint32_t(pl.pair ? pl.MT / 2 : pl.MT)}, es[2] = {1, 1};
    if (enc(&maps[4], bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, gathered, dims,
            strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
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
  kp.MT = pl.MT; kp.S = pl.S; kp.nk = pl.nk; kp.ncs = pl.ncs; kp.n_os = pl.n_os; kp.tiles_n = pl.tiles_n;
  kp.tiles_pad = pl.tiles_pad;
  kp.pregather = pl.pregather ? 1 : 0;
  kp.act_stages = pl.act_stages; kp.code_stages = pl.code_stages; kp.issuers = pl.issuers;
  kp.a_slots = pl.a_slots;
  kp.idesc = idesc_f16(bf16, pl.pair ? 2 * kRows : kRows, pl.MT);  // M = 256 over a pair
  kp.tmem_cols = pl.tmem_cols;
  kp.act_stage_bytes = pl.act_stage_bytes;
  // shared memory: act slots | code slots | sz slots | barriers (all 1024-aligned
  // regions: act slots are multiples of 2 KB, code and sz slots of 8 KB)
  kp.off_act = 0;
  kp.off_code = pl.act_stages * pl.act_stage_bytes;
  kp.off_sz = kp.off_code + pl.code_stages * kCodeBytes;
  kp.off_oidx = kp.off_sz + kSzSlots * kSzSlot;
  kp.off_bar = kp.off_oidx + pl.n_os * kStep * 4;
  if (pl.S > 1) {
    kp.counters = reinterpret_cast<int*>(ws);
    kp.partials = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + pl.partials_off);
  }
  if (pl.pregather) {
    const int cols = pl.n_os * kStep;
    const int64_t threads = int64_t(a.M) * (cols / 8);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned((threads + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gather_outlier_acts_kernel, static_cast<const uint16_t*>(a.a),
                                             int64_t(a.a_rs), a.idx, a.idx_dtype, a.n_out, a.K, a.M, cols, gathered);
    if (e != cudaSuccess) return cuda_status(e);
  }
  if (pl.pair) {
    if (bf16)
      return sz_tma ? launch_variant<true, true, true>(pl, maps, kp, st) : launch_variant<true, false, true>(pl, maps, kp, st);
    return sz_tma ? launch_variant<false, true, true>(pl, maps, kp, st) : launch_variant<false, false, true>(pl, maps, kp, st);
  }
  if (bf16)
    return sz_tma ? launch_variant<true, true, false>(pl, maps, kp, st) : launch_variant<true, false, false>(pl, maps, kp, st);
  return sz_tma ? launch_variant<false, true, false>(pl, maps, kp, st) : launch_variant<false, false, false>(pl, maps, kp, st);
}

int gemm_noalloc_scratch(void** ptr, size_t* bytes) {
  // The array's device address, looked up once per device and again whenever
  // that device's context was recreated (cudaDeviceReset reloads the module,
  // and the array may then live elsewhere).  The address is stored before the
  // context id, so a reader that sees its own context's id reads its address.
  static std::atomic<unsigned long long> ctx_of[kMaxDevices];
  static std::atomic<void*> addr[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return SPECTRA_ERR_UNSUPPORTED;
  const unsigned long long id = current_context_id();
  void* p = nullptr;
  if (id != 0 && ctx_of[dev].load(std::memory_order_acquire) == id) p = addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    e = cudaGetSymbolAddress((void**)&p, g_gemm_noalloc_scratch);  // with `dev` current
    if (e != cudaSuccess) return cuda_status(e);
    addr[dev].store(p, std::memory_order_release);
    ctx_of[dev].store(current_context_id(), std::memory_order_release);
  }
  *ptr = p;
  *bytes = sizeof(g_gemm_noalloc_scratch);
  return SPECTRA_OK;
}

int gemm_timeouts(long long* out, bool reset) { return read_timeout_counter(g_gemm_timeouts, out, reset); }

int gemm_pair_capacity(int* clusters) {
  auto kern = gemm_w4a16_tc_kernel<true, true, true>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMaxDynSmem));
  if (e != cudaSuccess) return cuda_status(e);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * 74);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kMaxDynSmem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaOccupancyMaxActiveClusters(clusters, kern, &cfg));
}

}  // namespace spectra
