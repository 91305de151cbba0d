// M=1 W4A16 decode GEMV for sm_100a (replaces spectra/kernels.py:16-184).
//
// Work decomposition
//   A "pass" covers 32 consecutive quantisation groups (1024 input features):
//   lane l of a warp owns group (pass*32 + l), so one 128-bit load per lane
//   streams 512 contiguous bytes of a weight row per warp instruction.
//   A CTA owns RG*R consecutive output rows.  Its S*RG warps are S k-splits x
//   RG row-groups; warp (ks, rg) runs passes ks, ks+S, ... for its R rows, so
//   every row of the CTA sees all of K inside the CTA and the split-K reduce
//   is a fixed-order sum through shared memory (deterministic, no workspace).
//
// Activation staging
//   Each CTA stages x once per K-window into shared memory as fp32, permuted
//   into the order the dequant consumes codes and pre-scaled by 16^-i for a
//   code sitting at nibble i of its 16-bit half-word, plus the per-group sum
//   X_g = sum_k x[k].  Rows of a warp reuse the staged x from registers.
//
// Dequant (exact)
//   A code q at nibble i of a half-word h becomes the float 2^23 + q*16^i with
//   one LOP3 ((h & 0xF<<4i) | 0x4B000000); subtracting 2^23 (packed f32x2 add)
//   leaves q*16^i exactly, and the f32x2 FMA with x*16^-i accumulates q*x.
//   Per group:  sum_k (q_k - z) * s * x_k  =  s * (sum_k q_k x_k  -  z * X_g).
//   Every product q*x is exact in fp32; the only roundings are the fp32
//   accumulations (the reference also accumulates in fp32).
//
// Fused epilogue: outlier columns  sum_j x[idx_j]*ow[n,j]  (fp32, as
// spectra/kernels.py:102-120), bias (:122-124), one rounding to y's dtype.
#include "common.cuh"
#include "gemv.h"
#include "sm100_ptx.cuh"

namespace spectra {

namespace {

constexpr int kXpStride = 36;  // floats per staged group: 32 + 4 pad (bank-conflict-free LDS.128)

struct GemvKParams {
  GemvArgs a;
  int S, RG, win_groups;
  bool vec_x;          // x contiguous, 16-byte aligned, fp16/bf16
  int rows_max;        // max rows of one CTA (bulk kernel)
  int off_bars, off_xs, off_xsum, off_xos, off_red;  // bulk kernel smem layout
  int red_passes;      // passes over all of K (bulk kernel partial-sum slots)
  int off_ow;          // bulk kernel: shared copy of this CTA's outlier-weight rows (-1: not staged)
  int smem_xs_floats;  // win_groups * kXpStride
};

// slot s = j*8 + i*2 + h of a staged group <-> code of word j (bytes 4j..4j+3),
// half-word h, nibble i inside that half-word.
__device__ __forceinline__ int slot_byte(int s) { return 4 * (s >> 3) + 2 * (s & 1) + (((s >> 1) & 3) >> 1); }
__device__ __forceinline__ int slot_hi(int s) { return (s >> 1) & 1; }
__device__ __forceinline__ float slot_scale(int s) {
  const int i = (s >> 1) & 3;
  return i == 0 ? 1.0f : (i == 1 ? 0.0625f : (i == 2 ? 0.00390625f : 0.000244140625f));
}

// (h & (0xF << 4I)) | magic in one LOP3: the mask is an immediate and the
// magic lives in a register, so the AND/OR pair cannot be split in two.
template <int I>
__device__ __forceinline__ uint32_t nib_magic(uint32_t h, uint32_t magic_reg) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(h), "n"(0xFu << (4 * I)), "r"(magic_reg));
  return r;
}

// sum_k q_k * x_k over one 32-code group (x pre-scaled, slot order).  Four
// independent f32x2 accumulators (one per nibble position) keep the FMA pipe
// busy without a serial dependency chain.
__device__ __forceinline__ float group_qdot(const uint4 w, const float2 (&xr)[16], uint32_t magic_reg) {
  const float2 neg_magic = make_float2(-8388608.0f, -8388608.0f);
  float2 acc[4];
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t a = words[j];
    const uint32_t b = a >> 16;
#define SPECTRA_QSTEP(I)                                                                                \
  {                                                                                                   \
    float2 v = make_float2(__uint_as_float(nib_magic<I>(a, magic_reg)),                               \
                           __uint_as_float(nib_magic<I>(b, magic_reg)));                              \
    v = __fadd2_rn(v, neg_magic);                                                                     \
    acc[I] = (j == 0) ? __fmul2_rn(v, xr[j * 4 + I]) : __ffma2_rn(v, xr[j * 4 + I], acc[I]);        \
  }
    SPECTRA_QSTEP(0) SPECTRA_QSTEP(1) SPECTRA_QSTEP(2) SPECTRA_QSTEP(3)
#undef SPECTRA_QSTEP
  }
  const float2 s01 = __fadd2_rn(acc[0], acc[1]);
  const float2 s23 = __fadd2_rn(acc[2], acc[3]);
  const float2 t = __fadd2_rn(s01, s23);
  return t.x + t.y;
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

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Inverse of the slot map: staged slot of the code for k (0..31) in its group.
__device__ __forceinline__ int k_slot(int k, int layout) {
  int byte, hi;
  if (layout == SPECTRA_LAYOUT_MARLIN) { byte = k & 15; hi = k >> 4; }
  else { byte = k >> 1; hi = k & 1; }
  const int j = byte >> 2, h = (byte >> 1) & 1, i = 2 * (byte & 1) + hi;
  return 8 * j + 2 * i + h;
}

// Stage x[wg0*32 .. (wg0+wgn)*32) into shared memory: fp32, permuted into the
// order group_qdot consumes codes, pre-scaled by 16^-i, plus per-group sums.
__device__ __forceinline__ void stage_x_window(const GemvArgs& p, bool vec_x, float* xs, float* xsum, int wg0, int wgn,
                                               int tid, int nthreads, int lane) {
  // With 16-byte vector loads a thread always stages the same 8-element
  // quarter (tid % 4) of a group.
  const int quarter = tid & 3;
  int vslot[8];
  float vscale[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    vslot[e] = k_slot(8 * quarter + e, p.layout);
    vscale[e] = slot_scale(vslot[e]);
  }
  const int sslot = k_slot(lane, p.layout);
  const float sscale = slot_scale(sslot);
    if (vec_x) {
      // 8 consecutive elements per thread (one 16-byte load); the 4 threads of
      // a group are consecutive lanes, so two shuffles finish its sum.
      const int nchunk = wgn * 4;
      const int rounds = (nchunk + nthreads - 1) / nthreads;  // CTA-uniform
      const uint4* xv = reinterpret_cast<const uint4*>(p.x) + int64_t(wg0) * 4;
      for (int r0 = 0; r0 < rounds; r0 += 4) {
        uint4 raw[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int c = (r0 + b) * nthreads + tid;
          raw[b] = (r0 + b < rounds && c < nchunk) ? __ldg(xv + c) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          if (r0 + b >= rounds) break;  // CTA-uniform: every lane reaches the shuffles below
          const int c = (r0 + b) * nthreads + tid;
          const uint32_t w4[4] = {raw[b].x, raw[b].y, raw[b].z, raw[b].w};
          float v[8];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (p.x_dtype == SPECTRA_DT_BF16) {
              v[2 * q] = __uint_as_float(w4[q] << 16);
              v[2 * q + 1] = __uint_as_float(w4[q] & 0xFFFF0000u);
            } else {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[q]));
              v[2 * q] = f.x;
              v[2 * q + 1] = f.y;
            }
          }
          float t = 0.f;
          const int gl = c >> 2;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            t += v[e];
            if (c < nchunk) xs[gl * kXpStride + vslot[e]] = v[e] * vscale[e];
          }
          t += __shfl_xor_sync(0xffffffffu, t, 1);
          t += __shfl_xor_sync(0xffffffffu, t, 2);
          if (quarter == 0 && c < nchunk) xsum[gl] = t;
        }
      }
    } else {
      // Strided or fp32 x: one element per lane, a warp stages whole groups.
      const int n = wgn * kGroup;
      constexpr int kBatch = 8;
      for (int e0 = tid; e0 < n; e0 += kBatch * nthreads) {
        float v[kBatch];
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
          const int e = e0 + b * nthreads;
          v[b] = (e < n) ? load_as_float(p.x, int64_t(wg0 * kGroup + e) * p.x_stride, p.x_dtype) : 0.f;
        }
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
          const int e = e0 + b * nthreads;  // warp-uniform validity (n is a multiple of 32)
          if (e < n) {
            const int gl = e >> 5;
            xs[gl * kXpStride + sslot] = v[b] * sscale;
            float t = v[b];
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
            if (lane == 0) xsum[gl] = t;
          }
        }
      }
    }
}

// Persistent kernel: CTA b owns the contiguous rows [N*b/grid, N*(b+1)/grid),
// processed in tiles of RG*R rows.  x is staged once per CTA and K-window.
template <int R, int ALIGN>
__global__ void __launch_bounds__(256, 2) gemv_w4a16_kernel(const __grid_constant__ GemvKParams kp) {
  const GemvArgs& p = kp.a;
  extern __shared__ __align__(16) float smem[];
  const int rows_cta = kp.RG * R;
  float* xs = smem;                                   // [win_groups][36]
  float* xsum = xs + kp.smem_xs_floats;               // [win_groups]
  float* xos = xsum + kp.win_groups;                  // [n_out]
  float* red = xos + ((p.n_out + 3) & ~3);            // [2][S][rows_cta]
  float* acc_rows = red + 2 * kp.S * rows_cta;        // [max_tiles][rows_cta] (multi-window K only)

  // Only weights are read before griddepcontrol.wait; let the next kernel in
  // the stream start its own weight prefetch as soon as SMs free up.
  griddep_launch_dependents();

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nthreads = blockDim.x;
  const int S = kp.S;
  const int ks = warp % S;
  const int rg = warp / S;
  const int G = p.K / kGroup;
  const int64_t r_begin = (int64_t(p.N) * blockIdx.x) / gridDim.x;
  const int64_t r_end = (int64_t(p.N) * (blockIdx.x + 1)) / gridDim.x;
  const int ntiles = int((r_end - r_begin + rows_cta - 1) / rows_cta);

  uint32_t magic_reg;
  asm volatile("mov.b32 %0, 0x4B000000;" : "=r"(magic_reg));

  // Weight registers of the unit being computed (cur) and of the next unit
  // (nxt), loaded one unit ahead so a warp always has a load batch in flight.
  uint4 nw[R];
  float ns[R], nz[R];
  auto load_unit = [&](int t, int g_first, int wgn, int pp) {
    const int gl = pp * 32 + lane;
    const int g = g_first + gl;
    const bool gv = gl < wgn;
    const int64_t row0 = r_begin + int64_t(t) * rows_cta + rg * R;
    const uint8_t* wp = p.packed + row0 * p.w_rs + int64_t(g) * kGroupBytes;
    const __half* sp = p.scales + row0 * p.s_rs + int64_t(g) * p.s_cs;
    const uint8_t* zp = p.zeros + row0 * p.z_rs + int64_t(g) * p.z_cs;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (gv && row0 + r < r_end) {
        nw[r] = load_group16<ALIGN>(wp + r * p.w_rs);
        ns[r] = __half2float(__ldg(sp + r * p.s_rs));
        // u8 -> float with the same magic (ALU) instead of an I2F conversion
        nz[r] = __uint_as_float(uint32_t(__ldg(zp + r * p.z_rs)) | kMagic) - 8388608.0f;
      } else {
        nw[r] = make_uint4(0u, 0u, 0u, 0u);
        ns[r] = 0.f;
        nz[r] = 0.f;
      }
    }
  };

  if (ntiles > 0) load_unit(0, 0, min(kp.win_groups, G), ks);

  // Outlier column indices are weights-side data: read them before the wait.
  constexpr int kOutPerThread = 4;
  int64_t oidx[kOutPerThread];
#pragma unroll
  for (int m = 0; m < kOutPerThread; ++m) {
    const int j = tid + m * nthreads;
    oidx[m] = (j < p.n_out) ? load_index(p.idx, j, p.idx_dtype) : -1;
  }

  griddep_wait();  // x (and the output buffer) belong to the previous kernel

#pragma unroll
  for (int m = 0; m < kOutPerThread; ++m) {
    const int j = tid + m * nthreads;
    if (j < p.n_out) xos[j] = (oidx[m] >= 0 && oidx[m] < p.K) ? load_as_float(p.x, oidx[m] * p.x_stride, p.x_dtype) : 0.f;
  }
  for (int j = tid + kOutPerThread * nthreads; j < p.n_out; j += nthreads) {
    const int64_t k = load_index(p.idx, j, p.idx_dtype);
    xos[j] = (k >= 0 && k < p.K) ? load_as_float(p.x, k * p.x_stride, p.x_dtype) : 0.f;
  }

  const bool vec_x = kp.vec_x;

  int buf = 0;
  const int nwin = (G + kp.win_groups - 1) / kp.win_groups;
  for (int w = 0; w < nwin; ++w) {
    const int wg0 = w * kp.win_groups;
    const int wgn = min(kp.win_groups, G - wg0);
    if (w > 0) __syncthreads();  // every tile is done with the previous window
    stage_x_window(p, vec_x, xs, xsum, wg0, wgn, tid, nthreads, lane);
    __syncthreads();

    const int wpass = (wgn + 31) / 32;
    if (w > 0 && ntiles > 0) load_unit(0, wg0, wgn, ks);
    const bool last_win = (w == nwin - 1);
    for (int t = 0; t < ntiles; ++t) {
      float acc[R];
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = 0.f;
      for (int pp = ks; pp < wpass; pp += S) {
        uint4 cw[R];
        float cs[R], cz[R];
#pragma unroll
        for (int r = 0; r < R; ++r) { cw[r] = nw[r]; cs[r] = ns[r]; cz[r] = nz[r]; }
        // Prefetch the next unit of work before computing this one.
        if (pp + S < wpass) load_unit(t, wg0, wgn, pp + S);
        else if (t + 1 < ntiles) load_unit(t + 1, wg0, wgn, ks);
        const int gl = pp * 32 + lane;
        if (gl < wgn) {
          float2 xr[16];
          const float4* src = reinterpret_cast<const float4*>(xs + gl * kXpStride);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 f = src[c];
            xr[2 * c] = make_float2(f.x, f.y);
            xr[2 * c + 1] = make_float2(f.z, f.w);
          }
          const float xg = xsum[gl];
#pragma unroll
          for (int r = 0; r < R; ++r) {
            float q = group_qdot(cw[r], xr, magic_reg);
            q = fmaf(-cz[r], xg, q);
            acc[r] = fmaf(q, cs[r], acc[r]);
          }
        }
      }
      const int64_t row0 = r_begin + int64_t(t) * rows_cta + rg * R;
      if (last_win) {
        // Outlier columns: chunk c of 32 columns is handled by k-split warp c % S.
        const int nch = (p.n_out + 31) / 32;
        for (int c = ks; c < nch; c += S) {
          const int j = c * 32 + lane;
          if (j < p.n_out) {
            const float xo = xos[j];
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const int64_t row = row0 + r;
              if (row < r_end)
                acc[r] = fmaf(xo, load_as_float(p.ow, row * p.ow_rs + int64_t(j) * p.ow_cs, p.ow_dtype), acc[r]);
            }
          }
        }
      }
      warp_transpose_reduce<R>(acc, lane);
      constexpr int kLeaderMask = (32 / R) - 1;
      float* rb = red + buf * S * rows_cta;
      if ((lane & kLeaderMask) == 0) rb[ks * rows_cta + rg * R + reduced_row<R>(lane)] = acc[0];
      __syncthreads();
      for (int i = tid; i < rows_cta; i += nthreads) {
        const int64_t row = r_begin + int64_t(t) * rows_cta + i;
        float v = 0.f;
        for (int q = 0; q < S; ++q) v += rb[q * rows_cta + i];
        if (nwin > 1) {
          if (w > 0) v += acc_rows[t * rows_cta + i];
          if (!last_win) {
            acc_rows[t * rows_cta + i] = v;
            continue;
          }
        }
        if (row < r_end) {
          if (p.bias) v += load_as_float(p.bias, row, p.bias_dtype);
          store_from_float(p.y, row * p.y_stride, p.y_dtype, v);
        }
      }
      buf ^= 1;
    }
  }
}

// ---------------------------------------------------------------------------
// Bulk-copy pipeline (main path).
//
// Each warp owns a ring of kBulkStages shared-memory stages.  A stage holds
// one unit of work -- R rows x one pass (32 groups): 512 packed bytes, 64
// scale bytes and 32 zero bytes per row -- filled by cp.async.bulk (the TMA
// engine's non-tensor copy) issued by lane 0 and completed on an mbarrier.
// Bytes in flight are bounded by shared memory, not registers, and the warp
// never waits on a CTA barrier inside the main loop: partial sums of each
// (k-split, row) go to shared memory once per row batch and are combined
// after a single barrier at the end.
// ---------------------------------------------------------------------------
constexpr int kBulkStages = 4;

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(bytes), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
               : "memory");
}

__device__ int g_gemv_timeouts;  // stuck pipeline waits since load (diagnostic)

template <int R>
__global__ void __launch_bounds__(256, 1) gemv_bulk_kernel(const __grid_constant__ GemvKParams kp) {
  using namespace sm100;
  const GemvArgs& p = kp.a;
  constexpr int kStageBytes = R * (512 + 64 + 32);
  constexpr int kWarps = 8;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nstages = kp.S;  // ring depth of each warp
  uint8_t* my_stages = smem_raw + size_t(warp) * nstages * kStageBytes;
  uint64_t* my_bars = reinterpret_cast<uint64_t*>(smem_raw + kp.off_bars) + warp * nstages;
  float* xs = reinterpret_cast<float*>(smem_raw + kp.off_xs);
  float* xsum = reinterpret_cast<float*>(smem_raw + kp.off_xsum);
  float* xos = reinterpret_cast<float*>(smem_raw + kp.off_xos);
  float* red = reinterpret_cast<float*>(smem_raw + kp.off_red);  // [passes][rows_max]
  float* ored = red + kp.red_passes * kp.rows_max;               // [rows_max]
  __shared__ int s_abort;
  __shared__ __align__(8) uint64_t s_ow_bar;

  griddep_launch_dependents();

  const int64_t r_begin = (int64_t(p.N) * blockIdx.x) / gridDim.x;
  const int64_t r_end = (int64_t(p.N) * (blockIdx.x + 1)) / gridDim.x;
  const int nrows = int(r_end - r_begin);
  const int nb = (nrows + R - 1) / R;
  const int G = p.K / kGroup;

  if (tid == 0) s_abort = 0;
  if (lane == 0) {
    for (int i = 0; i < nstages; ++i) mbar_init(my_bars + i, 1);
    fence_mbar_init();
  }
  for (int i = tid; i < (kp.red_passes + 1) * kp.rows_max; i += blockDim.x) red[i] = 0.f;
  // This CTA's outlier-weight rows are one contiguous byte range: bring its
  // 16-byte-aligned body over with one bulk copy now (weights-side data, no
  // dependency on the previous kernel) and read the ragged tail directly.
  const int ow_es = p.ow_dtype == SPECTRA_DT_F32 ? 4 : 2;
  const bool ow_staged = kp.off_ow >= 0 && p.n_out > 0;
  const uint8_t* ow_src = reinterpret_cast<const uint8_t*>(p.ow);
  const int64_t ow_b0 = r_begin * p.n_out * ow_es;
  const int64_t ow_b1 = r_end * p.n_out * ow_es;
  const int64_t ow_a0 = ow_b0 & ~int64_t(15);
  const int64_t ow_a1 = ow_b1 & ~int64_t(15);
  uint8_t* ow_smem = smem_raw + (kp.off_ow >= 0 ? kp.off_ow : 0);
  if (ow_staged && tid == 0) {
    mbar_init(&s_ow_bar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&s_ow_bar, uint32_t(ow_a1 - ow_a0));
    if (ow_a1 > ow_a0) bulk_g2s(ow_smem, ow_src + ow_a0, uint32_t(ow_a1 - ow_a0), &s_ow_bar);
  }
  __syncwarp();

  // Copy roles of the lanes when a unit is issued: lane l < R copies row l's
  // codes, R <= l < 2R its scales, 2R <= l < 3R its zero-points.
  const int role = lane / R;
  const int rrow = lane % R;
  // Unit (b, pass) of a window = rows [b*R, b*R+R) x groups [pass*32, pass*32+32).
  auto issue = [&](int ub, int upass, int wg0, int wgn, int slot) {
    const int gl0 = upass * 32;
    const int ng = min(32, wgn - gl0);
    const int nr = min(R, nrows - ub * R);
    uint8_t* st = my_stages + slot * kStageBytes;
    uint64_t* bar = my_bars + slot;
    if (lane == 0) mbar_arrive_expect_tx(bar, uint32_t(nr * ng * (kGroupBytes + 2 + 1)));
    __syncwarp();
    if (role < 3 && rrow < nr) {
      const int64_t row = r_begin + int64_t(ub) * R + rrow;
      const int64_t g = int64_t(wg0 + gl0);
      const void* src;
      void* dst;
      uint32_t bytes;
      if (role == 0) {
        src = p.packed + row * p.w_rs + g * kGroupBytes;
        dst = st + rrow * 512;
        bytes = uint32_t(ng * kGroupBytes);
      } else if (role == 1) {
        src = p.scales + row * p.s_rs + g;
        dst = st + R * 512 + rrow * 64;
        bytes = uint32_t(ng * 2);
      } else {
        src = p.zeros + row * p.z_rs + g;
        dst = st + R * 576 + rrow * 32;
        bytes = uint32_t(ng);
      }
      bulk_g2s(dst, src, bytes, bar);
    }
  };
  // Units are dealt round-robin to the CTA's warps: v = warp, warp+8, ...
  // with v = b*P + pass.  Advance (b, pass) by 8 units without dividing.
  auto advance = [](int& ub, int& upass, int P) {
    upass += kWarps;
    while (upass >= P) { upass -= P; ++ub; }
  };

  const int nwin = (G + kp.win_groups - 1) / kp.win_groups;
  uint32_t seq = 0;  // units consumed by this warp (stage = seq % nstages)

  // Window-0 prologue before the dependency wait: weights are immutable.
  int ib = 0, ip = 0;  // next unit to issue
  {
    const int wgn = min(kp.win_groups, G);
    const int P = (wgn + 31) / 32;
    ib = warp / P;
    ip = warp % P;
    for (int i = 0; i < nstages && ib < nb; ++i) {
      issue(ib, ip, 0, wgn, i);
      advance(ib, ip, P);
    }
  }

  constexpr int kOutPerThread = 4;
  int64_t oidx[kOutPerThread];
#pragma unroll
  for (int m = 0; m < kOutPerThread; ++m) {
    const int j = tid + m * blockDim.x;
    oidx[m] = (j < p.n_out) ? load_index(p.idx, j, p.idx_dtype) : -1;
  }

  griddep_wait();

#pragma unroll
  for (int m = 0; m < kOutPerThread; ++m) {
    const int j = tid + m * blockDim.x;
    if (j < p.n_out) xos[j] = (oidx[m] >= 0 && oidx[m] < p.K) ? load_as_float(p.x, oidx[m] * p.x_stride, p.x_dtype) : 0.f;
  }
  for (int j = tid + kOutPerThread * blockDim.x; j < p.n_out; j += blockDim.x) {
    const int64_t k = load_index(p.idx, j, p.idx_dtype);
    xos[j] = (k >= 0 && k < p.K) ? load_as_float(p.x, k * p.x_stride, p.x_dtype) : 0.f;
  }

  uint32_t magic_reg;
  asm volatile("mov.b32 %0, 0x4B000000;" : "=r"(magic_reg));

  for (int w = 0; w < nwin; ++w) {
    const int wg0 = w * kp.win_groups;
    const int wgn = min(kp.win_groups, G - wg0);
    const int P = (wgn + 31) / 32;
    const int pass_base = w * ((kp.win_groups + 31) / 32);
    if (w > 0) {
      __syncthreads();  // every warp is done with the previous window's x
      ib = warp / P;
      ip = warp % P;
      for (int i = 0; i < nstages && ib < nb; ++i) {
        issue(ib, ip, wg0, wgn, int((seq + i) % nstages));
        advance(ib, ip, P);
      }
    }
    stage_x_window(p, kp.vec_x, xs, xsum, wg0, wgn, tid, blockDim.x, lane);
    __syncthreads();
    int cb = warp / P, cp = warp % P;  // unit being consumed
    while (cb < nb) {
      const uint32_t slot = seq % nstages;
      uint64_t* bar = my_bars + slot;
      if (!mbar_wait(bar, (seq / nstages) & 1u, &s_abort)) {
        if (lane == 0) { s_abort = 1; atomicAdd(&g_gemv_timeouts, 1); }
        break;
      }
      const uint8_t* st = my_stages + slot * kStageBytes;
      const int gl = cp * 32 + lane;
      const int nr = min(R, nrows - cb * R);
      const bool lv = gl < wgn;
      uint4 cw[R];
      float cs[R], cz[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const bool ok = lv && r < nr;
        cw[r] = ok ? *reinterpret_cast<const uint4*>(st + r * 512 + lane * 16) : make_uint4(0u, 0u, 0u, 0u);
        cs[r] = ok ? __half2float(*reinterpret_cast<const __half*>(st + R * 512 + r * 64 + lane * 2)) : 0.f;
        cz[r] = ok ? __uint_as_float(uint32_t(st[R * 576 + r * 32 + lane]) | kMagic) - 8388608.0f : 0.f;
      }
      // Refill this stage with the unit nstages ahead before computing.
      if (ib < nb) {
        fence_proxy_async_smem();
        issue(ib, ip, wg0, wgn, int(slot));
        advance(ib, ip, P);
      }
      float acc[R];
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = 0.f;
      if (lv) {
        float2 xr[16];
        const float4* src = reinterpret_cast<const float4*>(xs + gl * kXpStride);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 f = src[c];
          xr[2 * c] = make_float2(f.x, f.y);
          xr[2 * c + 1] = make_float2(f.z, f.w);
        }
        const float xg = xsum[gl];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float q = group_qdot(cw[r], xr, magic_reg);
          q = fmaf(-cz[r], xg, q);
          acc[r] = q * cs[r];
        }
      }
      warp_transpose_reduce<R>(acc, lane);
      constexpr int kLeaderMask = (32 / R) - 1;
      const int rr = reduced_row<R>(lane);
      if ((lane & kLeaderMask) == 0 && rr < nr) red[(pass_base + cp) * kp.rows_max + cb * R + rr] = acc[0];
      ++seq;
      advance(cb, cp, P);
    }
  }
  // Outlier columns: warp v takes rows 8v.., 8 rows per batch, read from the
  // staged copy (or, when it could not be staged, straight from memory).
  if (p.n_out > 0) {
    if (ow_staged) {
      if (!mbar_wait(&s_ow_bar, 0, &s_abort)) {
        if (lane == 0) { s_abort = 1; atomicAdd(&g_gemv_timeouts, 1); }
      } else {
        // ragged tail (< 16 bytes) that the bulk copy left out
        for (int64_t bt = ow_a1 + tid; bt < ow_b1; bt += blockDim.x) ow_smem[bt - ow_a0] = ow_src[bt];
      }
    }
    __syncthreads();
    for (int i0 = warp * 8; i0 < nrows; i0 += kWarps * 8) {
      float oacc[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) oacc[r] = 0.f;
      for (int j0 = 0; j0 < p.n_out; j0 += 32) {
        const int j = j0 + lane;
        float ov[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          if (j < p.n_out && i0 + r < nrows) {
            if (ow_staged) {
              const int64_t off = (int64_t(i0 + r) * p.n_out + j) * ow_es + (ow_b0 - ow_a0);
              ov[r] = ow_es == 4 ? *reinterpret_cast<const float*>(ow_smem + off)
                      : p.ow_dtype == SPECTRA_DT_BF16
                          ? __uint_as_float(uint32_t(*reinterpret_cast<const uint16_t*>(ow_smem + off)) << 16)
                          : __half2float(*reinterpret_cast<const __half*>(ow_smem + off));
            } else {
              ov[r] = load_as_float(p.ow, (r_begin + i0 + r) * p.ow_rs + int64_t(j) * p.ow_cs, p.ow_dtype);
            }
          } else {
            ov[r] = 0.f;
          }
        }
        const float xo = j < p.n_out ? xos[j] : 0.f;
#pragma unroll
        for (int r = 0; r < 8; ++r) oacc[r] = fmaf(xo, ov[r], oacc[r]);
      }
      warp_transpose_reduce<8>(oacc, lane);
      const int rr = reduced_row<8>(lane);
      if ((lane & 3) == 0 && i0 + rr < nrows) ored[i0 + rr] = oacc[0];
    }
  }
  __syncthreads();
  for (int i = tid; i < nrows; i += blockDim.x) {
    float v = ored[i];
    for (int q = 0; q < kp.red_passes; ++q) v += red[q * kp.rows_max + i];
    const int64_t row = r_begin + i;
    if (p.bias) v += load_as_float(p.bias, row, p.bias_dtype);
    store_from_float(p.y, row * p.y_stride, p.y_dtype, v);
  }
}

template <int R, int ALIGN>
int launch_r(GemvKParams kp, const GemvPlan& pl, cudaStream_t st) {
  auto kern = gemv_w4a16_kernel<R, ALIGN>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  // Per-device caches: opt-in shared-memory size and resident CTAs per SM.
  static size_t set_bytes[kMaxDevices] = {};
  static int occ_cache[kMaxDevices][4] = {};  // keyed by smem bucket
  static int sms[kMaxDevices] = {};
  if (dev >= kMaxDevices) return SPECTRA_ERR_UNSUPPORTED;
  if (pl.smem > 48 * 1024 && set_bytes[dev] < pl.smem) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGemvMaxSmem));
    if (e != cudaSuccess) return cuda_status(e);
    set_bytes[dev] = kGemvMaxSmem;
  }
  if (sms[dev] == 0) {
    e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_status(e);
  }
  const int bucket = pl.smem <= 32 * 1024 ? 0 : pl.smem <= 64 * 1024 ? 1 : pl.smem <= 112 * 1024 ? 2 : 3;
  const size_t bucket_bytes[4] = {32 * 1024, 64 * 1024, 112 * 1024, kGemvMaxSmem};
  if (occ_cache[dev][bucket] == 0) {
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 256, bucket_bytes[bucket]);
    if (e != cudaSuccess) return cuda_status(e);
    occ_cache[dev][bucket] = occ < 1 ? 1 : occ;
  }
  const int64_t rows_cta = int64_t(pl.RG) * R;
  const int64_t max_grid = int64_t(sms[dev]) * occ_cache[dev][bucket];
  const int64_t want = (int64_t(kp.a.N) + rows_cta - 1) / rows_cta;
  const int grid = int(want < max_grid ? want : max_grid);
  // Multi-window K keeps per-row partial sums in shared memory across windows.
  const int max_tiles = int(((int64_t(kp.a.N) + grid - 1) / grid + rows_cta - 1) / rows_cta);
  size_t smem = pl.smem + (pl.win_groups < kp.a.K / kGroup ? size_t(max_tiles) * rows_cta * 4 : 0);
  if (smem > kGemvMaxSmem) return SPECTRA_ERR_UNSUPPORTED;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(unsigned(pl.threads));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, kp);
  return cuda_status(e);
}

struct DevInfo {
  int sms = 0;
};
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

template <int R>
int launch_bulk(GemvKParams kp, const GemvPlan& pl, cudaStream_t st) {
  auto kern = gemv_bulk_kernel<R>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev >= kMaxDevices) return SPECTRA_ERR_UNSUPPORTED;
  static bool attr_set[kMaxDevices] = {};
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGemvMaxSmem));
    if (e != cudaSuccess) return cuda_status(e);
    attr_set[dev] = true;
  }
  const GemvArgs& a = kp.a;
  constexpr int kWarps = 8;
  const int stage_bytes = R * (512 + 64 + 32);
  auto r16 = [](size_t v) { return (v + 15) & ~size_t(15); };
  const int G = a.K / kGroup;
  const int passes = (G + 31) / 32;
  int64_t grid = std::min<int64_t>((a.N + R - 1) / R, device_sms(dev));
  if (grid < 1) grid = 1;
  kp.rows_max = int((a.N + grid - 1) / grid);
  kp.red_passes = passes;
  const size_t tail = size_t(pl.win_groups) * kXpStride * 4 + r16(size_t(pl.win_groups) * 4) + r16(size_t(a.n_out) * 4) +
                      size_t(passes + 1) * kp.rows_max * 4;
  // Deepest ring (<= 4 stages per warp) that fits next to the staged x.
  int nst = 4;
  while (nst > 2 && size_t(kWarps) * nst * stage_bytes + r16(size_t(kWarps) * nst * 8) + tail > kGemvMaxSmem) --nst;
  kp.S = nst;
  kp.off_bars = kWarps * nst * stage_bytes;
  kp.off_xs = int(kp.off_bars + r16(size_t(kWarps) * nst * 8));
  kp.off_xsum = int(kp.off_xs + size_t(pl.win_groups) * kXpStride * 4);
  kp.off_xos = int(kp.off_xsum + r16(size_t(pl.win_groups) * 4));
  kp.off_red = int(kp.off_xos + r16(size_t(a.n_out) * 4));
  size_t smem = size_t(kp.off_red) + size_t(passes + 1) * kp.rows_max * 4;
  if (smem > kGemvMaxSmem) return SPECTRA_ERR_UNSUPPORTED;
  // Stage the outlier weights when they are one contiguous, 16-byte aligned
  // row-major block and the CTA's share fits (plus 32 bytes of alignment slack).
  kp.off_ow = -1;
  const int ow_es = a.ow_dtype == SPECTRA_DT_F32 ? 4 : 2;
  if (a.n_out > 0 && a.ow_cs == 1 && a.ow_rs == a.n_out && reinterpret_cast<uintptr_t>(a.ow) % 16 == 0) {
    const size_t need = r16(size_t(kp.rows_max) * a.n_out * ow_es + 32);
    if (r16(smem) + need <= kGemvMaxSmem) {
      kp.off_ow = int(r16(smem));
      smem = r16(smem) + need;
    }
  }

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, kp));
}

// The bulk path needs 16-byte aligned row segments of packed codes, scales
// and zeros (cp.async.bulk sizes and addresses are multiples of 16).
bool bulk_eligible(const GemvArgs& a) {
  const uintptr_t wp = reinterpret_cast<uintptr_t>(a.packed);
  const uintptr_t sp = reinterpret_cast<uintptr_t>(a.scales);
  const uintptr_t zp = reinterpret_cast<uintptr_t>(a.zeros);
  const int G = a.K / kGroup;
  return (G % 16) == 0 && wp % 16 == 0 && a.w_rs % 16 == 0 && sp % 16 == 0 && a.s_cs == 1 && a.s_rs % 8 == 0 &&
         zp % 16 == 0 && a.z_cs == 1 && a.z_rs % 16 == 0 && a.w_rs >= 0 && a.s_rs >= 0 && a.z_rs >= 0;
}

template <int ALIGN>
int launch_align(const GemvKParams& kp, const GemvPlan& pl, cudaStream_t st) {
  switch (pl.R) {
    case 4: return launch_r<4, ALIGN>(kp, pl, st);
    case 2: return launch_r<2, ALIGN>(kp, pl, st);
    default: return launch_r<1, ALIGN>(kp, pl, st);
  }
}

}  // namespace

GemvPlan plan_gemv(int64_t N, int64_t K, int64_t n_out) {
  GemvPlan pl{};
  const int G = int(K / kGroup);
  pl.win_groups = std::min(((G + 31) / 32) * 32, kGemvMaxWindowGroups);
  const int P = (pl.win_groups + 31) / 32;          // passes per window
  const int per = (P + 7) / 8;                       // passes per warp
  pl.S = (P + per - 1) / per;                        // k-split warps (<= 8)
  pl.RG = std::max(1, 8 / pl.S);
  pl.threads = pl.S * pl.RG * 32;
  // Rows per warp: the largest R (<= 4: the double-buffered weight registers
  // of R=8 do not fit in 128 registers) whose tile (RG*R rows) still fits in
  // the rows each of ~2 CTAs per SM on 148 SMs will own.
  const int64_t rows_per_cta = std::max<int64_t>(1, N / (148 * 2));
  pl.R = 1;
  for (int r : {4, 2}) {
    if (int64_t(pl.RG) * r <= rows_per_cta) { pl.R = r; break; }
  }
  const int64_t rows = int64_t(pl.RG) * pl.R;
  pl.grid = (N + rows - 1) / rows;
  pl.smem = size_t(pl.win_groups) * kXpStride * 4 + size_t(pl.win_groups) * 4 +
            size_t((n_out + 3) & ~3) * 4 + 2 * size_t(pl.S) * rows * 4;
  return pl;
}

int launch_gemv(const GemvArgs& a, cudaStream_t st) {
  const GemvPlan pl = plan_gemv(a.N, a.K, a.n_out);
  if (pl.smem > kGemvMaxSmem) return SPECTRA_ERR_UNSUPPORTED;
  GemvKParams kp;
  kp.a = a;
  kp.S = pl.S;
  kp.RG = pl.RG;
  kp.win_groups = pl.win_groups;
  kp.smem_xs_floats = pl.win_groups * kXpStride;
  kp.vec_x = a.x_stride == 1 && (reinterpret_cast<uintptr_t>(a.x) % 16) == 0 &&
             (a.x_dtype == SPECTRA_DT_BF16 || a.x_dtype == SPECTRA_DT_F16);
  if (bulk_eligible(a) && bulk_path_enabled()) return launch_bulk<8>(kp, pl, st);
  const uintptr_t base = reinterpret_cast<uintptr_t>(a.packed);
  const int align = ((base | uintptr_t(a.w_rs)) % 16 == 0) ? 16 : (((base | uintptr_t(a.w_rs)) % 4 == 0) ? 4 : 1);
  if (align == 16) return launch_align<16>(kp, pl, st);
  if (align == 4) return launch_align<4>(kp, pl, st);
  return launch_align<1>(kp, pl, st);
}

}  // namespace spectra
