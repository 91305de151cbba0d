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
#include "gemv_mma.cuh"

namespace spectra {

namespace {

constexpr int kXpStride = 36;  // floats per staged group: 32 + 4 pad (bank-conflict-free LDS.128)

struct GemvKParams {
  GemvArgs a;
  int S, RG, win_groups;
  bool vec_x;          // x contiguous, 16-byte aligned, fp16/bf16
  int rows_max;        // max rows of one CTA (bulk kernel)
  int off_xs, off_xsum, off_xos, off_red;  // dynamic shared-memory layout
  int red_passes;      // partial-sum slots per row (passes or 8-group blocks of K)
  int off_ow;          // shared copy of this CTA's outlier-weight rows (-1: not staged)
  int smem_xs_floats;  // win_groups * kXpStride
};

// Staged-x slot s = j*8 + i*2 + h of a group holds the code of word j
// (bytes 4j..4j+3), half-word h, nibble i inside that half-word.
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

__device__ int g_gemv_timeouts;  // stuck pipeline waits since load (diagnostic)

// ---------------------------------------------------------------------------
// Rows kernel (main path).
//
// Warp (ks, rg) of a CTA owns passes ks, ks+S, ... of each K-window and the
// rows of row-group rg.  For each of its passes it loads the staged x of its
// lane's group into registers once, then streams every row of its row-group
// in batches of R rows, keeping the next batch's loads in flight.  The
// per-(pass, row) partial sums go to shared memory; one barrier at the end
// precedes the fixed-order sum over passes (deterministic).
// ---------------------------------------------------------------------------
template <int R, int ALIGN>
__global__ void __launch_bounds__(256, 2) gemv_rows_kernel(const __grid_constant__ GemvKParams kp) {
  using namespace sm100;
  const GemvArgs& p = kp.a;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  float* xs = reinterpret_cast<float*>(smem_raw + kp.off_xs);
  float* xsum = reinterpret_cast<float*>(smem_raw + kp.off_xsum);
  float* xos = reinterpret_cast<float*>(smem_raw + kp.off_xos);
  float* red = reinterpret_cast<float*>(smem_raw + kp.off_red);  // [passes][rows_max]
  float* ored = red + kp.red_passes * kp.rows_max;               // [rows_max]
  __shared__ int s_abort;
  __shared__ __align__(8) uint64_t s_ow_bar;

  griddep_launch_dependents();

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int S = kp.S;
  const int ks = warp % S;
  const int rg = warp / S;
  const int64_t r_begin = (int64_t(p.N) * blockIdx.x) / gridDim.x;
  const int64_t r_end = (int64_t(p.N) * (blockIdx.x + 1)) / gridDim.x;
  const int nrows = int(r_end - r_begin);
  const int gb = (nrows * rg) / kp.RG;        // row-group rows, relative to r_begin
  const int ge = (nrows * (rg + 1)) / kp.RG;
  const int G = p.K / kGroup;

  if (tid == 0) s_abort = 0;
  for (int i = tid; i < (kp.red_passes + 1) * kp.rows_max; i += blockDim.x) red[i] = 0.f;

  // Outlier-weight rows of this CTA: one bulk copy of the aligned body.
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

  // Weight registers: the batch being computed (c*) and the next one (n*).
  uint4 nw[R];
  float ns[R], nz[R];
  auto load_batch = [&](int g, int row_rel) {  // g: absolute group; rows r_begin+row_rel..
    const int64_t row0 = r_begin + row_rel;
    const uint8_t* wp = p.packed + row0 * p.w_rs + int64_t(g) * kGroupBytes;
    const __half* sp = p.scales + row0 * p.s_rs + int64_t(g) * p.s_cs;
    const uint8_t* zp = p.zeros + row0 * p.z_rs + int64_t(g) * p.z_cs;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (row_rel + r < ge) {
        nw[r] = load_group16<ALIGN>(wp + r * p.w_rs);
        ns[r] = __half2float(__ldg(sp + r * p.s_rs));
        nz[r] = __uint_as_float(uint32_t(__ldg(zp + r * p.z_rs)) | kMagic) - 8388608.0f;
      } else {
        nw[r] = make_uint4(0u, 0u, 0u, 0u);
        ns[r] = 0.f;
        nz[r] = 0.f;
      }
    }
  };

#pragma unroll
  for (int r = 0; r < R; ++r) { nw[r] = make_uint4(0u, 0u, 0u, 0u); ns[r] = 0.f; nz[r] = 0.f; }
  // First batch of window 0, before the dependency wait (weights only).
  {
    const int wgn0 = min(kp.win_groups, G);
    const int gl = ks * 32 + lane;
    if (gl < wgn0 && gb < ge) load_batch(gl, gb);
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

  const int nwin = (G + kp.win_groups - 1) / kp.win_groups;
  for (int w = 0; w < nwin; ++w) {
    const int wg0 = w * kp.win_groups;
    const int wgn = min(kp.win_groups, G - wg0);
    const int wpass = (wgn + 31) / 32;
    const int pass_base = w * (kp.win_groups / 32);
    if (w > 0) __syncthreads();  // every warp is done with the previous window's x
    stage_x_window(p, kp.vec_x, xs, xsum, wg0, wgn, tid, blockDim.x, lane);
    __syncthreads();
    if (w > 0 && ks * 32 + lane < wgn && gb < ge) load_batch(wg0 + ks * 32 + lane, gb);

    for (int pp = ks; pp < wpass; pp += S) {
      const int gl = pp * 32 + lane;
      const bool lv = gl < wgn;
      float2 xr[16];
      float xg = 0.f;
      if (lv) {
        const float4* src = reinterpret_cast<const float4*>(xs + gl * kXpStride);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 f = src[c];
          xr[2 * c] = make_float2(f.x, f.y);
          xr[2 * c + 1] = make_float2(f.z, f.w);
        }
        xg = xsum[gl];
      }
      for (int rb = gb; rb < ge; rb += R) {
        uint4 cw[R];
        float cs[R], cz[R];
#pragma unroll
        for (int r = 0; r < R; ++r) { cw[r] = nw[r]; cs[r] = ns[r]; cz[r] = nz[r]; }
        // Keep the next batch in flight: next rows of this pass, else the
        // first rows of this warp's next pass in the window.
        if (rb + R < ge) {
          if (lv) load_batch(wg0 + gl, rb + R);
        } else if (pp + S < wpass) {
          const int gn = (pp + S) * 32 + lane;
          if (gn < wgn) load_batch(wg0 + gn, gb);
        }
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float q = lv ? group_qdot(cw[r], xr, magic_reg) : 0.f;
          q = fmaf(-cz[r], xg, q);
          acc[r] = q * cs[r];
        }
        warp_transpose_reduce<R>(acc, lane);
        constexpr int kLeaderMask = (32 / R) - 1;
        const int rr = reduced_row<R>(lane);
        if ((lane & kLeaderMask) == 0 && rb + rr < ge) red[(pass_base + pp) * kp.rows_max + rb + rr] = acc[0];
      }
    }
  }

  // Outlier columns (staged copy if available), 8 rows per warp batch.
  if (p.n_out > 0) {
    if (ow_staged) {
      if (!mbar_wait(&s_ow_bar, 0, &s_abort)) {
        if (lane == 0) { s_abort = 1; atomicAdd(&g_gemv_timeouts, 1); }
      } else {
        for (int64_t bt = ow_a1 + tid; bt < ow_b1; bt += blockDim.x) ow_smem[bt - ow_a0] = ow_src[bt];
      }
    }
    __syncthreads();
    for (int i0 = warp * 8; i0 < nrows; i0 += nwarps * 8) {
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
int launch_rows(GemvKParams kp, const GemvPlan& pl, cudaStream_t st) {
  auto kern = gemv_rows_kernel<R, ALIGN>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev >= kMaxDevices) return SPECTRA_ERR_UNSUPPORTED;
  static PerContextOnce attrs;
  e = attrs.run(dev, [&] { return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGemvMaxSmem)); });
  if (e != cudaSuccess) return cuda_status(e);
  const GemvArgs& a = kp.a;
  auto r16 = [](size_t v) { return (v + 15) & ~size_t(15); };
  const int G = a.K / kGroup;
  const int passes = kp.red_passes = (G + 31) / 32;
  (void)passes;
  const size_t xs_bytes = size_t(pl.win_groups) * kXpStride * 4 + r16(size_t(pl.win_groups) * 4) + r16(size_t(a.n_out) * 4);
  // two CTAs per SM when the staged x leaves room, else one
  const int per_sm = xs_bytes + 16 * 1024 <= 100 * 1024 ? 2 : 1;
  const int64_t rows_group = int64_t(pl.RG) * R;
  int64_t grid = std::min<int64_t>((a.N + rows_group - 1) / rows_group, int64_t(device_sms(dev)) * per_sm);
  if (grid < 1) grid = 1;
  kp.rows_max = int((a.N + grid - 1) / grid);
  kp.off_xs = 0;
  kp.off_xsum = int(size_t(pl.win_groups) * kXpStride * 4);
  kp.off_xos = int(kp.off_xsum + r16(size_t(pl.win_groups) * 4));
  kp.off_red = int(kp.off_xos + r16(size_t(a.n_out) * 4));
  size_t smem = size_t(kp.off_red) + size_t(kp.red_passes + 1) * kp.rows_max * 4;
  kp.off_ow = -1;
  const int ow_es = a.ow_dtype == SPECTRA_DT_F32 ? 4 : 2;
  if (a.n_out > 0 && a.ow_cs == 1 && a.ow_rs == a.n_out && reinterpret_cast<uintptr_t>(a.ow) % 16 == 0) {
    const size_t need = r16(size_t(kp.rows_max) * a.n_out * ow_es + 32);
    if (r16(smem) + need <= (per_sm == 2 ? 110 * 1024 : kGemvMaxSmem)) {
      kp.off_ow = int(r16(smem));
      smem = r16(smem) + need;
    }
  }
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
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, kp));
}

template <int ALIGN>
int launch_rows_align(const GemvKParams& kp, const GemvPlan& pl, cudaStream_t st) {
  switch (pl.R) {
    case 4: return launch_rows<4, ALIGN>(kp, pl, st);
    case 2: return launch_rows<2, ALIGN>(kp, pl, st);
    default: return launch_rows<1, ALIGN>(kp, pl, st);
  }
}

// ---------------------------------------------------------------------------
// Tensor-core kernel (main path for bf16 / fp16 activations).
//
// The dot products run on mma.sync.m16n8k16 with fp32 accumulation:
//   A (16 x 16): codes of 16 weight rows, as 16-bit pairs OFF+q built with one
//                LOP3 (plus a shift) per pair -- exact small integers;
//   B (16 x 8):  block-diagonal x -- column n carries x only in the k-slots
//                that belong to quantisation group n of an 8-group block, so
//                after the 16 MMAs of a block D[row][n] is group n's dot;
//   thread (g, c) loads the codes of groups 2c and 2c+1 of rows g and g+8 and
//   ends up holding exactly their four dots, to which it applies the group's
//   scale and zero point in fp32:  s * (D - (OFF + z) * X_g),  X_g = sum of x.
// A unit of work is 16 rows x 8 groups (4096 codes); a CTA's units are dealt
// round-robin to its warps and each unit's partial row sums go to shared
// memory, summed in a fixed order at the end (deterministic).
// ---------------------------------------------------------------------------
struct MmaUnitRegs {
  uint4 w[4];     // codes: [grpA row g, grpA row g+8, grpB row g, grpB row g+8]
  uint32_t s[2];  // scales (fp16 pairs {grpA, grpB}) of rows g, g+8
  uint32_t z[2];  // zero points (byte pairs {grpA, grpB}) of rows g, g+8
};

template <bool BF16, int ALIGN>
__global__ void __launch_bounds__(256, 2) gemv_mma_kernel(const __grid_constant__ GemvKParams kp) {
  using namespace sm100;
  const GemvArgs& p = kp.a;
  constexpr uint32_t kMagic2 = BF16 ? 0x41804180u : 0x4C004C00u;  // 16.0 in both halves
  constexpr float kOff = 16.0f;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint32_t* xp = reinterpret_cast<uint32_t*>(smem_raw + kp.off_xs);  // [win_groups + 1][16] pairs (+ zero pad)
  float* xsum = reinterpret_cast<float*>(smem_raw + kp.off_xsum);     // [win_groups]
  float* xos = reinterpret_cast<float*>(smem_raw + kp.off_xos);
  float* red = reinterpret_cast<float*>(smem_raw + kp.off_red);       // [G/8 blocks][rows_max]
  float* ored = red + kp.red_passes * kp.rows_max;                    // [rows_max]
  __shared__ int s_abort;
  __shared__ __align__(8) uint64_t s_ow_bar;

  griddep_launch_dependents();

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  // 16-row blocks are dealt to CTAs evenly; only the matrix's last block is ragged.
  const int64_t nblk = (int64_t(p.N) + 15) / 16;
  const int64_t b0 = (nblk * blockIdx.x) / gridDim.x;
  const int64_t b1 = (nblk * (blockIdx.x + 1)) / gridDim.x;
  const int nrb = int(b1 - b0);
  const int64_t r_begin = b0 * 16;
  const int64_t r_end = (int64_t(p.N) < b1 * 16) ? int64_t(p.N) : b1 * 16;
  const int nrows = int(r_end - r_begin);
  const int G = p.K / kGroup;

  if (tid == 0) s_abort = 0;
  for (int i = tid; i < (kp.red_passes + 1) * kp.rows_max; i += blockDim.x) red[i] = 0.f;

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

  // Load unit (rbi, kb): rows r_begin + 16*rbi + {g, g+8}, groups 8*kb + {2c, 2c+1} of the window.
  auto load_unit = [&](MmaUnitRegs& u, int rbi, int kb, int wg0, int wgn) {
    const int gA = kb * 8 + 2 * c;
    const bool va = gA < wgn, vb = gA + 1 < wgn;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t row = r_begin + rbi * 16 + g + 8 * h;
      const bool vr = row < r_end;
      const int64_t gabs = int64_t(wg0 + gA);
      const uint8_t* wp = p.packed + row * p.w_rs + gabs * kGroupBytes;
      u.w[h] = (vr && va) ? load_group16<ALIGN>(wp) : make_uint4(0u, 0u, 0u, 0u);
      u.w[2 + h] = (vr && vb) ? load_group16<ALIGN>(wp + kGroupBytes) : make_uint4(0u, 0u, 0u, 0u);
      const uint16_t* sp = reinterpret_cast<const uint16_t*>(p.scales) + row * p.s_rs + gabs * p.s_cs;
      const uint8_t* zp = p.zeros + row * p.z_rs + gabs * p.z_cs;
      const uint32_t sa = (vr && va) ? uint32_t(__ldg(sp)) : 0u;
      const uint32_t sb = (vr && vb) ? uint32_t(__ldg(sp + p.s_cs)) : 0u;
      const uint32_t za = (vr && va) ? uint32_t(__ldg(zp)) : 0u;
      const uint32_t zb = (vr && vb) ? uint32_t(__ldg(zp + p.z_cs)) : 0u;
      u.s[h] = sa | (sb << 16);
      u.z[h] = za | (zb << 16);
    }
  };

  constexpr int kOutPerThread = 4;
  int64_t oidx[kOutPerThread];
#pragma unroll
  for (int m = 0; m < kOutPerThread; ++m) {
    const int j = tid + m * blockDim.x;
    oidx[m] = (j < p.n_out) ? load_index(p.idx, j, p.idx_dtype) : -1;
  }

  const int nwin = (G + kp.win_groups - 1) / kp.win_groups;
  MmaUnitRegs nxt;
  // first unit of window 0 before the dependency wait (weights only)
  int cb = 0, ck = 0;  // unit being consumed: row-block cb, 8-group block ck
  {
    const int wgn = min(kp.win_groups, G);
    const int KB = (wgn + 7) / 8;
    cb = warp / KB;
    ck = warp % KB;
    if (cb < nrb) load_unit(nxt, cb, ck, 0, wgn);
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
  asm volatile("mov.b32 %0, %1;" : "=r"(magic_reg) : "n"(kMagic2));
  const uint16_t* xh = reinterpret_cast<const uint16_t*>(p.x);

  for (int w = 0; w < nwin; ++w) {
    const int wg0 = w * kp.win_groups;
    const int wgn = min(kp.win_groups, G - wg0);
    const int KB = (wgn + 7) / 8;
    const int kb_base = w * (kp.win_groups / 8);
    if (w > 0) {
      __syncthreads();  // every warp is done with the previous window's x
      cb = warp / KB;
      ck = warp % KB;
      if (cb < nrb) load_unit(nxt, cb, ck, wg0, wgn);
    }
    // Stage x as 16 pairs per group in MMA order (x in the MMA's dtype is
    // copied bit-exactly) and the per-group sums X_g, plus a zero pad group.
    const int nstage = (wgn + 1) * 16;
    for (int e0 = tid - lane; e0 < nstage; e0 += blockDim.x) {  // warp-uniform trip count
      const int e = e0 + lane;
      const int gl = e >> 4, kk = e & 15;
      uint32_t v = 0u;
      float sum2 = 0.f;
      if (gl < wgn) {
        const int64_t kbase = int64_t(wg0 + gl) * kGroup;
        const int64_t klo = kbase + pair_k(kk, 0, p.layout), khi = kbase + pair_k(kk, 1, p.layout);
        const uint32_t lo = __ldg(xh + klo * p.x_stride), hi = __ldg(xh + khi * p.x_stride);
        v = lo | (hi << 16);
        sum2 = BF16 ? (__uint_as_float(lo << 16) + __uint_as_float(hi << 16))
                    : (__half2float(__ushort_as_half(uint16_t(lo))) + __half2float(__ushort_as_half(uint16_t(hi))));
      }
      if (e < nstage) xp[e] = v;
      // 16 consecutive lanes hold one group's pairs
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) sum2 += __shfl_xor_sync(0xffffffffu, sum2, o);
      if ((lane & 15) == 0 && gl < wgn) xsum[gl] = sum2;
    }
    __syncthreads();

    const uint32_t* xzero = xp + wgn * 16;
    const bool lane_a = (lane % 9) == 0;        // lanes 0, 9, 18, 27: B column 2c
    const bool lane_b = (lane % 9) == 4;        // lanes 4, 13, 22, 31: B column 2c+1
    while (cb < nrb) {
      MmaUnitRegs cur = nxt;
      const int rbi = cb, kbi = ck;
      // next unit of this warp: 8-group block ck + nwarps (row-block advances)
      ck += nwarps;
      while (ck >= KB) { ck -= KB; ++cb; }
      if (cb < nrb) load_unit(nxt, cb, ck, wg0, wgn);

      const int gA = kbi * 8 + 2 * c;  // this thread's groups (window-relative)
      // B fragments: x pairs of group gA (lane_a) or gA+1 (lane_b), else zero
      const uint4* srcA = reinterpret_cast<const uint4*>(lane_a && gA < wgn ? xp + gA * 16 : xzero);
      const uint4* srcB = reinterpret_cast<const uint4*>(lane_b && gA + 1 < wgn ? xp + (gA + 1) * 16 : xzero);
      uint32_t bA[16], bB[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 ta = srcA[q], tb = srcB[q];
        bA[4 * q] = ta.x; bA[4 * q + 1] = ta.y; bA[4 * q + 2] = ta.z; bA[4 * q + 3] = ta.w;
        bB[4 * q] = tb.x; bB[4 * q + 1] = tb.y; bB[4 * q + 2] = tb.z; bB[4 * q + 3] = tb.w;
      }
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t wa[4][4] = {{cur.w[0].x, cur.w[0].y, cur.w[0].z, cur.w[0].w},
                                 {cur.w[1].x, cur.w[1].y, cur.w[1].z, cur.w[1].w},
                                 {cur.w[2].x, cur.w[2].y, cur.w[2].z, cur.w[2].w},
                                 {cur.w[3].x, cur.w[3].y, cur.w[3].z, cur.w[3].w}};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#define SPECTRA_MMA_STEP(T)                                                                                   \
  mma16816<BF16>(d, pair_code<BF16, T>(wa[0][j], magic_reg), pair_code<BF16, T>(wa[1][j], magic_reg),           \
                 pair_code<BF16, T>(wa[2][j], magic_reg), pair_code<BF16, T>(wa[3][j], magic_reg),              \
                 bA[4 * j + T], bB[4 * j + T]);
        SPECTRA_MMA_STEP(0) SPECTRA_MMA_STEP(1) SPECTRA_MMA_STEP(2) SPECTRA_MMA_STEP(3)
#undef SPECTRA_MMA_STEP
      }
      // d = {D[g][gA], D[g][gA+1], D[g+8][gA], D[g+8][gA+1]}
      const float XA = (gA < wgn) ? xsum[gA] : 0.f;
      const float XB = (gA + 1 < wgn) ? xsum[gA + 1] : 0.f;
      float rs[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float sa = __half2float(__ushort_as_half(uint16_t(cur.s[h] & 0xFFFFu)));
        const float sb = __half2float(__ushort_as_half(uint16_t(cur.s[h] >> 16)));
        const float za = __uint_as_float((cur.z[h] & 0xFFu) | kMagic) - 8388608.0f + kOff;
        const float zb = __uint_as_float(((cur.z[h] >> 16) & 0xFFu) | kMagic) - 8388608.0f + kOff;
        rs[h] = sa * fmaf(-za, XA, d[2 * h]) + sb * fmaf(-zb, XB, d[2 * h + 1]);
      }
      // sum the 4 threads of a quad: rows g and g+8 over this unit's 8 groups
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
        rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
      }
      if (c == 0) {
        float* rr = red + (kb_base + kbi) * kp.rows_max + rbi * 16 + g;
        if (rbi * 16 + g < nrows) rr[0] = rs[0];
        if (rbi * 16 + g + 8 < nrows) rr[8] = rs[1];
      }
    }
  }

  // Outlier columns (staged copy if available), 8 rows per warp batch.
  if (p.n_out > 0) {
    if (ow_staged) {
      if (!mbar_wait(&s_ow_bar, 0, &s_abort)) {
        if (lane == 0) { s_abort = 1; atomicAdd(&g_gemv_timeouts, 1); }
      } else {
        for (int64_t bt = ow_a1 + tid; bt < ow_b1; bt += blockDim.x) ow_smem[bt - ow_a0] = ow_src[bt];
      }
    }
    __syncthreads();
    const bool ow_bf16 = p.ow_dtype == SPECTRA_DT_BF16;
    for (int i0 = warp * 8; i0 < nrows; i0 += nwarps * 8) {
      float oacc[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) oacc[r] = 0.f;
      for (int j0 = 0; j0 < p.n_out; j0 += 32) {
        const int j = j0 + lane;
        float ov[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          ov[r] = 0.f;
          if (j < p.n_out && i0 + r < nrows) {
            if (ow_staged) {
              const uint8_t* q = ow_smem + (int64_t(i0 + r) * p.n_out + j) * ow_es + (ow_b0 - ow_a0);
              ov[r] = ow_es == 4 ? *reinterpret_cast<const float*>(q)
                      : ow_bf16 ? __uint_as_float(uint32_t(*reinterpret_cast<const uint16_t*>(q)) << 16)
                                : __half2float(*reinterpret_cast<const __half*>(q));
            } else {
              ov[r] = load_as_float(p.ow, (r_begin + i0 + r) * p.ow_rs + int64_t(j) * p.ow_cs, p.ow_dtype);
            }
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
    const int64_t row = r_begin + i;
    float v = ored[i];
    for (int q = 0; q < kp.red_passes; ++q) v += red[q * kp.rows_max + i];
    if (p.bias) v += load_as_float(p.bias, row, p.bias_dtype);
    store_from_float(p.y, row * p.y_stride, p.y_dtype, v);
  }
}

template <bool BF16, int ALIGN>
int launch_mma(GemvKParams kp, const GemvPlan& pl, cudaStream_t st) {
  auto kern = gemv_mma_kernel<BF16, ALIGN>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev >= kMaxDevices) return SPECTRA_ERR_UNSUPPORTED;
  static PerContextOnce attrs;
  e = attrs.run(dev, [&] { return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGemvMaxSmem)); });
  if (e != cudaSuccess) return cuda_status(e);
  const GemvArgs& a = kp.a;
  auto r16 = [](size_t v) { return (v + 15) & ~size_t(15); };
  const int G = a.K / kGroup;
  kp.red_passes = (G + 7) / 8;  // partial-sum slots: one per 8-group block of K
  const int64_t nblk = (int64_t(a.N) + 15) / 16;
  int64_t grid = std::min<int64_t>(nblk, int64_t(device_sms(dev)) * 2);
  if (grid < 1) grid = 1;
  kp.rows_max = int(((nblk + grid - 1) / grid) * 16);
  kp.off_xs = 0;
  kp.off_xsum = int(r16(size_t(pl.win_groups + 1) * 64));
  kp.off_xos = int(kp.off_xsum + r16(size_t(pl.win_groups) * 4));
  kp.off_red = int(kp.off_xos + r16(size_t(a.n_out) * 4));
  size_t smem = size_t(kp.off_red) + size_t(kp.red_passes + 1) * kp.rows_max * 4;
  kp.off_ow = -1;
  const int ow_es = a.ow_dtype == SPECTRA_DT_F32 ? 4 : 2;
  if (a.n_out > 0 && a.ow_cs == 1 && a.ow_rs == a.n_out && reinterpret_cast<uintptr_t>(a.ow) % 16 == 0) {
    const size_t need = r16(size_t(kp.rows_max) * a.n_out * ow_es + 32);
    if (r16(smem) + need <= 110 * 1024) {
      kp.off_ow = int(r16(smem));
      smem = r16(smem) + need;
    }
  }
  if (smem > kGemvMaxSmem) return SPECTRA_ERR_UNSUPPORTED;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, kp));
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
  const uintptr_t base = reinterpret_cast<uintptr_t>(a.packed);
  const int align = ((base | uintptr_t(a.w_rs)) % 16 == 0) ? 16 : (((base | uintptr_t(a.w_rs)) % 4 == 0) ? 4 : 1);
  // bf16 / fp16 activations: tensor-core kernel; fp32 activations keep the
  // exact CUDA-core kernel (an fp32 x cannot be an MMA operand unrounded).
  if (mma_path_enabled() && (a.x_dtype == SPECTRA_DT_BF16 || a.x_dtype == SPECTRA_DT_F16)) {
    const int r = launch_gemv_pf(a, st);
    if (r != SPECTRA_ERR_UNSUPPORTED) return r;
    const bool bf = a.x_dtype == SPECTRA_DT_BF16;
    if (align == 16) return bf ? launch_mma<true, 16>(kp, pl, st) : launch_mma<false, 16>(kp, pl, st);
    if (align == 4) return bf ? launch_mma<true, 4>(kp, pl, st) : launch_mma<false, 4>(kp, pl, st);
    return bf ? launch_mma<true, 1>(kp, pl, st) : launch_mma<false, 1>(kp, pl, st);
  }
  if (align == 16) return launch_rows_align<16>(kp, pl, st);
  if (align == 4) return launch_rows_align<4>(kp, pl, st);
  return launch_rows_align<1>(kp, pl, st);
}

int gemv_timeouts(long long* out, bool reset) { return read_timeout_counter(g_gemv_timeouts, out, reset); }

}  // namespace spectra
