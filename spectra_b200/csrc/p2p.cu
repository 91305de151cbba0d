// All-gather of an N-sharded layer's output slices over NVLink peer memory,
// for sm_100a: the exchange step of spectra_b200.sharded in place of an NCCL
// all-gather (the reference has no multi-GPU path; this is the collective the
// column-sharded large layers need, one per layer call).
//
// Every rank owns an exchange buffer of the same layout, allocated with
// cudaMalloc and opened in every peer's address space through CUDA IPC
// handles (plain peer memory, no NVLS):
//   [kP2pSignalBytes]  epoch flags [rank][cta]: flag (r, b) = the last call
//                      whose chunk b rank r has finished pushing here
//   [2][world][pitch]  the gathered slices, double-buffered by call parity.
// The slice (pitch bytes) is cut into G chunks, G a function of the slice size
// alone (so it is the same on every rank).  CTA b of one launch:
//   1. pushes chunk b of this rank's slice into region [parity][rank] of every
//      peer's buffer with 16-byte stores over NVLink (st.global to peer
//      addresses, no TMA);
//   2. after a CTA barrier, writes the call's epoch into flag (rank, b) of
//      every peer (release, system scope: the barrier orders the CTA's stores
//      before it; lane r of warp 0 writes peer r's, all in one instruction);
//   3. waits until flag (r, b) of its own buffer holds the epoch for every
//      peer r (lane r polls peer r's; acquire, system scope; bounded by
//      wait_limit_ns -- on time-out
//      it counts the event in g_p2p_timeouts, read by spectra_device_timeouts,
//      and returns), then copies chunk b of every rank's slice into the [M, N]
//      output: this rank's from `src`, each peer's from its region.
// No CTA waits for another CTA of the same launch: the only waits are on the
// peers' CTAs of the same index.  The epoch of CTA b is its own call counter in
// `state` (device memory, so the kernel replays from a CUDA graph); every CTA
// counts the same calls, so parity agrees across CTAs and ranks.
// Why two regions: a rank can run one call ahead of a slow peer (it needs only
// the peer's flag, which the peer sends before its own copy-out), so its next
// push must not land where the slow peer is still reading; two calls ahead is
// impossible, since that needs the peer's next flag, sent only after the peer's
// copy-out has finished (stream order).
#include <algorithm>

#include "common.cuh"
#include "p2p.h"
#include "sm100_ptx.cuh"

namespace spectra {

namespace {

__device__ int g_p2p_timeouts;  // waits for a peer's flag that gave up (diagnostic)

constexpr int kP2pThreads = 256;

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kP2pThreads) p2p_allgather_kernel(P2pArgs a) {
  // the next kernel on this stream may start its own prologue (a GEMV's weight
  // prefetch) now; it reads nothing of ours before its griddepcontrol.wait
  sm100::pdl_trigger();
  sm100::pdl_wait();  // src is the previous kernel's output
  __shared__ int s_epoch, s_ok;
  const int b = blockIdx.x;
  if (threadIdx.x == 0) {
    s_epoch = a.state[b] + 1;  // only this CTA touches its counter
    a.state[b] = s_epoch;
  }
  __syncthreads();
  const int epoch = s_epoch;
  const int64_t region0 = kP2pSignalBytes + int64_t(epoch & 1) * a.world * a.slice_pitch;
  const int64_t n16 = a.slice_pitch / 16;
  const int64_t u0 = n16 * b / gridDim.x, u1 = n16 * (b + 1) / gridDim.x;

  // 1. chunk b of this rank's slice into every peer's region [parity][rank]
  const uint4* src = reinterpret_cast<const uint4*>(a.src);
  const int64_t dst_off = region0 + int64_t(a.rank) * a.slice_pitch;
  for (int64_t i = u0 + threadIdx.x; i < u1; i += kP2pThreads) {
    const uint4 v = __ldcg(src + i);
#pragma unroll 1
    for (int r = 0; r < a.world; ++r)
      if (r != a.rank) __stcg(reinterpret_cast<uint4*>(a.peer[r] + dst_off) + i, v);
  }
  __syncthreads();

  // 2./3. flag the chunk to every peer, then wait for theirs: lane r of warp 0
  // serves peer r, so the world-1 release stores go out as one instruction
  // (one system-scope fence for all peers, not one per peer in turn) and the
  // peers' flags are polled side by side
  if (threadIdx.x < 32) {
    const int r = threadIdx.x;
    const bool peer_lane = r < a.world && r != a.rank;
    if (peer_lane) st_release_sys(reinterpret_cast<int*>(a.peer[r]) + a.rank * kP2pMaxCtas + b, epoch);
    const int* flags = reinterpret_cast<const int*>(a.peer[a.rank]);
    bool ok = true;
    if (peer_lane) {
      uint64_t t0 = 0;
      for (uint32_t polls = 1; int(unsigned(ld_acquire_sys(flags + r * kP2pMaxCtas + b)) - unsigned(epoch)) < 0;
           ++polls) {
        if ((polls & 63) == 0) {
          const uint64_t now = sm100::global_ns();
          if (t0 == 0) {
            t0 = now;
          } else if (now - t0 > a.wait_limit_ns) {
            ok = false;
            break;
          }
        }
      }
    }
    ok = __all_sync(0xffffffffu, ok);
    if (r == 0) {
      if (!ok) atomicAdd(&g_p2p_timeouts, 1);  // once per CTA that gave up
      s_ok = ok ? 1 : 0;
    }
  }
  __syncthreads();
  if (!s_ok) return;  // output undefined; the host reads the counter between steps

  // chunk b of every rank's slice into the [M, N] output
  const int eb = a.elem_bytes;
  const int64_t slice_bytes = int64_t(a.M) * a.ns * eb;
  const int per16 = 16 / eb;
  for (int r = 0; r < a.world; ++r) {
    const int64_t col0 = int64_t(r) * a.ns;
    if (col0 >= a.N) break;  // empty shards
    const uint4* from = r == a.rank ? src
                                    : reinterpret_cast<const uint4*>(a.peer[a.rank] + region0 +
                                                                     int64_t(r) * a.slice_pitch);
    for (int64_t i = u0 + threadIdx.x; i < u1; i += kP2pThreads) {
      if (i * 16 >= slice_bytes) break;  // the pitch's padding
      const uint4 v = __ldcg(from + i);
      const int64_t e0 = i * per16;  // first element of the unit in the [M, ns] slice
      const int64_t m = e0 / a.ns, j = e0 - m * a.ns;
      if (a.unit == 16 && col0 + j + per16 <= a.N) {
        // the whole unit lies in one output row (ns, out_rs and the output's
        // address are 16-byte aligned, so no unit straddles a row)
        *reinterpret_cast<uint4*>(a.out + (m * a.out_rs + col0 + j) * eb) = v;
        continue;
      }
      const uint8_t* bytes = reinterpret_cast<const uint8_t*>(&v);
      for (int k = 0; k < per16; ++k) {
        const int64_t e = e0 + k;
        if (e * eb >= slice_bytes) break;
        const int64_t mm = e / a.ns, jj = e - mm * a.ns;
        if (col0 + jj >= a.N) continue;  // ragged last shard
        uint8_t* dst = a.out + (mm * a.out_rs + col0 + jj) * eb;
        switch (eb) {
          case 8: *reinterpret_cast<uint64_t*>(dst) = *reinterpret_cast<const uint64_t*>(bytes + k * 8); break;
          case 4: *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(bytes + k * 4); break;
          default: *reinterpret_cast<uint16_t*>(dst) = *reinterpret_cast<const uint16_t*>(bytes + k * 2); break;
        }
      }
    }
  }
}

}  // namespace

int p2p_timeouts(long long* out, bool reset) { return read_timeout_counter(g_p2p_timeouts, out, reset); }

int64_t p2p_slice_pitch(int M, int ns, int elem_bytes) { return (int64_t(M) * ns * elem_bytes + 15) / 16 * 16; }

int64_t p2p_buffer_bytes(int M, int ns, int elem_bytes, int world) {
  return kP2pSignalBytes + 2 * int64_t(world) * p2p_slice_pitch(M, ns, elem_bytes);
}

int p2p_ctas(int64_t slice_pitch) {
  // ~2 16-byte units per thread; a function of the slice size only, so every
  // rank launches the same grid
  const int64_t n16 = slice_pitch / 16;
  return int(std::max<int64_t>(1, std::min<int64_t>(kP2pMaxCtas, (n16 + 2 * kP2pThreads - 1) / (2 * kP2pThreads))));
}

int launch_p2p_allgather(P2pArgs a, cudaStream_t st) {
  const int64_t eb = a.elem_bytes;
  const bool vec = (int64_t(a.ns) * eb) % 16 == 0 && (a.out_rs * eb) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(a.out) % 16 == 0;
  a.unit = vec ? 16 : int(eb);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(p2p_ctas(a.slice_pitch)));
  cfg.blockDim = dim3(kP2pThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, p2p_allgather_kernel, a));
}

}  // namespace spectra
