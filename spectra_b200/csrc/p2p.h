// Internal interface of the NVLink peer-memory all-gather (p2p.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace spectra {

constexpr int kP2pMaxRanks = 8;
constexpr int kP2pMaxCtas = 128;  // CTAs of one exchange launch, at most
// epoch flags [rank][cta] at the start of every exchange buffer
constexpr int64_t kP2pSignalBytes = int64_t(kP2pMaxRanks) * kP2pMaxCtas * 4;

struct P2pArgs {
  const uint8_t* src;             // this rank's slice [M][ns], slice_pitch bytes readable
  uint8_t* peer[kP2pMaxRanks];    // every rank's exchange buffer as mapped here (peer[rank]: own)
  uint8_t* out;                   // [M][out_rs] elements; columns [0, N) written
  int64_t out_rs;                 // output row stride, elements
  int64_t slice_pitch;            // bytes per slice region, multiple of 16, >= M*ns*elem_bytes
  int* state;                     // device int[kP2pMaxCtas]: each CTA's call counter
  int M, ns, N, elem_bytes;
  int unit;                       // 16: whole 16-byte units go to the output (set by the launcher)
  int rank, world;
  uint64_t wait_limit_ns;
};

int64_t p2p_slice_pitch(int M, int ns, int elem_bytes);
int64_t p2p_buffer_bytes(int M, int ns, int elem_bytes, int world);
int p2p_ctas(int64_t slice_pitch);
int launch_p2p_allgather(P2pArgs a, cudaStream_t st);
int p2p_timeouts(long long* out, bool reset);

}  // namespace spectra
