// tp_p2p.cuh -- the peer-memory all-reduce of the row-split projections (tp_p2p.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>

namespace lrs {

struct TpArgs {
  float* residual;             // [n], updated in place
  size_t n;                    // items * hidden
  const float* const* parts0;  // [world] exchange buffers, parity 0 (peers' mapped over IPC)
  const float* const* parts1;  // [world] parity 1
  int parity;
  int* local_sig;              // [world] this rank's signal words (peers store into them)
  int* const* peer_sig;        // [world] every rank's signal words
  unsigned* tickets;           // this rank's launch counter (zero at creation)
  int rank, world;
  int* error_flag;
};

constexpr int kTpGrid = 128;  // blocks of every launch (fixed: see tp_p2p.cu)

// residual += sum over ranks of parts[rank], in rank order, after every peer
// signalled that its part of this launch is complete (bounded waits).
cudaError_t launch_tp_allreduce_add(const TpArgs& a, cudaStream_t st);

}  // namespace lrs
