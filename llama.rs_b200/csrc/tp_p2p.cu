// tp_p2p.cu -- the tensor-parallel all-reduce of the row-split projections
// (o_proj, down_proj) over peer memory, in place of an NCCL all-reduce.
//
// Every rank's projection stores its partial sum y_r into its own exchange
// buffer (one of two, alternating per call).  One kernel then, on every rank:
//  1. takes a ticket; with a fixed grid the launch index L = ticket / kTpGrid
//     is the same on all ranks because every rank runs the same sequence of
//     these launches (and the blocks of one launch take their tickets before
//     the next launch starts: stream order);
//  2. the first block of the launch stores L + 1 into sig[rank] of every peer
//     (a P2P store with release semantics at system scope): this rank's
//     partial of launch L is complete (the projection kernel before it on the
//     stream has finished);
//  3. every block waits, bounded, until its own sig[p] >= L + 1 for all
//     peers p (acquire at system scope);
//  4. residual[i] += y_0[i] + y_1[i] + ... + y_{N-1}[i], read over NVLink
//     with plain loads, in rank order, so every rank gets the same bits.
// A rank overwrites an exchange buffer two launches later, after every peer
// has signalled the launch in between, i.e. after the peers finished reading
// it.  Peer memory is only read with plain loads and written with plain stores.
#include <cuda_runtime.h>

#include "../../include/llamars.h"
#include "device_common.cuh"
#include "tp_p2p.cuh"

namespace lrs {
namespace {

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) tp_allreduce_add_kernel(const TpArgs a) {
  __shared__ unsigned ticket_sh;
  __shared__ int abort_sh;
  if (threadIdx.x == 0) {
    ticket_sh = atomicAdd(a.tickets, 1u);
    abort_sh = 0;
  }
  __syncthreads();
  const int epoch = (int)(ticket_sh / gridDim.x) + 1;
  const int t = threadIdx.x;
  if (ticket_sh % gridDim.x == 0 && t < a.world && t != a.rank)
    st_release_sys(a.peer_sig[t] + a.rank, epoch);
  if (t < a.world && t != a.rank) {
    bool ok = false;
    for (uint32_t i = 0; i < kSpinLimit; i++)
      if (ld_acquire_sys(a.local_sig + t) >= epoch) {
        ok = true;
        break;
      }
    if (!ok) {
      abort_sh = 1;
      if (a.error_flag) atomicExch(a.error_flag, LRS_ERR_DEVICE_TIMEOUT);
    }
  }
  __syncthreads();
  if (abort_sh) return;
  const float* const* parts = a.parity ? a.parts1 : a.parts0;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + t; i < a.n; i += (size_t)gridDim.x * blockDim.x) {
    float s = a.residual[i];
    for (int q = 0; q < a.world; q++) s += parts[q][i];
    a.residual[i] = s;
  }
}

}  // namespace

cudaError_t launch_tp_allreduce_add(const TpArgs& a, cudaStream_t st) {
  // a fixed grid: the launch index is ticket / gridDim.x
  tp_allreduce_add_kernel<<<kTpGrid, 256, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace lrs
