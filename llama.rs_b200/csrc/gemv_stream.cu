// gemv_stream.cu -- batch-1 quantized GEMV with the weights streamed through a
// shared-memory ring by bulk copies (sm_100a).
//
// Replaces the per-row dots of CpuBackend::matvec at batch 1 (src/backend.rs:
// 143-162; dot_row_scalar, src/quant.rs:458-648) like gemv5_kernel (gemv.cu),
// with the same factored dot (gemv_fast.cuh) but a different memory scheme:
//
// * Persistent grid, one or two CTAs per SM.  CTA b owns the contiguous range
//   of row tiles [b*T/G, (b+1)*T/G); a tile is RT = R*ng rows (R = 4, or 2 rows
//   of each matrix of a gate/up pair) and is consumed in K-chunks of kc block
//   units, so an item (tile, chunk) is NM*RT row pieces of at most ~32 KB.
// * One producer warp issues, per item, one cp.async.bulk per (matrix, row)
//   chunk into a ring of `stages` items, completing on the item's "full"
//   mbarrier.  Every copy starts on the 16-byte boundary at or below the
//   chunk's first byte and ends on the one at or above its last byte; the
//   offset of the chunk inside its slot is the address modulo 16, so the block
//   alignment the piece loaders rely on is the same as in global memory.  The
//   first `stages` items are in flight before griddepcontrol.wait: the weights
//   do not depend on the previous kernel.
// * Eight consumer warps stage x once (prep_x), then for each item: warp w
//   takes row group w / wpg of the tile (wpg = 8 / ng warps per group), lane l
//   the pieces l + 32*(w % wpg), step 32*wpg, of the chunk, for all R rows of
//   the group (each x fragment is read once for R rows), and accumulates in
//   registers across the chunks of a tile.  After a tile's last chunk the
//   warp's row sums go to a per-stage slot of shared memory; every warp then
//   releases the stage on its "empty" mbarrier.
// * The producer, before refilling a stage (or at the end), waits for its
//   release and runs the epilogue of the tile that ended there: lane l sums
//   row l's wpg partials in a fixed order (deterministic) and applies the bias
//   / residual add / SwiGLU / argmax of gemv5.
// Every mbarrier wait is bounded; a wait that gives up writes
// LRS_ERR_DEVICE_TIMEOUT to the error flag and the CTA drains its copies and
// returns.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.h"
#include "device_common.cuh"
#include "gemv.cuh"
#include "gemv_fast.cuh"

namespace lrs {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = 32 * kConsumerWarps;
constexpr int kStreamThreads = kConsumers + 32;
constexpr int kStreamMaxStages = 16;
constexpr int kItemMaxBytes = 32 * 1024;

// Launch shape of one stream GEMV (host-chosen, read-only on the device).
struct StreamShape {
  int rt;       // rows per tile (R * ng)
  int ng;       // row groups per tile
  int wpg;      // consumer warps per row group (8 / ng)
  int kc;       // block units per chunk
  int nchunk;   // chunks per row
  int units;    // block units per row
  int mreg;     // shared-memory bytes per (matrix, row) slot of an item
  int stages;   // items in the ring
  int item_bytes;  // NM * rt * mreg
  int red_off, bar_off, x_off, ring_off;  // shared-memory layout
};

__device__ __forceinline__ void mbar_arrive_cta(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}

__device__ __forceinline__ GemvSeg seg_of(const GemvParams& p, int tile) {
  if (p.nseg > 2 && tile >= p.seg[2].tile0) return p.seg[2];
  if (p.nseg > 1 && tile >= p.seg[1].tile0) return p.seg[1];
  return p.seg[0];
}

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int o) {
  const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, o);
  const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), o);
  return ((unsigned long long)hi << 32) | lo;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <int T, bool PAIR, bool TPX>
__global__ void __launch_bounds__(kStreamThreads)
    gemv_stream_kernel(const __grid_constant__ GemvParams p, const __grid_constant__ StreamShape sh,
                       const __grid_constant__ StreamTp tp) {
  using BT = BlockTraits<T>;
  using P = fast::Piece<T>;
  using XL = XLayout<T>;
  constexpr int NM = PAIR ? 2 : 1;
  constexpr int R = PAIR ? 2 : 4;
  constexpr int PV = XL::PV, NRUN = XL::NRUN, CH = XL::CH, NW = P::kWords;
  constexpr bool kDense = XL::kDense;
  extern __shared__ __align__(128) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem + sh.red_off);  // [stages][8 warps][NM*R]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + sh.bar_off);
  uint64_t* empty = full + sh.stages;
  uint8_t* xq = smem + sh.x_off;
  uint8_t* ring = smem + sh.ring_off;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int npieces = p.cols / PV;

  const int tA = (int)((long long)blockIdx.x * p.total_tiles / gridDim.x);
  const int tB = (int)((long long)(blockIdx.x + 1) * p.total_tiles / gridDim.x);
  const int nitems = (tB - tA) * sh.nchunk;
  const int NS = sh.stages;

  if (tid == 0) {
    for (int s = 0; s < NS; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer warp ----------------
    const uint64_t policy = evict_first_policy();
    bool ok = true;
    unsigned long long key = 0ull;
    int issued = 0;
    // Epilogue of item j, in two halves so that the refill copies go out in
    // between: gather() reads the row sums of the tile that ended with item j
    // from shared memory (before the consumers can reuse its slot) and starts
    // the bias load; apply() writes the outputs.  Lane l owns tile row l.
    struct Rows {
      float y[NM];
      float bias;
      float* out;
      int row;
      bool live, has_bias;
    };
    auto gather = [&](int j) {
      Rows e;
      e.live = false;
      if (j % sh.nchunk != sh.nchunk - 1) return e;
      const int t = tA + j / sh.nchunk, s = j % NS;
      const GemvSeg sg = seg_of(p, t);
      const int r0 = (t - sg.tile0) * sh.rt;
      const int nr = min(sh.rt, sg.rows - r0);
      if (lane >= nr) return e;
      const int gw = lane / R, jr = lane % R;
#pragma unroll
      for (int m = 0; m < NM; m++) {
        float acc = 0.0f;
        for (int u = 0; u < sh.wpg; u++)  // fixed order: deterministic
          acc += red[((s * kConsumerWarps) + gw * sh.wpg + u) * (NM * R) + m * R + jr];
        e.y[m] = acc;
      }
      e.row = r0 + lane;
      e.out = sg.out ? sg.out + e.row : nullptr;
      e.has_bias = p.epi == EPI_STORE && sg.bias;
      e.bias = e.has_bias ? __ldg(sg.bias + e.row) : 0.0f;
      e.live = true;
      return e;
    };
    auto apply = [&](const Rows& e) {
      if (!e.live) return;
      if constexpr (TPX) {
        // this rank's partial of the row, into every rank's exchange buffer
        // (peers' over NVLink): x_q[rank][row]
        for (int q = 0; q < tp.world; q++) tp.peer_x[q][(size_t)tp.rank * tp.rows + e.row] = e.y[0];
        return;
      }
      switch (p.epi) {
        case EPI_STORE:
          *e.out = e.has_bias ? e.y[0] + e.bias : e.y[0];
          break;
        case EPI_ADD:
          // the only update of this element in the launch: one rounding, as
          // out += y, without waiting for the load
          atomicAdd(e.out, e.y[0]);
          break;
        case EPI_SWIGLU:
          *e.out = (e.y[0] / (1.0f + expf(-e.y[0]))) * e.y[NM - 1];
          break;
        default: {
          if (e.out) *e.out = e.y[0];
          const unsigned long long k2 = argmax_pack(e.y[0], (uint32_t)e.row);
          key = k2 > key ? k2 : key;
        }
      }
    };
    for (int i = 0; i < nitems && ok; i++) {
      const int s = i % NS, k = i / NS;
      Rows e;
      e.live = false;
      if (k >= 1) {
        if (lane == 0) ok = mbar_wait_bounded(&empty[s], (uint32_t)((k - 1) & 1));
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        e = gather(i - NS);
        __syncwarp();
      }
      if (lane == 0) {
        const int t = tA + i / sh.nchunk, c = i % sh.nchunk;
        const GemvSeg sg = seg_of(p, t);
        const int r0 = (t - sg.tile0) * sh.rt;
        const int nr = min(sh.rt, sg.rows - r0);
        const int u0 = c * sh.kc, nu = min(sh.kc, sh.units - u0);
        // copy r of matrix m: [lo, hi) around the chunk's bytes, both 16-byte aligned
        auto span = [&](int m, int r, uintptr_t& lo) -> uint32_t {
          const uint8_t* w = m == 0 ? sg.w : sg.w2;
          const uintptr_t a = reinterpret_cast<uintptr_t>(w + (size_t)(r0 + r) * sg.rb +
                                                          (size_t)u0 * BT::kBytes);
          lo = a & ~uintptr_t(15);
          return (uint32_t)(((a + (uintptr_t)nu * BT::kBytes + 15) & ~uintptr_t(15)) - lo);
        };
        uint32_t total = 0;
        uintptr_t lo;
        for (int m = 0; m < NM; m++)
          for (int r = 0; r < nr; r++) total += span(m, r, lo);
        if (k >= 1) fence_proxy_async();  // consumers' reads of the slot before the copy's writes
        mbar_expect_tx(&full[s], total);
        uint8_t* item = ring + (size_t)s * sh.item_bytes;
        for (int m = 0; m < NM; m++)
          for (int r = 0; r < nr; r++) {
            const uint32_t bytes = span(m, r, lo);
            tma_load_1d(item + (size_t)(m * sh.rt + r) * sh.mreg, reinterpret_cast<const void*>(lo),
                        bytes, &full[s], policy);
          }
      }
      issued = i + 1;
      // the epilogues write outputs that the previous kernel may still read
      if (i == min(NS, nitems) - 1) pdl_wait();
      apply(e);
    }
    if (ok) {
      for (int i = max(0, nitems - NS); i < nitems && ok; i++) {
        const int s = i % NS, k = i / NS;
        if (lane == 0) ok = mbar_wait_bounded(&empty[s], (uint32_t)(k & 1));
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (ok) apply(gather(i));
        __syncwarp();
      }
    }
    if (!ok) {
      if (lane == 0 && p.error_flag) atomicExch(p.error_flag, LRS_ERR_DEVICE_TIMEOUT);
      // let the copies already issued land before the CTA leaves
      if (lane == 0)
        for (int i = max(0, issued - NS); i < issued; i++)
          mbar_wait_bounded(&full[i % NS], (uint32_t)((i / NS) & 1));
      return;
    }
    if constexpr (TPX) {
      // every partial of this CTA's rows is stored: make them visible to the
      // peers, signal the same CTA index there, wait for theirs, reduce
      __threadfence_system();
      __syncwarp();
      const int b = blockIdx.x;
      int epoch = 0;
      if (lane == 0) epoch = (int)(++tp.counters[b]);
      epoch = __shfl_sync(0xffffffffu, epoch, 0);
      if (lane < tp.world && lane != tp.rank)
        st_release_sys(tp.peer_sig[lane] + kTpSigFused + tp.rank * kTpMaxGrid + b, epoch);
      bool got = true;
      if (lane < tp.world && lane != tp.rank) {
        got = false;
        for (uint32_t it = 0; it < kSpinLimit; it++)
          if (ld_acquire_sys(tp.local_sig + lane * kTpMaxGrid + b) >= epoch) {
            got = true;
            break;
          }
      }
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0 && tp.error_flag) atomicExch(tp.error_flag, LRS_ERR_DEVICE_TIMEOUT);
        return;
      }
      // rows of this CTA's tiles (one segment): out[row] += sum over ranks in rank order
      const GemvSeg sg = p.seg[0];
      const int rA = (tA - sg.tile0) * sh.rt, rB = min(sg.rows, (tB - sg.tile0) * sh.rt);
      const float* mine = tp.peer_x[tp.rank];
      for (int row = rA + lane; row < rB; row += 32) {
        float acc = sg.out[row];
        for (int q = 0; q < tp.world; q++) acc += mine[(size_t)q * tp.rows + row];
        sg.out[row] = acc;
      }
      return;
    }
    if (p.epi == EPI_ARGMAX) {
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        const unsigned long long k2 = shfl_xor_u64(key, o);
        key = k2 > key ? k2 : key;
      }
      if (lane == 0 && key) atomicMax(&p.argmax_keys[0], key);
    }
    return;
  }

  // ---------------- consumer warps ----------------
  pdl_wait();  // x / residual come from the previous kernel
  prep_x<T, kConsumers>(p.x, p.norm_w, p.norm_eps, p.cols, xq, red, tid, [] { consumer_sync(); });
  pdl_launch_dependents();
  const XView<T> xv(xq, npieces);
  const int gw = warp / sh.wpg, sub_w = warp % sh.wpg;
  float acc[NM][R];
#pragma unroll
  for (int m = 0; m < NM; m++)
#pragma unroll
    for (int r = 0; r < R; r++) acc[m][r] = 0.0f;
  for (int i = 0; i < nitems; i++) {
    const int s = i % NS, k = i / NS;
    const int t = tA + i / sh.nchunk, c = i % sh.nchunk;
    const GemvSeg sg = seg_of(p, t);
    const int r0 = (t - sg.tile0) * sh.rt;
    const int nr = min(sh.rt, sg.rows - r0);
    const int u0 = c * sh.kc, nu = min(sh.kc, sh.units - u0);
    bool ok = true;
    if (lane == 0) ok = mbar_wait_bounded(&full[s], (uint32_t)(k & 1));
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) {
      if (lane == 0 && p.error_flag) atomicExch(p.error_flag, LRS_ERR_DEVICE_TIMEOUT);
      return;
    }
    const int g0 = gw * R;  // first tile row of this warp's group
    if (g0 < nr) {
      const uint8_t* item = ring + (size_t)s * sh.item_bytes;
      const uint8_t* base[NM][R];
#pragma unroll
      for (int m = 0; m < NM; m++) {
        const uint8_t* w = m == 0 ? sg.w : sg.w2;
#pragma unroll
        for (int j = 0; j < R; j++) {
          const int r = g0 + j < nr ? g0 + j : g0;  // rows past nr re-read the group's first (discarded)
          const uintptr_t a = reinterpret_cast<uintptr_t>(w + (size_t)(r0 + r) * sg.rb +
                                                          (size_t)u0 * BT::kBytes);
          base[m][j] = item + (size_t)(m * sh.rt + r) * sh.mreg + (a & 15);
        }
      }
      const int npc = nu * P::kPieces;
      for (int pl = lane + 32 * sub_w; pl < npc; pl += 32 * sh.wpg) {
        const int ul = pl / P::kPieces, sub = pl % P::kPieces;
        const int pc = u0 * P::kPieces + pl;  // piece index of x
        P pr[NM][R];
#pragma unroll
        for (int m = 0; m < NM; m++)
#pragma unroll
          for (int j = 0; j < R; j++) pr[m][j].template load<true>(base[m][j] + ul * BT::kBytes, sub);
        if constexpr (kDense) {
          const float4* xp = reinterpret_cast<const float4*>(xv.xf + (size_t)pc * PV);
          fast::f2 xa[NW], xb[NW];
#pragma unroll
          for (int q = 0; q < NW; q++) {
            const float4 v = xp[q];
            xa[q] = fast::pk(v.x, v.y);
            xb[q] = fast::pk(v.z, v.w);
          }
#pragma unroll
          for (int m = 0; m < NM; m++)
#pragma unroll
            for (int j = 0; j < R; j++) {
              fast::f2 S0 = 0ull, S1 = 0ull;
#pragma unroll
              for (int q = 0; q < NW; q++) {
                fast::f2 a, b;
                pr[m][j].weights(q, a, b);
                fast::fma2(S0, a, xa[q]);
                fast::fma2(S1, b, xb[q]);
              }
              acc[m][j] += fast::hsum2(S0) + fast::hsum2(S1);
            }
        } else {
          uint32_t xh[PV / 4], xl[PV / 4];
#pragma unroll
          for (int q = 0; q < CH; q++) {
            const uint4 h = xv.xh4[(size_t)q * npieces + pc], l = xv.xl4[(size_t)q * npieces + pc];
            xh[4 * q] = h.x, xh[4 * q + 1] = h.y, xh[4 * q + 2] = h.z, xh[4 * q + 3] = h.w;
            xl[4 * q] = l.x, xl[4 * q + 1] = l.y, xl[4 * q + 2] = l.z, xl[4 * q + 3] = l.w;
          }
          float sx[NRUN], X8[NRUN];
#pragma unroll
          for (int r = 0; r < NRUN; r++) {
            sx[r] = xv.sxa[(size_t)r * npieces + pc];
            X8[r] = xv.Xa[(size_t)r * npieces + pc];
          }
#pragma unroll
          for (int m = 0; m < NM; m++)
#pragma unroll
            for (int j = 0; j < R; j++) {
              float qx[NRUN];
#pragma unroll
              for (int u = 0; u < NRUN; u++) {
                const uint32_t c0 = pr[m][j].icode(2 * u, sub), c1 = pr[m][j].icode(2 * u + 1, sub);
                int hs = __dp4a((int)c0, (int)xh[2 * u], 0);
                hs = __dp4a((int)c1, (int)xh[2 * u + 1], hs);
                int ls = __dp4a((int)c0, (int)xl[2 * u], hs << 8);
                ls = __dp4a((int)c1, (int)xl[2 * u + 1], ls);
                qx[u] = sx[u] * (float)ls;
              }
              acc[m][j] += pr[m][j].finish_i(qx, X8, sub);
            }
        }
      }
    }
    if (c == sh.nchunk - 1) {  // the tile ends here: hand the row sums to the producer
#pragma unroll
      for (int m = 0; m < NM; m++)
#pragma unroll
        for (int j = 0; j < R; j++) {
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) acc[m][j] += __shfl_xor_sync(0xffffffffu, acc[m][j], o);
          if (lane == 0) red[(s * kConsumerWarps + warp) * (NM * R) + m * R + j] = acc[m][j];
          acc[m][j] = 0.0f;
        }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive_cta(&empty[s]);
  }
}

template <int T>
const void* stream_kernel_of(bool pair, bool tpx) {
  if (tpx) return pair ? nullptr : (const void*)gemv_stream_kernel<T, false, true>;
  return pair ? (const void*)gemv_stream_kernel<T, true, false>
              : (const void*)gemv_stream_kernel<T, false, false>;
}

const void* stream_kernel(int type, bool pair, bool tpx) {
  switch (type) {
    case LRS_GGML_F32: return stream_kernel_of<LRS_GGML_F32>(pair, tpx);
    case LRS_GGML_F16: return stream_kernel_of<LRS_GGML_F16>(pair, tpx);
    case LRS_GGML_BF16: return stream_kernel_of<LRS_GGML_BF16>(pair, tpx);
    case LRS_GGML_Q4_0: return stream_kernel_of<LRS_GGML_Q4_0>(pair, tpx);
    case LRS_GGML_Q4_1: return stream_kernel_of<LRS_GGML_Q4_1>(pair, tpx);
    case LRS_GGML_Q5_0: return stream_kernel_of<LRS_GGML_Q5_0>(pair, tpx);
    case LRS_GGML_Q5_1: return stream_kernel_of<LRS_GGML_Q5_1>(pair, tpx);
    case LRS_GGML_Q8_0: return stream_kernel_of<LRS_GGML_Q8_0>(pair, tpx);
    case LRS_GGML_Q4_K: return stream_kernel_of<LRS_GGML_Q4_K>(pair, tpx);
    case LRS_GGML_Q5_K: return stream_kernel_of<LRS_GGML_Q5_K>(pair, tpx);
    case LRS_GGML_Q6_K: return stream_kernel_of<LRS_GGML_Q6_K>(pair, tpx);
  }
  return nullptr;
}

template <int T>
size_t stream_x_bytes(int cols) {
  return XLayout<T>::bytes(cols / XLayout<T>::PV);
}

size_t x_bytes_of(int type, int cols) {
  switch (type) {
    case LRS_GGML_F32: return stream_x_bytes<LRS_GGML_F32>(cols);
    case LRS_GGML_F16: return stream_x_bytes<LRS_GGML_F16>(cols);
    case LRS_GGML_BF16: return stream_x_bytes<LRS_GGML_BF16>(cols);
    case LRS_GGML_Q4_0: return stream_x_bytes<LRS_GGML_Q4_0>(cols);
    case LRS_GGML_Q4_1: return stream_x_bytes<LRS_GGML_Q4_1>(cols);
    case LRS_GGML_Q5_0: return stream_x_bytes<LRS_GGML_Q5_0>(cols);
    case LRS_GGML_Q5_1: return stream_x_bytes<LRS_GGML_Q5_1>(cols);
    case LRS_GGML_Q8_0: return stream_x_bytes<LRS_GGML_Q8_0>(cols);
    case LRS_GGML_Q4_K: return stream_x_bytes<LRS_GGML_Q4_K>(cols);
    case LRS_GGML_Q5_K: return stream_x_bytes<LRS_GGML_Q5_K>(cols);
    case LRS_GGML_Q6_K: return stream_x_bytes<LRS_GGML_Q6_K>(cols);
  }
  return 0;
}

// Resident CTAs per SM of `kernel` with `smem` bytes (cached).
int stream_occupancy(const void* kernel, int smem) {
  struct Entry {
    int dev;
    const void* k;
    int smem, blocks;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  for (auto& c : cache)
    if (c.dev == dev && c.k == kernel && c.smem == smem) return c.blocks;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  int blocks = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, kStreamThreads, smem);
  cache.push_back({dev, kernel, smem, blocks});
  return blocks;
}

// Shared-memory layout for `stages` items; returns the total bytes.
int stream_layout(StreamShape& sh, size_t xbytes) {
  sh.red_off = 0;
  const int red = sh.stages * kConsumerWarps * 4 * 4;  // NM * R = 4 floats per warp
  sh.bar_off = (red + 15) & ~15;
  sh.x_off = (sh.bar_off + 2 * sh.stages * 8 + 127) & ~127;
  sh.ring_off = (int)((sh.x_off + xbytes + 127) & ~size_t(127));
  return sh.ring_off + sh.stages * sh.item_bytes;
}

}  // namespace

bool gemv_stream_enabled() {
  const char* e = getenv("LRS_GEMV_STREAM");
  return e && e[0] == '1';
}

cudaError_t gemv_stream_launch(const GemvParams& p0, cudaStream_t stream, int num_sms, bool pdl,
                               const StreamTp* tp) {
  const bool pair = p0.epi == EPI_SWIGLU;
  const int nm = pair ? 2 : 1, R = pair ? 2 : 4;
  const int type = p0.seg[0].type;
  uint32_t bv, bb;
  if (!type_geometry((uint32_t)type, &bv, &bb)) return cudaErrorInvalidValue;
  // BlockTraits units: 32-value units for the dense types
  const bool dense = type == LRS_GGML_F32 || type == LRS_GGML_F16 || type == LRS_GGML_BF16;
  const int ub = dense ? (int)(bb * 32) : (int)bb;
  const int uv = dense ? 32 : (int)bv;
  const int units = p0.cols / uv;
  if (tp && (pair || p0.nseg != 1 || p0.batch != 1 || tp->plan_cols < p0.cols))
    return cudaErrorInvalidValue;
  const void* kernel = stream_kernel(type, pair, tp != nullptr);
  // The tensor-parallel variant reduces CTA b's rows after CTA b of every
  // peer signalled, so all ranks need the same tiles and grid: those are
  // planned from plan_cols, the same on every rank (windowed shards of one
  // projection may cover different numbers of blocks).
  const int plan_cols = tp ? tp->plan_cols : p0.cols;
  const int plan_units = plan_cols / uv;
  const size_t xbytes = x_bytes_of(type, plan_cols);
  if (!kernel || units < 1) return cudaErrorInvalidValue;

  StreamShape sh = {};
  // K-chunks: whole rows while R rows of every matrix fit one item.
  auto chunk = [&](int n, int cap) {
    sh.units = n;
    sh.kc = std::max(1, std::min(n, cap));
    sh.nchunk = (n + sh.kc - 1) / sh.kc;
    sh.kc = (n + sh.nchunk - 1) / sh.nchunk;  // even chunks
    sh.mreg = ((sh.kc * ub + 15) & ~15) + 32;
  };
  chunk(plan_units, kItemMaxBytes / (nm * R * ub));

  int total_rows = 0;
  for (int i = 0; i < p0.nseg; i++) total_rows += p0.seg[i].rows;

  // Two CTAs per SM when x is small and the registers allow, else one.
  int occ = 1;
  for (int want = 2; want >= 1; want--) {
    const int budget = 227 * 1024 / want - 1024;
    // groups per tile: widen the tile while the item stays small and every CTA keeps >= 4 tiles
    int ng = 1;
    while (ng < kConsumerWarps && 2 * ng * nm * R * sh.mreg <= kItemMaxBytes &&
           total_rows / (2 * ng * R) >= 4 * num_sms * want)
      ng *= 2;
    sh.ng = ng;
    sh.wpg = kConsumerWarps / ng;
    sh.rt = R * ng;
    sh.item_bytes = nm * sh.rt * sh.mreg;
    sh.stages = kStreamMaxStages;
    while (sh.stages > 2 && stream_layout(sh, xbytes) > budget) sh.stages--;
    const int smem = stream_layout(sh, xbytes);
    if (smem > budget) continue;
    if (want == 1 || (sh.stages >= 3 && stream_occupancy(kernel, smem) >= 2)) {
      occ = want;
      break;
    }
  }
  if (stream_layout(sh, xbytes) > 227 * 1024) return cudaErrorNotSupported;  // x too wide
  if (units != plan_units) {
    // this rank's shard: chunks no longer than the plan's, so the item and
    // the staged x stay within the planned layout (same stages and tiles)
    chunk(units, sh.kc);
    sh.item_bytes = nm * sh.rt * sh.mreg;
  }
  const int smem = stream_layout(sh, x_bytes_of(type, p0.cols));

  GemvParams q = p0;
  int tile0 = 0;
  for (int i = 0; i < q.nseg; i++) {
    GemvSeg& s = q.seg[i];
    s.rt = sh.rt;
    s.tiles = (s.rows + sh.rt - 1) / sh.rt;
    s.tile0 = tile0;
    tile0 += s.tiles;
  }
  q.total_tiles = tile0;
  const int grid = std::min(q.total_tiles, num_sms * occ);
  if (grid < 1) return cudaSuccess;
  if (grid > kTpMaxGrid) return cudaErrorInvalidValue;
  stream_occupancy(kernel, smem);  // sets the dynamic shared-memory limit

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kStreamThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  StreamTp none = {};
  void* args[] = {&q, &sh, tp ? const_cast<StreamTp*>(tp) : &none};
  return cudaLaunchKernelExC(&cfg, kernel, args);
}

}  // namespace lrs
