// gemm_tc.cu -- batched Q4_K / Q6_K matmul (4..64 items: decode batches and
// prefill chunks) on the 5th-generation tensor cores: tcgen05.mma with the
// accumulators in tensor memory (TMEM).
//
// Replaces B independent CpuBackend::matvec calls (src/backend.rs:143-162)
// for Q4_K and Q6_K weights, the bulk of the q4k/q4km models (q, k, o, gate,
// up in Q4_K; down in Q6_K under q4km).
//
// Arithmetic.  A Q4_K super-block row is w_k = d*sc_g*q_k - dmin*m_g
// (value_at, src/quant.rs:404-440) with 6-bit sc_g, m_g per 32-column group g.
// sc_g*q_k <= 63*15 = 945 is an exact f16 integer, so the A tile holds
// f16(sc_g*q_k) and the whole 256-column super-block accumulates in one TMEM
// accumulator; per super-block and element the epilogue adds
//     d * T - dmin * M,   T = sum_k sc q_k x_k,   M = sum_g m_g sum_{k in g} x_k
// where M comes from a second, K = 16 MMA of A_min = 32*m_g (exact f16) with
// B_min = (group sums of x)/32.  x is scaled per item by a power of two (max
// |x/s| in [2^13, 2^14)) and split into f16 hi + lo; the B tile stacks the
// two as rows 2i and 2i+1 (N = 128 for 64 items), so one MMA covers both and
// the epilogue adds the pair.  Every product is exact and accumulates in f32.
//
// Layout.  A, B, A_min and B_min are K-major, no swizzle: 8x8 f16 core
// matrices (8 rows of 16 contiguous bytes), K-adjacent core matrices 128 B
// apart (LBO), 8-row groups 16 core matrices apart (SBO = 2048 B for a
// 128-column K chunk).  Inside every 4 columns the order is (0, 2, 1, 3): the
// order in which a nibble mask of a 4-byte word yields f16 pairs.  The split x
// is written by xsplit_tc_kernel in exactly the shared-memory image, so it is
// staged with one cp.async.bulk per 128-column chunk.
//
// Pipeline (416 threads, one CTA per SM):
//   warps 0-7 (two threads per weight row, two 32-column groups each) decode
//     each half super-block into an A tile (three buffers);
//   warp 12 (one thread) issues the bulk copies of the x tiles two half steps
//     ahead (three buffers) and, once an A tile is complete, its MMAs
//     (8 x K=16, plus the A_min MMA per super-block) and tcgen05.commit;
//   warps 8-11 (TMEM lanes 32*(w-8)...) read the finished super-block's
//     accumulators with tcgen05.ld and update 64 per-item f32 sums;
//   TMEM holds two super-blocks (2 x (128 + 128) columns) so the epilogue of
//   super-block s overlaps the MMAs of s+1.
// Results are partial sums per K group (grid.y), reduced with the epilogue of
// gemm_mma.cu (fixed order).  Every mbarrier wait is bounded; a timeout sets
// the error word, the kernel stops issuing work, frees its TMEM and returns.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "common.h"
#include "device_common.cuh"
#include "gemv.cuh"

namespace lrs {
namespace {

constexpr int kMaxItems = 64;
constexpr int kRows = 128;           // weight rows per CTA = TMEM lanes
constexpr int kKC = 128;             // columns per A/B tile (half a super-block)
constexpr int kTileA = kRows * kKC * 2;  // 32 KB
// x tile of NI items: N = 2 NI rows (item, hi/lo) x 128 columns
__host__ __device__ constexpr int tile_b(int ni) { return 2 * ni * kKC * 2; }
// B_min tile: N rows x 16 positions
__host__ __device__ constexpr int tile_bmin(int ni) { return 2 * ni * 16 * 2; }
constexpr int kTileMin = 128 * 16 * 2;   // 4 KB (A_min or B_min)
constexpr int kSBO = (kKC / 8) * 128;    // 2048
constexpr uint32_t kTmemCols = 512;
constexpr int kTcAhead = 2;  // super-blocks of weight rows prefetched into L2 ahead

// Per-type pipeline shape.  Q4_K: one A tile (sc*q) per half super-block plus
// the A_min MMA; three A and three x buffers.  Q6_K: two A tiles per half
// super-block, (q-32)*(sc & 15) and (q-32)*(sc - (sc & 15)), both exact in
// f16, accumulated into the same TMEM columns; two A and two x buffers.
template <int T, int NI>
struct TcShape {
  static constexpr int kN = 2 * NI;
  static constexpr int kTileB = tile_b(NI);
  static constexpr int kTileBmin = tile_bmin(NI);
  static constexpr bool kMins = T == LRS_GGML_Q4_K;
  static constexpr int kAParts = T == LRS_GGML_Q6_K ? 2 : 1;  // A tiles per half step
  static constexpr int kAB = T == LRS_GGML_Q6_K ? 2 : 3;  // A buffers
  static constexpr int kBB = T == LRS_GGML_Q6_K ? 2 : 3;  // x buffers
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kAB * kAParts * kTileA;
  static constexpr int kOffAmin = kOffB + kBB * kTileB;
  static constexpr int kOffBmin = kOffAmin + (kMins ? 2 * kTileMin : 0);
  static constexpr int kOffBar = kOffBmin + (kMins ? 2 * kTileBmin : 0);
  static constexpr int kSmem = kOffBar + 128;
  static constexpr int kBytes = T == LRS_GGML_Q6_K ? 210 : 144;
  static constexpr int kThreads = 416;
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, no swizzle, version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor, kind::f16: f16 A and B, f32 D, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
  __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b),
                      *reinterpret_cast<const __half2*>(&c));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t h2u(float a, float b) {
  __half2 r = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint4 ldg128(const uint8_t* p) {
  uint4 v;
  asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t byte_of(uint32_t w, int j) { return (w >> (8 * j)) & 0xffu; }


// ---- x preparation: one CTA per item slot (64, zero-padded) -------------------
// xt: [cols/128][N x 128] f16 tiles; xm: [cols/256][N x 16] group-sum tiles;
// xscale: [64] item scales.
__global__ void __launch_bounds__(256)
    xsplit_tc_kernel(const float* x, int x_ld, int cols, int batch, int ni, uint8_t* xt,
                     uint8_t* xm, float* xscale, const float* norm_w, float norm_eps) {
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* xr = x + (size_t)b * x_ld;
  __shared__ float red[8];
  // fused RMSNorm (RMSNorm::forward, src/model.rs:65-73): x * (inv * w)
  float inv_rms = 1.0f;
  if (norm_w && b < batch) {
    float ss = 0.0f;
    for (int c = threadIdx.x; c < cols; c += 256) ss = fmaf(xr[c], xr[c], ss);
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int k = 0; k < 8; k++) tot += red[k];
    inv_rms = 1.0f / sqrtf(tot / (float)cols + norm_eps);
    __syncthreads();
  }
  auto xval = [&](int c) { return norm_w ? xr[c] * (inv_rms * norm_w[c]) : xr[c]; };
  float mx = 0.0f;
  if (b < batch)
    for (int c = threadIdx.x; c < cols; c += 256) mx = fmaxf(mx, fabsf(xval(c)));
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < 8; w++) mx = fmaxf(mx, red[w]);
  int e = 14;
  if (mx > 0.0f && isfinite(mx)) frexpf(mx, &e);
  const float inv = ldexpf(1.0f, 14 - e);
  if (threadIdx.x == 0 && blockIdx.y == 0) xscale[b] = ldexpf(1.0f, e - 14);
  // one warp per super-block (256 columns), 8 columns per lane: f16 hi / lo in
  // tile order (one 16-byte store each), group sums / 32 into B_min
  for (int sb = blockIdx.y * 8 + warp; sb * 256 < cols; sb += 8 * gridDim.y) {
    const int k0 = sb * 256 + 8 * lane;
    float v[8];
    if (b < batch) {
      const float4 p0 = *reinterpret_cast<const float4*>(xr + k0);
      const float4 p1 = *reinterpret_cast<const float4*>(xr + k0 + 4);
      v[0] = p0.x, v[1] = p0.y, v[2] = p0.z, v[3] = p0.w, v[4] = p1.x, v[5] = p1.y, v[6] = p1.z,
      v[7] = p1.w;
      if (norm_w) {
        const float4 w0 = *reinterpret_cast<const float4*>(norm_w + k0);
        const float4 w1 = *reinterpret_cast<const float4*>(norm_w + k0 + 4);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = v[i] * (inv_rms * wv[i]);
      }
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] *= inv;
    } else {
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = 0.0f;
    }
    __half h[8], l[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      h[i] = __float2half_rn(v[i]);
      l[i] = __float2half_rn(v[i] - __half2float(h[i]));
    }
    // column order inside 4 columns: (0, 2, 1, 3)
    auto pack = [](const __half* q, int i0, int i1) {
      return (uint32_t)__half_as_ushort(q[i0]) | ((uint32_t)__half_as_ushort(q[i1]) << 16);
    };
    const uint4 hv = make_uint4(pack(h, 0, 2), pack(h, 1, 3), pack(h, 4, 6), pack(h, 5, 7));
    const uint4 lv = make_uint4(pack(l, 0, 2), pack(l, 1, 3), pack(l, 4, 6), pack(l, 5, 7));
    uint8_t* tile = xt + (size_t)(k0 / kKC) * tile_b(ni) + (lane & 15) * 128;
    const int nh = 2 * b, nl = 2 * b + 1;
    *reinterpret_cast<uint4*>(tile + (nh >> 3) * kSBO + (nh & 7) * 16) = hv;
    *reinterpret_cast<uint4*>(tile + (nl >> 3) * kSBO + (nl & 7) * 16) = lv;
    float sum = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    uint8_t* mt = xm + (size_t)sb * tile_bmin(ni);
    if ((lane & 3) == 0) {
      const float sg = sum * (1.0f / 32.0f);
      const __half sh = __float2half_rn(sg);
      const __half sl = __float2half_rn(sg - __half2float(sh));
      const int pos = lane >> 2;
      *reinterpret_cast<__half*>(mt + (nh >> 3) * 256 + (nh & 7) * 16 + pos * 2) = sh;
      *reinterpret_cast<__half*>(mt + (nl >> 3) * 256 + (nl & 7) * 16 + pos * 2) = sl;
    }
    if (lane == 0) {  // positions 8..15 (second core matrix) are zero
      *reinterpret_cast<uint4*>(mt + (nh >> 3) * 256 + 128 + (nh & 7) * 16) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(mt + (nl >> 3) * 256 + 128 + (nl & 7) * 16) = make_uint4(0, 0, 0, 0);
    }
  }
}

struct TcArgs {
  const uint8_t* w;  // block rows
  int rows, rb, cols, batch, kgroups;
  const uint8_t* xt;
  const uint8_t* xm;
  const float* xscale;
  float* part;  // [kgroups][batch][rows]
  int* error_flag;
};

// Four bytes at a 2-byte aligned address (Q6_K blocks are 210 bytes).
__device__ __forceinline__ uint32_t ldg32_a2(const uint8_t* p) {
  const uintptr_t ad = reinterpret_cast<uintptr_t>(p);
  const uint8_t* b = reinterpret_cast<const uint8_t*>(ad & ~uintptr_t(3));
  uint32_t lo, hi;
  asm("ld.global.nc.b32 %0, [%1];" : "=r"(lo) : "l"(b));
  asm("ld.global.nc.b32 %0, [%1];" : "=r"(hi) : "l"(b + 4));
  return __funnelshift_r(lo, hi, (uint32_t)(ad & 3) * 8);
}
__device__ __forceinline__ uint32_t h2sub(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t h2mul(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// Raw bytes one producer thread (c, r) needs from one super-block.
template <int T>
struct Raw;
template <>
struct Raw<LRS_GGML_Q4_K> {
  uint4 v[5];  // header, then 32 code bytes of pair c (half 0) and pair 2+c (half 1)
  __device__ __forceinline__ void load(const uint8_t* u, int c) {
    v[0] = ldg128(u);
    v[1] = ldg128(u + 16 + 32 * c);
    v[2] = ldg128(u + 32 + 32 * c);
    v[3] = ldg128(u + 80 + 32 * c);
    v[4] = ldg128(u + 96 + 32 * c);
  }
};
template <>
struct Raw<LRS_GGML_Q6_K> {
  uint32_t ql[2][8], qh[2][8], sc[2][2];  // per half: ql bytes of quarters c, c+2; qh; scales
  __device__ __forceinline__ void load(const uint8_t* u, int c) {
#pragma unroll
    for (int h = 0; h < 2; h++) {
#pragma unroll
      for (int i = 0; i < 8; i++) {
        ql[h][i] = ldg32_a2(u + 64 * h + 32 * c + 4 * i);
        qh[h][i] = ldg32_a2(u + 128 + 32 * h + 4 * i);
      }
      sc[h][0] = ldg32_a2(u + 192 + 8 * h);
      sc[h][1] = ldg32_a2(u + 196 + 8 * h);
    }
  }
};

template <int T, int NI>
__global__ void __launch_bounds__(TcShape<T, NI>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ TcArgs a) {
  using S = TcShape<T, NI>;
  constexpr int kN = S::kN, kTileB = S::kTileB;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint32_t tmem_base_sh;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kOffBar);
  uint64_t* full_b = bars;          // [kBB] x tile landed
  uint64_t* a_full = bars + 3;      // [kAB] the 256 producer threads wrote an A tile
  uint64_t* mma_done = bars + 6;    // [kAB] MMAs of a half step finished (A, x buffers free)
  uint64_t* acc_full = bars + 9;    // [2] super-block accumulator ready
  uint64_t* acc_empty = bars + 11;  // [2] epilogue finished reading it
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t sbase = smem_u32(smem);

  if (tid == 0) {
    for (int i = 0; i < 3; i++) {
      mbar_init(&full_b[i], 1);
      mbar_init(&a_full[i], 256);
      mbar_init(&mma_done[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_base_sh)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  const int nsb_all = a.cols / 256;
  const int s0 = (int)((long long)blockIdx.y * nsb_all / a.kgroups);
  const int s1 = (int)((long long)(blockIdx.y + 1) * nsb_all / a.kgroups);
  const int nsb = s1 - s0, nhs = 2 * nsb;
  const int row0 = blockIdx.x * kRows;
  bool ok = true;

  if (warp < 8) {
    // ---------------- producers: decode the A tiles ----------------
    // thread (c, r): row r, 32-column groups 2c, 2c+1 (Q4_K) or quarters c, c+2
    // (Q6_K) of every half super-block
    const int r = tid & 127, c = tid >> 7;
    const uint8_t* rp = a.w + (size_t)min(row0 + r, a.rows - 1) * a.rb;
    Raw<T> cur, nxt;
    if (nsb > 0) cur.load(rp + (size_t)s0 * S::kBytes, c);
    for (int sb = 0; sb < nsb && ok; sb++) {
      if (sb + 1 < nsb) nxt.load(rp + (size_t)(s0 + sb + 1) * S::kBytes, c);
      if (sb + kTcAhead < nsb) {  // kTcAhead super-blocks ahead into L2
        const uint8_t* pf = rp + (size_t)(s0 + sb + kTcAhead) * S::kBytes + c * 128;
        if (c * 128 < S::kBytes) asm volatile("prefetch.global.L2 [%0];" ::"l"(pf));
      }
#pragma unroll
      for (int half = 0; half < 2; half++) {
        const int hs = 2 * sb + half, ab = hs % S::kAB;
        if (hs >= S::kAB) ok = ok && mbar_wait_bounded(&mma_done[ab], ((hs - S::kAB) / S::kAB) & 1);
        if (!ok) break;
        uint8_t* A = smem + S::kOffA + ab * S::kAParts * kTileA;
        if constexpr (T == LRS_GGML_Q4_K) {
          const uint4 hd = cur.v[0];
          uint4 q[2] = {cur.v[1 + 2 * half], cur.v[2 + 2 * half]};
#pragma unroll
          for (int gl = 0; gl < 2; gl++) {
            const int g = 4 * half + 2 * c + gl;
            uint32_t sc;
            if (g < 4) {
              sc = byte_of(hd.y, g) & 63u;
            } else {
              sc = (byte_of(hd.w, g - 4) & 15u) | ((byte_of(hd.y, g - 4) >> 6) << 4);
            }
            const uint32_t sc2 = h2u((float)sc, (float)sc);
            const uint32_t nb2 = h2u(-1024.0f * (float)sc, -1024.0f * (float)sc);
            // groups 2p and 2p+1 share the 32 code bytes of pair p: low, high nibbles
            const int sh = 4 * gl;
            const uint32_t* wq = reinterpret_cast<const uint32_t*>(q);
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const uint32_t w0 = wq[2 * e] >> sh, w1 = wq[2 * e + 1] >> sh;
              uint4 v;
              v.x = hfma2u((w0 & 0x000F000Fu) | 0x64006400u, sc2, nb2);
              v.y = hfma2u(((w0 >> 8) & 0x000F000Fu) | 0x64006400u, sc2, nb2);
              v.z = hfma2u((w1 & 0x000F000Fu) | 0x64006400u, sc2, nb2);
              v.w = hfma2u(((w1 >> 8) & 0x000F000Fu) | 0x64006400u, sc2, nb2);
              const int j = (2 * c + gl) * 4 + e;  // k-group within the 128-column tile
              *reinterpret_cast<uint4*>(A + (r >> 3) * kSBO + j * 128 + (r & 7) * 16) = v;
            }
          }
          if (half == 0 && c == 0) {
            // A_min row: 32*m_g for the 8 groups, then 8 zeros
            uint32_t mw[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
              float m2[2];
#pragma unroll
              for (int k = 0; k < 2; k++) {
                const int g = 2 * i + k;
                const uint32_t mn =
                    g < 4 ? (byte_of(hd.z, g) & 63u)
                          : ((byte_of(hd.w, g - 4) >> 4) | ((byte_of(hd.z, g - 4) >> 6) << 4));
                m2[k] = 32.0f * (float)mn;
              }
              mw[i] = h2u(m2[0], m2[1]);
            }
            uint8_t* Am = smem + S::kOffAmin + (sb & 1) * kTileMin;
            *reinterpret_cast<uint4*>(Am + (r >> 3) * 256 + (r & 7) * 16) =
                make_uint4(mw[0], mw[1], mw[2], mw[3]);
            *reinterpret_cast<uint4*>(Am + (r >> 3) * 256 + 128 + (r & 7) * 16) =
                make_uint4(0, 0, 0, 0);
          }
        } else {
          // Q6_K half `half`: quarter qq of 32 columns: code = nibble (qq >> 1) of
          // ql[32 (qq & 1) + l] | 2 bits (2 qq) of qh[l] << 4; scale sc[2 qq + l / 16]
#pragma unroll
          for (int k = 0; k < 2; k++) {
            const int qq = c + 2 * k;
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const uint32_t scw = cur.sc[half][(2 * qq + (e >> 1)) >> 2];
              const int scv = (int)(int8_t)byte_of(scw, (2 * qq + (e >> 1)) & 3);
              const float sl = (float)(scv & 15), sr = (float)(scv - (scv & 15));
              const uint32_t sl2 = h2u(sl, sl), sr2 = h2u(sr, sr);
              uint32_t u[4];
#pragma unroll
              for (int m = 0; m < 2; m++) {
                const uint32_t lw = cur.ql[half][2 * e + m] >> (4 * k);
                const uint32_t hw = cur.qh[half][2 * e + m] >> (2 * qq);
                const uint32_t p0 = (lw & 0x000F000Fu) | ((hw & 0x00030003u) << 4);
                const uint32_t p1 = ((lw >> 8) & 0x000F000Fu) | (((hw >> 8) & 0x00030003u) << 4);
                u[2 * m] = h2sub(p0 | 0x64006400u, 0x64206420u);      // q - 32
                u[2 * m + 1] = h2sub(p1 | 0x64006400u, 0x64206420u);
              }
              const int j = qq * 4 + e;
              uint8_t* dst = A + (r >> 3) * kSBO + j * 128 + (r & 7) * 16;
              *reinterpret_cast<uint4*>(dst) =
                  make_uint4(h2mul(u[0], sl2), h2mul(u[1], sl2), h2mul(u[2], sl2), h2mul(u[3], sl2));
              *reinterpret_cast<uint4*>(dst + kTileA) =
                  make_uint4(h2mul(u[0], sr2), h2mul(u[1], sr2), h2mul(u[2], sr2), h2mul(u[3], sr2));
            }
          }
        }
        fence_proxy_async();
        mbar_arrive(&a_full[ab]);
      }
      cur = nxt;
    }
  } else if (warp < 12) {
    // ---------------- epilogue: TMEM -> per-item sums ----------------
    const int r = tid - 256;  // TMEM lane / row
    const uint32_t lane_off = (uint32_t)((warp - 8) * 32) << 16;
    const uint8_t* rp = a.w + (size_t)min(row0 + r, a.rows - 1) * a.rb;
    float acc[NI];
#pragma unroll
    for (int i = 0; i < NI; i++) acc[i] = 0.0f;
    for (int sb = 0; sb < nsb && ok; sb++) {
      const int tb = sb & 1;
      float d, dmin = 0.0f;
      if constexpr (T == LRS_GGML_Q4_K) {
        const uint32_t hx = *reinterpret_cast<const uint32_t*>(rp + (size_t)(s0 + sb) * 144);
        d = f16_bits((uint16_t)(hx & 0xffffu));
        dmin = f16_bits((uint16_t)(hx >> 16));
      } else {
        d = f16_bits(*reinterpret_cast<const uint16_t*>(rp + (size_t)(s0 + sb) * 210 + 208));
      }
      ok = mbar_wait_bounded(&acc_full[tb], (sb >> 1) & 1);
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < kN / 32; cc++) {
        float Tv[32];
        tc_ld32(tmem + lane_off + tb * 256 + 32 * cc, Tv);
        if constexpr (S::kMins) {
          float M[32];
          tc_ld32(tmem + lane_off + tb * 256 + kN + 32 * cc, M);
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const int item = 16 * cc + i;
            acc[item] = fmaf(d, Tv[2 * i] + Tv[2 * i + 1],
                             fmaf(-dmin, M[2 * i] + M[2 * i + 1], acc[item]));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const int item = 16 * cc + i;
            acc[item] = fmaf(d, Tv[2 * i] + Tv[2 * i + 1], acc[item]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[tb]);
    }
    // partial sums, in units of the true x (item scales are powers of two)
    const int row = row0 + r;
    const bool live = row < a.rows;
    if (ok && live) {
      float* pp = a.part + (size_t)blockIdx.y * a.batch * a.rows + row;
#pragma unroll
      for (int i = 0; i < NI; i++)
        if (i < a.batch) pp[(size_t)i * a.rows] = acc[i] * a.xscale[i];
    }
    if (!ok && a.error_flag) atomicExch(a.error_flag, LRS_ERR_DEVICE_TIMEOUT);
  } else if (warp == 12 && lane == 0) {
    // ---------------- issuer: x copies and MMAs ----------------
    const uint64_t pol = evict_first_policy();
    constexpr uint32_t idesc = idesc_f16(kRows, kN);
    // x tile of half step h (and, at even h, the super-block's B_min) into B[h % kBB]
    auto issue_x = [&](int h) {
      const int sbg = s0 + (h >> 1), bi = h % S::kBB;
      const bool mins = S::kMins && (h & 1) == 0;
      mbar_expect_tx(&full_b[bi], kTileB + (mins ? S::kTileBmin : 0));
      tma_load_1d(smem + S::kOffB + bi * kTileB, a.xt + (size_t)(2 * sbg + (h & 1)) * kTileB,
                  kTileB, &full_b[bi], pol);
      if (mins)
        tma_load_1d(smem + S::kOffBmin + ((h >> 1) & 1) * S::kTileBmin,
                    a.xm + (size_t)sbg * S::kTileBmin, S::kTileBmin, &full_b[bi], pol);
    };
    for (int h = 0; h < S::kBB - 1 && h < nhs; h++) issue_x(h);
    for (int hs = 0; hs < nhs && ok; hs++) {
      const int sb = hs >> 1, half = hs & 1, ab = hs % S::kAB, bb = hs % S::kBB, tb = sb & 1;
      ok = mbar_wait_bounded(&a_full[ab], (hs / S::kAB) & 1) &&
           mbar_wait_bounded(&full_b[bb], (hs / S::kBB) & 1);
      if (ok && half == 0 && sb >= 2) ok = mbar_wait_bounded(&acc_empty[tb], ((sb - 2) >> 1) & 1);
      if (!ok) break;
      tc_fence_after();
      const uint32_t d_main = tmem + tb * 256, d_min = d_main + kN;
      const uint32_t a0 = sbase + S::kOffA + ab * S::kAParts * kTileA,
                     b0 = sbase + S::kOffB + bb * kTileB;
#pragma unroll
      for (int t = 0; t < kKC / 16; t++)
#pragma unroll
        for (int part = 0; part < S::kAParts; part++)
          tc_mma(d_main, smem_desc(a0 + part * kTileA + t * 256, 128, kSBO),
                 smem_desc(b0 + t * 256, 128, kSBO), idesc, (half | t | part) != 0);
      if (S::kMins && half == 0)
        tc_mma(d_min, smem_desc(sbase + S::kOffAmin + tb * kTileMin, 128, 256),
               smem_desc(sbase + S::kOffBmin + tb * S::kTileBmin, 128, 256), idesc, 0);
      tc_commit(&mma_done[ab]);
      if (half == 1) tc_commit(&acc_full[tb]);
      // B[(hs + kBB - 1) % kBB] was last read by half step hs - 1
      const int hn = hs + S::kBB - 1;
      if (hn < nhs) {
        if (hs >= 1) ok = mbar_wait_bounded(&mma_done[(hs - 1) % S::kAB], ((hs - 1) / S::kAB) & 1);
        if (!ok) break;
        issue_x(hn);
      }
    }
    if (!ok && a.error_flag) atomicExch(a.error_flag, LRS_ERR_DEVICE_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace

bool gemm_tc_supported(const GemvParams& p) {
  // measured: Q4_K gains from 4 items up, Q6_K (two MMAs per K step) from 17
  if (p.batch < 4 || p.batch > kMaxItems || p.cols % 256) return false;
  for (int i = 0; i < p.nseg; i++) {
    if (p.seg[i].type == LRS_GGML_Q6_K && p.batch <= 16) return false;
    if (p.seg[i].type != LRS_GGML_Q4_K && p.seg[i].type != LRS_GGML_Q6_K) return false;
  }
  for (int i = 1; i < p.nseg; i++)
    if (p.seg[i].type != p.seg[0].type) return false;
  return true;
}

namespace {
int tc_items(int batch) { return batch <= 16 ? 16 : batch <= 32 ? 32 : 64; }
int tc_kgroups(const GemvParams& p, int sms) {
  int ctas = 0;
  for (int i = 0; i < p.nseg; i++) ctas += (p.seg[i].rows + kRows - 1) / kRows;
  const int nsb = p.cols / 256;
  return ctas >= sms ? 1 : std::max(1, std::min(nsb, sms / ctas));
}

template <int T, int NI>
cudaError_t launch_tc(const TcArgs& a, dim3 grid, cudaStream_t st) {
  using S = TcShape<T, NI>;
  static std::atomic<uint64_t> attr{0};
  cudaError_t e = set_smem_once(attr, (const void*)gemm_tc_kernel<T, NI>, S::kSmem);
  if (e != cudaSuccess) return e;
  gemm_tc_kernel<T, NI><<<grid, S::kThreads, S::kSmem, st>>>(a);
  return cudaGetLastError();
}

template <int NI>
cudaError_t launch_tc_type(int type, const TcArgs& a, dim3 grid, cudaStream_t st) {
  if (type == LRS_GGML_Q6_K) return launch_tc<LRS_GGML_Q6_K, NI>(a, grid, st);
  return launch_tc<LRS_GGML_Q4_K, NI>(a, grid, st);
}
}  // namespace

size_t gemm_tc_scratch_bytes(const GemvParams& p, int sms) {
  const int kg = tc_kgroups(p, sms), ni = tc_items(p.batch);
  size_t rows = 0;
  for (int i = 0; i < p.nseg; i++) rows += p.seg[i].rows;
  return (size_t)(p.cols / kKC) * tile_b(ni) + (size_t)(p.cols / 256) * tile_bmin(ni) +
         kMaxItems * 4 + (size_t)kg * p.batch * rows * 4 * (p.epi == EPI_SWIGLU ? 2 : 1) + 1024;
}

// Partial sums for every segment (and the pair's second matrix), then the
// fixed-order epilogue shared with gemm_mma.cu.
cudaError_t gemm_tc_launch(const GemvParams& p, void* scratch, int sms, cudaStream_t st) {
  const int cols = p.cols, B = p.batch, ni = tc_items(B);
  const bool pair = p.epi == EPI_SWIGLU;
  auto align = [](void* q) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(q) + 255) & ~uintptr_t(255));
  };
  uint8_t* xt = align(scratch);
  uint8_t* xm = xt + (size_t)(cols / kKC) * tile_b(ni);
  float* xscale = reinterpret_cast<float*>(xm + (size_t)(cols / 256) * tile_bmin(ni));
  float* part = xscale + kMaxItems;
  const int kgroups = tc_kgroups(p, sms);
  xsplit_tc_kernel<<<dim3(ni, 4), 256, 0, st>>>(p.x, p.x_ld, cols, B, ni, xt, xm, xscale,
                                                p.norm_w, p.norm_eps);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const float* parts[kGemvMaxSeg];
  float* cur = part;
  for (int i = 0; i < p.nseg; i++) {
    parts[i] = cur;
    for (int m = 0; m < (pair ? 2 : 1); m++) {
      TcArgs a{};
      a.w = m ? p.seg[i].w2 : p.seg[i].w;
      a.rows = p.seg[i].rows;
      a.rb = p.seg[i].rb;
      a.cols = cols;
      a.batch = B;
      a.kgroups = kgroups;
      a.xt = xt;
      a.xm = xm;
      a.xscale = xscale;
      a.part = cur;
      a.error_flag = p.error_flag;
      cur += (size_t)kgroups * B * a.rows;
      const dim3 grid((a.rows + kRows - 1) / kRows, kgroups);
      e = ni == 16 ? launch_tc_type<16>(p.seg[i].type, a, grid, st)
                   : ni == 32 ? launch_tc_type<32>(p.seg[i].type, a, grid, st)
                              : launch_tc_type<64>(p.seg[i].type, a, grid, st);
      if (e != cudaSuccess) return e;
    }
  }
  return gemm_partials_epilogue(p, parts, kgroups, st);
}

}  // namespace lrs
