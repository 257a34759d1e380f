// decode.cu -- embedding, RMSNorm, RoPE + paged KV store, split-K GQA decode
// attention and greedy bookkeeping for the Qwen2 token step (sm_100a).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <math.h>
#include <cstdlib>

#include "common.h"
#include "decode.cuh"
#include "device_common.cuh"

namespace lrs {
namespace {

// ---- embedding / dequantization (value_at, bit-exact) ---------------------
template <int T>
__global__ void __launch_bounds__(128)
    embed_kernel(const uint8_t* w, int cols, const int* rows, int row0, float* out,
                 unsigned long long* keys) {
  using BT = BlockTraits<T>;
  const int b = blockIdx.x;
  const size_t rb = (size_t)(cols / BT::kValues) * BT::kBytes;
  const int row = rows ? rows[b] : row0 + b;
  const uint8_t* rp = w + (size_t)row * rb;
  float* o = out + (size_t)b * cols;
  if (keys && threadIdx.x == 0) keys[b] = 0ull;
  for (int pc = threadIdx.x; pc < cols / 32; pc += blockDim.x) {
    const int unit = pc / BT::kPieces, sub = pc % BT::kPieces;
    float v[32];
    decode_piece<T>(rp + (size_t)unit * BT::kBytes, sub, v);
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int col = unit * BT::kValues + run_col<T>(sub, r);
#pragma unroll
      for (int i = 0; i < 8; i++) o[col + i] = v[r * 8 + i];
    }
  }
}

cudaError_t embed_dispatch(const uint8_t* w, uint32_t type, int cols, const int* rows, int row0,
                           int n, float* out, unsigned long long* keys, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  dim3 g(n), b(128);
#define LRS_EMBED(T) \
  case T: embed_kernel<T><<<g, b, 0, st>>>(w, cols, rows, row0, out, keys); break;
  switch (type) {
    LRS_EMBED(LRS_GGML_F32)
    LRS_EMBED(LRS_GGML_F16)
    LRS_EMBED(LRS_GGML_BF16)
    LRS_EMBED(LRS_GGML_Q4_0)
    LRS_EMBED(LRS_GGML_Q4_1)
    LRS_EMBED(LRS_GGML_Q5_0)
    LRS_EMBED(LRS_GGML_Q5_1)
    LRS_EMBED(LRS_GGML_Q8_0)
    LRS_EMBED(LRS_GGML_Q4_K)
    LRS_EMBED(LRS_GGML_Q5_K)
    LRS_EMBED(LRS_GGML_Q6_K)
    default: return cudaErrorInvalidValue;
  }
#undef LRS_EMBED
  return cudaGetLastError();
}

// ---- RMSNorm ---------------------------------------------------------------
__global__ void __launch_bounds__(256)
    rmsnorm_kernel(const float* x, const float* w, float eps, int n, float* out) {
  __shared__ float red[8];
  const float* xb = x + (size_t)blockIdx.x * n;
  float* ob = out + (size_t)blockIdx.x * n;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < n; i += 256) ss = fmaf(xb[i], xb[i], ss);
  for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int k = 0; k < 8; k++) tot += red[k];
  const float inv = 1.0f / sqrtf(tot / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += 256) ob[i] = xb[i] * (inv * w[i]);
}

// ---- RoPE + KV store --------------------------------------------------------
__device__ __forceinline__ size_t kv_offset(const StepIO& io, int b, int p, int nkv, int kvh,
                                            int hd) {
  const int page = io.pages[io.seq[b] * io.max_pages + p / kPageSize];
  return (((size_t)page * nkv + kvh) * kPageSize + (p % kPageSize)) * hd;
}

// One CTA per (item, head): heads [0, nh) rotate q in place; heads
// [nh, nh + nkv) rotate k and store k and v of the item's position.
__global__ void __launch_bounds__(64)
    rope_store_kernel(float* q, const float* k, const float* v, const float* cos_t,
                      const float* sin_t, StepIO io, int nh, int nkv, int hd, void* kpool,
                      void* vpool, int kv_bf16) {
  const int b = blockIdx.x, h = blockIdx.y;
  const int half = hd / 2;
  const int pos = io.pos[b];
  const float* c = cos_t + (size_t)pos * half;
  const float* s = sin_t + (size_t)pos * half;
  // apply_rope_inplace, src/model.rs:86-95 (unfused, as the reference)
  if (h < nh) {
    float* qh = q + ((size_t)b * nh + h) * hd;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      const float re = qh[i], im = qh[i + half];
      qh[i] = __fsub_rn(__fmul_rn(re, c[i]), __fmul_rn(im, s[i]));
      qh[i + half] = __fadd_rn(__fmul_rn(re, s[i]), __fmul_rn(im, c[i]));
    }
    return;
  }
  const int kvh = h - nh;
  const float* kh = k + ((size_t)b * nkv + kvh) * hd;
  const float* vh = v + ((size_t)b * nkv + kvh) * hd;
  const size_t o = kv_offset(io, b, pos, nkv, kvh, hd);
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float re = kh[i], im = kh[i + half];
    const float k0 = __fsub_rn(__fmul_rn(re, c[i]), __fmul_rn(im, s[i]));
    const float k1 = __fadd_rn(__fmul_rn(re, s[i]), __fmul_rn(im, c[i]));
    if (kv_bf16) {
      __nv_bfloat16* kp = reinterpret_cast<__nv_bfloat16*>(kpool) + o;
      __nv_bfloat16* vp = reinterpret_cast<__nv_bfloat16*>(vpool) + o;
      kp[i] = __float2bfloat16_rn(k0);
      kp[i + half] = __float2bfloat16_rn(k1);
      vp[i] = __float2bfloat16_rn(vh[i]);
      vp[i + half] = __float2bfloat16_rn(vh[i + half]);
    } else {
      float* kp = reinterpret_cast<float*>(kpool) + o;
      float* vp = reinterpret_cast<float*>(vpool) + o;
      kp[i] = k0;
      kp[i + half] = k1;
      vp[i] = vh[i];
      vp[i + half] = vh[i + half];
    }
  }
}

// ---- split-K GQA decode attention ------------------------------------------
constexpr int kMaxGroup = 8;    // query heads per KV head handled by one CTA
constexpr int kAttnWarps = 8;   // consumer warps; one more warp issues the copies
constexpr int kAttnCons = 32 * kAttnWarps;
constexpr int kAttnThreads = kAttnCons + 32;
constexpr int kTile = 32;       // positions per staged K / V tile
constexpr int kMinSplit = kTile;

// Positions of split `split` of a context of L positions: [s0, s1) with
// chunks a multiple of 32 (tiles of 32 positions never straddle a KV page).
__device__ __forceinline__ int split_chunk(int L, int nsplit) {
  const int c = max((L + nsplit - 1) / nsplit, kMinSplit);
  return (c + kTile - 1) & ~(kTile - 1);
}

// Shared-memory plan of the attention kernel for head_dim HD and KV element size.
struct AttnSmem {
  int tile, stages, ring, bars, qs, sc, pw, corr, om, total;
};
__host__ __device__ inline AttnSmem attn_smem(int hd, int esz) {
  AttnSmem a;
  a.tile = kTile * hd * esz;                      // bytes of one K (or V) tile
  a.stages = esz == 4 ? 2 : 4;                    // 64 KB of K/V in flight per CTA
  a.ring = 0;
  a.bars = a.stages * 2 * a.tile;
  a.qs = a.bars + 2 * 8 * a.stages;               // [kMaxGroup][hd] scaled q
  a.sc = a.qs + kMaxGroup * hd * 4;               // [kMaxGroup][kTile] scores
  a.pw = a.sc + kMaxGroup * kTile * 4;            // [2][kMaxGroup][kTile] probabilities
  a.corr = a.pw + 2 * kMaxGroup * kTile * 4;      // [2][kMaxGroup] rescale factors
  a.om = a.ring;                                  // [kMaxGroup][hd] merge area (after the ring's last use)
  a.total = a.corr + 2 * kMaxGroup * 4;
  return a;
}

__device__ __forceinline__ void attn_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void attn_consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kAttnCons) : "memory");
}
// Consumer barrier that also returns whether any consumer thread passed `flag`.
__device__ __forceinline__ bool attn_consumer_sync_or(bool flag) {
  uint32_t n;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.u32 p, %2, 0;\n bar.red.popc.u32 %0, 1, %1, p;\n}"
      : "=r"(n)
      : "n"(kAttnCons), "r"((uint32_t)flag)
      : "memory");
  return n != 0;
}

// Four consecutive K values of a staged row, as floats.
template <bool BF16>
__device__ __forceinline__ float4 smem4(const uint8_t* row, int f) {
  if constexpr (BF16) {
    const uint2 u = reinterpret_cast<const uint2*>(row)[f];
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
  } else {
    return reinterpret_cast<const float4*>(row)[f];
  }
}
template <bool BF16>
__device__ __forceinline__ float smem1(const uint8_t* row, int d) {
  if constexpr (BF16)
    return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(row)[d] << 16);
  else
    return reinterpret_cast<const float*>(row)[d];
}

// One CTA per (split, kv head, item) serves all G query heads of the GQA
// group, so each K/V row is read from HBM once per group
// (src/model.rs:206-231, softmax_inplace :298-313, as an online softmax over
// tiles).  A producer warp streams the split's K and V tiles (32 positions of
// one page, contiguous in the pool) into a shared-memory ring with bulk
// copies; the eight consumer warps work on every tile together:
// * scores: thread (pos, e) dots pieces e, e + 8, ... of K row `pos` with the
//   G scaled q rows (bf16 rows rotated by position so the staged rows are
//   read without bank conflicts); three shuffles finish the dot;
// * softmax: warp g keeps the running max / sum of head g and publishes the
//   tile's probabilities and the rescale factor of the earlier tiles;
// * PV: thread (d, half) accumulates o[g][d] over its half of the tile's
//   positions (quarters for HD = 64); the halves merge at the end.
// Scores, probabilities and factors are double-buffered by tile parity, so a
// tile costs two consumer barriers.  The split's (max, sum, o) go to `part`.
//
// FUSED (decode steps, one item per sequence): the kernel also does the work
// of rope_store_kernel and attn_combine_kernel.  Every CTA rotates its q rows
// itself (the same products as rope_store_kernel); the CTA whose split holds
// the item's position rotates k, stores k and v into the cache and writes the
// rounded row over the (older) staged copy of that position; the last CTA of
// an (item, kv head) to finish, found with a counter, merges the splits into
// att and resets the counter.
struct AttnArgs {
  const float* q;      // [B][nh][HD]: rotated (unfused) or as projected (FUSED)
  const float* k;      // FUSED: [B][nkv][HD] as projected
  const float* v;
  const float* cos_t;  // FUSED: [max_seq][HD / 2]
  const float* sin_t;
  StepIO io;
  int nh, nkv, nsplit;
  float scale;
  void* kpool;
  void* vpool;
  float* part;         // [B][nh][nsplit][2 + HD]
  float* att;          // FUSED: [B][nh][HD]
  unsigned* cnt;       // FUSED: [B][nkv] finished splits (zero between launches)
  int* err;
};

template <int HD, bool BF16, bool FUSED>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(const __grid_constant__ AttnArgs a) {
  constexpr int ESZ = BF16 ? 2 : 4;
  constexpr int NI = HD / 32;               // 4-value pieces of a row per thread
  constexpr int NJ = kAttnCons / HD;        // position ranges of the PV product
  constexpr int JR = kTile / NJ;            // positions per range
  constexpr int ROWB = HD * ESZ;
  constexpr int HALF = HD / 2;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint8_t newrow[2 * ROWB];      // FUSED: the position's K and V row as stored
  __shared__ int last_cta;
  const AttnSmem sp = attn_smem(HD, ESZ);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + sp.bars);
  uint64_t* empty = full + sp.stages;
  float* qs = reinterpret_cast<float*>(smem + sp.qs);
  float* sc = reinterpret_cast<float*>(smem + sp.sc);
  float* pwb = reinterpret_cast<float*>(smem + sp.pw);
  float* corrb = reinterpret_cast<float*>(smem + sp.corr);
  float* om = reinterpret_cast<float*>(smem + sp.om);

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int nh = a.nh, nkv = a.nkv, nsplit = a.nsplit;
  const int G = nh / nkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int L = a.io.pos[b] + 1, pos_new = L - 1;
  const int chunk = split_chunk(L, nsplit);
  const int s0 = split * chunk, s1 = min(L, s0 + chunk);
  const int ntiles = s0 < s1 ? (s1 - s0 + kTile - 1) / kTile : 0;
  const bool own = FUSED && s0 <= pos_new && pos_new < s1;

  if (tid == 0) {
    for (int i = 0; i < sp.stages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kAttnWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kAttnWarps) {  // producer
    if (lane == 0) {
      // decode steps: the tiles hold earlier positions only (the new one is
      // written over its staged copy), so they stream before the projection
      // that precedes this kernel has finished; prefill chunks read rows
      // rope_store_kernel just wrote
      if constexpr (!FUSED) pdl_wait();
      const uint64_t pol = evict_first_policy();
      const uint8_t* kb = reinterpret_cast<const uint8_t*>(a.kpool);
      const uint8_t* vb = reinterpret_cast<const uint8_t*>(a.vpool);
      for (int i = 0; i < ntiles; i++) {
        const int st = i % sp.stages;
        if (i >= sp.stages && !mbar_wait_bounded(&empty[st], ((i / sp.stages) - 1) & 1)) {
          atomicExch(a.err, 1);
          break;
        }
        const size_t off = kv_offset(a.io, b, s0 + kTile * i, nkv, kvh, HD) * ESZ;
        uint8_t* dst = smem + sp.ring + (size_t)st * 2 * sp.tile;
        mbar_expect_tx(&full[st], 2u * sp.tile);
        tma_load_1d(dst, kb + off, sp.tile, &full[st], pol);
        tma_load_1d(dst + sp.tile, vb + off, sp.tile, &full[st], pol);
      }
      // stay until the last copies have landed (they may outlive the consumers
      // on an error exit)
      for (int i = max(0, ntiles - sp.stages); i < ntiles; i++)
        if (!mbar_wait_bounded(&full[i % sp.stages], (i / sp.stages) & 1)) atomicExch(a.err, 1);
    }
    return;
  }


  pdl_wait();  // q, k, v come from the projection launched before this kernel
  const float* cs = FUSED ? a.cos_t + (size_t)pos_new * HALF : nullptr;
  const float* sn = FUSED ? a.sin_t + (size_t)pos_new * HALF : nullptr;
  // RoPE (apply_rope_inplace, src/model.rs:86-95) of element d of a head row
  auto rope = [&](const float* r, int d) {
    const int i = d % HALF;
    const float re = r[i], im = r[i + HALF];
    return d < HALF ? __fsub_rn(__fmul_rn(re, cs[i]), __fmul_rn(im, sn[i]))
                    : __fadd_rn(__fmul_rn(re, sn[i]), __fmul_rn(im, cs[i]));
  };
  for (int i = tid; i < kMaxGroup * HD; i += kAttnCons) {
    const int g = i / HD, d = i % HD;
    float val = 0.0f;
    if (g < G) {
      const float* qh = a.q + ((size_t)b * nh + kvh * G + g) * HD;
      val = (FUSED ? rope(qh, d) : qh[d]) * a.scale;
    }
    qs[i] = val;
  }
  if (own && tid < HD) {  // KVCache::update (src/cache.rs:38-53) of this head
    const float* kh = a.k + ((size_t)b * nkv + kvh) * HD;
    const float kr = rope(kh, tid), vr = a.v[((size_t)b * nkv + kvh) * HD + tid];
    const size_t o = kv_offset(a.io, b, pos_new, nkv, kvh, HD) + tid;
    if constexpr (BF16) {
      const __nv_bfloat16 kb = __float2bfloat16_rn(kr), vb = __float2bfloat16_rn(vr);
      reinterpret_cast<__nv_bfloat16*>(a.kpool)[o] = kb;
      reinterpret_cast<__nv_bfloat16*>(a.vpool)[o] = vb;
      reinterpret_cast<__nv_bfloat16*>(newrow)[tid] = kb;
      reinterpret_cast<__nv_bfloat16*>(newrow + ROWB)[tid] = vb;
    } else {
      reinterpret_cast<float*>(a.kpool)[o] = kr;
      reinterpret_cast<float*>(a.vpool)[o] = vr;
      reinterpret_cast<float*>(newrow)[tid] = kr;
      reinterpret_cast<float*>(newrow + ROWB)[tid] = vr;
    }
  }
  attn_consumer_sync();

  float m = -INFINITY, l = 0.0f;  // running state of head `warp` (softmax warps)
  float o[kMaxGroup];
#pragma unroll
  for (int g = 0; g < kMaxGroup; g++) o[g] = 0.0f;
  const int pos = tid >> 3, e8 = tid & 7;
  const int rot = BF16 ? (pos & 1) : 0;
  const int d = tid % HD, jr = tid / HD;
  bool ok = true;
  for (int i = 0; i < ntiles; i++) {
    const int st = i % sp.stages;
    const bool got = mbar_wait_bounded(&full[st], (i / sp.stages) & 1);
    uint8_t* K = smem + sp.ring + (size_t)st * 2 * sp.tile;
    uint8_t* V = K + sp.tile;
    const int t0 = s0 + kTile * i;
    const int nv = min(kTile, s1 - t0);
    float* pw = pwb + (i & 1) * kMaxGroup * kTile;
    float* corr = corrb + (i & 1) * kMaxGroup;
    if (own && pos_new - t0 < kTile && pos_new >= t0) {
      // the staged copy of the new position predates this step's store
      const int r = pos_new - t0;
      for (int u = tid; u < ROWB / 4; u += kAttnCons) {
        reinterpret_cast<uint32_t*>(K + r * ROWB)[u] = reinterpret_cast<const uint32_t*>(newrow)[u];
        reinterpret_cast<uint32_t*>(V + r * ROWB)[u] =
            reinterpret_cast<const uint32_t*>(newrow + ROWB)[u];
      }
      fence_proxy_async();  // the slot is refilled by bulk copies later
      attn_consumer_sync();
    }
    // scores of the tile
    {
      float acc[kMaxGroup];
#pragma unroll
      for (int g = 0; g < kMaxGroup; g++) acc[g] = 0.0f;
      const uint8_t* krow = K + pos * ROWB;
#pragma unroll
      for (int ii = 0; ii < NI; ii++) {
        const int f = ((ii + rot) % NI) * 8 + e8;
        const float4 kv = smem4<BF16>(krow, f);
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
          if (g < G) {
            const float4 qq = reinterpret_cast<const float4*>(qs + g * HD)[f];
            acc[g] = fmaf(qq.x, kv.x, fmaf(qq.y, kv.y, fmaf(qq.z, kv.z, fmaf(qq.w, kv.w, acc[g]))));
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kMaxGroup; g++) {
        if (g < G) {
          acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 1);
          acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 2);
          acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 4);
          if (e8 == 0) sc[g * kTile + pos] = acc[g];
        }
      }
    }
    if (attn_consumer_sync_or(!got)) {  // a copy never landed: every consumer leaves
      if (tid == 0) atomicExch(a.err, 1);
      ok = false;
      break;
    }
    // online softmax of head `warp` over the tile (lane = position)
    if (warp < G) {
      const bool valid = lane < nv;
      const float s = valid ? sc[warp * kTile + lane] : -INFINITY;
      float bm = s;
#pragma unroll
      for (int w = 16; w >= 1; w >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, w));
      const float mn = fmaxf(m, bm);  // finite: position 0 of a tile is valid
      const float cf = m == -INFINITY ? 0.0f : expf(m - mn);
      const float ev = valid ? expf(s - mn) : 0.0f;
      float es = ev;
#pragma unroll
      for (int w = 16; w >= 1; w >>= 1) es += __shfl_xor_sync(0xffffffffu, es, w);
      l = l * cf + es;
      m = mn;
      pw[warp * kTile + lane] = ev;
      if (lane == 0) corr[warp] = cf;
    }
    attn_consumer_sync();
    // PV over this thread's position range: o[g][d] = o[g][d] * corr[g] + sum_j p[g][j] V[j][d]
#pragma unroll
    for (int g = 0; g < kMaxGroup; g++)
      if (g < G) o[g] *= corr[g];
    const int j0 = jr * JR, j1 = min(nv, j0 + JR);
    if (j1 - j0 == JR) {
#pragma unroll
      for (int j = j0; j < j0 + JR; j += 4) {
        const float v0 = smem1<BF16>(V + (j + 0) * ROWB, d), v1 = smem1<BF16>(V + (j + 1) * ROWB, d);
        const float v2 = smem1<BF16>(V + (j + 2) * ROWB, d), v3 = smem1<BF16>(V + (j + 3) * ROWB, d);
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
          if (g < G) {
            const float4 pp = *reinterpret_cast<const float4*>(pw + g * kTile + j);
            o[g] = fmaf(pp.w, v3, fmaf(pp.z, v2, fmaf(pp.y, v1, fmaf(pp.x, v0, o[g]))));
          }
        }
      }
    } else {
      for (int j = j0; j < j1; j++) {
        const float v = smem1<BF16>(V + j * ROWB, d);
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++)
          if (g < G) o[g] = fmaf(pw[g * kTile + j], v, o[g]);
      }
    }
    __syncwarp();
    if (lane == 0) attn_arrive(&empty[st]);
  }
  pdl_launch_dependents();
  // per-head totals, then merge the position ranges and write (max, sum, o)
  if (warp < G && lane == 0) {
    om[warp * 2] = m;  // om is free until the merge below
    om[warp * 2 + 1] = l;
  }
  attn_consumer_sync();
  float Mg[kMaxGroup], Lg[kMaxGroup];
#pragma unroll
  for (int g = 0; g < kMaxGroup; g++) {
    Mg[g] = g < G ? om[g * 2] : 0.0f;
    Lg[g] = g < G ? om[g * 2 + 1] : 0.0f;
  }
  for (int r = 1; r < NJ; r++) {
    attn_consumer_sync();
    if (jr == r)
#pragma unroll
      for (int g = 0; g < kMaxGroup; g++)
        if (g < G) om[g * HD + d] = o[g];
    attn_consumer_sync();
    if (jr == 0)
#pragma unroll
      for (int g = 0; g < kMaxGroup; g++)
        if (g < G) o[g] += om[g * HD + d];
  }
  if (jr == 0) {
    const bool any = ok && ntiles > 0;
#pragma unroll
    for (int g = 0; g < kMaxGroup; g++) {
      if (g < G) {
        float* pp = a.part + (((size_t)b * nh + kvh * G + g) * nsplit + split) * (HD + 2);
        if (d == 0) {
          pp[0] = any ? Mg[g] : -INFINITY;
          pp[1] = any ? Lg[g] : 0.0f;
        }
        pp[2 + d] = any ? o[g] : 0.0f;
      }
    }
  }
  if constexpr (FUSED) {
    // the last split of (item, kv head) to finish merges them (threadfence
    // reduction: partials visible before the count, read after it)
    attn_consumer_sync();
    if (tid == 0) {
      __threadfence();
      unsigned* c = a.cnt + (size_t)b * nkv + kvh;
      last_cta = atomicAdd(c, 1u) == (unsigned)(nsplit - 1);
      if (last_cta) *c = 0u;
    }
    attn_consumer_sync();
    if (last_cta) {
      __threadfence();
      // warp g merges head g: lanes weigh the splits, then sweep the dims
      const int nact = min(nsplit, (L + chunk - 1) / chunk);  // splits that saw positions
      if (warp < G) {
        const float* pp = a.part + ((size_t)b * nh + kvh * G + warp) * nsplit * (HD + 2);
        float* w = pwb + warp * 64;  // the probabilities are no longer needed
        const float m0 = lane < nact ? __ldcg(pp + lane * (HD + 2)) : -INFINITY;
        const float m1 = lane + 32 < nact ? __ldcg(pp + (lane + 32) * (HD + 2)) : -INFINITY;
        float M = fmaxf(m0, m1);
#pragma unroll
        for (int o2 = 16; o2 >= 1; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
        const float w0 = m0 == -INFINITY ? 0.0f : expf(m0 - M);
        const float w1 = m1 == -INFINITY ? 0.0f : expf(m1 - M);
        float Ls = (lane < nact ? __ldcg(pp + lane * (HD + 2) + 1) * w0 : 0.0f) +
                   (lane + 32 < nact ? __ldcg(pp + (lane + 32) * (HD + 2) + 1) * w1 : 0.0f);
#pragma unroll
        for (int o2 = 16; o2 >= 1; o2 >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, o2);
        w[lane] = w0;
        w[lane + 32] = w1;
        __syncwarp();
        float O[HD / 32];
#pragma unroll
        for (int k = 0; k < HD / 32; k++) O[k] = 0.0f;
#pragma unroll 4
        for (int s2 = 0; s2 < nact; s2++) {
          const float ws = w[s2];
#pragma unroll
          for (int k = 0; k < HD / 32; k++)
            O[k] = fmaf(__ldcg(pp + s2 * (HD + 2) + 2 + lane + 32 * k), ws, O[k]);
        }
        float* out = a.att + ((size_t)b * nh + kvh * G + warp) * HD;
#pragma unroll
        for (int k = 0; k < HD / 32; k++) out[lane + 32 * k] = O[k] / Ls;
      }
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(HD) attn_combine_kernel(const float* part, const int* pos,
                                                          int nh, int nsplit, float* att) {
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const float* pp = part + ((size_t)b * nh + h) * nsplit * (HD + 2);
  const int L = pos[b] + 1;
  const int chunk = split_chunk(L, nsplit);
  const int nact = min(nsplit, (L + chunk - 1) / chunk);  // splits that saw positions
  __shared__ float wsh[64];
  __shared__ float Lsum;
  if (d < 32) {
    // weights exp(m_s - M) of the active splits, and the total softmax denominator
    float m0 = d < nact ? pp[d * (HD + 2)] : -INFINITY;
    float m1 = d + 32 < nact ? pp[(d + 32) * (HD + 2)] : -INFINITY;
    float M = fmaxf(m0, m1);
    for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float w0 = m0 == -INFINITY ? 0.0f : expf(m0 - M);
    const float w1 = m1 == -INFINITY ? 0.0f : expf(m1 - M);
    float l = (d < nact ? pp[d * (HD + 2) + 1] * w0 : 0.0f) +
              (d + 32 < nact ? pp[(d + 32) * (HD + 2) + 1] * w1 : 0.0f);
    for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    wsh[d] = w0;
    wsh[d + 32] = w1;
    if (d == 0) Lsum = l;
  }
  __syncthreads();
  float O = 0.0f;
  for (int s = 0; s < nact; s++) O += pp[s * (HD + 2) + 2 + d] * wsh[s];
  att[((size_t)b * nh + h) * HD + d] = O / Lsum;
}

__global__ void advance_kernel(const unsigned long long* keys, int* tok, int* pos, int batch,
                               int* step, int n_steps, uint32_t* tokens_out, uint32_t* last) {
  const int s = *step;
  for (int b = threadIdx.x; b < batch; b += blockDim.x) {
    const uint32_t t = (uint32_t)(keys[b] & 0xffffffffull);
    tok[b] = (int)t;
    pos[b] += 1;
    if (last) last[b] = t;
    if (tokens_out && s < n_steps) tokens_out[(size_t)s * batch + b] = t;
  }
  __syncthreads();
  if (threadIdx.x == 0) *step = s + 1;
}

}  // namespace

cudaError_t launch_embed(const uint8_t* w, uint32_t type, int cols, const int* rows, int n,
                         float* out, unsigned long long* keys, cudaStream_t st) {
  return embed_dispatch(w, type, cols, rows, 0, n, out, keys, st);
}

cudaError_t launch_dequant_rows(const uint8_t* w, uint32_t type, int cols, int row0, int n,
                                float* out, cudaStream_t st) {
  return embed_dispatch(w, type, cols, nullptr, row0, n, out, nullptr, st);
}

cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int n, int batch, float* out,
                           cudaStream_t st) {
  rmsnorm_kernel<<<batch, 256, 0, st>>>(x, w, eps, n, out);
  return cudaGetLastError();
}

cudaError_t launch_rope_store(float* q, const float* k, const float* v, const float* cos_t,
                              const float* sin_t, StepIO io, int batch, int nh, int nkv, int hd,
                              void* kpool, void* vpool, int kv_bf16, cudaStream_t st) {
  rope_store_kernel<<<dim3(batch, nh + nkv), 64, 0, st>>>(q, k, v, cos_t, sin_t, io, nh, nkv, hd,
                                                          kpool, vpool, kv_bf16);
  return cudaGetLastError();
}

const void* attn_kernel_for(int hd, int kv_bf16, bool fused) {
#define LRS_AK(HD, BF)                                                                   \
  return fused ? (const void*)attn_split_kernel<HD, BF, true>                            \
               : (const void*)attn_split_kernel<HD, BF, false>;
  if (hd == 128) {
    if (kv_bf16) { LRS_AK(128, true) }
    LRS_AK(128, false)
  }
  if (hd == 64) {
    if (kv_bf16) { LRS_AK(64, true) }
    LRS_AK(64, false)
  }
#undef LRS_AK
  return nullptr;
}

// Sets the shared-memory attributes of every variant (once per device).
cudaError_t attn_attributes() {
  static thread_local int attr_dev = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || attr_dev == dev) return e;
  for (int h : {64, 128})
    for (int bf : {0, 1})
      for (bool fu : {false, true}) {
        const void* k = attn_kernel_for(h, bf, fu);
        if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      attn_smem(h, bf ? 2 : 4).total)) != cudaSuccess ||
            (e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100)) !=
                cudaSuccess)
          return e;
      }
  attr_dev = dev;
  return cudaSuccess;
}

int attention_ctas_per_sm(int hd, int kv_bf16) {
  const void* k = attn_kernel_for(hd, kv_bf16, true);
  if (!k || attn_attributes() != cudaSuccess) return 1;
  int n = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kAttnThreads,
                                                    attn_smem(hd, kv_bf16 ? 2 : 4).total) !=
      cudaSuccess)
    return 1;
  return n < 1 ? 1 : n;
}

cudaError_t launch_attention(const AttnLaunch& l, cudaStream_t st) {
  if (l.nh / l.nkv > kMaxGroup || l.nsplit > 64) return cudaErrorInvalidValue;
  const void* k = attn_kernel_for(l.hd, l.kv_bf16, l.fused);
  if (!k) return cudaErrorInvalidValue;
  cudaError_t e = attn_attributes();
  if (e != cudaSuccess) return e;
  AttnArgs a;
  a.q = l.q, a.k = l.k, a.v = l.v, a.cos_t = l.cos_t, a.sin_t = l.sin_t;
  a.io = l.io;
  a.nh = l.nh, a.nkv = l.nkv, a.nsplit = l.nsplit;
  a.scale = 1.0f / sqrtf((float)l.hd);
  a.kpool = l.kpool, a.vpool = l.vpool;
  a.part = l.part, a.att = l.att, a.cnt = l.cnt, a.err = l.err;
  void* args[] = {&a};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(l.nsplit, l.nkv, l.batch);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = attn_smem(l.hd, l.kv_bf16 ? 2 : 4).total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelExC(&cfg, k, args);
  if (e != cudaSuccess || l.fused) return e;
  if (l.hd == 128)
    attn_combine_kernel<128><<<dim3(l.nh, l.batch), 128, 0, st>>>(l.part, l.io.pos, l.nh, l.nsplit,
                                                                  l.att);
  else
    attn_combine_kernel<64><<<dim3(l.nh, l.batch), 64, 0, st>>>(l.part, l.io.pos, l.nh, l.nsplit,
                                                                l.att);
  return cudaGetLastError();
}

// dst[b][j] = src[b][j - lo] for lo <= j < lo + n, else 0 (j < width): the
// rank's x of a windowed column shard, zero outside its columns.
__global__ void pad_copy_kernel(const float* src, int n, float* dst, int width, int lo, int batch) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)batch * width) return;
  const int b = (int)(i / width), j = (int)(i % width) - lo;
  dst[i] = j >= 0 && j < n ? src[(size_t)b * n + j] : 0.0f;
}

// g[i] = silu(g[i]) * u[i] (src/model.rs:251-254), for gate and up
// projections of different GGML types that ran as two launches.
__global__ void swiglu_kernel(float* g, const float* u, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float y = g[i];
    g[i] = (y / (1.0f + expf(-y))) * u[i];
  }
}

__global__ void key_offset_kernel(unsigned long long* keys, int n, uint32_t offset) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n && keys[i]) keys[i] += offset;
}

cudaError_t launch_pad_copy(const float* src, int n, float* dst, int width, int lo, int batch,
                            cudaStream_t st) {
  const size_t total = (size_t)batch * width;
  if (total == 0) return cudaSuccess;
  pad_copy_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(src, n, dst, width, lo, batch);
  return cudaGetLastError();
}

cudaError_t launch_swiglu(float* g, const float* u, size_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  swiglu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(g, u, n);
  return cudaGetLastError();
}

cudaError_t launch_key_offset(unsigned long long* keys, int n, uint32_t offset, cudaStream_t st) {
  key_offset_kernel<<<(n + 63) / 64, 64, 0, st>>>(keys, n, offset);
  return cudaGetLastError();
}

cudaError_t launch_advance(const unsigned long long* keys, int* tok, int* pos, int batch,
                           int* step, int n_steps, uint32_t* tokens_out, uint32_t* last,
                           cudaStream_t st) {
  advance_kernel<<<1, 64, 0, st>>>(keys, tok, pos, batch, step, n_steps, tokens_out, last);
  return cudaGetLastError();
}

}  // namespace lrs
