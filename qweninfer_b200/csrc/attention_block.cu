// Prefill attention over blocks of query tokens on the tensor cores
// (qweninfer/models/qwen2.py:184-199 with S > 1: causal attention of a prompt's tokens over
// the cache row they were just written to, kv_cache.py:48-63).
//
// The per-token kernel (attention.cu) gives every query token its own CTA, so a prompt of
// P tokens streams its K/V prefix P times, and its CUDA-core dot products are bound by
// shared-memory reads. Here one CTA takes a block of 16 consecutive query tokens and one
// KV head. When the block's tokens share a cache row (the tokens of one prompt), its 128
// query rows (token j, head h) -> row 8 j + h (h = 7 is padding) form the M = 128 operand
// of tcgen05 UMMAs, and the keys stream in 64-key tiles:
//   S = Q K^T      M 128 x N 64 (keys) x K 64 (dims), fp32 in TMEM columns 0..63
//   O_t = P V      M 128 x N 64 (dims) x K 64 (keys), fp32 in TMEM columns 64..127
// q and p carry fp32 precision as hi + lo bf16 halves (two UMMA chains into one
// accumulator: hi*b + lo*b, ~16 mantissa bits); K and V are the cache's bf16 values. Thread
// r (4 warps, warp w on TMEM lanes 32w..) owns query row r: it reads its 64 scores, runs
// the fp32 online softmax of its row (keys after the token's position masked), writes its
// p row (hi/lo) as the A operand of the P.V product, and accumulates O = O * alpha + O_t
// in registers. Operands sit in shared memory in the SWIZZLE_NONE K-major layout of
// tcgen05 descriptors (core matrices of 8 rows x 16 bytes; 1 KB per 8-row group, 128 B
// between core matrices along K): K rows are copied in 16-byte chunks, V is transposed on
// the way (its K dimension is the key). The next tile's K/V are loaded into registers
// while the current tile's products run and stored into the other buffer.
//
// A block whose tokens lie in several rows (a prompt boundary, or the prompts' last tokens
// that a batched prefill places after all other tokens) runs token by token on CUDA cores:
// warp w takes tokens w, w + 4, .., streaming each token's keys in 32-key chunks through a
// private shared-memory slice.
//
// Token t's output is written like the per-token kernel's (fp32 rows and/or the o
// projection's activation tiles); a position or row outside the cache is reported as
// QI_ERR_INDEX and nothing is read or written for that token.
#include "common.cuh"
#include "internal.h"
#include "tc_proj.h"
#include "tc_device.cuh"
#include "attention_device.cuh"

namespace qi {

namespace {

using namespace tc;

constexpr int kQB = 16;          // query tokens per block
constexpr int kThreads = 128;    // one thread per query row
constexpr int kKT = 64;          // keys per tile
constexpr int kChunk = 32;       // keys per step of the token-by-token path
constexpr uint32_t kTmemCols = 256;  // S double buffer (0..63, 64..127), O_t (128..191)

// shared memory (byte offsets)
constexpr uint32_t kQhi = 0, kQlo = 16384;      // 128 x 64 bf16 each
constexpr uint32_t kK0 = 32768;                 // K tiles [2]: 64 keys x 64 dims, 8 KB each
constexpr uint32_t kVt0 = 49152;                // V^T tiles [2]: 64 dims x 64 keys
constexpr uint32_t kPhi = 65536, kPlo = 81920;  // 128 x 64 bf16 each
constexpr uint32_t kMisc = 98304;
constexpr uint32_t kSmemBytes = kMisc + 512;

// A block's valid tokens grouped by cache row: segment s = the tokens of row seg_row[s]
// (seg_n of them, keys 0 .. seg_kmax - 1); tok_seg[j] = segment of token j, or -1.
struct Misc {
  uint64_t bar_s[2], bar_o;
  uint32_t tmem;
  int nseg;
  int pos[kQB];  // position of each token, -1 when it is past M or outside the cache
  int row[kQB];
  int tok_seg[kQB];
  int seg_row[kQB], seg_kmax[kQB], seg_n[kQB];
};
static_assert(sizeof(Misc) <= 512, "misc area");

// token-by-token path: per warp, q of 7 heads [h][half][chunk][4] (fp32, scaled), the V
// rows of a 32-key chunk and its probabilities; the slices reuse the P area
constexpr int kSliceQ = kGqa * kHeadDim * 4;
constexpr int kSliceV = kChunk * kHeadDim * 2;
constexpr int kSliceBytes = kSliceQ + kSliceV + kGqa * kChunk * 4;
static_assert(4 * kSliceBytes <= 32768, "token slices fit the P area");

// K/V offset of (row, head g, first key k0 of a tile or chunk); an unmapped page is
// reported and read from the layer's start (in bounds)
__device__ __forceinline__ long long kv_base(const AttnParams& p, int row, int g, int k0) {
  const long long o = kv_offset(p.kv, p.max_len, row, g, k0);
  if (o < 0 && p.err) atomicExch(p.err, QI_ERR_INDEX);
  return o < 0 ? 0 : o;
}

// One tile's K and V (keys k0 .. k0 + nk - 1 of a row's head) as 4 + 4 16-byte chunks per
// thread: chunk q = tid + 128 j is key 8 (q >> 6) + (q & 7), dims 8 ((q >> 3) & 7) ..; keys
// past nk read as zeros. The 8 lanes of a store phase hold 8 keys of one chunk column.
struct TileRegs {
  uint4 k[4], v[4];
};

// kt / vt: the tile's first key (a tile never straddles a page)
__device__ __forceinline__ void tile_load(TileRegs& R, const uint16_t* kt, const uint16_t* vt, int nk, int tid) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = tid + 128 * j;
    const int n = ((q >> 6) << 3) | (q & 7), c = (q >> 3) & 7;
    if (n < nk) {
      const long long o = (long long)n * kHeadDim + c * 8;
      R.k[j] = __ldcg(reinterpret_cast<const uint4*>(kt + o));
      R.v[j] = __ldcg(reinterpret_cast<const uint4*>(vt + o));
    } else {
      R.k[j] = R.v[j] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

__device__ __forceinline__ void tile_store(const TileRegs& R, uint8_t* smem, int buf, int tid) {
  uint8_t* kt = smem + kK0 + buf * 8192;
  uint8_t* vt = smem + kVt0 + buf * 8192;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = tid + 128 * j;
    const int n = ((q >> 6) << 3) | (q & 7), c = (q >> 3) & 7;
    *reinterpret_cast<uint4*>(kt + kmaj(n, c)) = R.k[j];
    // V^T: element (dim 8c + e, key n) of the (dims x keys) K-major operand
    const uint32_t w[4] = {R.v[j].x, R.v[j].y, R.v[j].z, R.v[j].w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint16_t hv = (uint16_t)((e & 1) ? (w[e >> 1] >> 16) : (w[e >> 1] & 0xffffu));
      *reinterpret_cast<uint16_t*>(vt + c * 1024 + (n >> 3) * 128 + e * 16 + (n & 7) * 2) = hv;
    }
  }
}

// Tokens whose segment has one token, on CUDA cores: warp w takes the w-th, (w+4)-th, ..
// such token of the block.
__device__ __forceinline__ void token_path(const AttnParams& p, uint8_t* smem, const Misc& X, int t0, int g,
                                           int warp, int lane) {
  uint8_t* slice = smem + kPhi + warp * kSliceBytes;
  float* qs = reinterpret_cast<float*>(slice);                          // [7][2][8][4]
  uint16_t* vs = reinterpret_cast<uint16_t*>(slice + kSliceQ);          // [32 keys][64]
  float* ps_ = reinterpret_cast<float*>(slice + kSliceQ + kSliceV);     // [7 heads][32 keys]
  int nth = 0;  // singleton tokens seen so far
#pragma unroll 1
  for (int j = 0; j < kQB; ++j) {
    const int sg = X.tok_seg[j];
    if (sg < 0 || X.seg_n[sg] != 1) continue;
    if ((nth++ & 3) != warp) continue;
    const int ps = X.pos[j];
    const int t = t0 + j;
    {
      constexpr int kPerLane = kGqa * kHeadDim / 32;  // 14
      float qv[kPerLane];
#pragma unroll
      for (int i = 0; i < kPerLane; ++i)
        qv[i] = __ldcg(p.q + (long long)t * kHidden + g * kGqa * kHeadDim + lane + 32 * i);
      __syncwarp();  // the previous token's reads of the slice are done
#pragma unroll
      for (int i = 0; i < kPerLane; ++i) {
        const int idx = lane + 32 * i, h = idx >> 6, d = idx & 63;
        qs[((h * 2 + ((d & 7) >> 2)) * 8 + (d >> 3)) * 4 + (d & 3)] = qv[i] * 0.125f;
      }
      __syncwarp();
    }
    float m[kGqa], l[kGqa], acc[kGqa][2];
#pragma unroll
    for (int h = 0; h < kGqa; ++h) {
      m[h] = -INFINITY;
      l[h] = 0.f;
      acc[h][0] = acc[h][1] = 0.f;
    }
    for (int k0 = 0; k0 <= ps; k0 += kChunk) {
      const int key = k0 + lane;
      const bool valid = key <= ps;
      const long long cb = kv_base(p, X.row[j], g, k0) + (long long)(valid ? lane : 0) * kHeadDim;
      const uint4* krow = reinterpret_cast<const uint4*>(p.kc + cb);
      const uint4* vrow = reinterpret_cast<const uint4*>(p.vc + cb);
      // V chunks in rotated order (vx[c] = chunk (c + lane) & 7), so the stores of the 8
      // lanes of a phase hit distinct banks
      uint4 kx[8], vx[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        kx[c] = __ldcg(krow + c);
        vx[c] = __ldcg(vrow + ((c + lane) & 7));
      }
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(vs + lane * kHeadDim + ((c + lane) & 7) * 8) =
            valid ? vx[c] : make_uint4(0u, 0u, 0u, 0u);
      float s[kGqa];
#pragma unroll
      for (int h = 0; h < kGqa; ++h) s[h] = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 x = kx[c];
        const float a0 = bf16lo(x.x), a1 = bf16hi(x.x), a2 = bf16lo(x.y), a3 = bf16hi(x.y);
        const float a4 = bf16lo(x.z), a5 = bf16hi(x.z), a6 = bf16lo(x.w), a7 = bf16hi(x.w);
#pragma unroll
        for (int h = 0; h < kGqa; ++h) {
          const float4 qa = *reinterpret_cast<const float4*>(&qs[((h * 2 + 0) * 8 + c) * 4]);
          const float4 qb = *reinterpret_cast<const float4*>(&qs[((h * 2 + 1) * 8 + c) * 4]);
          float u = s[h];
          u = fmaf(qa.x, a0, u);
          u = fmaf(qa.y, a1, u);
          u = fmaf(qa.z, a2, u);
          u = fmaf(qa.w, a3, u);
          u = fmaf(qb.x, a4, u);
          u = fmaf(qb.y, a5, u);
          u = fmaf(qb.z, a6, u);
          u = fmaf(qb.w, a7, u);
          s[h] = u;
        }
      }
#pragma unroll
      for (int h = 0; h < kGqa; ++h) {
        const float sv = valid ? s[h] : -INFINITY;
        const float mn = fmaxf(m[h], warp_max(sv));  // key 0 is always valid: mn is finite
        const float alpha = expf(m[h] - mn);
        const float pr = valid ? expf(sv - mn) : 0.f;
        l[h] = l[h] * alpha + warp_sum(pr);
        acc[h][0] *= alpha;
        acc[h][1] *= alpha;
        m[h] = mn;
        ps_[h * kChunk + lane] = pr;
      }
      __syncwarp();
      const int nk = min(kChunk, ps + 1 - k0);
      for (int jj = 0; jj < nk; ++jj) {
        const uint32_t v2 = *reinterpret_cast<const uint32_t*>(vs + jj * kHeadDim + 2 * lane);
        const float v0 = bf16lo(v2), v1 = bf16hi(v2);
#pragma unroll
        for (int h = 0; h < kGqa; ++h) {
          const float pr = ps_[h * kChunk + jj];
          acc[h][0] = fmaf(pr, v0, acc[h][0]);
          acc[h][1] = fmaf(pr, v1, acc[h][1]);
        }
      }
      __syncwarp();
    }
#pragma unroll
    for (int h = 0; h < kGqa; ++h) {
      const float inv = 1.f / l[h];
      const int f = (g * kGqa + h) * kHeadDim + 2 * lane;
      attn::emit(p, t, f, acc[h][0] * inv);
      attn::emit(p, t, f + 1, acc[h][1] * inv);
    }
  }
}

// The tensor-core path for segment sg of the block (its tokens' rows are live, the other
// rows zero). nb_s0 / nb_s1 / nb_o count the completions of bar_s[0], bar_s[1] and bar_o
// so far (their parities), carried across the block's segments.
__device__ __forceinline__ void tc_segment(const AttnParams& p, uint8_t* smem, Misc& X, int t0, int g, int tid,
                                           int sg, uint32_t& nb_s0, uint32_t& nb_s1, uint32_t& nb_o) {
  const int warp = tid >> 5;
  const int kmax = X.seg_kmax[sg];
  // this thread's query row: token j, head h (h = 7 and tokens of other segments are zero rows)
  const int j = tid >> 3, h = tid & 7;
  const int ps = X.pos[j];
  const bool live = h < kGqa && X.tok_seg[j] == sg;
  {
    uint4 hi[8], lo[8];
    const float4* qrow = reinterpret_cast<const float4*>(p.q + (long long)min(t0 + j, p.M - 1) * kHidden +
                                                         (g * kGqa + min(h, kGqa - 1)) * kHeadDim);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
      if (live) {
        a = __ldcg(qrow + 2 * c);
        b = __ldcg(qrow + 2 * c + 1);
      }
      const float v[8] = {a.x * 0.125f, a.y * 0.125f, a.z * 0.125f, a.w * 0.125f,
                          b.x * 0.125f, b.y * 0.125f, b.z * 0.125f, b.w * 0.125f};
      split8(v, hi[c], lo[c]);
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      *reinterpret_cast<uint4*>(smem + kQhi + kmaj(tid, c)) = hi[c];
      *reinterpret_cast<uint4*>(smem + kQlo + kmaj(tid, c)) = lo[c];
    }
  }
  const int srow = X.seg_row[sg];
  auto load = [&](TileRegs& T, int k0, int nk) {
    const long long o = kv_base(p, srow, g, k0);
    tile_load(T, p.kc + o, p.vc + o, nk, tid);
  };
  const int ntiles = (kmax + kKT - 1) / kKT;
  TileRegs R;
  load(R, 0, min(kKT, kmax));
  tile_store(R, smem, 0, tid);
  if (ntiles > 1) load(R, kKT, min(kKT, kmax - kKT));
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = X.tmem;
  const uint32_t t_row = tmem + ((uint32_t)(warp * 32) << 16);  // this warp's TMEM lanes
  const uint32_t idesc = idesc_bf16(128, 64);
  const uint32_t sb = smem_u32(smem);
  // S(i) = (q_hi + q_lo) K(i)^T into TMEM columns 64 (i & 1)
  auto issue_qk = [&](int i) {
    tc_fence_after();
    const uint64_t kd = kmajor_desc(sb + kK0 + (i & 1) * 8192);
    const uint32_t d = tmem + (uint32_t)(64 * (i & 1));
    umma_bf16_kblock(d, kmajor_desc(sb + kQhi), kd, idesc, 0u);
    umma_bf16_kblock(d, kmajor_desc(sb + kQlo), kd, idesc, 1u);
    umma_commit(&X.bar_s[i & 1]);
  };
  if (tid == 0) issue_qk(0);

  float m = -INFINITY, l = 0.f, acc[64];
#pragma unroll
  for (int d = 0; d < 64; ++d) acc[d] = 0.f;

  for (int i = 0; i < ntiles; ++i) {
    const int b = i & 1, k0 = i * kKT;
    // tile i + 1 into the other buffer (its last readers, QK(i-1) and PV(i-1), are done),
    // tile i + 2 requested
    if (i + 1 < ntiles) {
      tile_store(R, smem, b ^ 1, tid);
      if (i + 2 < ntiles) load(R, k0 + 2 * kKT, min(kKT, kmax - k0 - 2 * kKT));
    }
    const uint32_t par = b ? (nb_s1++ & 1u) : (nb_s0++ & 1u);
    mbar_wait(&X.bar_s[b], par, p.err);
    tc_fence_after();
    float s[64];
    tmem_ld64(t_row + (uint32_t)(64 * b), s);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();  // S(i) read by every thread; K/V(i + 1) in place
    if (tid == 0 && i + 1 < ntiles) issue_qk(i + 1);  // runs during this tile's softmax
    // online softmax of this row over the tile's keys k0 .. k0 + 63 (valid: <= ps)
    const int nv = live ? min(64, ps + 1 - k0) : 0;  // valid keys of the tile (a prefix)
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < 64; ++k)
      if (k < nv) mx = fmaxf(mx, s[k]);
    const float mn = fmaxf(m, mx);
    const float alpha = mn == -INFINITY ? 1.f : __expf(m - mn);
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float pv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int k = 8 * c + e;
        pv[e] = k < nv ? __expf(s[k] - mn) : 0.f;
        sum += pv[e];
      }
      uint4 ph, pl;
      split8(pv, ph, pl);
      *reinterpret_cast<uint4*>(smem + kPhi + kmaj(tid, c)) = ph;
      *reinterpret_cast<uint4*>(smem + kPlo + kmaj(tid, c)) = pl;
    }
    l = l * alpha + sum;
    m = mn;
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {  // O_t = (p_hi + p_lo) V
      tc_fence_after();
      const uint64_t vd = kmajor_desc(sb + kVt0 + b * 8192);
      umma_bf16_kblock(tmem + 128, kmajor_desc(sb + kPhi), vd, idesc, 0u);
      umma_bf16_kblock(tmem + 128, kmajor_desc(sb + kPlo), vd, idesc, 1u);
      umma_commit(&X.bar_o);
    }
    mbar_wait(&X.bar_o, nb_o & 1u, p.err);
    ++nb_o;
    tc_fence_after();
    float o[64];
    tmem_ld64(t_row + 128, o);
#pragma unroll
    for (int d = 0; d < 64; ++d) acc[d] = fmaf(acc[d], alpha, o[d]);
  }

  if (live) {
    const float inv = 1.f / l;
    const int t = t0 + j;
    const int f = (g * kGqa + h) * kHeadDim;
#pragma unroll
    for (int d = 0; d < 64; ++d) attn::emit(p, t, f + d, acc[d] * inv);
  }
  // the next segment rewrites Q, K/V and P: every thread is past its reads
  tc_fence_before();
  __syncthreads();
}

__global__ void __launch_bounds__(kThreads) attention_block_kernel(const AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  Misc& X = *reinterpret_cast<Misc*>(smem + kMisc);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.x * kQB;
  const int g = blockIdx.y;
  grid_dep_wait();
  // TMEM before the dependent launch: the next kernel's CTAs may take TMEM of this SM as
  // soon as every CTA here has signalled, and they hold it until this grid completes
  if (warp == 0) {
    tmem_alloc(&X.tmem, kTmemCols);
    tmem_relinquish();
  }
  grid_dep_launch();
  if (tid == 0) {
    mbar_init(&X.bar_s[0], 1);
    mbar_init(&X.bar_s[1], 1);
    mbar_init(&X.bar_o, 1);
    fence_barrier_init();
  }
  if (tid < kQB) {
    const int t = t0 + tid;
    int ps = -1, rw = -1;
    if (t < p.M) {
      ps = p.pos[t];
      rw = p.rows[t];
      if (ps < 0 || ps >= p.max_len || rw < 0 || (p.cache_rows > 0 && rw >= p.cache_rows)) {
        if (g == 0 && p.err) atomicExch(p.err, QI_ERR_INDEX);
        ps = -1;
      }
    }
    X.pos[tid] = ps;
    X.row[tid] = rw;
  }
  __syncthreads();
  if (tid == 0) {
    int ns = 0;
    for (int i = 0; i < kQB; ++i) {
      X.tok_seg[i] = -1;
      if (X.pos[i] < 0) continue;
      int sg = 0;
      while (sg < ns && X.seg_row[sg] != X.row[i]) ++sg;
      if (sg == ns) {
        X.seg_row[ns] = X.row[i];
        X.seg_kmax[ns] = 0;
        X.seg_n[ns] = 0;
        ++ns;
      }
      X.tok_seg[i] = sg;
      X.seg_kmax[sg] = max(X.seg_kmax[sg], X.pos[i] + 1);
      ++X.seg_n[sg];
    }
    X.nseg = ns;
  }
  __syncthreads();
  {
    // segments of two or more tokens on the tensor cores, one after another; then the
    // single-token segments (a batched prefill's last tokens) token by token
    uint32_t nb_s0 = 0u, nb_s1 = 0u, nb_o = 0u;
    bool singles = false;
    for (int sg = 0; sg < X.nseg; ++sg) {
      if (X.seg_n[sg] >= 2) tc_segment(p, smem, X, t0, g, tid, sg, nb_s0, nb_s1, nb_o);
      else singles = true;
    }
    if (singles) token_path(p, smem, X, t0, g, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(X.tmem, kTmemCols);
  }
}

}  // namespace

cudaError_t launch_attention_block(const AttnParams& p, cudaStream_t stream, bool pdl) {
  cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(attention_block_kernel), (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.M + kQB - 1) / kQB, kKvHeads, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n++].val.programmaticStreamSerializationAllowed = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, attention_block_kernel, p);
}

}  // namespace qi
