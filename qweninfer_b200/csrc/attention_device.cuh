// One attention work unit — (key split, KV head, query token) — of the ragged decode
// attention kernel (attention.cu), on the tensor cores with warp-level mma.sync.
//
// The 7 query heads of a KV group are the rows of an m16n8k16 A operand: row h holds
// bf16(q_h) and row h + 8 holds bf16(q_h - bf16(q_h)) (row 7 and 15 are zero), so one
// MMA multiplies both halves and the thread that owns row h also owns row h + 8: adding
// the two accumulator rows restores ~16 mantissa bits of the fp32 query with fp32
// accumulation. The probabilities go back into the same A layout (p_hi in row h, p_lo in
// row h + 8) for O += P V, straight from the score accumulators, without leaving the
// registers. 8 warps: warp w takes keys 16w .. 16w + 15 of every 128-key tile (two
// 8-key n-tiles), keeps its own fp32 online softmax per head (m, l over its keys) and its
// own O (16 x 64 fp32 accumulators); the warps and then the key splits are merged with
// max-rescaled sums.
//
// K and V tiles are copied with cp.async (16 bytes per thread and copy) into shared
// memory rows of 128 bytes whose 16-byte chunks are XOR-swizzled by the key index
// (chunk c of key r sits at c ^ (r & 7)), so the ldmatrix reads of 8 keys at one chunk
// hit 8 different bank groups: K through ldmatrix (B of S = Q K^T, keys as columns), V
// through ldmatrix.trans (B of O = P V). Two stages; the copies of tile i + 2 are issued
// after tile i.
//
// Positions and cache rows are read before the programmatic-launch wait, so key splits
// without keys end at once instead of holding SM slots while the previous kernel runs.
// Decode steps (AttnParams::decode: every query token is the only one of its cache row in
// the forward) also copy the first two tiles' cached keys (positions < the query's own)
// before the wait: those were written by earlier forwards. Only the query and the key at
// the query's own position, which the preceding QKV launch writes, are read after it.
#pragma once

#include "common.cuh"
#include "internal.h"
#include "tc_proj.h"

namespace qi {
namespace attn {

constexpr int kAttnThreads = 256;  // 8 warps
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kTile = 128;                         // keys per stage
constexpr int kWarpKeys = kTile / kAttnWarps;      // 16 keys of a tile per warp
constexpr int kPartStride = kGqa * (kHeadDim + 2);  // floats per (token, head, split) partial
static_assert(kWarpKeys == 16, "two 8-key n-tiles per warp");
static_assert(2 * kGqa * kMaxAttnSplits + kGqa <= kAttnWarps * kGqa * (kHeadDim + 2), "split merge scratch");

struct AttnSmem {
  uint16_t k[2][kTile * kHeadDim];  // swizzled rows (see above)
  uint16_t v[2][kTile * kHeadDim];
  int last;
};

// Split merge in a thread-block cluster (AttnParams::cluster): the partials of splits 0..
// of one (token, KV head) in split 0's shared memory, and the barrier that the other
// splits' threads arrive on once theirs is stored.
constexpr int kMaxClusterSplits = 8;
struct ClusterMerge {
  float recv[kMaxClusterSplits][kPartStride];
  uint64_t bar;
};

// Output element (token, feature f = head * 64 + d): fp32 and/or the o projection's
// activation tiles (hi/lo bf16 halves).
__device__ __forceinline__ void emit(const AttnParams& p, int tok, int f, float v) {
  if (p.out) p.out[(long long)tok * kHidden + f] = v;
  if (p.out_act) {
    const uint16_t hi = f32_to_bf16_rn(v);
    p.out_act[act_offset(tok, f, 0, kHidden, p.out_nt)] = hi;
    p.out_act[act_offset(tok, f, 1, kHidden, p.out_nt)] = f32_to_bf16_rn(v - bf16_to_f32(hi));
  }
}

// {bf16(a) in the low half, bf16(b) in the high half}
__device__ __forceinline__ uint32_t bf16x2(float a, float b);

// Output elements f and f + 1 (f even): one 8-byte fp32 store and one 4-byte store per
// activation-tile half (the two features are neighbours in the tile layout).
__device__ __forceinline__ void emit2(const AttnParams& p, int tok, int f, float v0, float v1) {
  if (p.out) *reinterpret_cast<float2*>(p.out + (long long)tok * kHidden + f) = make_float2(v0, v1);
  if (p.out_act) {
    const uint32_t hi = bf16x2(v0, v1);
    const uint32_t lo = bf16x2(v0 - __uint_as_float(hi << 16), v1 - __uint_as_float(hi & 0xffff0000u));
    *reinterpret_cast<uint32_t*>(p.out_act + act_offset(tok, f, 0, kHidden, p.out_nt)) = hi;
    *reinterpret_cast<uint32_t*>(p.out_act + act_offset(tok, f, 1, kHidden, p.out_nt)) = lo;
  }
}

// {bf16(a) in the low half, bf16(b) in the high half}
__device__ __forceinline__ uint32_t bf16x2(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
// hi/lo halves of the pair (a, b): hi = bf16(x), lo = bf16(x - hi)
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = bf16x2(a, b);
  lo = bf16x2(a - bf16lo(hi), b - bf16hi(hi));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// 16-byte asynchronous copy global -> shared; src_bytes 0 writes zeros (nothing is read)
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// byte offset of (key r, 16-byte chunk c) in a swizzled tile
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// Runs unit (split, g, tok); returns true when it wrote the final output of (tok, g)
// (a single split, or the last split to arrive, which merges all of them).
// cm: the cluster merge buffer (AttnParams::cluster), else null; *waited is set when the
// unit waited on the cluster barrier (a split that pushes its partial to split 0 does so
// before its first remote store). `ps` and `row` are the query's position and cache row,
// read by the caller before the programmatic-launch wait. The wait is taken here: before
// the first copy (p.decode == 0) or after the first two tiles' cached keys are requested
// (p.decode == 1); units without keys (and queries outside the cache) return without it.
template <bool kPaged = false>
__device__ __forceinline__ bool attention_unit(const AttnParams& p, AttnSmem& S, int split, int g, int tok, int ps,
                                               int row, int tid, ClusterMerge* cm, bool* waited) {
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int gq = lane >> 2;  // accumulator row (head) of this thread, and row + 8
  const int qd = lane & 3;   // its column pair
  const bool early = p.decode != 0;
  auto dep_wait = [&] {
    grid_dep_wait();
    grid_dep_launch();
  };
  if (ps < 0 || ps >= p.max_len || row < 0 || (p.cache_rows > 0 && row >= p.cache_rows)) {
    // outside the cache: reported, nothing read or written; split 0 still counts the
    // (token, head) as finished for callers that wait on completions
    if (split == 0 && tid == 0 && p.err) atomicExch(p.err, QI_ERR_INDEX);
    return split == 0;
  }
  const int nkeys = ps + 1;
  const int nsplit = (nkeys + p.split_keys - 1) / p.split_keys;
  if (split >= nsplit) return false;
  const int kbeg = split * p.split_keys;
  const int kend = min(nkeys, kbeg + p.split_keys);
  const int ntiles = (kend - kbeg + kTile - 1) / kTile;
  // tile i's keys start at K/V offset tile_base(k0): packed, one run per (row, head);
  // paged, a tile never straddles a page, and an unmapped page is reported and read from
  // the layer's start (in bounds)
  const long long head_base = (((long long)row * kKvHeads + g) * p.max_len) * kHeadDim;
  auto tile_base = [&](int k0) -> long long {
    if constexpr (!kPaged) {
      return head_base + (long long)k0 * kHeadDim;
    } else {
      const long long o = kv_offset(p.kv, p.max_len, row, g, k0);
      if (o < 0 && p.err) atomicExch(p.err, QI_ERR_INDEX);
      return o < 0 ? 0 : o;
    }
  };
  const uint32_t sk0 = smem_u32(&S.k[0][0]), sv0 = smem_u32(&S.v[0][0]);
  constexpr uint32_t kStageBytes = kTile * kHeadDim * 2;
  // Tile i into stage i & 1: keys k0 + r for r < min(nk, lim - k0) are copied; V rows
  // nk .. (the rest of the last warp's 16 keys) are zero-filled so that P = 0 never meets
  // a stale non-finite value. 8 chunks of 16 bytes per thread (K then V, key-major).
  auto issue = [&](int i, int lim) {
    const int k0 = kbeg + i * kTile;
    const int nk = min(kTile, kend - k0);
    const int ncopy = min(nk, lim - k0);
    const int nzero = (nk + kWarpKeys - 1) / kWarpKeys * kWarpKeys;
    const long long base = tile_base(k0);
    const uint32_t st = (uint32_t)(i & 1) * kStageBytes;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = tid + j * kAttnThreads;  // 0 .. 2047
      const int isv = c >> 10, r = (c >> 3) & (kTile - 1), ch = c & 7;
      const uint16_t* src = (isv ? p.vc : p.kc) + base + (long long)r * kHeadDim + ch * 8;
      const uint32_t dst = (isv ? sv0 : sk0) + st + swz(r, ch);
      if (r < ncopy) cp_async16(dst, src, 16u);
      else if (isv && r >= nk && r < nzero) cp_async16(dst, p.vc + base, 0u);
    }
  };

  if (early) {
    issue(0, ps);
    cp_async_commit();
    if (ntiles > 1) issue(1, ps);
    cp_async_commit();
    dep_wait();
    // the key at the query's own position, written by the preceding launch, if its tile
    // was requested above (the last split's last tile when that is tile 0 or 1)
    const int it = (ps - kbeg) / kTile;
    if (kend == nkeys && it < 2 && tid < 16) {
      const int r = ps - kbeg - it * kTile, isv = tid >> 3, ch = tid & 7;
      const long long base = tile_base(kbeg + it * kTile);
      cp_async16((isv ? sv0 : sk0) + (uint32_t)(it & 1) * kStageBytes + swz(r, ch),
                 (isv ? p.vc : p.kc) + base + (long long)r * kHeadDim + ch * 8, 16u);
    }
    cp_async_commit();
  } else {
    dep_wait();
    issue(0, kend);
    cp_async_commit();
    if (ntiles > 1) issue(1, kend);
    cp_async_commit();
  }

  // A operand: q of head gq (hi row gq, lo row gq + 8) pre-scaled by 1/8 (exact), per
  // 16-dim k-step s: columns 2qd, 2qd + 1 and 2qd + 8, 2qd + 9
  uint32_t qa[4][4];
  {
    const float* qrow = p.q + (long long)tok * kHidden + (g * kGqa + (gq < kGqa ? gq : 0)) * kHeadDim + 2 * qd;
    float2 x[8];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      x[2 * s] = __ldcg(reinterpret_cast<const float2*>(qrow + 16 * s));
      x[2 * s + 1] = __ldcg(reinterpret_cast<const float2*>(qrow + 16 * s + 8));
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const float sc = gq < kGqa ? 0.125f : 0.f;
      split2(x[2 * s].x * sc, x[2 * s].y * sc, qa[s][0], qa[s][1]);
      split2(x[2 * s + 1].x * sc, x[2 * s + 1].y * sc, qa[s][2], qa[s][3]);
    }
  }

  float m = -INFINITY, l = 0.f;  // running max and this thread's share of the sum (head gq)
  float o[8][4];                 // O: dim tile d, rows gq (hi part) and gq + 8 (lo part)
#pragma unroll
  for (int d = 0; d < 8; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;

  const int kw = warp * kWarpKeys;
  // ldmatrix row addresses of this lane: matrix j = lane >> 3, row lane & 7
  const int lj = lane >> 3, lr = lane & 7;
  for (int i = 0; i < ntiles; ++i) {
    if (i == ntiles - 1) cp_async_wait<0>();
    else cp_async_wait<1>();
    __syncthreads();
    const int k0 = kbeg + i * kTile;
    const int nk = min(kTile, kend - k0);
    if (kw < nk) {
      const uint32_t st = (uint32_t)(i & 1) * kStageBytes;
      // S = Q K^T for the warp's two 8-key n-tiles: ldmatrix of keys kw + 8t + lr, chunks
      // 4h + lj (k-steps 2h and 2h + 1)
      float sacc[2][4];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        sacc[t][0] = sacc[t][1] = sacc[t][2] = sacc[t][3] = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t b[4];
          ldsm4(sk0 + st + swz(kw + 8 * t + lr, 4 * h + lj), b);
          mma16816(sacc[t], qa[2 * h][0], qa[2 * h][1], qa[2 * h][2], qa[2 * h][3], b[0], b[1]);
          mma16816(sacc[t], qa[2 * h + 1][0], qa[2 * h + 1][1], qa[2 * h + 1][2], qa[2 * h + 1][3], b[2], b[3]);
        }
      }
      // scores of head gq for keys kw + 8t + 2qd + e (hi row + lo row), masked past nk
      float sc[2][2];
      float mx = -INFINITY;
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const bool valid = kw + 8 * t + 2 * qd + e < nk;
          sc[t][e] = valid ? sacc[t][e] + sacc[t][2 + e] : -INFINITY;
          mx = fmaxf(mx, sc[t][e]);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m, mx);
      const float alpha = expf(m - mn);
      m = mn;
      float pr[2][2];
      float ps_ = 0.f;
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          pr[t][e] = sc[t][e] == -INFINITY ? 0.f : expf(sc[t][e] - mn);
          ps_ += pr[t][e];
        }
      l = l * alpha + ps_;
#pragma unroll
      for (int d = 0; d < 8; ++d) {
        o[d][0] *= alpha;
        o[d][1] *= alpha;
        o[d][2] *= alpha;
        o[d][3] *= alpha;
      }
      // P as the A operand over the warp's 16 keys: k columns 2qd, 2qd + 1 = n-tile 0,
      // 2qd + 8, 2qd + 9 = n-tile 1; row gq = p_hi, row gq + 8 = p_lo
      uint32_t pa[4];
      split2(pr[0][0], pr[0][1], pa[0], pa[1]);
      split2(pr[1][0], pr[1][1], pa[2], pa[3]);
      // O += P V: ldmatrix.trans of keys kw + 8 (lj & 1) + lr, chunks 2h + (lj >> 1)
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        uint32_t b[4];
        ldsm4_t(sv0 + st + swz(kw + 8 * (lj & 1) + lr, 2 * h + (lj >> 1)), b);
        mma16816(o[2 * h], pa[0], pa[1], pa[2], pa[3], b[0], b[1]);
        mma16816(o[2 * h + 1], pa[0], pa[1], pa[2], pa[3], b[2], b[3]);
      }
    }
    __syncthreads();  // stage i & 1 fully consumed
    if (i + 2 < ntiles) {
      issue(i + 2, kend);
      cp_async_commit();
    }
  }

  // Merge the 8 warps. Their partials (O[64], m, l per warp and head) take the place of
  // K tile 0, whose last reader was the loop above.
  float (&cmb)[kAttnWarps][kGqa][kHeadDim + 2] =
      *reinterpret_cast<float (*)[kAttnWarps][kGqa][kHeadDim + 2]>(&S.k[0][0]);
  static_assert(sizeof(float) * kAttnWarps * kGqa * (kHeadDim + 2) <= sizeof(S.k[0]), "warp partials fit a K tile");
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  if (gq < kGqa) {
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      cmb[warp][gq][8 * d + 2 * qd] = o[d][0] + o[d][2];
      cmb[warp][gq][8 * d + 2 * qd + 1] = o[d][1] + o[d][3];
    }
    if (qd == 0) {
      cmb[warp][gq][kHeadDim] = m;
      cmb[warp][gq][kHeadDim + 1] = l;
    }
  }
  __syncthreads();
  // this split's partial: (A[64], m, l) per head, in global scratch, in split 0's
  // shared memory (cluster: split 0 writes its own, the others over distributed shared
  // memory), or straight to the output when there is a single split
  float* part = p.part + (((long long)tok * kKvHeads + g) * p.max_splits + split) * kPartStride;
  const bool push = cm && nsplit > 1 && split > 0;
  if (push) {
    cluster_wait();  // split 0's barrier initialisation is visible (uniform over the CTA)
    *waited = true;
  }
  const uint32_t remote = push ? map_rank(&cm->recv[split][0], 0) : 0u;
  // (1) per head: the max over the warps, each warp's weight exp(m_w - max) and the
  // weighted sum; (2) per pair of output dims: the weighted sum of the warps' O
  float* wsc = &cmb[0][0][0] + kAttnWarps * kGqa * (kHeadDim + 2);  // [7][8] weights, [7] max, [7] sum
  static_assert(sizeof(float) * (kAttnWarps * kGqa * (kHeadDim + 2) + kGqa * (kAttnWarps + 2)) <= sizeof(S.k[0]),
                "warp weights fit after the partials");
  if (tid < kGqa) {
    const int h = tid;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, cmb[w][h][kHeadDim]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float mw = cmb[w][h][kHeadDim];
      const float sc = mw == -INFINITY ? 0.f : expf(mw - mx);
      L = fmaf(sc, cmb[w][h][kHeadDim + 1], L);
      wsc[h * kAttnWarps + w] = sc;
    }
    wsc[kGqa * kAttnWarps + h] = mx;
    wsc[kGqa * (kAttnWarps + 1) + h] = L;
    const int off = h * (kHeadDim + 2) + kHeadDim;  // m and l of the split's partial
    if (nsplit > 1) {
      if (!cm) {
        part[off] = mx;
        part[off + 1] = L;
      } else if (split == 0) {
        cm->recv[0][off] = mx;
        cm->recv[0][off + 1] = L;
      } else {
        st_cluster_f32(remote + (uint32_t)off * 4u, mx);
        st_cluster_f32(remote + (uint32_t)(off + 1) * 4u, L);
      }
    }
  }
  __syncthreads();
  for (int e = tid; e < kGqa * kHeadDim / 2; e += kAttnThreads) {
    const int h = e / (kHeadDim / 2), d = 2 * (e - h * (kHeadDim / 2));
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float sc = wsc[h * kAttnWarps + w];
      const float2 v = *reinterpret_cast<const float2*>(&cmb[w][h][d]);
      a0 = fmaf(sc, v.x, a0);
      a1 = fmaf(sc, v.y, a1);
    }
    const int off = h * (kHeadDim + 2) + d;
    if (nsplit == 1) {
      const float L = wsc[kGqa * (kAttnWarps + 1) + h];
      emit2(p, tok, (g * kGqa + h) * kHeadDim + d, a0 / L, a1 / L);
    } else if (!cm) {
      *reinterpret_cast<float2*>(part + off) = make_float2(a0, a1);
    } else if (split == 0) {
      *reinterpret_cast<float2*>(&cm->recv[0][off]) = make_float2(a0, a1);
    } else {
      st_cluster_f32(remote + (uint32_t)off * 4u, a0);
      st_cluster_f32(remote + (uint32_t)(off + 1) * 4u, a1);
    }
  }
  if (nsplit == 1) return true;
  if (cm && split > 0) {
    // every thread's stores are released to split 0 by its own arrival
    mbar_arrive_remote(map_rank(&cm->bar, 0));
    return false;
  }

  if (cm) {
    // split 0: its own partial is in place (barrier) and every other split's has arrived
    __syncthreads();
    mbar_wait_cluster(&cm->bar, 0, p.err);
  } else {
    // Split merge by the last-arriving CTA of this (token, head): the barrier orders every
    // thread's partial stores before thread 0's acq_rel arrival.
    __syncthreads();
    if (tid == 0) S.last = atomic_add_acq_rel(&p.counters[tok * kKvHeads + g], 1u) == (unsigned int)(nsplit - 1);
    __syncthreads();
    if (!S.last) return false;
  }
  const float* base = p.part + (((long long)tok * kKvHeads + g) * p.max_splits) * kPartStride;
  // partial value `off` of split s
  auto load = [&](int s, int off) -> float {
    return cm ? cm->recv[s][off] : __ldcg(base + (long long)s * kPartStride + off);
  };
  // (1) every split's running max and sum into shared memory (reusing the warp-merge
  // area: 2 * 7 * nsplit + 7 floats), (2) per head the max and the split weights
  // exp(m_s - max), (3) the weighted sum of the split outputs, loads before stores.
  float* sm = &cmb[0][0][0];
  for (int idx = tid; idx < kGqa * nsplit; idx += kAttnThreads) {
    const int h = idx / nsplit, s = idx - h * nsplit;
    const float mv = load(s, h * (kHeadDim + 2) + kHeadDim), lv = load(s, h * (kHeadDim + 2) + kHeadDim + 1);
    sm[idx] = mv;
    sm[kGqa * nsplit + idx] = lv;
  }
  __syncthreads();
  if (tid < kGqa) {
    const int h = tid;
    float mx = -INFINITY;
    for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, sm[h * nsplit + s]);
    float L = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float sc = expf(sm[h * nsplit + s] - mx);
      L = fmaf(sc, sm[kGqa * nsplit + h * nsplit + s], L);
      sm[h * nsplit + s] = sc;
    }
    sm[2 * kGqa * nsplit + h] = L;
  }
  __syncthreads();
  for (int e = tid; e < kGqa * kHeadDim / 2; e += kAttnThreads) {
    const int h = e / (kHeadDim / 2), d = 2 * (e - h * (kHeadDim / 2));
    const int off = h * (kHeadDim + 2) + d;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll 4
    for (int s = 0; s < nsplit; ++s) {
      const float sc = sm[h * nsplit + s];
      const float2 v = cm ? *reinterpret_cast<const float2*>(&cm->recv[s][off])
                          : __ldcg(reinterpret_cast<const float2*>(base + (long long)s * kPartStride + off));
      a0 = fmaf(sc, v.x, a0);
      a1 = fmaf(sc, v.y, a1);
    }
    const float L = sm[2 * kGqa * nsplit + h];
    emit2(p, tok, (g * kGqa + h) * kHeadDim + d, a0 / L, a1 / L);
  }
  if (!cm && tid == 0) p.counters[tok * kKvHeads + g] = 0u;
  return true;
}

}  // namespace attn
}  // namespace qi
