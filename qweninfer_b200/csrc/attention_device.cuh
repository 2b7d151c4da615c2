// One attention work unit — (key split, KV head, query token) — as a device function of
// the standalone attention kernel (attention.cu). NW warps run a unit: warp w takes keys
// 32*(w % 4).. of every 128-key tile and, with NW = 8, half of the 7 query heads (w / 4
// picks the half). With one CTA per SM the per-warp chain of dependent shared-memory
// loads, FMAs and shuffles sets the tile time, so the kernel uses 8 warps (NW = 4 runs all
// heads per warp, with `sync` a named barrier of those 4 warps when kNamedBarrier is set;
// otherwise the whole CTA). The two K/V stage mbarriers are initialised once per CTA;
// `uses` carries their phase counts from unit to unit.
#pragma once

#include "common.cuh"
#include "internal.h"
#include "tc_proj.h"

namespace qi {
namespace attn {

constexpr int kAttnThreads = 256;  // the standalone kernel (NW = 8)
constexpr int kTile = 128;  // keys per stage
constexpr int kPartStride = kGqa * (kHeadDim + 2);  // floats per (token, head, split) partial
static_assert(2 * kGqa * kMaxAttnSplits + kGqa <= 4 * kGqa * (kHeadDim + 2), "split merge scratch");

struct AttnSmem {
  uint16_t k[2][kTile * kHeadDim];
  uint16_t v[2][kTile * kHeadDim];
  float q[kGqa * 2 * 8 * 4];          // per head: [half][chunk][4], scaled by 1/sqrt(64)
  float p[4][32][8];                  // per key group: probabilities of its 32 keys, 7 heads
  uint64_t bar[2];
  int last;
};

// Split merge in a thread-block cluster (standalone kernel, AttnParams::cluster): the
// partials of splits 0.. of one (token, KV head) in split 0's shared memory, and the
// barrier that the other splits' threads arrive on once theirs is stored.
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

// Runs unit (split, g, tok); returns true when it wrote the final output of (tok, g)
// (a single split, or the last split to arrive, which merges all of them).
// cm: the cluster merge buffer (standalone kernel with AttnParams::cluster), else null;
// *waited is set when the unit waited on the cluster barrier (a split that pushes its
// partial to split 0 does so before its first remote store).
template <bool kNamedBarrier, int NW, bool kPaged = false>
__device__ __forceinline__ bool attention_unit(const AttnParams& p, AttnSmem& S, int split, int g, int tok,
                                               int tid, uint32_t (&uses)[2], ClusterMerge* cm = nullptr,
                                               bool* waited = nullptr) {
  static_assert(NW == 4 || NW == 8, "4 or 8 warps");
  static_assert(!kNamedBarrier || NW == 4, "the named barrier spans 4 warps");
  constexpr int NT = NW * 32;
  constexpr int HPG = NW == 4 ? kGqa : (kGqa + 1) / 2;  // heads per warp
  auto sync = [] {
    if constexpr (kNamedBarrier) asm volatile("bar.sync 1, 128;" ::: "memory");
    else __syncthreads();
  };
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int kgrp = warp & 3;                // key group: keys 32 * kgrp .. of each tile
  const int h0 = (warp >> 2) * HPG;         // first head of this warp
  const int nh = min(HPG, kGqa - h0);       // heads of this warp
  const int ps = p.pos[tok];
  const int row = p.rows[tok];
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

  const int ntiles = (kend - kbeg + kTile - 1) / kTile;
  // mbarrier phases continue across the units a CTA runs: tile i uses stage i & 1
  const uint32_t u0s = uses[0], u1s = uses[1];
  uses[0] += (uint32_t)((ntiles + 1) >> 1);
  uses[1] += (uint32_t)(ntiles >> 1);
  auto parity = [&](int i) { return (uint32_t)((((i & 1) ? u1s : u0s) + (uint32_t)(i >> 1)) & 1u); };
  // Tile i's K and V rows as 8 bulk copies (4 key quarters x K/V), one per thread
  // 0..7: the copies one thread issues are processed one after another, so a single
  // issuing thread would serialise them.
  auto issue = [&](int i) {
    const int k0 = kbeg + i * kTile;
    const int nk = min(kTile, kend - k0);
    const int st = i & 1;
    if (tid == 0) mbar_arrive_expect_tx(&S.bar[st], (uint32_t)nk * kHeadDim * 2 * 2);
    __syncwarp(0xffu);
    const int q = tid & 3, kq = (nk + 3) >> 2;
    const int a = min(nk, q * kq), b = min(nk, a + kq);
    if (b > a) {
      const long long o = tile_base(k0) + (long long)a * kHeadDim;
      if (tid < 4) bulk_g2s(S.k[st] + a * kHeadDim, p.kc + o, (uint32_t)(b - a) * kHeadDim * 2, &S.bar[st]);
      else bulk_g2s(S.v[st] + a * kHeadDim, p.vc + o, (uint32_t)(b - a) * kHeadDim * 2, &S.bar[st]);
    }
  };
  // the first two tiles are requested before q is staged: the copies do not depend on
  // it, so their latency overlaps the q loads
  if (tid < 8) {
    issue(0);
    if (ntiles > 1) issue(1);
  }

  // q of the 7 heads sharing KV head g, pre-scaled by 1/8 (exact), laid out so that the
  // eight 8-dim chunks' first halves are 16-byte neighbours (conflict-free rotated reads).
  // (all four loads of a thread are issued before its shared-memory stores)
  {
    constexpr int kRounds = (kGqa * kHeadDim + NT - 1) / NT;
    float qv[kRounds];
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      const int idx = tid + r * NT;
      qv[r] = __ldcg(p.q + (long long)tok * kHidden + g * kGqa * kHeadDim + (idx < kGqa * kHeadDim ? idx : 0));
    }
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      const int idx = tid + r * NT;
      if (idx < kGqa * kHeadDim) {
        const int h = idx >> 6, d = idx & 63;
        const int cc = d >> 3, e = d & 7;
        S.q[((h * 2 + (e >> 2)) * 8 + cc) * 4 + (e & 3)] = qv[r] * 0.125f;
      }
    }
  }
  sync();

  float m[HPG], l[HPG], acc[HPG][2];
#pragma unroll
  for (int hi = 0; hi < HPG; ++hi) {
    m[hi] = -INFINITY;
    l[hi] = 0.f;
    acc[hi][0] = acc[hi][1] = 0.f;
  }

  for (int i = 0; i < ntiles; ++i) {
    const int st = i & 1;
    mbar_wait(&S.bar[st], parity(i), p.err);
    const int k0 = kbeg + i * kTile;
    const int nk = min(kTile, kend - k0);
    const int kw = 32 * kgrp;
    const int nkw = max(0, min(32, nk - kw));
    if (nkw > 0) {
      const bool valid = lane < nkw;
      float s[HPG];
#pragma unroll
      for (int hi = 0; hi < HPG; ++hi) s[hi] = 0.f;
      const uint16_t* krow = S.k[st] + (kw + lane) * kHeadDim;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int cc = (c + lane) & 7;
        const uint4 kv = *reinterpret_cast<const uint4*>(krow + cc * 8);
        const float k0f = bf16lo(kv.x), k1f = bf16hi(kv.x), k2f = bf16lo(kv.y), k3f = bf16hi(kv.y);
        const float k4f = bf16lo(kv.z), k5f = bf16hi(kv.z), k6f = bf16lo(kv.w), k7f = bf16hi(kv.w);
#pragma unroll
        for (int hi = 0; hi < HPG; ++hi) {
          if (hi < nh) {
            const int h = h0 + hi;
            const float4 qa = *reinterpret_cast<const float4*>(&S.q[((h * 2 + 0) * 8 + cc) * 4]);
            const float4 qb = *reinterpret_cast<const float4*>(&S.q[((h * 2 + 1) * 8 + cc) * 4]);
            float a = s[hi];
            a = fmaf(qa.x, k0f, a);
            a = fmaf(qa.y, k1f, a);
            a = fmaf(qa.z, k2f, a);
            a = fmaf(qa.w, k3f, a);
            a = fmaf(qb.x, k4f, a);
            a = fmaf(qb.y, k5f, a);
            a = fmaf(qb.z, k6f, a);
            a = fmaf(qb.w, k7f, a);
            s[hi] = a;
          }
        }
      }
#pragma unroll
      for (int hi = 0; hi < HPG; ++hi) {
        if (hi < nh) {
          const float sv = valid ? s[hi] : -INFINITY;
          const float mn = fmaxf(m[hi], warp_max(sv));
          const float alpha = expf(m[hi] - mn);
          const float pr = valid ? expf(sv - mn) : 0.f;
          l[hi] = l[hi] * alpha + warp_sum(pr);
          acc[hi][0] *= alpha;
          acc[hi][1] *= alpha;
          m[hi] = mn;
          S.p[kgrp][lane][h0 + hi] = pr;
        }
      }
      __syncwarp();
      const uint16_t* vt = S.v[st] + kw * kHeadDim + 2 * lane;
#pragma unroll 4
      for (int j = 0; j < nkw; ++j) {
        const uint32_t v2 = *reinterpret_cast<const uint32_t*>(vt + j * kHeadDim);
        const float v0 = bf16lo(v2), v1 = bf16hi(v2);
        float pv[HPG];
        if constexpr (HPG == 4) {
          const float4 pa = *reinterpret_cast<const float4*>(&S.p[kgrp][j][h0]);
          pv[0] = pa.x; pv[1] = pa.y; pv[2] = pa.z; pv[3] = pa.w;
        } else {
          const float4 pa = *reinterpret_cast<const float4*>(&S.p[kgrp][j][0]);
          const float4 pb = *reinterpret_cast<const float4*>(&S.p[kgrp][j][4]);
          pv[0] = pa.x; pv[1] = pa.y; pv[2] = pa.z; pv[3] = pa.w; pv[4] = pb.x; pv[5] = pb.y; pv[6] = pb.z;
        }
#pragma unroll
        for (int hi = 0; hi < HPG; ++hi) {
          acc[hi][0] = fmaf(pv[hi], v0, acc[hi][0]);
          acc[hi][1] = fmaf(pv[hi], v1, acc[hi][1]);
        }
      }
      __syncwarp();
    }
    sync();  // stage st fully consumed
    if (tid < 8 && i + 2 < ntiles) issue(i + 2);
  }

  // Merge the 4 key groups. Their partials (acc[64], m, l per key group and head) take the
  // place of K tile 0, whose last reader was the loop above: the CTA's shared memory then
  // fits three CTAs per SM.
  float (&cmb)[4][kGqa][kHeadDim + 2] = *reinterpret_cast<float (*)[4][kGqa][kHeadDim + 2]>(&S.k[0][0]);
  static_assert(sizeof(float) * 4 * kGqa * (kHeadDim + 2) <= sizeof(S.k[0]), "key-group partials fit a K tile");
#pragma unroll
  for (int hi = 0; hi < HPG; ++hi) {
    if (hi < nh) {
      const int h = h0 + hi;
      cmb[kgrp][h][2 * lane] = acc[hi][0];
      cmb[kgrp][h][2 * lane + 1] = acc[hi][1];
      if (lane == 0) {
        cmb[kgrp][h][kHeadDim] = m[hi];
        cmb[kgrp][h][kHeadDim + 1] = l[hi];
      }
    }
  }
  sync();
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
  for (int idx = tid; idx < kGqa * (kHeadDim + 2); idx += NT) {
    const int h = idx / (kHeadDim + 2);
    const int d = idx - h * (kHeadDim + 2);
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) mx = fmaxf(mx, cmb[w][h][kHeadDim]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = cmb[w][h][kHeadDim];
      if (mw == -INFINITY) continue;
      const float sc = expf(mw - mx);
      L = fmaf(sc, cmb[w][h][kHeadDim + 1], L);
      if (d < kHeadDim) A = fmaf(sc, cmb[w][h][d], A);
    }
    const float val = d < kHeadDim ? A : (d == kHeadDim ? mx : L);
    if (nsplit == 1) {
      if (d < kHeadDim) emit(p, tok, (g * kGqa + h) * kHeadDim + d, A / L);
    } else if (!cm) {
      part[idx] = val;
    } else if (split == 0) {
      cm->recv[0][idx] = val;
    } else {
      st_cluster_f32(remote + (uint32_t)idx * 4u, val);
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
    sync();
    mbar_wait_cluster(&cm->bar, 0, p.err);
  } else {
    // Split merge by the last-arriving CTA of this (token, head): the barrier orders every
    // thread's partial stores before thread 0's acq_rel arrival.
    sync();
    if (tid == 0) S.last = atomic_add_acq_rel(&p.counters[tok * kKvHeads + g], 1u) == (unsigned int)(nsplit - 1);
    sync();
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
  for (int idx = tid; idx < kGqa * nsplit; idx += NT) {
    const int h = idx / nsplit, s = idx - h * nsplit;
    const float mv = load(s, h * (kHeadDim + 2) + kHeadDim), lv = load(s, h * (kHeadDim + 2) + kHeadDim + 1);
    sm[idx] = mv;
    sm[kGqa * nsplit + idx] = lv;
  }
  sync();
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
  sync();
  {
    constexpr int kRounds = (kGqa * kHeadDim + NT - 1) / NT;
    float A[kRounds];
#pragma unroll
    for (int r = 0; r < kRounds; ++r) A[r] = 0.f;
#pragma unroll 4
    for (int s = 0; s < nsplit; ++s) {
#pragma unroll
      for (int r = 0; r < kRounds; ++r) {
        const int idx = tid + r * NT;
        if (idx < kGqa * kHeadDim) {
          const int h = idx >> 6, d = idx & 63;
          A[r] = fmaf(sm[h * nsplit + s], load(s, h * (kHeadDim + 2) + d), A[r]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      const int idx = tid + r * NT;
      if (idx < kGqa * kHeadDim) emit(p, tok, g * kGqa * kHeadDim + idx, A[r] / sm[2 * kGqa * nsplit + (idx >> 6)]);
    }
  }
  if (!cm && tid == 0) p.counters[tok * kKvHeads + g] = 0u;
  return true;
}

}  // namespace attn
}  // namespace qi
