// Work partition of the decode-step kernel (step.cu), shared by host and device code so
// that the host can check it (tests/native/step_plan_check.cpp).
//
// The step kernel runs on 148 CTAs, one per SM. For each projection with K = 896 (QKV, o,
// gate/up and the tied head) a CTA owns a contiguous range of 8-row weight groups and
// multiplies them over the whole of K, so every output row is finished by the CTA that
// computes it (no partial sums cross CTAs). The down projection (K = 4864) is split over
// 147 CTAs instead: m-tile i (128 rows) x k range j of 21 ranges, partial sums added by
// the reduce phase.
//
// Weight pieces: the part of one 128 x 64 weight block (one m-tile, one k block) that a
// CTA multiplies is `rows / 8` contiguous 1 KB groups of the tiled layout. Pieces are
// packed in order into ring slots of kSlotKB KB; a piece never straddles two slots.
#pragma once

#include <stdint.h>

#ifndef __CUDACC__  // plain C++ (the host-side partition check)
#define __host__
#define __device__
#endif

namespace qi {
namespace step {

constexpr int kGrid = 148;            // CTAs: one per SM
constexpr int kSlotKB = 18;           // ring slot (KB): the pieces of two k blocks of a CTA's gate/up rows
constexpr int kMaxTokens = 32;        // tokens of one decode step
constexpr int kDownRanges = 21;       // k ranges of the down projection
constexpr int kDownCtas = 7 * kDownRanges;
constexpr int kMaxLayers = 32;
constexpr int kPhasesPerLayer = 6;    // counters: qkv, attention, o, gate/up, down, reduce

enum Op : int { kQkv = 0, kAttn = 1, kO = 2, kGateUp = 3, kDown = 4, kHead = 5 };

// 8-row weight groups and 64-column k blocks of each projection.
__host__ __device__ inline int op_groups(int op, int vocab) {
  return op == kQkv ? 144 : op == kO ? 112 : op == kGateUp ? 1216 : op == kDown ? 112 : vocab / 8;
}
__host__ __device__ inline int op_kblocks(int op) { return op == kDown ? 76 : 14; }

// A CTA's share of one projection: weight groups [g0, g1), k blocks [kb0, kb1).
// tile_major: pieces ordered tile by tile (the head, whose tiles are finished one by one),
// else k block by k block (one accumulation unit).
struct Part {
  int g0, g1, kb0, kb1;
  bool tile_major;
  __host__ __device__ bool empty() const { return g1 <= g0 || kb1 <= kb0; }
  __host__ __device__ int tile0() const { return g0 >> 4; }
  __host__ __device__ int ntiles() const { return empty() ? 0 : ((g1 - 1) >> 4) - (g0 >> 4) + 1; }
  // groups of tile u (relative): [lo, hi)
  __host__ __device__ int seg_lo(int u) const {
    const int a = (tile0() + u) * 16;
    return g0 > a ? g0 : a;
  }
  __host__ __device__ int seg_hi(int u) const {
    const int b = (tile0() + u + 1) * 16;
    return g1 < b ? g1 : b;
  }
};

__host__ __device__ inline Part part_of(int op, int cta, int vocab) {
  Part P;
  P.tile_major = op == kHead;
  if (op == kDown) {
    if (cta >= kDownCtas) {
      P.g0 = P.g1 = P.kb0 = P.kb1 = 0;
      return P;
    }
    const int i = cta / kDownRanges, j = cta - i * kDownRanges;
    P.g0 = 16 * i;
    P.g1 = 16 * i + 16;
    P.kb0 = j * 76 / kDownRanges;
    P.kb1 = (j + 1) * 76 / kDownRanges;
    return P;
  }
  const long long G = op_groups(op, vocab);
  P.g0 = (int)(G * cta / kGrid);
  P.g1 = (int)(G * (cta + 1) / kGrid);
  P.kb0 = 0;
  P.kb1 = 14;
  return P;
}

// Accumulation units of a share: the head has one per tile (finished one by one); the
// layer projections one for all their tiles (at most 2).
constexpr int kMaxLayerTiles = 2;
__host__ __device__ inline int units_of(const Part& P) { return P.empty() ? 0 : (P.tile_major ? P.ntiles() : 1); }

// One weight piece: tile u (relative), k block kb, groups [lo, hi) of the tile's 16.
struct Piece {
  int u, kb, lo, hi;
  __host__ __device__ int kbytes() const { return hi - lo; }
};

// Calls f(piece, slot, offset_kb, first_of_unit, last_of_unit) for each piece of a share
// in order, packing pieces greedily into slots numbered from slot0; returns the slot
// count. A unit's first piece is where its accumulator starts (k block kb0 of its first
// tile), its last where the accumulator is complete.
template <class F>
__host__ __device__ inline int for_each_piece(const Part& P, int slot0, F&& f) {
  if (P.empty()) return 0;
  const int nt = P.ntiles();
  int slot = slot0, used = 0;
  bool open = false;
  auto emit = [&](int u, int kb, bool first, bool last) {
    Piece pc;
    pc.u = u;
    pc.kb = kb;
    pc.lo = P.seg_lo(u) - (P.tile0() + u) * 16;
    pc.hi = P.seg_hi(u) - (P.tile0() + u) * 16;
    if (open && used + pc.kbytes() > kSlotKB) {
      ++slot;
      used = 0;
    }
    open = true;
    f(pc, slot, used, first, last);
    used += pc.kbytes();
  };
  if (P.tile_major) {
    for (int u = 0; u < nt; ++u)
      for (int kb = P.kb0; kb < P.kb1; ++kb) emit(u, kb, kb == P.kb0, kb == P.kb1 - 1);
  } else {
    for (int kb = P.kb0; kb < P.kb1; ++kb)
      for (int u = 0; u < nt; ++u) emit(u, kb, kb == P.kb0 && u == 0, kb == P.kb1 - 1 && u == nt - 1);
  }
  return slot - slot0 + 1;
}

// Attention units of one layer: (token t, KV head g, key split s), numbered
// u = (s * M + t) * 2 + g so that every token's first split comes first; unit u runs on
// CTA kGrid - 1 - (u % kGrid) (the down projection leaves the last CTA idle).
__host__ __device__ inline int attn_cta(int u) { return kGrid - 1 - (u % kGrid); }
__host__ __device__ inline int attn_first_unit(int cta) { return kGrid - 1 - cta; }

// Key splits of a token at position ps (keys 0..ps) with split_keys keys per split.
__host__ __device__ inline int attn_nsplit(int ps, int split_keys) { return (ps + split_keys) / split_keys; }

// Reduce / embedding units (m-tile i of the hidden size, token t): u = t * 7 + i on CTA u % kGrid.
__host__ __device__ inline int reduce_units(int M) { return 7 * M; }

// Counter of phase `ph` of layer l (1 + 6 l + ph); counter 0 is the embedding phase.
__host__ __device__ inline int counter_index(int l, int ph) { return 1 + kPhasesPerLayer * l + ph; }
constexpr int kCounterStride = 32;  // counters one 128-byte line apart

}  // namespace step
}  // namespace qi
