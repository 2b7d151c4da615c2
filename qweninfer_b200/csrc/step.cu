// The whole forward of a decode step (qweninfer/models/qwen2.py:263-292 for B <= 32 rows
// at S = 1, as driven by qweninfer/engine/engine.py:140-155) in ONE cooperative launch.
//
// Why one launch: a decode step is ~120 dependent projections and attention passes over
// 0.99 GB of weights. Launched one by one, each pays its own ramp-up, first-byte latency
// and drain, far more than its share of the ~150 us weight stream. Here 148 resident CTAs
// (one per SM) walk the same fixed program and:
//
//  * stream their weight pieces (step_plan.h) through a ring of shared-memory slots, one
//    issuing lane per slot, in program order. Weights do not depend on activations, so
//    the stream runs ahead across every phase boundary and is never drained; the K/V
//    tiles of a CTA's attention units (keys written by earlier steps) ride in the same
//    ring;
//  * wait for a phase's inputs on a global counter (every CTA adds 1 when it has written
//    its outputs of a phase; the waiting CTA polls for 148 with acquire semantics), then
//    bulk-copy the activation tiles they multiply (UMMA B operand, hi/lo bf16 halves);
//  * multiply with tcgen05 UMMAs (M = 128 weight rows, N = 2 x token tile, K = 16) into
//    TMEM accumulators, consecutive k blocks into independent accumulator chains (one
//    chain's UMMAs wait on each other, ~170 ns apiece at these shapes); every CTA owns
//    whole output rows over all of K (the down projection excepted), so it runs the fused
//    epilogue itself (RMSNorm scale, bias + RoPE + KV append, residual + next norm
//    operands, SwiGLU, logits + argmax) with no partial sums crossing CTAs.
//
// Phases per layer: QKV -> attention -> o -> gate/up -> down (partials over 21 k ranges)
// -> reduce (sum the down partials + residual, next norm operands). The embedding is a
// reduce-like phase before layer 0; the head follows the last reduce.
//
// Every wait is bounded: after a timeout the kernel records QI_ERR_TIMEOUT and every later
// wait of every CTA returns at once, so a failure ends the launch instead of hanging.
#include <cstddef>

#include "common.cuh"
#include "internal.h"
#include "tc_proj.h"
#include "tc_device.cuh"
#include "step.h"

namespace qi {

namespace {

using namespace tc;
using namespace step;

constexpr int kStepThreads = 320;      // warp 0 producer, warp 1 MMA, warps 2-9 workers
constexpr int kWorkers = 256;
constexpr uint32_t kSlotBytes = kSlotKB * 1024;
constexpr int kMaxSlots = 12;
constexpr int kPartStride = kGqa * (kHeadDim + 2);  // floats per (token, head, split) partial

// The CTA's share of each projection (the same in every layer) and its ring slot count.
struct Shares {
  Part P[6];
  int slots[6];
  __device__ void init(int cta, int vocab) {
    for (int op = 0; op < 6; ++op) {
      if (op == kAttn) {
        slots[op] = 0;
        continue;
      }
      P[op] = part_of(op, cta, vocab);
      slots[op] = for_each_piece(P[op], 0, [](const Piece&, int, int, bool, bool) {});
    }
  }
};

// The fixed part of shared memory (before the ring). At least 16 KB: the UMMA A operand of
// a piece that starts mid-tile is addressed from below the piece (rows outside the piece
// are read but never used), which may reach up to 15 KB before the first slot.
struct StepSmem {
  uint64_t full[kMaxSlots];
  uint64_t empty[kMaxSlots];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t b_full;
  uint64_t b_empty;
  uint32_t tmem_slot;
  int alast;
  Shares sh;                    // this CTA's share of every projection
  int tpos[kMaxTokens];
  int trow[kMaxTokens];
  float rsm[kMaxTokens];
  unsigned long long abest[kMaxTokens];
  float red[4][kMaxTokens];     // per lane-quadrant partial sums of squares
  float red2[2][4];             // reduce units: per half, per warp
  // attention scratch (aq and ap are read as float4)
  alignas(16) float aq[kGqa * 2 * 8 * 4];   // q of the 7 heads, scaled, [head][half][chunk][4]
  alignas(16) float ap[4][32][8];           // probabilities per key group
  alignas(16) float acmb[4][kGqa][kHeadDim + 2];
};
static_assert(offsetof(StepSmem, aq) % 16 == 0 && offsetof(StepSmem, ap) % 16 == 0 &&
                  offsetof(StepSmem, abest) % 8 == 0,
              "vector-accessed shared arrays are aligned");
// >= 16 KB: the UMMA A operand of a piece that starts mid-tile is addressed from below the
// piece (rows outside the piece are read, never used), up to 15 KB before the first slot
constexpr size_t kFixedBytes = ((sizeof(StepSmem) + 1023) / 1024 * 1024) < 16384
                                   ? 16384
                                   : (sizeof(StepSmem) + 1023) / 1024 * 1024;

// The activation tiles of a whole K = 896 (14 k blocks of NT tokens, hi/lo); >= 16 KB so
// that operand rows read past the last ring slot stay inside shared memory.
__host__ __device__ inline uint32_t b_region_bytes(int NT) {
  const uint32_t b = 14u * (uint32_t)NT * 256u;
  return b < 16384u ? 16384u : b;
}

// ------------------------------------------------------------------ helpers

// A wait that gave up records QI_ERR_TIMEOUT; every later wait of every CTA then returns at
// once (the launch is failing). An index outside the cache is only reported (below) and
// does not stop the other tokens.
__device__ __forceinline__ bool err_set(const int* err) {
  return *reinterpret_cast<const volatile int*>(err) == QI_ERR_TIMEOUT;
}
__device__ __forceinline__ void report_index(int* err) { atomicCAS(err, 0, QI_ERR_INDEX); }

// Bounded mbarrier wait that also gives up once any CTA has recorded a timeout. The error
// word (a global load) is only read every kErrPollNs of waiting, so a completed phase is
// seen within one try_wait instead of behind a memory round trip.
constexpr uint64_t kErrPollNs = 16000;

__device__ __noinline__ bool swait(uint64_t* bar, uint32_t parity, int* err) {
  for (int i = 0; i < 64; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  uint64_t next = t0 + kErrPollNs;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t now = global_timer_ns();
    if (now >= next) {
      if (err_set(err)) return false;
      if (now - t0 > kWaitLimitNs) {
        atomicExch(err, QI_ERR_TIMEOUT);
        return false;
      }
      next = now + kErrPollNs;
    }
  }
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// named barrier of the 256 worker threads
__device__ __forceinline__ void wbar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// named barrier of one 128-thread half of the workers (reduce units)
__device__ __forceinline__ void hbar(int h) { asm volatile("bar.sync %0, 128;" ::"r"(2 + h) : "memory"); }

// Poll a phase counter until all CTAs have added their 1 (bounded; one thread; the error
// word is read every kErrPollNs).
__device__ __noinline__ bool wait_phase(const unsigned* ctr, int* err) {
  if (ld_acquire_gpu(ctr) >= (unsigned)kGrid) return true;
  const uint64_t t0 = global_timer_ns();
  uint64_t next = t0 + kErrPollNs;
  while (true) {
    if (ld_acquire_gpu(ctr) >= (unsigned)kGrid) return true;
    const uint64_t now = global_timer_ns();
    if (now >= next) {
      if (err_set(err)) return false;
      if (now - t0 > kWaitLimitNs) {
        atomicExch(err, QI_ERR_TIMEOUT);
        return false;
      }
      next = now + kErrPollNs;
    }
  }
}

// Position in the ring of the slot sequence: ring slot `idx` in its `lap`-th use (parity
// lap & 1); advanced slot by slot, so no division by the slot count per piece.
struct RingPos {
  int idx = 0;
  uint32_t lap = 0;
  int ns;
  __device__ explicit RingPos(int n) : ns(n) {}
  __device__ __forceinline__ void next() {
    if (++idx == ns) {
      idx = 0;
      ++lap;
    }
  }
  __device__ __forceinline__ void advance(int n) {
    for (int i = 0; i < n; ++i) next();
  }
};

// Timeline stamp (one thread; no effect without a trace buffer).
__device__ __forceinline__ void stamp(const StepParams& p, int cta, int phase, int event) {
  if (p.trace) p.trace[((long long)cta * kTracePhases + phase) * kTraceEvents + event] = global_timer_ns();
}
__device__ __forceinline__ int phase_of(int op, int l, int n_layers) {
  return op == kHead ? 1 + kPhasesPerLayer * n_layers
                     : counter_index(l, op == kQkv ? 0 : op == kO ? 2 : op == kGateUp ? 3 : 4);
}

__device__ __forceinline__ const uint16_t* weights_of(const StepParams& p, int op, int l) {
  if (op == kHead) return p.embed;
  const StepLayer& L = p.L[l];
  return op == kQkv ? L.w_qkv : op == kO ? L.w_o : op == kGateUp ? L.w_gu : L.w_down;
}

__device__ __forceinline__ bool slot_ok(const StepParams& p, int ps, int row) {
  return ps >= 0 && ps < p.max_len && row >= 0 && row < p.cache_rows;
}

// Attention units of this CTA and their K/V slots. Calls f(t, g, split, kbeg, kend) for
// each unit with keys (kend > kbeg); units of a token outside the cache have none.
template <class F>
__device__ __forceinline__ void for_each_attn_unit(const StepParams& p, const StepSmem& S, int cta, F&& f) {
  const int U = p.max_splits * 2 * p.M;
  for (int u = attn_first_unit(cta); u < U; u += kGrid) {
    const int g = u & 1, t = (u >> 1) % p.M, s = (u >> 1) / p.M;
    const int ps = S.tpos[t];
    if (!slot_ok(p, ps, S.trow[t])) {
      f(t, g, s, 0, 0);
      continue;
    }
    if (s >= attn_nsplit(ps, p.split_keys)) continue;
    const int kbeg = s * p.split_keys;
    const int kend = min(ps + 1, kbeg + p.split_keys);
    f(t, g, s, kbeg, kend);
  }
}

__device__ __forceinline__ int attn_slot_count(const StepParams& p, const StepSmem& S, int cta) {
  int n = 0;
  for_each_attn_unit(p, S, cta, [&](int, int, int, int kbeg, int kend) { n += 2 * ((kend - kbeg + 127) / 128); });
  return n;
}

// ------------------------------------------------------------------ producer

// The producer warp walks the slot sequence in order. Lane 0 alone waits until a ring slot
// is free and posts the bytes each piece will bring; after a __syncwarp the piece's 1 KB
// groups are copied by up to 16 lanes at once (one thread's bulk copies are processed one
// after another, so spreading a slot over lanes keeps several copies in flight). No lane
// ever waits inside a branch the others skipped. Slots are freed in order, so walking them
// in order loses nothing.
__device__ void run_producer(const StepParams& p, StepSmem& S, uint8_t* ring, int cta, int lane,
                             const Shares& sh) {
  RingPos rp(p.slots);
  auto open_slot = [&]() {
    if (lane == 0) swait(&S.empty[rp.idx], (rp.lap & 1u) ^ 1u, p.err);
    __syncwarp();
  };
  auto gemm = [&](int op, int l) {
    const Part& P = sh.P[op];
    if (P.empty()) return;
    const uint16_t* w = weights_of(p, op, l);
    const int KB = op_kblocks(op);
    int cur = -1;
    for_each_piece(P, 0, [&](const Piece& pc, int slot, int off, bool, bool) {
      if (slot != cur) {
        if (cur >= 0) {
          if (lane == 0) mbar_arrive(&S.full[rp.idx]);
          rp.next();
        }
        cur = slot;
        open_slot();
      }
      const int n = pc.kbytes();  // 1 KB groups
      if (lane == 0) mbar_expect_tx(&S.full[rp.idx], (uint32_t)n * 1024u);
      __syncwarp();
      if (lane < n) {
        const int mt = P.tile0() + pc.u;
        bulk_g2s(ring + (size_t)rp.idx * kSlotBytes + (size_t)(off + lane) * 1024,
                 w + ((long long)mt * KB + pc.kb) * 8192 + (long long)(pc.lo + lane) * 512, 1024u, &S.full[rp.idx]);
      }
    });
    if (lane == 0) mbar_arrive(&S.full[rp.idx]);
    rp.next();
  };
  auto attn = [&](int l) {
    for_each_attn_unit(p, S, cta, [&](int t, int g, int, int kbeg, int kend) {
      const long long hb = p.layer_elems * l + ((long long)S.trow[t] * kKvHeads + g) * p.max_len * kHeadDim;
      for (int k0 = kbeg; k0 < kend; k0 += 128) {
        const int nk = min(128, kend - k0);
        for (int kv = 0; kv < 2; ++kv) {
          open_slot();
          if (lane == 0) mbar_arrive_expect_tx(&S.full[rp.idx], (uint32_t)nk * kHeadDim * 2);
          __syncwarp();
          // 8 keys (1 KB) per lane
          const int k8 = lane * 8;
          if (k8 < nk) {
            const int nkl = min(8, nk - k8);
            bulk_g2s(ring + (size_t)rp.idx * kSlotBytes + (size_t)k8 * kHeadDim * 2,
                     (kv ? p.vc : p.kc) + hb + (long long)(k0 + k8) * kHeadDim, (uint32_t)nkl * kHeadDim * 2,
                     &S.full[rp.idx]);
          }
          rp.next();
        }
      }
    });
  };
  for (int l = 0; l < p.n_layers; ++l) {
    gemm(kQkv, l);
    attn(l);
    gemm(kO, l);
    gemm(kGateUp, l);
    gemm(kDown, l);
  }
  gemm(kHead, 0);
}

// ----------------------------------------------------------------------- MMA

// Accumulators: the UMMAs of consecutive k blocks go to `chains` independent accumulators
// (k block kb -> chain (kb - kb0) % chains) so that they do not wait on one another; the
// epilogue adds the chains in order. A layer projection's unit (<= 2 tiles) takes TMEM
// columns [0, 2 * chains * 2NT); the head's one-tile units alternate between buffer 0
// (columns of tile 0) and buffer 1 (columns of tile 1), so a tile's epilogue overlaps the
// next tile's UMMAs. Per buffer, acc_full / acc_empty count its uses.
__device__ __forceinline__ uint32_t tile_cols(const StepParams& p) { return (uint32_t)p.chains * 2u * (uint32_t)p.NT; }

__device__ void run_mma(const StepParams& p, StepSmem& S, uint8_t* ring, uint8_t* bbuf, uint32_t tmem_base,
                        int cta, const Shares& sh) {
  const int NT = p.NT, CH = p.chains;
  const uint32_t idesc = idesc_bf16(128, 2 * NT);
  const uint32_t ring_a = smem_u32(ring), b_a = smem_u32(bbuf);
  const uint32_t tcols = tile_cols(p);
  const int n_attn = attn_slot_count(p, S, cta);
  RingPos rp(p.slots);
  uint32_t use0 = 0, use1 = 0, ops = 0;  // uses of accumulator buffer 0 / 1
  int cur_l = 0;
  auto gemm = [&](int op) {
    const Part& P = sh.P[op];
    if (P.empty()) return;
    const int ph = phase_of(op, cur_l, p.n_layers);
    swait(&S.b_full, ops & 1u, p.err);
    stamp(p, cta, ph, kTrMmaB);
    tc_fence_after();
    bool first_unit = true;
    int cur = -1;
    uint32_t b = 0, head_units = 0;
    for_each_piece(P, 0, [&](const Piece& pc, int slot, int off, bool first, bool last) {
      if (slot != cur) {
        if (cur >= 0) {
          umma_commit(&S.empty[rp.idx]);
          rp.next();
        }
        cur = slot;
        swait(&S.full[rp.idx], rp.lap & 1u, p.err);
        tc_fence_after();
      }
      if (first) {
        b = P.tile_major ? (head_units & 1u) : 0u;
        swait(&S.acc_empty[b], ((b ? use1 : use0) & 1u) ^ 1u, p.err);
        tc_fence_after();
      }
      const int kr = pc.kb - P.kb0;
      const uint32_t d = tmem_base + (P.tile_major ? b : (uint32_t)pc.u) * tcols +
                         (uint32_t)(kr & (CH - 1)) * 2u * (uint32_t)NT;
      // row 0 of the piece's tile (rows outside the piece are read but not used)
      const int a_off = rp.idx * (int)kSlotBytes + (off - pc.lo) * 1024;
      const uint32_t a0 = (uint32_t)((int)ring_a + a_off);
      const uint32_t b0 = b_a + (uint32_t)kr * (uint32_t)NT * 256u;
      umma_bf16_kblock(d, kmajor_desc(a0), kmajor_desc(b0), idesc, kr >= CH ? 1u : 0u);
      if (last) {
        if (first_unit) stamp(p, cta, ph, kTrMmaLast);
        first_unit = false;
        umma_commit(&S.acc_full[b]);
        if (b) ++use1; else ++use0;
        ++head_units;
      }
    });
    umma_commit(&S.empty[rp.idx]);
    rp.next();
    umma_commit(&S.b_empty);
    ++ops;
  };
  for (int l = 0; l < p.n_layers; ++l) {
    cur_l = l;
    gemm(kQkv);
    rp.advance(n_attn);  // K/V slots: consumed by the workers
    gemm(kO);
    gemm(kGateUp);
    gemm(kDown);
  }
  gemm(kHead);
}

// -------------------------------------------------------------------- workers

struct Worker {
  const StepParams& p;
  StepSmem& S;
  uint8_t* ring;
  uint8_t* bbuf;
  uint32_t tmem_base;
  int cta, wt, ww, lane;
  int slot_i = 0;
  uint32_t use0 = 0, use1 = 0, ops = 0;  // uses of accumulator buffer 0 / 1

  __device__ Worker(const StepParams& p_, StepSmem& S_, uint8_t* ring_, uint8_t* bbuf_, uint32_t tb, int cta_, int wt_)
      : p(p_), S(S_), ring(ring_), bbuf(bbuf_), tmem_base(tb), cta(cta_), wt(wt_), ww(wt_ >> 5), lane(wt_ & 31) {
  }

  __device__ void signal(int idx) {
    fence_proxy_async_global();  // outputs may be read by bulk copies in other CTAs
    wbar();
    if (wt == 0) red_release_gpu(p.ctr + (size_t)idx * kCounterStride, 1u);
  }
  __device__ void wait_for(int idx) {
    if (wt == 0) {
      wait_phase(p.ctr + (size_t)idx * kCounterStride, p.err);
      fence_proxy_async_global();
    }
    wbar();
  }

  // ---------------------------------------------------------- reduce / embed
  // Unit (i, t): features f = 128 i + 0..127 of token t. x = embedding row (l < 0) or
  // x + sum of the 21 down partials in k order (reduce of layer l); writes x, the tile's
  // sum of squares ss[i][t] and the next projection's activation tiles of w * x.
  __device__ void reduce_phase(int l) {
    const int M = p.M, NT = p.NT;
    const int h = wt >> 7, tid = wt & 127;
    const int U = reduce_units(M);
    const float* w = l < 0 ? p.L[0].ln1 : (l + 1 < p.n_layers ? p.L[l + 1].ln1 : p.norm_w);
    if (l < 0 && cta == 0 && wt < M) p.argmax[wt] = 0ull;
    // two units at a time, one per 128-thread half
    for (int k = 0;; k += 2) {
      const int u = cta + (k + h) * kGrid;
      const int u_other = cta + (k + (h ^ 1)) * kGrid;
      if (u >= U && u_other >= U) break;
      if (u < U) {
        const int t = u / 7, i = u - t * 7;
        const int f = 128 * i + tid;
        float v;
        if (l < 0) {
          int id = p.ids[t];
          if (id < 0 || id >= p.vocab) {
            if (tid == 0) report_index(p.err);
            id = 0;
          }
          v = bf16_to_f32(p.embed[tiled_offset(id, f, kHidden)]);
        } else {
          v = __ldcg(p.x + (long long)t * kHidden + f);
          float acc = 0.f;
          float part[kDownRanges];  // all loads in flight, then added in k order
#pragma unroll
          for (int j = 0; j < kDownRanges; ++j) part[j] = __ldcg(p.dpart + ((long long)j * NT + t) * kHidden + f);
#pragma unroll
          for (int j = 0; j < kDownRanges; ++j) acc += part[j];
          v += acc;
        }
        p.x[(long long)t * kHidden + f] = v;
        float sq = warp_sum(v * v);
        if ((tid & 31) == 0) S.red2[h][tid >> 5] = sq;
        const float a = v * __ldg(w + f);
        const uint16_t hi = f32_to_bf16_rn(a);
        p.act_x[act_offset(t, f, 0, kHidden, NT)] = hi;
        p.act_x[act_offset(t, f, 1, kHidden, NT)] = f32_to_bf16_rn(a - bf16_to_f32(hi));
        hbar(h);
        if (tid == 0) p.ss[i * NT + t] = (S.red2[h][0] + S.red2[h][1]) + (S.red2[h][2] + S.red2[h][3]);
        hbar(h);
      }
    }
  }

  // ------------------------------------------------------------- attention
  // One unit: keys [kbeg, kend) of token t's row for KV head g (split s of nsplit), K/V
  // tiles from the ring (slots slot_i, slot_i + 1, ...), the key at the token's own
  // position patched in from the cache (written by this step's QKV phase).
  __device__ void attention_unit(int l, int t, int g, int split, int kbeg, int kend) {
    const int ns = p.slots;
    const int ps = S.tpos[t], row = S.trow[t];
    if (kend <= kbeg) {  // outside the cache: reported, nothing read or written
      if (split == 0 && wt == 0) report_index(p.err);
      return;
    }
    const int nsplit = attn_nsplit(ps, p.split_keys);
    const int kgrp = ww & 3, h0 = (ww >> 2) * 4, nh = min(4, kGqa - h0);
    // q of the 7 heads of group g, scaled by 1/8 (exact), chunk-interleaved layout
    {
      constexpr int kRounds = (kGqa * kHeadDim + kWorkers - 1) / kWorkers;
      float qv[kRounds];
#pragma unroll
      for (int r = 0; r < kRounds; ++r) {
        const int idx = wt + r * kWorkers;
        qv[r] = __ldcg(p.q + (long long)t * kHidden + g * kGqa * kHeadDim + (idx < kGqa * kHeadDim ? idx : 0));
      }
#pragma unroll
      for (int r = 0; r < kRounds; ++r) {
        const int idx = wt + r * kWorkers;
        if (idx < kGqa * kHeadDim) {
          const int hh = idx >> 6, d = idx & 63, cc = d >> 3, e = d & 7;
          S.aq[((hh * 2 + (e >> 2)) * 8 + cc) * 4 + (e & 3)] = qv[r] * 0.125f;
        }
      }
    }
    wbar();
    float m[4], lsum[4], acc[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      m[i] = -INFINITY;
      lsum[i] = 0.f;
      acc[i][0] = acc[i][1] = 0.f;
    }
    const long long hb = p.layer_elems * l + ((long long)row * kKvHeads + g) * p.max_len * kHeadDim;
    const int ntiles = (kend - kbeg + 127) / 128;
    for (int i = 0; i < ntiles; ++i, slot_i += 2) {
      const int sk = slot_i % ns, sv = (slot_i + 1) % ns;
      swait(&S.full[sk], (uint32_t)((slot_i / ns) & 1), p.err);
      swait(&S.full[sv], (uint32_t)(((slot_i + 1) / ns) & 1), p.err);
      uint16_t* Kt = reinterpret_cast<uint16_t*>(ring + (size_t)sk * kSlotBytes);
      uint16_t* Vt = reinterpret_cast<uint16_t*>(ring + (size_t)sv * kSlotBytes);
      const int k0 = kbeg + i * 128;
      const int nk = min(128, kend - k0);
      if (ps >= k0 && ps < k0 + nk) {
        // the token's own key and value, written by this step's QKV phase
        if (wt < 16) {
          const uint16_t* src = (wt < 8 ? p.kc : p.vc) + hb + (long long)ps * kHeadDim + (wt & 7) * 8;
          const uint4 val = __ldcg(reinterpret_cast<const uint4*>(src));
          *reinterpret_cast<uint4*>((wt < 8 ? Kt : Vt) + (ps - k0) * kHeadDim + (wt & 7) * 8) = val;
        }
        wbar();
      }
      const int kw = 32 * kgrp;
      const int nkw = max(0, min(32, nk - kw));
      if (nkw > 0) {
        const bool valid = lane < nkw;
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        const uint16_t* krow = Kt + (kw + lane) * kHeadDim;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int cc = (c + lane) & 7;
          const uint4 kv = *reinterpret_cast<const uint4*>(krow + cc * 8);
          const float k0f = bf16lo(kv.x), k1f = bf16hi(kv.x), k2f = bf16lo(kv.y), k3f = bf16hi(kv.y);
          const float k4f = bf16lo(kv.z), k5f = bf16hi(kv.z), k6f = bf16lo(kv.w), k7f = bf16hi(kv.w);
#pragma unroll
          for (int hi = 0; hi < 4; ++hi) {
            if (hi < nh) {
              const int hh = h0 + hi;
              const float4 qa = *reinterpret_cast<const float4*>(&S.aq[((hh * 2 + 0) * 8 + cc) * 4]);
              const float4 qb = *reinterpret_cast<const float4*>(&S.aq[((hh * 2 + 1) * 8 + cc) * 4]);
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
        for (int hi = 0; hi < 4; ++hi) {
          if (hi < nh) {
            const float sv2 = valid ? s[hi] : -INFINITY;
            const float mn = fmaxf(m[hi], warp_max(sv2));
            const float alpha = expf(m[hi] - mn);
            const float pr = valid ? expf(sv2 - mn) : 0.f;
            lsum[hi] = lsum[hi] * alpha + warp_sum(pr);
            acc[hi][0] *= alpha;
            acc[hi][1] *= alpha;
            m[hi] = mn;
            S.ap[kgrp][lane][h0 + hi] = pr;
          }
        }
        __syncwarp();
        const uint16_t* vt = Vt + kw * kHeadDim + 2 * lane;
#pragma unroll 4
        for (int j = 0; j < nkw; ++j) {
          const uint32_t v2 = *reinterpret_cast<const uint32_t*>(vt + j * kHeadDim);
          const float v0 = bf16lo(v2), v1 = bf16hi(v2);
          const float4 pa = *reinterpret_cast<const float4*>(&S.ap[kgrp][j][h0]);
          const float pv[4] = {pa.x, pa.y, pa.z, pa.w};
#pragma unroll
          for (int hi = 0; hi < 4; ++hi) {
            acc[hi][0] = fmaf(pv[hi], v0, acc[hi][0]);
            acc[hi][1] = fmaf(pv[hi], v1, acc[hi][1]);
          }
        }
        __syncwarp();
      }
      wbar();  // both slots fully read
      if (wt == 0) {
        fence_proxy_async_smem();
        mbar_arrive(&S.empty[sk]);
        mbar_arrive(&S.empty[sv]);
      }
    }
    // merge the 4 key groups (as the standalone attention kernel)
#pragma unroll
    for (int hi = 0; hi < 4; ++hi) {
      if (hi < nh) {
        const int hh = h0 + hi;
        S.acmb[kgrp][hh][2 * lane] = acc[hi][0];
        S.acmb[kgrp][hh][2 * lane + 1] = acc[hi][1];
        if (lane == 0) {
          S.acmb[kgrp][hh][kHeadDim] = m[hi];
          S.acmb[kgrp][hh][kHeadDim + 1] = lsum[hi];
        }
      }
    }
    wbar();
    float* part = p.apart + (((long long)t * kKvHeads + g) * p.max_splits + split) * kPartStride;
    for (int idx = wt; idx < kPartStride; idx += kWorkers) {
      const int hh = idx / (kHeadDim + 2), d = idx - hh * (kHeadDim + 2);
      float mx = -INFINITY;
#pragma unroll
      for (int w4 = 0; w4 < 4; ++w4) mx = fmaxf(mx, S.acmb[w4][hh][kHeadDim]);
      float L = 0.f, A = 0.f;
#pragma unroll
      for (int w4 = 0; w4 < 4; ++w4) {
        const float mw = S.acmb[w4][hh][kHeadDim];
        if (mw == -INFINITY) continue;
        const float sc = expf(mw - mx);
        L = fmaf(sc, S.acmb[w4][hh][kHeadDim + 1], L);
        if (d < kHeadDim) A = fmaf(sc, S.acmb[w4][hh][d], A);
      }
      if (nsplit == 1) {
        if (d < kHeadDim) emit_attn(t, (g * kGqa + hh) * kHeadDim + d, A / L);
      } else {
        part[idx] = d < kHeadDim ? A : (d == kHeadDim ? mx : L);
      }
    }
    if (nsplit == 1) return;
    // split merge by the last-arriving unit of (t, g): the barrier orders every thread's
    // partial stores before thread 0's acq_rel arrival
    wbar();
    if (wt == 0) S.alast = atomic_add_acq_rel(&p.acnt[t * kKvHeads + g], 1u) == (unsigned)(nsplit - 1);
    wbar();
    if (!S.alast) return;
    const float* base = p.apart + (((long long)t * kKvHeads + g) * p.max_splits) * kPartStride;
    float* sm = &S.acmb[0][0][0];  // 2 * 7 * nsplit + 7 floats (nsplit <= max_splits <= 128)
    for (int idx = wt; idx < kGqa * nsplit; idx += kWorkers) {
      const int hh = idx / nsplit, s = idx - hh * nsplit;
      sm[idx] = __ldcg(base + (long long)s * kPartStride + hh * (kHeadDim + 2) + kHeadDim);
      sm[kGqa * nsplit + idx] = __ldcg(base + (long long)s * kPartStride + hh * (kHeadDim + 2) + kHeadDim + 1);
    }
    wbar();
    if (wt < kGqa) {
      const int hh = wt;
      float mx = -INFINITY;
      for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, sm[hh * nsplit + s]);
      float L = 0.f;
      for (int s = 0; s < nsplit; ++s) {
        const float sc = expf(sm[hh * nsplit + s] - mx);
        L = fmaf(sc, sm[kGqa * nsplit + hh * nsplit + s], L);
        sm[hh * nsplit + s] = sc;
      }
      sm[2 * kGqa * nsplit + hh] = L;
    }
    wbar();
    {
      constexpr int kRounds = (kGqa * kHeadDim + kWorkers - 1) / kWorkers;
      float A[kRounds];
#pragma unroll
      for (int r = 0; r < kRounds; ++r) A[r] = 0.f;
      for (int s = 0; s < nsplit; ++s) {
#pragma unroll
        for (int r = 0; r < kRounds; ++r) {
          const int idx = wt + r * kWorkers;
          if (idx < kGqa * kHeadDim) {
            const int hh = idx >> 6, d = idx & 63;
            A[r] = fmaf(sm[hh * nsplit + s], __ldcg(base + (long long)s * kPartStride + hh * (kHeadDim + 2) + d), A[r]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kRounds; ++r) {
        const int idx = wt + r * kWorkers;
        if (idx < kGqa * kHeadDim) emit_attn(t, g * kGqa * kHeadDim + idx, A[r] / sm[2 * kGqa * nsplit + (idx >> 6)]);
      }
    }
    wbar();
    if (wt == 0) p.acnt[t * kKvHeads + g] = 0u;
  }

  __device__ __forceinline__ void emit_attn(int t, int f, float v) {
    const uint16_t hi = f32_to_bf16_rn(v);
    p.act_attn[act_offset(t, f, 0, kHidden, p.NT)] = hi;
    p.act_attn[act_offset(t, f, 1, kHidden, p.NT)] = f32_to_bf16_rn(v - bf16_to_f32(hi));
  }

  __device__ void attention_phase(int l) {
    for_each_attn_unit(p, S, cta, [&](int t, int g, int s, int kbeg, int kend) {
      attention_unit(l, t, g, s, kbeg, kend);
      wbar();  // the unit's shared scratch is free
    });
  }

  // ------------------------------------------------------------ projections

  // Accumulator columns [8 tokens of chunk c] of this warp's 32 rows: hi + lo of every
  // chain that received a k block, added chain by chain (a fixed order).
  __device__ __forceinline__ void tmem_chunk(uint32_t t_tile, int c, int nchains, float (&v)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    for (int ch = 0; ch < nchains; ++ch) {
      float a[8], b[8];
      const uint32_t t = t_tile + (uint32_t)(ch * 2 * p.NT + c * 8);
      tmem_ld8(t, a);
      tmem_ld8(t + (uint32_t)p.NT, b);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] += a[i] + b[i];
    }
  }

  // Fused epilogue of weight row n (valid) for tokens c*8 .. c*8+nlive-1.
  __device__ __forceinline__ void finish(int op, int l, int n, bool valid, int c, int nlive, const float (&v)[8],
                                         float (&sq)[8]) {
    const int t0 = c * 8;
    if (op == kQkv) {
      // RMSNorm scale, bias, RoPE (qwen2.py:160-171, 86-99), q out / KV append
      // (kv_cache.py:59-60); rows 2j, 2j+1 are a RoPE pair (adjacent lanes)
      const int head = n >> 6, half = n & 1, d = ((n & 63) >> 1) + 32 * half, j = (n & 63) >> 1;
      const bool rope = head < kHeads + kKvHeads;
      const float bias = valid ? __ldg(p.L[l].b_qkv + n) : 0.f;
      float x[8], partner[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = v[i] * S.rsm[t0 + i] + bias;
#pragma unroll
      for (int i = 0; i < 8; ++i) partner[i] = __shfl_xor_sync(0xffffffffu, x[i], 1);
      uint16_t* kvbase = (head < kHeads + kKvHeads ? p.kc : p.vc) + p.layer_elems * l;
      const int kvh = (head - kHeads) & 1;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (valid && i < nlive) {
          const int t = t0 + i, ps = S.tpos[t], rw = S.trow[t];
          const bool ok = slot_ok(p, ps, rw);
          if (rope) {
            const long long o = (long long)(ok ? ps : 0) * kHeadDim + j;
            const float cs = __ldg(p.rope_cos + o), sn = __ldg(p.rope_sin + o);
            x[i] = half ? (x[i] * cs + partner[i] * sn) : (x[i] * cs - partner[i] * sn);
          }
          if (head < kHeads) {
            p.q[(long long)t * kHidden + head * kHeadDim + d] = x[i];
          } else if (ok) {
            kvbase[(((long long)rw * kKvHeads + kvh) * p.max_len + ps) * kHeadDim + d] = f32_to_bf16_rn(x[i]);
          } else if (d == 0) {
            report_index(p.err);
          }
        }
      }
    } else if (op == kO) {
      // residual add into the fp32 stream (qwen2.py:237-238), then the gate/up
      // activations hi/lo(ln2 * x) and this row's share of the sums of squares
      const float wn = valid ? __ldg(p.L[l].ln2 + n) : 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        sq[i] = 0.f;
        if (valid && i < nlive) {
          const int t = t0 + i;
          const float xn = __ldcg(p.x + (long long)t * kHidden + n) + v[i];
          p.x[(long long)t * kHidden + n] = xn;
          sq[i] = xn * xn;
          const float a = xn * wn;
          const uint16_t hi = f32_to_bf16_rn(a);
          p.act_x[act_offset(t, n, 0, kHidden, p.NT)] = hi;
          p.act_x[act_offset(t, n, 1, kHidden, p.NT)] = f32_to_bf16_rn(a - bf16_to_f32(hi));
        }
      }
    } else if (op == kGateUp) {
      // silu(gate) * up (qwen2.py:114-116); gate row 2i (even lane), up row 2i+1
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xg = v[i] * S.rsm[t0 + i];
        const float up = __shfl_xor_sync(0xffffffffu, xg, 1);
        if (valid && !(n & 1) && i < nlive) {
          const float hval = __fdividef(xg, 1.0f + __expf(-xg)) * up;
          const uint16_t hi = f32_to_bf16_rn(hval);
          const int t = t0 + i, f = n >> 1;
          p.act_h[act_offset(t, f, 0, kInter, p.NT)] = hi;
          p.act_h[act_offset(t, f, 1, kInter, p.NT)] = f32_to_bf16_rn(hval - bf16_to_f32(hi));
        }
      }
    } else {  // kHead: final norm scale, logits, greedy argmax (qwen2.py:282-292, engine.py:155)
      unsigned long long key[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float x = v[i] * S.rsm[t0 + i];
        const bool live = valid && i < nlive;
        if (live && p.logits) {
          const long long o = (long long)(t0 + i) * p.logits_ld + n;
          if (p.logits_bf16) reinterpret_cast<uint16_t*>(p.logits)[o] = f32_to_bf16_rn(x);
          else reinterpret_cast<float*>(p.logits)[o] = x;
        }
        key[i] = live ? argmax_pack(x, n) : 0ull;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, key[i], o);
          key[i] = other > key[i] ? other : key[i];
        }
      if (lane == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (key[i]) atomicMax(&S.abest[t0 + i], key[i]);
      }
    }
  }

  // One projection phase of this CTA: activation tiles in, accumulation unit(s), the
  // pair exchange and the fused epilogue (or the down partials).
  __device__ void gemm_phase(int op, int l, int dep) {
    const Part& P = S.sh.P[op];
    slot_i += S.sh.slots[op];
    const int M = p.M, NT = p.NT;
    const int nch = (M + 7) / 8;
    if (P.empty()) {
      wait_for(dep);  // keep the phase order (nothing to multiply here)
      if (op == kO && wt < M) p.ss_o[cta * NT + wt] = 0.f;
      return;
    }
    const int nkb = P.kb1 - P.kb0;
    const uint16_t* act = op == kO ? p.act_attn : op == kDown ? p.act_h : p.act_x;
    const int ph = phase_of(op, l, p.n_layers);
    if (wt == 0) {
      stamp(p, cta, ph, kTrEnter);
      wait_phase(p.ctr + (size_t)dep * kCounterStride, p.err);
      stamp(p, cta, ph, kTrInputs);
      fence_proxy_async_global();
      swait(&S.b_empty, (ops & 1u) ^ 1u, p.err);
      mbar_arrive_expect_tx(&S.b_full, (uint32_t)(nkb * NT * 256));
    }
    wbar();
    if (wt < nkb) {
      // the activation tiles were written by other CTAs (generic proxy) and are read by a
      // bulk copy (async proxy): the issuing thread acquires the phase counter itself and
      // fences the proxies before its copy
      (void)ld_acquire_gpu(p.ctr + (size_t)dep * kCounterStride);
      fence_proxy_async_global();
      bulk_g2s(bbuf + (size_t)wt * NT * 256, act + (long long)(P.kb0 + wt) * NT * 128, (uint32_t)(NT * 256), &S.b_full);
    }
    // per-token RMSNorm scale of the multiplied activations (qwen2.py:44-48)
    if (wt < M && (op == kQkv || op == kHead || op == kGateUp)) {
      float ss = 0.f;
      if (op == kGateUp) {
        for (int j = 0; j < kGrid; ++j) ss += __ldcg(p.ss_o + j * NT + wt);
      } else {
#pragma unroll
        for (int j = 0; j < 7; ++j) ss += __ldcg(p.ss + j * NT + wt);
      }
      S.rsm[wt] = 1.0f / sqrtf(ss / (float)kHidden + p.eps);
    }
    if (op == kHead && wt < kMaxTokens) S.abest[wt] = 0ull;
    wbar();
    // a warp reads the TMEM lane quadrant (its warp index within the CTA) % 4: worker
    // warps 2..9 cover quadrants 2, 3, 0, 1 (half 0) and again (half 1)
    const int quad = (ww + 2) & 3, half = ww >> 2;
    const int row = quad * 32 + lane;
    const int nt = P.ntiles(), nu = units_of(P);
    const int nchains = min(p.chains, nkb);
    const uint32_t tcols = tile_cols(p);
    if (op == kO) {
      // per lane quadrant, this CTA's share of each token's sum of squares (accumulated
      // over its tiles; each (quadrant, token) entry belongs to one warp)
      if (wt < 4 * kMaxTokens) S.red[wt / kMaxTokens][wt % kMaxTokens] = 0.f;
      wbar();
    }
    for (int uu = 0; uu < nu; ++uu) {
      const uint32_t b = P.tile_major ? (uint32_t)(uu & 1) : 0u;
      swait(&S.acc_full[b], (b ? use1 : use0) & 1u, p.err);
      if (wt == 0 && uu == 0) stamp(p, cta, ph, kTrAcc);
      tc_fence_after();
      const int v_lo = P.tile_major ? uu : 0, v_hi = P.tile_major ? uu + 1 : nt;
      for (int v = v_lo; v < v_hi; ++v) {
        const int mt = P.tile0() + v;
        const int r_lo = 8 * (P.seg_lo(v) - 16 * mt), r_hi = 8 * (P.seg_hi(v) - 16 * mt);
        const bool valid = row >= r_lo && row < r_hi;
        const int n = mt * 128 + row;
        const uint32_t t_tile =
            tmem_base + ((uint32_t)(quad * 32) << 16) + (P.tile_major ? b : (uint32_t)v) * tcols;
        for (int c = half; c < nch; c += 2) {
          float val[8];
          tmem_chunk(t_tile, c, nchains, val);
          const int nlive = min(8, M - c * 8);
          if (op == kDown) {
            const int j = cta % kDownRanges;
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (i < nlive) p.dpart[((long long)j * NT + c * 8 + i) * kHidden + n] = val[i];
            continue;
          }
          float sq[8];
          finish(op, l, n, valid, c, nlive, val, sq);
          if (op == kO) {
#pragma unroll
            for (int i = 0; i < 8; ++i) sq[i] = warp_sum(sq[i]);
            if (lane == 0) {
#pragma unroll
              for (int i = 0; i < 8; ++i)
                if (c * 8 + i < M) S.red[quad][c * 8 + i] += sq[i];
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.acc_empty[b]);
      if (b) ++use1; else ++use0;
    }
    if (op == kO) {
      // this CTA's slot of the o projection's sums of squares (zero if it has no rows)
      wbar();
      if (wt < M) p.ss_o[cta * NT + wt] = (S.red[2][wt] + S.red[3][wt]) + (S.red[0][wt] + S.red[1][wt]);
    }
    if (op == kHead) {
      wbar();
      if (wt < M && S.abest[wt]) atomicMax(&p.argmax[wt], S.abest[wt]);
    }
    if (wt == 0) stamp(p, cta, ph, kTrDone);
    ++ops;
  }

  __device__ void run() {
    if (wt == 0) stamp(p, cta, 0, kTrEnter);
    reduce_phase(-1);  // embedding
    if (wt == 0) stamp(p, cta, 0, kTrDone);
    signal(0);
    for (int l = 0; l < p.n_layers; ++l) {
      gemm_phase(kQkv, l, l == 0 ? 0 : counter_index(l - 1, 5));
      signal(counter_index(l, 0));
      if (wt == 0) stamp(p, cta, counter_index(l, 1), kTrEnter);
      wait_for(counter_index(l, 0));
      if (wt == 0) stamp(p, cta, counter_index(l, 1), kTrInputs);
      attention_phase(l);
      if (wt == 0) stamp(p, cta, counter_index(l, 1), kTrDone);
      signal(counter_index(l, 1));
      gemm_phase(kO, l, counter_index(l, 1));
      signal(counter_index(l, 2));
      gemm_phase(kGateUp, l, counter_index(l, 2));
      signal(counter_index(l, 3));
      gemm_phase(kDown, l, counter_index(l, 3));
      signal(counter_index(l, 4));
      if (wt == 0) stamp(p, cta, counter_index(l, 5), kTrEnter);
      wait_for(counter_index(l, 4));
      if (wt == 0) stamp(p, cta, counter_index(l, 5), kTrInputs);
      reduce_phase(l);
      if (wt == 0) stamp(p, cta, counter_index(l, 5), kTrDone);
      signal(counter_index(l, 5));
    }
    gemm_phase(kHead, 0, counter_index(p.n_layers - 1, 5));
  }
};

__global__ void __launch_bounds__(kStepThreads, 1) step_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  StepSmem& S = *reinterpret_cast<StepSmem*>(smem);
  uint8_t* ring = smem + kFixedBytes;
  uint8_t* bbuf = ring + (size_t)p.slots * kSlotBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.slots; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    mbar_init(&S.acc_full[0], 1);
    mbar_init(&S.acc_full[1], 1);
    mbar_init(&S.acc_empty[0], kWorkers / 32);
    mbar_init(&S.acc_empty[1], kWorkers / 32);
    mbar_init(&S.b_full, 1);
    mbar_init(&S.b_empty, 1);
    fence_barrier_init();
  }
  if (threadIdx.x == 32) S.sh.init(cta, p.vocab);
  if (threadIdx.x < kMaxTokens) {
    const int t = threadIdx.x;
    S.tpos[t] = t < p.M ? p.pos[t] : 0;
    S.trow[t] = t < p.M ? p.rows[t] : 0;
    S.abest[t] = 0ull;
  }
  if (warp == 1) {
    tmem_alloc(&S.tmem_slot, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = S.tmem_slot;

  if (warp == 0) {
    run_producer(p, S, ring, cta, lane, S.sh);
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) run_mma(p, S, ring, bbuf, tmem_base, cta, S.sh);
    __syncwarp();
  } else {
    Worker w(p, S, ring, bbuf, tmem_base, cta, threadIdx.x - 64);
    w.run();
  }

  if (err_set(p.err)) {
    // a wait gave up and the loops ran on without waiting: let the copies and MMAs
    // already issued land before shared memory and TMEM are released
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 200000ull) __nanosleep(1000);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

}  // namespace

int step_ring_slots(int NT) {
  const size_t room = 227 * 1024 - kFixedBytes - b_region_bytes(NT);
  int slots = (int)(room / kSlotBytes);
  return slots > kMaxSlots ? kMaxSlots : slots;
}

size_t step_smem_bytes(int NT) {
  return kFixedBytes + (size_t)step_ring_slots(NT) * kSlotBytes + b_region_bytes(NT);
}

int step_chains(int NT) { return NT <= 16 ? 8 : 4; }

uint32_t step_tmem_cols(int NT) {
  // two tiles of `chains` accumulators of 2 NT columns each, rounded to a power of two
  uint32_t need = 2u * (uint32_t)step_chains(NT) * 2u * (uint32_t)NT, cols = 32;
  while (cols < need) cols <<= 1;
  return cols;
}

bool step_supported() { return sm_count() == kGrid; }

cudaError_t launch_step(const StepParams& p, cudaStream_t stream) {
  const size_t smem = step_smem_bytes(p.NT);
  if (p.slots != step_ring_slots(p.NT) || p.chains != step_chains(p.NT) || p.tmem_cols != step_tmem_cols(p.NT) ||
      p.tmem_cols > 512)
    return cudaErrorInvalidValue;
  cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(step_kernel), (int)smem);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(p.ctr, 0, sizeof(unsigned) * kCounterStride * (size_t)(1 + kPhasesPerLayer * p.n_layers),
                      stream);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kGrid, 1, 1);
  cfg.blockDim = dim3(kStepThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: phases wait on each other
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, step_kernel, p);
}

}  // namespace qi
