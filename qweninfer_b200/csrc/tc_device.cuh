// Device-side building blocks of the tensor-core kernels (tc_proj.cu, and the tcgen05 /
// TMEM wrappers and descriptors the prefill attention in attention_block.cu uses): UMMA
// descriptors, the stream-K partition, activation-tile addressing and the fused
// epilogues of every projection.
#pragma once

#include "common.cuh"
#include "internal.h"
#include "tc_proj.h"

namespace qi {
namespace tc {

constexpr int kProjEpiWarps = 8;      // epilogue warps of tc_proj_kernel: two per TMEM lane quadrant
constexpr int kProjThreads = 64 + 32 * kProjEpiWarps;
constexpr int kEpiWarp0 = 2;
constexpr uint32_t kABytes = 128 * 64 * 2;  // one 128x64 weight block

// ------------------------------------------------------------ tcgen05 wrappers

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void umma_bf16(uint32_t d_taddr, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_taddr),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}
// The four UMMAs (K = 16 each) of one 64-column k block: A and B descriptors of the block's
// first core-matrix column, stepped by 256 bytes (16 in the descriptors' address field,
// which cannot carry: shared addresses stay below 256 KB). `acc0` is the accumulate flag of
// the first UMMA; the other three always accumulate.
__device__ __forceinline__ void umma_bf16_kblock(uint32_t d_taddr, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t acc0) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.eq.b32 q, %4, %4;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %5, %6, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %7, %8, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %9, %10, %3, q;\n\t}" ::"r"(d_taddr),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc0), "l"(adesc + 16), "l"(bdesc + 16), "l"(adesc + 32),
      "l"(bdesc + 32), "l"(adesc + 48), "l"(bdesc + 48)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// named barrier of EW epilogue warps
template <int EW>
__device__ __forceinline__ void epi_bar_n() {
  if constexpr (EW == 4) asm volatile("bar.sync 1, 128;" ::: "memory");
  else asm volatile("bar.sync 1, 256;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// SWIZZLE_NONE K-major shared-memory descriptor: LBO 128 B, SBO 1024 B, version bit (sm_100).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
         (1ull << 46);
}

// Instruction descriptor of kind::f16: bf16 A and B, both K-major, fp32 D, shape M x N.
__device__ __forceinline__ uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------- operand staging by threads

// byte offset of (row r, 8-element chunk c) in a K-major operand with 1 KB per 8-row group
__device__ __forceinline__ uint32_t kmaj(int r, int c) { return (uint32_t)((r >> 3) * 1024 + c * 128 + (r & 7) * 16); }

// bf16 pair (a at the lower address), round to nearest even
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}

// hi/lo bf16 halves of 8 consecutive values (hi = bf16(v), lo = bf16(v - hi))
__device__ __forceinline__ void split8(const float (&v)[8], uint4& hi, uint4& lo) {
  const uint32_t h0 = pack_bf16(v[0], v[1]), h1 = pack_bf16(v[2], v[3]);
  const uint32_t h2 = pack_bf16(v[4], v[5]), h3 = pack_bf16(v[6], v[7]);
  hi = make_uint4(h0, h1, h2, h3);
  lo = make_uint4(pack_bf16(v[0] - bf16lo(h0), v[1] - bf16hi(h0)), pack_bf16(v[2] - bf16lo(h1), v[3] - bf16hi(h1)),
                  pack_bf16(v[4] - bf16lo(h2), v[5] - bf16hi(h2)), pack_bf16(v[6] - bf16lo(h3), v[7] - bf16hi(h3)));
}

// 64 consecutive TMEM columns of this thread's lane (two x32 loads, one wait)
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr + 32u));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------- stream-K geometry

struct Geom {
  int U, G;
  __device__ int start(int c) const { return (int)(((long long)c * U) / G); }
  // CTA whose range holds unit u: the largest c with start(c) <= u
  __device__ int owner(int u) const { return (int)(((long long)(u + 1) * G - 1) / U); }
};

// ------------------------------------------------------------------ epilogues

// Shared-memory scratch of the four epilogue warps (carve_epi lays it out).
struct EpiSmem {
  unsigned long long* abest;  // 128 packed argmax candidates of the token tile
  float* sred;                // [4 lane quadrants][128 tokens] partial sums of squares
  float* rsm;                 // 128 per-token reciprocal RMS of the current token tile
  int* tpos;                  // 128 positions of the current token tile
  int* trow;                  // 128 cache rows of the current token tile
  int* flag;                  // last-contributor broadcast
  uint16_t* stage;            // 4096: per-warp staging of activation-tile stores
  // cluster split tiles (tc_proj_kernel only): partials of ranks 1.. ((cluster - 1) x 128 x
  // NT floats, the partial layout) and the barrier their epilogue threads arrive on
  float* recv;
  uint64_t* red_full;
};
constexpr size_t kEpiSmemBytes = 128 * 8 + 4 * 128 * 4 + 128 * 4 + 128 * 4 + 128 * 4 + 16 + 4096 * 2;

__device__ __forceinline__ EpiSmem carve_epi(uint8_t* base) {  // base 8-byte aligned
  EpiSmem e;
  e.abest = reinterpret_cast<unsigned long long*>(base);
  e.sred = reinterpret_cast<float*>(base + 1024);
  e.rsm = e.sred + 4 * 128;
  e.tpos = reinterpret_cast<int*>(e.rsm + 128);
  e.trow = e.tpos + 128;
  e.flag = e.trow + 128;
  e.stage = reinterpret_cast<uint16_t*>(base + 4624);  // 16-byte aligned when base is
  e.recv = nullptr;
  e.red_full = nullptr;
  return e;
}

// Activation-tile store of one warp for the CT tokens tbase.. of a chunk: lane L holds
// val[i] for column k0 + (L >> SHIFT) (SHIFT 1: the even lanes hold 16 columns; SHIFT 0:
// all lanes, 32 columns; the columns lie in one 64-column block). The hi/lo halves go to
// the warp's staging buffer in the tile layout, then out as 16-byte rows of core matrices
// (2-4 vector stores per lane instead of 2 * CT scattered 2-byte stores). Live tokens only.
template <int CT, int SHIFT>
__device__ __forceinline__ void act_store_warp(uint16_t* act, int K, int NT, int lg, int k0, int tbase, int nlive,
                                               const float (&val)[CT], uint16_t* wbuf, int lane) {
  constexpr int KG = (32 >> SHIFT) / 8;  // 8-column groups of the warp
  constexpr int TG = CT / 8;             // 8-token groups of the chunk
  if ((lane & ((1 << SHIFT) - 1)) == 0) {
    const int col = lane >> SHIFT, kg = col >> 3, kk = col & 7;
#pragma unroll
    for (int i = 0; i < CT; ++i) {
      const uint16_t hi = f32_to_bf16_rn(val[i]);
      const uint16_t lo = f32_to_bf16_rn(val[i] - bf16_to_f32(hi));
      wbuf[((0 * TG + (i >> 3)) * KG + kg) * 64 + (i & 7) * 8 + kk] = hi;
      wbuf[((1 * TG + (i >> 3)) * KG + kg) * 64 + (i & 7) * 8 + kk] = lo;
    }
  }
  __syncwarp();
  const long long kpart = (long long)(k0 >> 6) * (2LL * NT * 64) + ((k0 & 63) >> 3) * 64;
  const long long ntile = (long long)(K / 64) * 2LL * NT * 64;
#pragma unroll
  for (int r = 0; r < (2 * TG * KG * 8) / 32; ++r) {
    const int v = lane + 32 * r;
    const int t = v & 7, kg = (v >> 3) % KG, tg = ((v >> 3) / KG) % TG, part = (v >> 3) / (KG * TG);
    const int i = tg * 8 + t;
    if (i < nlive) {
      const int tok = tbase + i, tl = tok & ((1 << lg) - 1);
      const long long o = (long long)(tok >> lg) * ntile + kpart + (long long)part * NT * 64 + (tl >> 3) * 512 +
                          kg * 64 + (tl & 7) * 8;
      *reinterpret_cast<uint4*>(act + o) =
          *reinterpret_cast<const uint4*>(wbuf + ((part * TG + tg) * KG + kg) * 64 + t * 8);
    }
  }
  __syncwarp();
}

// Whether the K/V of a token at position ps of cache row rw can be stored. Positions
// outside [0, max_len) and rows outside the cache are reported (QI_ERR_INDEX) and their
// K/V store skipped; the RoPE table lookups use position 0 for them.
__device__ __forceinline__ bool kv_slot_ok(const TcParams& p, int ps, int rw) {
  return ps >= 0 && ps < p.max_len && rw >= 0 && (p.cache_rows == 0 || rw < p.cache_rows);
}

// Epilogue operands of one chunk that do not depend on the accumulator: loaded before the
// accumulator wait (first chunk) or ahead of the previous chunk's stores, so that their
// latency overlaps the MMAs and the split-tile fix-up instead of following them.
template <int EPI, int CT>
struct ChunkPre {};
template <int CT>
struct ChunkPre<kTcQkvRope, CT> {
  float cs[CT], sn[CT], b;
};
template <int CT>
struct ChunkPre<kTcQkvRopePaged, CT> : ChunkPre<kTcQkvRope, CT> {};
template <int CT>
struct ChunkPre<kTcResidual, CT> {
  float xo[CT], wn;
};

// Operands of weight row n for the nlive tokens tbase.. (tpos/trow: the chunk's positions
// and cache rows in shared memory).
template <int EPI, int CT>
__device__ __forceinline__ void pre_load(const TcParams& p, int n, int tbase, int nlive, const int* tpos,
                                         const int* trow, ChunkPre<EPI, CT>& pre) {
  if constexpr (kIsQkv<EPI>) {
    const int head = n >> 6, j = (n & 63) >> 1;
    const bool rope = head < kHeads + kKvHeads;
    pre.b = __ldg(p.bias + n);
#pragma unroll
    for (int i = 0; i < CT; ++i) {
      const int ps = i < nlive ? tpos[i] : 0;
      const int rw = i < nlive ? trow[i] : 0;
      const long long o = (long long)(kv_slot_ok(p, ps, rw) ? ps : 0) * kHeadDim + j;
      pre.cs[i] = rope ? __ldg(p.rope_cos + o) : 1.0f;
      pre.sn[i] = rope ? __ldg(p.rope_sin + o) : 0.0f;
    }
  } else if constexpr (EPI == kTcResidual) {
    pre.wn = p.next_norm_w ? __ldg(p.next_norm_w + n) : 1.0f;
#pragma unroll
    for (int i = 0; i < CT; ++i) pre.xo[i] = __ldcg(p.x + (long long)(tbase + (i < nlive ? i : 0)) * kHidden + n);
  }
}

// Final epilogue of weight row n (this thread) for tokens tbase .. tbase+nlive-1 (the
// live prefix of a chunk of CT). `v` holds D with its hi and lo columns summed; rs, tpos
// and trow are the chunk's per-token reciprocal RMS, positions and cache rows (shared
// memory), `pre` its operands from pre_load. The 32 lanes of a warp hold 32 consecutive
// rows.
template <int EPI, int CT>
__device__ __forceinline__ void finish_rows(const TcParams& p, int n, int tbase, int nlive, const float (&v)[CT],
                                            const float* rs, const int* tpos, const int* trow,
                                            const ChunkPre<EPI, CT>& pre, int lane, int ew, float* sred,
                                            unsigned long long* abest, uint16_t* wbuf) {
  if constexpr (EPI == kTcPlain) {
#pragma unroll
    for (int i = 0; i < CT; ++i)
      if (i < nlive) p.out[(long long)(tbase + i) * p.out_ld + n] = v[i] * rs[i];
  } else if constexpr (kIsQkv<EPI>) {
    // bias, RoPE (qwen2.py:160-171, 86-99), q out / KV append (kv_cache.py:59-60)
    const int head = n >> 6, half = n & 1, d = ((n & 63) >> 1) + 32 * half;
    const bool rope = head < kHeads + kKvHeads;
    uint16_t* kvbase = head < kHeads + kKvHeads ? p.kc : p.vc;
    const int kvh = (head - kHeads) & 1;
    // the chunk's tokens as independent chains (no early exit: predicated stores)
    float x[CT], partner[CT];
#pragma unroll
    for (int i = 0; i < CT; ++i) x[i] = v[i] * rs[i] + pre.b;
#pragma unroll
    for (int i = 0; i < CT; ++i) partner[i] = __shfl_xor_sync(0xffffffffu, x[i], 1);
#pragma unroll
    for (int i = 0; i < CT; ++i) {
      if (rope) x[i] = half ? (x[i] * pre.cs[i] + partner[i] * pre.sn[i]) : (x[i] * pre.cs[i] - partner[i] * pre.sn[i]);
      if (i < nlive) {
        const int t = tbase + i;
        if (head < kHeads) {
          p.q[(long long)t * kHidden + head * kHeadDim + d] = x[i];
        } else if constexpr (EPI == kTcQkvRopePaged) {
          const long long o = kv_slot_ok(p, tpos[i], trow[i]) ? kv_offset(p.kv, p.max_len, trow[i], kvh, tpos[i]) : -1;
          if (o >= 0) kvbase[o + d] = f32_to_bf16_rn(x[i]);
          else if (d == 0 && p.err) atomicExch(p.err, QI_ERR_INDEX);
        } else if (kv_slot_ok(p, tpos[i], trow[i])) {
          kvbase[(((long long)trow[i] * kKvHeads + kvh) * p.max_len + tpos[i]) * kHeadDim + d] = f32_to_bf16_rn(x[i]);
        } else if (d == 0 && p.err) {
          atomicExch(p.err, QI_ERR_INDEX);
        }
      }
    }
  } else if constexpr (EPI == kTcSwiglu) {
    // silu(gate) * up (qwen2.py:114-116); gate row 2i, up row 2i+1
    float h[CT];
#pragma unroll
    for (int i = 0; i < CT; ++i) {
      const float x = v[i] * rs[i];
      const float up = __shfl_xor_sync(0xffffffffu, x, 1);
      h[i] = __fdividef(x, 1.0f + __expf(-x)) * up;
    }
    act_store_warp<CT, 1>(p.act_out, kInter, p.out_nt, p.lg_out_nt, (n - lane) >> 1, tbase, nlive, h, wbuf, lane);
  } else if constexpr (EPI == kTcResidual) {
    // residual add into the fp32 stream (qwen2.py:237-239), then the next projection's
    // activations hi/lo(w_next * x) and this tile's partial sums of squares of x
    // the chunk's tokens as independent chains: predicated stores, and the sums of squares
    // as interleaved butterflies (each token's in the order of warp_sum)
    float an[CT], sq[CT];
#pragma unroll
    for (int i = 0; i < CT; ++i) {
      const float xv = pre.xo[i] + v[i];
      an[i] = i < nlive ? xv * pre.wn : 0.f;
      sq[i] = xv * xv;
      if (i < nlive) p.x[(long long)(tbase + i) * kHidden + n] = xv;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < CT; ++i) sq[i] += __shfl_xor_sync(0xffffffffu, sq[i], o);
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < CT; ++i)
        if (i < nlive) sred[i] = sq[i];  // this lane quadrant's partial of token tbase + i
    }
    if (p.act_out) act_store_warp<CT, 0>(p.act_out, kHidden, p.out_nt, p.lg_out_nt, n - lane, tbase, nlive, an, wbuf, lane);
  } else {  // kTcLogits: tied head (qwen2.py:282-292) + greedy argmax (engine.py:155)
    // the chunk's tokens reduce as independent butterflies (one chain per token would
    // serialise 16 x 5 dependent shuffle pairs); a token counts only if it is a live
    // head token
    unsigned long long key[CT];
#pragma unroll
    for (int i = 0; i < CT; ++i) {
      const int t = tbase + i;
      const float x = v[i] * rs[i];
      const bool head = i < nlive && t >= p.head_lo && t < p.head_hi && (t - p.head_lo) % p.head_stride == 0;
      if (head && p.logits) {
        const long long o = (long long)((t - p.head_lo) / p.head_stride) * p.logits_ld + n;
        if (p.logits_bf16) reinterpret_cast<uint16_t*>(p.logits)[o] = f32_to_bf16_rn(x);
        else reinterpret_cast<float*>(p.logits)[o] = x;
      }
      key[i] = head ? argmax_pack(x, n) : 0ull;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < CT; ++i) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key[i], o);
        key[i] = other > key[i] ? other : key[i];
      }
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < CT; ++i)
        if (key[i]) atomicMax(&abest[(tbase + i) & (p.NT - 1)], key[i]);
    }
  }
}

// Reads the kernel parameters a projection's finish uses before the accumulator wait, so
// that their constant-cache lines are filled while the MMAs run rather than on the
// finish's first use. (Measured without effect on the decode step: the finish of a chunk
// took ~1 us with and without it. It costs a few instructions per epilogue thread.)
template <int EPI>
__device__ __forceinline__ void warm_params(const TcParams& p) {
  asm volatile("" ::"l"(p.scratch), "l"(p.counters), "r"(p.cluster), "l"(p.err), "r"(p.M), "r"(p.n_ntiles),
               "r"(p.ntile0));
  if constexpr (EPI == kTcPlain) asm volatile("" ::"l"(p.out), "r"(p.out_ld));
  if constexpr (kIsQkv<EPI>)
    asm volatile("" ::"l"(p.q), "l"(p.kc), "l"(p.vc), "r"(p.max_len), "r"(p.cache_rows));
  if constexpr (EPI == kTcResidual)
    asm volatile("" ::"l"(p.x), "l"(p.act_out), "r"(p.out_nt), "r"(p.lg_out_nt), "l"(p.ss_out), "r"(p.ss_ld));
  if constexpr (EPI == kTcSwiglu) asm volatile("" ::"l"(p.act_out), "r"(p.out_nt), "r"(p.lg_out_nt));
  if constexpr (EPI == kTcLogits)
    asm volatile("" ::"l"(p.logits), "r"(p.logits_bf16), "l"(p.logits_ld), "l"(p.argmax), "r"(p.head_lo),
                 "r"(p.head_hi), "r"(p.head_stride));
}

// Epilogue of a CTA's stream-K units [u0, u1) of one projection, run by EW epilogue warps
// (4 or 8). Warp w reads TMEM lane quadrant w % 4 (rows 32 * (w % 4) ..) and, with 8
// warps, the token chunks c = w / 4, w / 4 + 2, .. of CT columns, so two warps share each
// sub-partition and hide each other's latencies. Per segment (the CTA's part of one
// output tile): wait for the MMA warp's accumulator, then either finish the tile (whole
// segment) or publish the partial sum and, if this CTA arrives last on the tile's
// counter, add all partials in k order (deterministic) and finish it. on_tile(et) runs
// on the epilogue threads after a tile's final outputs are written. `seg` counts the
// CTA's segments (accumulator buffer b = seg & 1) and carries over between calls.
template <int EPI, int EW, class OnTile>
__device__ __forceinline__ void epilogue_range(const TcParams& p, const Geom& geo, int cta, int u0, int u1, int& seg,
                                               uint64_t* acc_full, uint64_t* acc_empty, uint32_t tmem_base, int N,
                                               int warp, int lane, const EpiSmem& es, OnTile on_tile) {
  static_assert(EW == 4 || EW == 8, "4 or 8 epilogue warps");
  constexpr int CT = EW == 8 ? 8 : 16;  // token columns per chunk
  constexpr int CSTEP = EW / 4;         // chunk stride of one warp
  const int NT = p.NT;
  const int ew = warp - kEpiWarp0;
  const int quad = warp & 3;
  const int cfirst = ew / 4;            // this warp's first chunk
  const int row = quad * 32 + lane;
  const int et = ew * 32 + lane;
  uint16_t* wbuf = es.stage + ew * (4096 / EW);
  warm_params<EPI>(p);
  int cur_nt = -1;
  for (int u = u0; u < u1; ++seg) {
    const int tile = u / p.KB, kb0 = u - tile * p.KB;
    const int len = min(p.KB - kb0, u1 - u);
    const int mt = tile / p.n_ntiles;
    const int ntile = tile % p.n_ntiles + p.ntile0;
    const int n = mt * 128 + row;
    const int tok0 = ntile * NT;
    const int live = min(NT, p.M - tok0);  // tokens of this token tile that exist
    const bool whole = (kb0 == 0 && len == p.KB);
    if (cur_nt != ntile) {
      // per-token reciprocal RMS of this token tile (RMSNorm.forward, qwen2.py:44-48) from
      // the producer's 7 partial sums of squares (1 for unnormalised inputs), and for the
      // QKV epilogue the tokens' positions and cache rows; staged while the MMAs run
      epi_bar_n<EW>();
      if (et < 128) {  // every entry is written (tokens past `live`: neutral values)
        float r = 1.0f;
        if (p.ss_in && et < live) {
          float ss = 0.f;
#pragma unroll
          for (int jj = 0; jj < kHidden / 128; ++jj) ss += __ldcg(p.ss_in + (long long)jj * p.ss_ld + tok0 + et);
          r = 1.0f / sqrtf(ss / (float)kHidden + p.eps);
        }
        es.rsm[et] = r;
        if constexpr (kIsQkv<EPI>) {
          es.tpos[et] = et < live ? __ldg(p.pos + tok0 + et) : 0;
          es.trow[et] = et < live ? __ldg(p.rows + tok0 + et) : 0;
        }
      }
      cur_nt = ntile;
      epi_bar_n<EW>();
    }
    const int b = seg & 1;
    const int nchunks = (min(NT, live) + CT - 1) / CT;
    ChunkPre<EPI, CT> pre;
    if (cfirst < nchunks)
      pre_load<EPI, CT>(p, n, tok0 + cfirst * CT, min(CT, live - cfirst * CT), es.tpos + cfirst * CT,
                        es.trow + cfirst * CT, pre);
    mbar_wait(&acc_full[b], (uint32_t)((seg >> 1) & 1), p.err);
    tc_fence_after();
    const uint32_t t_base = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * N);
    // accumulator chunk c (columns c*CT..) with its hi and lo halves summed
    auto tmem_chunk = [&](int c, float (&v)[CT]) {
      if constexpr (CT == 16) {
        float r[16];
        if (NT == 8) {
          tmem_ld16(t_base, r);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = r[i] + r[8 + i];
#pragma unroll
          for (int i = 8; i < 16; ++i) v[i] = 0.f;
        } else {
          float lo[16];
          tmem_ld16(t_base + (uint32_t)(c * CT), r);
          tmem_ld16(t_base + (uint32_t)(NT + c * CT), lo);
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = r[i] + lo[i];
        }
      } else {
        float r[8], lo[8];
        tmem_ld8(t_base + (uint32_t)(c * CT), r);
        tmem_ld8(t_base + (uint32_t)(NT + c * CT), lo);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = r[i] + lo[i];
      }
    };
    bool finish = whole;
    int c_first = cta, c_last = cta;
    const bool clustered = !whole && p.cluster > 1;
    if (clustered) {
      // One cluster per tile: ranks 1.. push their partials into rank 0's receive buffer
      // (distributed shared memory, the partial layout) and arrive on its barrier with
      // release semantics; rank 0 finishes the tile.
      const uint32_t rank = cluster_rank();
      if (rank != 0) {
        const uint32_t dst = map_rank(es.recv + (rank - 1) * 128 * NT + row * 4, 0);
        for (int c = cfirst; c < nchunks; c += CSTEP) {
          float v[CT];
          tmem_chunk(c, v);
          const int nlive = min(CT, live - c * CT);
          for (int i = 0; i < nlive; i += 4)
            st_cluster_v4(dst + (uint32_t)(((c * CT + i) >> 2) * 512 * 4), v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[b]);
        mbar_arrive_remote(map_rank(es.red_full, 0));
      }
      finish = rank == 0;
    } else if (!whole) {
      // publish this CTA's partial sum of the tile, then arrive on the tile's counter
      // (acq_rel: releases the partial stores of all epilogue threads, ordered before it by
      // the barrier, and acquires the other contributors' if this arrival is the last).
      // Partial layout per (CTA, slot): [column / 4][row][column % 4], so the 32 lanes
      // (consecutive rows) of a warp store or load 512 contiguous bytes per float4.
      const int slot = (geo.start(cta) >= tile * p.KB) ? 0 : 1;
      float* my_part = p.scratch + ((long long)cta * 2 + slot) * 128 * NT + row * 4;
      for (int c = cfirst; c < nchunks; c += CSTEP) {
        float v[CT];
        tmem_chunk(c, v);
        const int nlive = min(CT, live - c * CT);
        for (int i = 0; i < nlive; i += 4)
          *reinterpret_cast<float4*>(my_part + (long long)((c * CT + i) >> 2) * 512) =
              make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      c_first = geo.owner(tile * p.KB);
      c_last = geo.owner(tile * p.KB + p.KB - 1);
      epi_bar_n<EW>();
      if (et == 0) *es.flag = atomic_add_acq_rel(&p.counters[tile], 1u) == (unsigned)(c_last - c_first);
      epi_bar_n<EW>();
      finish = *es.flag != 0;
    }
    if (finish) {
      // The tile's final values, chunk by chunk: from TMEM (whole segment) or the sum of
      // every contributor's partial in k order (deterministic whatever the arrival order).
      // The partial loads of the warp's next chunk are issued before this chunk's stores.
      constexpr int kBatch = 4;
      float4 q[kBatch][CT / 4];
      auto issue = [&](int c, int cc0) {
        const int nlive = min(CT, live - c * CT);
#pragma unroll
        for (int a = 0; a < kBatch; ++a) {
          const int cc = cc0 + a;
          const bool on = cc <= c_last;
          const int slot = (geo.start(on ? cc : c_first) >= tile * p.KB) ? 0 : 1;
          const float* src = p.scratch + ((long long)(on ? cc : c_first) * 2 + slot) * 128 * NT + row * 4 +
                              (long long)((c * CT) >> 2) * 512;
#pragma unroll
          for (int i4 = 0; i4 < CT / 4; ++i4)
            q[a][i4] = (on && 4 * i4 < nlive) ? __ldcg(reinterpret_cast<const float4*>(src + i4 * 512))
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      };
      auto reduce = [&](float (&v)[CT]) {
#pragma unroll
        for (int a = 0; a < kBatch; ++a)
#pragma unroll
          for (int i4 = 0; i4 < CT / 4; ++i4) {
            v[4 * i4] += q[a][i4].x;
            v[4 * i4 + 1] += q[a][i4].y;
            v[4 * i4 + 2] += q[a][i4].z;
            v[4 * i4 + 3] += q[a][i4].w;
          }
      };
      if (clustered) mbar_wait_cluster(es.red_full, 0, p.err);  // every rank's partial is in
      if (!whole && !clustered && cfirst < nchunks) issue(cfirst, c_first);
#pragma unroll 1
      for (int c = cfirst; c < nchunks; c += CSTEP) {
        float v[CT];
        if (whole) {
          tmem_chunk(c, v);
        } else if (clustered) {
          // rank 0's own partial (the first k range), then ranks 1.. in order
          tmem_chunk(c, v);
          const int nlive = min(CT, live - c * CT);
          for (int r = 1; r < p.cluster; ++r) {
            const float* src = es.recv + (r - 1) * 128 * NT + row * 4 + ((c * CT) >> 2) * 512;
#pragma unroll
            for (int i4 = 0; i4 < CT / 4; ++i4)
              if (4 * i4 < nlive) {
                const float4 q4 = *reinterpret_cast<const float4*>(src + i4 * 512);
                v[4 * i4] += q4.x;
                v[4 * i4 + 1] += q4.y;
                v[4 * i4 + 2] += q4.z;
                v[4 * i4 + 3] += q4.w;
              }
          }
        } else {
#pragma unroll
          for (int i = 0; i < CT; ++i) v[i] = 0.f;
          for (int cc0 = c_first;;) {
            reduce(v);
            cc0 += kBatch;
            if (cc0 <= c_last) issue(c, cc0);
            else break;
          }
          if (c + CSTEP < nchunks) issue(c + CSTEP, c_first);
        }
        ChunkPre<EPI, CT> nxt;
        const int cn = c + CSTEP;
        if (cn < nchunks)
          pre_load<EPI, CT>(p, n, tok0 + cn * CT, min(CT, live - cn * CT), es.tpos + cn * CT, es.trow + cn * CT, nxt);
        const int nlive = min(CT, live - c * CT);
        finish_rows<EPI, CT>(p, n, tok0 + c * CT, nlive, v, es.rsm + c * CT, es.tpos + c * CT, es.trow + c * CT, pre,
                             lane, ew, es.sred + quad * 128 + c * CT, es.abest, wbuf);
        pre = nxt;
      }
      if (whole || clustered) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[b]);
      } else if (et == 0) {
        p.counters[tile] = 0u;
      }
      if constexpr (EPI == kTcResidual) {
        // the tile's partial sums of squares per token: its four lane quadrants, added as
        // ((2 + 3) + (0 + 1)), for the next projection's RMSNorm
        if (p.ss_out) {
          epi_bar_n<EW>();
          if (et < live)
            p.ss_out[(long long)mt * p.ss_ld + tok0 + et] =
                (es.sred[2 * 128 + et] + es.sred[3 * 128 + et]) + (es.sred[et] + es.sred[128 + et]);
          epi_bar_n<EW>();
        }
      }
      on_tile(et);
    }
    u += len;
  }
  if constexpr (EPI == kTcLogits) {
    // one atomic per head token per CTA (a logits range covers a single token tile)
    epi_bar_n<EW>();
    if (ew == 0) {
      for (int i = lane; i < NT; i += 32) {
        const int t = p.ntile0 * NT + i;
        const unsigned long long k = es.abest[i];
        if (k && t < p.M && t >= p.head_lo && t < p.head_hi && (t - p.head_lo) % p.head_stride == 0)
          atomicMax(&p.argmax[(t - p.head_lo) / p.head_stride], k);
      }
    }
    epi_bar_n<EW>();
  }
}

}  // namespace tc
}  // namespace qi
