// Tensor-core projections of the model forward: tcgen05 UMMA with TMEM accumulators,
// fed by bulk copies (TMA), stream-K over (tile, 64-column block) units.
//
// D[n, t] = sum_k W[n, k] * X[t, k] for one weight matrix W (bf16, tiled layout) and
// the step's activations X, carried as two bf16 halves hi = bf16(x), lo = bf16(x - hi).
// One UMMA of shape M = 128 weight rows x N = 2*NT (hi tokens, then lo tokens) x K = 16
// multiplies both halves; the epilogue adds the two column halves, which restores ~16
// mantissa bits of the fp32 activations with fp32 accumulation.
//
// Shared-memory operands use the SWIZZLE_NONE K-major canonical layout (8x8 core
// matrices of 128 contiguous bytes; LBO = 128 B along K, SBO = 1024 B between 8-row
// groups). Weights sit in HBM already in that layout (128x64 blocks of 16 KB), and the
// producing kernel writes activations the same way (tc_proj.h), so a pipeline stage is
// two contiguous cp.async.bulk copies.
//
// Work split: U = (m-tiles x token tiles x k-blocks) units; CTA c of G takes units
// [c*U/G, (c+1)*U/G). A run of units inside one tile is a segment. A tile covered by a
// single segment is finished straight from TMEM; a tile shared by several CTAs is
// finished by the last contributor to arrive (per-tile counter), which sums the
// contributors' fp32 partials in k order — results do not depend on timing or on how
// many tokens are in the batch.
//
// Warp roles (6 warps): warp 0 streams stages (weights may be fetched before the
// programmatic-launch wait, activations only after it); warp 1 owns TMEM and one of its
// threads issues the UMMAs; warps 2-5 are the epilogue (TMEM lane quadrant = warp % 4,
// one weight row per thread). Two TMEM accumulators let the epilogue of one segment
// overlap the UMMAs of the next. Every mbarrier wait is bounded (error word on timeout).
#include "common.cuh"
#include "internal.h"
#include "tc_proj.h"

namespace qi {

namespace {

constexpr int kThreads = 192;
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
// named barrier of the four epilogue warps
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// SWIZZLE_NONE K-major shared-memory descriptor: LBO 128 B, SBO 1024 B, version bit (sm_100).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
         (1ull << 46);
}

// Instruction descriptor of kind::f16: bf16 A and B, both K-major, fp32 D, shape M x N.
__device__ __forceinline__ uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------- stream-K geometry

struct Geom {
  int U, G;
  __device__ int start(int c) const { return (int)(((long long)c * U) / G); }
  // CTA whose range holds unit u: the largest c with start(c) <= u
  __device__ int owner(int u) const { return (int)(((long long)(u + 1) * G - 1) / U); }
};

// ------------------------------------------------------------------ epilogues

// Address of (token t, column k) in activation tiles, split into a per-thread part (the
// column this thread writes) and a per-token part; NT is a power of two.
struct ActAddr {
  long long col;         // k-dependent offset (hi half)
  long long half;        // offset of the lo half
  long long ntile;       // elements per token tile
  int lg;
  __device__ __forceinline__ long long tok(int t) const {
    const int tl = t & ((1 << lg) - 1);
    return (long long)(t >> lg) * ntile + (tl >> 3) * 512 + (tl & 7) * 8;
  }
};

__device__ __forceinline__ ActAddr act_addr(int k, int K, int NT, int lg) {
  ActAddr a;
  a.col = (long long)(k >> 6) * (2LL * NT * 64) + ((k & 63) >> 3) * 64 + (k & 7);
  a.half = (long long)NT * 64;
  a.ntile = (long long)(K / 64) * 2LL * NT * 64;
  a.lg = lg;
  return a;
}

__device__ __forceinline__ void act_store(uint16_t* act, const ActAddr& a, int t, float v) {
  const uint16_t hi = f32_to_bf16_rn(v);
  const long long o = a.tok(t) + a.col;
  act[o] = hi;
  act[o + a.half] = f32_to_bf16_rn(v - bf16_to_f32(hi));
}

// Final epilogue of weight row n (this thread) for tokens tbase .. tbase+nlive-1 (the
// live prefix of a chunk of CT). `v` holds D with its hi and lo columns summed, `rs` the
// chunk's per-token reciprocal RMS. The 32 lanes of a warp hold 32 consecutive rows.
template <int EPI, int CT>
__device__ __forceinline__ void finish_rows(const TcParams& p, int n, int tbase, int nlive, const float (&v)[CT],
                                            const float* rs, int lane, int ew, float* sred,
                                            unsigned long long* abest) {
  if constexpr (EPI == kTcPlain) {
#pragma unroll
    for (int i = 0; i < CT; ++i)
      if (i < nlive) p.out[(long long)(tbase + i) * p.out_ld + n] = v[i] * rs[i];
  } else if constexpr (EPI == kTcQkvRope) {
    // bias, RoPE (qwen2.py:160-171, 86-99), q out / KV append (kv_cache.py:59-60)
    const int head = n >> 6, j = (n & 63) >> 1, half = n & 1, d = j + 32 * half;
    const float b = p.bias[n];
    const bool rope = head < kHeads + kKvHeads;
    uint16_t* kvbase = head < kHeads + kKvHeads ? p.kc : p.vc;
    const int kvh = (head - kHeads) & 1;
#pragma unroll
    for (int i = 0; i < CT; ++i) {
      if (i >= nlive) break;
      const int t = tbase + i;
      float x = v[i] * rs[i] + b;
      const float partner = __shfl_xor_sync(0xffffffffu, x, 1);
      const int ps = p.pos[t];
      if (rope) {
        const float cs = p.rope_cos[(long long)ps * kHeadDim + j];
        const float sn = p.rope_sin[(long long)ps * kHeadDim + j];
        x = half ? (x * cs + partner * sn) : (x * cs - partner * sn);
      }
      if (head < kHeads) p.q[(long long)t * kHidden + head * kHeadDim + d] = x;
      else kvbase[(((long long)p.rows[t] * kKvHeads + kvh) * p.max_len + ps) * kHeadDim + d] = f32_to_bf16_rn(x);
    }
  } else if constexpr (EPI == kTcSwiglu) {
    // silu(gate) * up (qwen2.py:114-116); gate row 2i, up row 2i+1
    const ActAddr a = act_addr(n >> 1, kInter, p.NT, p.lg_nt);
#pragma unroll
    for (int i = 0; i < CT; ++i) {
      if (i >= nlive) break;
      const float x = v[i] * rs[i];
      const float up = __shfl_xor_sync(0xffffffffu, x, 1);
      if (!(n & 1)) act_store(p.act_out, a, tbase + i, x / (1.0f + expf(-x)) * up);
    }
  } else if constexpr (EPI == kTcResidual) {
    // residual add into the fp32 stream (qwen2.py:237-239), then the next projection's
    // activations hi/lo(w_next * x) and this tile's partial sums of squares of x
    const float wn = p.next_norm_w ? p.next_norm_w[n] : 1.0f;
    const ActAddr a = act_addr(n, kHidden, p.NT, p.lg_nt);
#pragma unroll
    for (int i = 0; i < CT; ++i) {
      if (i >= nlive) break;
      const int t = tbase + i;
      float* xp = p.x + (long long)t * kHidden + n;
      const float xv = *xp + v[i];
      *xp = xv;
      if (p.act_out) act_store(p.act_out, a, t, xv * wn);
      const float s = warp_sum(xv * xv);
      if (lane == 0) sred[ew * 16 + i] = s;
    }
    if (p.ss_out) {
      epi_bar();
      if (ew == 0 && lane < nlive)
        p.ss_out[(long long)(n >> 7) * p.ss_ld + tbase + lane] =
            (sred[lane] + sred[16 + lane]) + (sred[32 + lane] + sred[48 + lane]);
      epi_bar();
    }
  } else {  // kTcLogits: tied head (qwen2.py:282-292) + greedy argmax (engine.py:155)
#pragma unroll
    for (int i = 0; i < CT; ++i) {
      if (i >= nlive) break;
      const int t = tbase + i;
      if (t < p.head_lo || t >= p.head_hi || (t - p.head_lo) % p.head_stride) continue;
      const float x = v[i] * rs[i];
      if (p.logits) {
        const long long o = (long long)((t - p.head_lo) / p.head_stride) * p.logits_ld + n;
        if (p.logits_bf16) reinterpret_cast<uint16_t*>(p.logits)[o] = f32_to_bf16_rn(x);
        else reinterpret_cast<float*>(p.logits)[o] = x;
      }
      unsigned long long key = argmax_pack(x, n);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
      }
      if (lane == 0) atomicMax(&abest[t & (p.NT - 1)], key);
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1) tc_proj_kernel(const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NT = p.NT;
  const int N = 2 * NT;
  const uint32_t b_bytes = (uint32_t)NT * 256;
  const uint32_t stage_bytes = kABytes + b_bytes;
  const int S = p.stages;

  uint8_t* stage_base = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;      // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* rs_tile = reinterpret_cast<int*>(tmem_slot + 2);
  float* sred = reinterpret_cast<float*>(tmem_slot + 4);                         // 4 x 16
  unsigned long long* abest = reinterpret_cast<unsigned long long*>(sred + 64);  // 128
  float* rsm = reinterpret_cast<float*>(abest + 128);                            // 128

  const Geom geo{p.n_mtiles * p.n_ntiles * p.KB, (int)gridDim.x};
  const int u0 = geo.start(blockIdx.x), u1 = geo.start(blockIdx.x + 1);
  const int nunits = u1 - u0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_full[1], 1);
    mbar_init(&acc_empty[0], 4);
    mbar_init(&acc_empty[1], 4);
    fence_barrier_init();
    *rs_tile = -1;
  }
  if (threadIdx.x < 128) abest[threadIdx.x] = 0ull;
  if (warp == 1) {
    tmem_alloc(tmem_slot, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      auto src_a = [&](int u) {
        const int tile = u / p.KB, kb = u - tile * p.KB;
        return p.w + ((long long)(tile / p.n_ntiles) * p.KB + kb) * (kABytes / 2);
      };
      auto src_b = [&](int u) {
        const int tile = u / p.KB, kb = u - tile * p.KB;
        const int nt = tile % p.n_ntiles + p.ntile0;
        return p.act_in + ((long long)nt * p.KB + kb) * (b_bytes / 2);
      };
      const int pre = nunits < S ? nunits : S;
      for (int i = 0; i < pre; ++i) {  // weights only: they do not depend on earlier kernels
        mbar_arrive_expect_tx(&full[i], stage_bytes);
        bulk_g2s(stage_base + (size_t)i * stage_bytes, src_a(u0 + i), kABytes, &full[i]);
      }
      grid_dep_wait();
      for (int i = 0; i < pre; ++i)
        bulk_g2s(stage_base + (size_t)i * stage_bytes + kABytes, src_b(u0 + i), b_bytes, &full[i]);
      for (int i = pre; i < nunits; ++i) {
        const int s = i % S;
        mbar_wait(&empty[s], (uint32_t)(((i / S) & 1) ^ 1), p.err);
        uint8_t* st = stage_base + (size_t)s * stage_bytes;
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        bulk_g2s(st, src_a(u0 + i), kABytes, &full[s]);
        bulk_g2s(st + kABytes, src_b(u0 + i), b_bytes, &full[s]);
      }
    } else {
      grid_dep_wait();
    }
    grid_dep_launch();
    __syncwarp();
  } else if (warp == 1) {
    // --------------------------------------------------------------------- MMA
    grid_dep_wait();
    grid_dep_launch();
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(128, N);
      int i = 0, seg = 0;
      for (int u = u0; u < u1; ++seg) {
        const int kb0 = u % p.KB;
        const int len = min(p.KB - kb0, u1 - u);
        const int b = seg & 1;
        mbar_wait(&acc_empty[b], (uint32_t)(((seg >> 1) & 1) ^ 1), p.err);
        tc_fence_after();
        const uint32_t d_taddr = tmem_base + (uint32_t)(b * N);
        for (int j = 0; j < len; ++j, ++i) {
          const int s = i % S;
          mbar_wait(&full[s], (uint32_t)((i / S) & 1), p.err);
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stage_base + (size_t)s * stage_bytes);
          const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(d_taddr, kmajor_desc(a_addr + kk * 256), kmajor_desc(b_addr + kk * 256), idesc,
                      (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[b]);
        u += len;
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue
    grid_dep_wait();
    grid_dep_launch();
    const int ew = warp - kEpiWarp0;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int et = ew * 32 + lane;  // 0..127 across the epilogue warps
    constexpr int CT = 16;
    int seg = 0;
    for (int u = u0; u < u1; ++seg) {
      const int tile = u / p.KB, kb0 = u - tile * p.KB;
      const int len = min(p.KB - kb0, u1 - u);
      const int mt = tile / p.n_ntiles;
      const int ntile = tile % p.n_ntiles + p.ntile0;
      const int n = mt * 128 + row;
      const int tok0 = ntile * NT;
      const int live = min(NT, p.M - tok0);  // tokens of this token tile that exist
      const bool whole = (kb0 == 0 && len == p.KB);
      if (*rs_tile != ntile) {
        // per-token reciprocal RMS of this token tile (RMSNorm.forward, qwen2.py:44-48),
        // from the producer's 7 partial sums of squares; 1 for unnormalised inputs
        epi_bar();
        if (et < NT) {
          float r = 1.0f;
          if (p.ss_in && et < live) {
            float ss = 0.f;
#pragma unroll
            for (int jj = 0; jj < kHidden / 128; ++jj) ss += p.ss_in[(long long)jj * p.ss_ld + tok0 + et];
            r = 1.0f / sqrtf(ss / (float)kHidden + p.eps);
          }
          rsm[et] = r;
        }
        if (et == 0) *rs_tile = ntile;
        epi_bar();
      }
      const int b = seg & 1;
      mbar_wait(&acc_full[b], (uint32_t)((seg >> 1) & 1), p.err);
      tc_fence_after();
      const uint32_t t_base = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * N);
      float* my_part = nullptr;
      if (!whole) {
        const int slot = (geo.start(blockIdx.x) >= tile * p.KB) ? 0 : 1;
        my_part = p.scratch + (((long long)blockIdx.x * 2 + slot) * 128 + row) * NT;
      }
      for (int c = 0; c < NT && c < live; c += CT) {
        float r[16], v[16];
        if (NT == 8) {
          tmem_ld16(t_base, r);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = r[i] + r[8 + i];
        } else {
          float lo[16];
          tmem_ld16(t_base + (uint32_t)c, r);
          tmem_ld16(t_base + (uint32_t)(NT + c), lo);
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = r[i] + lo[i];
        }
        const int nlive = min(min(CT, NT - c), live - c);
        if (whole) {
          finish_rows<EPI, CT>(p, n, tok0 + c, nlive, v, rsm + c, lane, ew, sred, abest);
        } else {
          for (int i = 0; i < nlive; i += 4)
            *reinterpret_cast<float4*>(my_part + c + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      if (!whole) {
        // arrive on the tile's counter; the last contributor sums the partials in k order
        __threadfence();
        epi_bar();
        const int c_first = geo.owner(tile * p.KB);
        const int c_last = geo.owner(tile * p.KB + p.KB - 1);
        if (et == 0) {
          const unsigned prev = atomicAdd(&p.counters[tile], 1u);
          *flag = (prev == (unsigned)(c_last - c_first));
        }
        epi_bar();
        if (*flag) {
          __threadfence();
          for (int c = 0; c < NT && c < live; c += CT) {
            const int nlive = min(min(CT, NT - c), live - c);
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
            // contributors are summed in k order; loads are issued 4 contributors ahead
            auto src_of = [&](int cc) {
              const int slot = (geo.start(cc) >= tile * p.KB) ? 0 : 1;
              return p.scratch + (((long long)cc * 2 + slot) * 128 + row) * NT + c;
            };
            int cc = c_first;
            for (; cc + 3 <= c_last; cc += 4) {
              float4 q[4][4];
#pragma unroll
              for (int a = 0; a < 4; ++a) {
                const float* src = src_of(cc + a);
#pragma unroll
                for (int i4 = 0; i4 < 4; ++i4)
                  q[a][i4] = (4 * i4 < nlive) ? __ldcg(reinterpret_cast<const float4*>(src + 4 * i4))
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int i4 = 0; i4 < 4; ++i4) {
                  v[4 * i4] += q[a][i4].x;
                  v[4 * i4 + 1] += q[a][i4].y;
                  v[4 * i4 + 2] += q[a][i4].z;
                  v[4 * i4 + 3] += q[a][i4].w;
                }
            }
            for (; cc <= c_last; ++cc) {
              const float* src = src_of(cc);
#pragma unroll
              for (int i = 0; i < 16; i += 4) {
                if (i < nlive) {
                  const float4 q4 = __ldcg(reinterpret_cast<const float4*>(src + i));
                  v[i] += q4.x;
                  v[i + 1] += q4.y;
                  v[i + 2] += q4.z;
                  v[i + 3] += q4.w;
                }
              }
            }
            finish_rows<EPI, CT>(p, n, tok0 + c, nlive, v, rsm + c, lane, ew, sred, abest);
          }
          if (et == 0) p.counters[tile] = 0u;
        }
        epi_bar();
      }
      u += len;
    }
    if constexpr (EPI == kTcLogits) {
      // one atomic per head token per CTA (a logits launch covers a single token tile)
      epi_bar();
      if (ew == 0) {
        for (int i = lane; i < NT; i += 32) {
          const int t = p.ntile0 * NT + i;
          const unsigned long long k = abest[i];
          if (k && t < p.M && t >= p.head_lo && t < p.head_hi && (t - p.head_lo) % p.head_stride == 0)
            atomicMax(&p.argmax[(t - p.head_lo) / p.head_stride], k);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

// x (M, K) fp32 -> activation tiles of norm_w * x; ss[0][t] = sum x^2 (ss[1..6][t] = 0).
// One warp per (token, 64-column block); lane = (8-column chunk, 4 of the 8 elements).
__global__ void __launch_bounds__(256) act_tiles_kernel(const float* __restrict__ x, const float* __restrict__ norm_w,
                                                         int M, int K, int NT, uint16_t* __restrict__ act,
                                                         float* __restrict__ ss, int ss_ld) {
  grid_dep_wait();
  grid_dep_launch();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int KB = K / 64;
  const int Mp = ((M + NT - 1) / NT) * NT;
  if (warp >= Mp * KB) return;
  const int t = warp / KB, kb = warp - t * KB;
  for (int e = lane; e < 64; e += 32) {
    const int k = kb * 64 + e;
    float v = t < M ? x[(long long)t * K + k] : 0.f;
    if (norm_w) v *= norm_w[k];
    const uint16_t hi = f32_to_bf16_rn(v);
    const uint16_t lo = f32_to_bf16_rn(v - bf16_to_f32(hi));
    act[act_offset(t, k, 0, K, NT)] = hi;
    act[act_offset(t, k, 1, K, NT)] = lo;
  }
  if (ss && kb == 0 && t < M) {
    float s = 0.f;
    for (int k = lane; k < K; k += 32) {
      const float a = x[(long long)t * K + k];
      s = fmaf(a, a, s);
    }
    s = warp_sum(s);
    if (lane < kHidden / 128) ss[(long long)lane * ss_ld + t] = lane == 0 ? s : 0.f;
  }
}

}  // namespace

size_t tc_proj_smem(int NT, int stages) {
  const size_t stage_bytes = kABytes + (size_t)NT * 256;
  return (size_t)stages * stage_bytes + (size_t)stages * 16 + 32 + 16 + 64 * 4 + 128 * 8 + 128 * 4;
}

cudaError_t launch_tc_proj(const TcParams& p, int ctas, cudaStream_t stream, bool pdl) {
  void (*kern)(TcParams) = nullptr;
  switch (p.epi) {
    case kTcPlain: kern = tc_proj_kernel<kTcPlain>; break;
    case kTcQkvRope: kern = tc_proj_kernel<kTcQkvRope>; break;
    case kTcResidual: kern = tc_proj_kernel<kTcResidual>; break;
    case kTcSwiglu: kern = tc_proj_kernel<kTcSwiglu>; break;
    case kTcLogits: kern = tc_proj_kernel<kTcLogits>; break;
    default: return cudaErrorInvalidValue;
  }
  static bool configured[5] = {false, false, false, false, false};
  if (!configured[p.epi]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    configured[p.epi] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = tc_proj_smem(p.NT, p.stages);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

cudaError_t launch_act_tiles(const float* x, const float* norm_w, int M, int K, int NT, uint16_t* act, float* ss,
                             int ss_ld, cudaStream_t stream, bool pdl) {
  const int Mp = ((M + NT - 1) / NT) * NT;
  const long long warps = (long long)Mp * (K / 64);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((warps * 32 + 255) / 256), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, act_tiles_kernel, x, norm_w, M, K, NT, act, ss, ss_ld);
}

}  // namespace qi
