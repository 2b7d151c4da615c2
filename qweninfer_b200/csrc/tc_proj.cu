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
// Work split: U = (m-tiles x token tiles x k-blocks) units. Stream-K: CTA c of G takes
// units [c*U/G, (c+1)*U/G); a run of units inside one tile is a segment. A tile covered
// by a single segment is finished straight from TMEM; a tile shared by several CTAs is
// finished by the last contributor to arrive (per-tile counter), which sums the
// contributors' fp32 partials in k order. Clusters (TcParams::cluster = C > 1): cluster q
// of C CTAs takes tile q, rank r the k blocks [r*KB/C, (r+1)*KB/C); ranks 1.. push their
// partials into rank 0's shared memory (distributed shared memory) and rank 0 finishes the
// tile, adding them in rank order. Either way the sums do not depend on timing.
//
// Warp roles (10 warps): warp 0 streams stages, one issuing lane per ring stage (weights
// may be fetched before the programmatic-launch wait, activations only after it); warp 1
// owns TMEM and one of its threads issues the UMMAs; warps 2-9 are the epilogue (TMEM lane
// quadrant = warp % 4, one weight row per thread, the two warps of a quadrant on
// alternate token chunks). Two TMEM accumulators let the epilogue of one segment overlap
// the UMMAs of the next. Every mbarrier wait is bounded (error word on timeout).
#include "common.cuh"
#include "internal.h"
#include "tc_proj.h"
#include "tc_device.cuh"

namespace qi {

namespace {

using namespace tc;

template <int EPI>
__global__ void __launch_bounds__(kProjThreads, 1) tc_proj_kernel(const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NT = p.NT;
  const int N = 2 * NT;
  const uint32_t b_bytes = (uint32_t)NT * 256;  // one 64-column block of the token tile
  // a pipeline unit is kpu consecutive 64-column k blocks: kpu weight blocks, then kpu
  // activation blocks (each run contiguous in HBM)
  const int kpu = p.kpu;
  const uint32_t a_unit = (uint32_t)kpu * kABytes, b_unit = (uint32_t)kpu * b_bytes;
  const uint32_t stage_bytes = a_unit + b_unit;
  const int S = p.stages;

  uint8_t* stage_base = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;      // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* red_full = acc_empty + 2;  // [1], cluster split tiles
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_full + 2);
  EpiSmem es = carve_epi(reinterpret_cast<uint8_t*>(tmem_slot + 4));
  es.recv = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(tmem_slot + 4) + kEpiSmemBytes);
  es.red_full = red_full;

  // stream-K: CTA c takes units [c*U/G, (c+1)*U/G); clusters of C: cluster q takes tile q,
  // its rank r the k blocks [r*KB/C, (r+1)*KB/C)
  const int C = p.cluster > 1 ? p.cluster : 1;
  const Geom geo{p.n_mtiles * p.n_ntiles * p.KB, (int)gridDim.x};
  int u0, u1;
  if (C > 1) {
    const int tile = blockIdx.x / C, r = blockIdx.x - tile * C;
    u0 = tile * p.KB + r * p.KB / C;
    u1 = tile * p.KB + (r + 1) * p.KB / C;
  } else {
    u0 = geo.start(blockIdx.x);
    u1 = geo.start(blockIdx.x + 1);
  }
  const int nunits = u1 - u0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_full[1], 1);
    mbar_init(&acc_empty[0], kProjEpiWarps);  // one arrival per epilogue warp
    mbar_init(&acc_empty[1], kProjEpiWarps);
    mbar_init(red_full, (uint32_t)((C - 1) * 32 * kProjEpiWarps));  // every epilogue thread of ranks 1..
    fence_barrier_init();
  }
  if (threadIdx.x < 128) es.abest[threadIdx.x] = 0ull;
  if (warp == 1) {
    tmem_alloc(tmem_slot, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the barrier initialisations are visible to the whole cluster before any remote arrival:
  // every thread arrives here and waits before its first remote access (epilogue) or
  // before it ends (producer, MMA)
  if (C > 1) cluster_arrive();

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane < S) {
      // Lane s owns ring stage s and streams the CTA's units i = s, s + S, ..: the bulk
      // copies issued by one thread are processed one after another (~23 GB/s per thread
      // for 16 KB copies), so one issuing lane per stage keeps S copies in flight.
      const int s = lane;
      uint8_t* st = stage_base + (size_t)s * stage_bytes;
      auto src_a = [&](int u) {
        const int tile = u / p.KB, ku = u - tile * p.KB;
        return p.w + ((long long)(tile / p.n_ntiles) * p.KB + ku) * (a_unit / 2);
      };
      auto src_b = [&](int u) {
        const int tile = u / p.KB, ku = u - tile * p.KB;
        const int nt = tile % p.n_ntiles + p.ntile0;
        return p.act_in + ((long long)nt * p.KB + ku) * (b_unit / 2);
      };
      if (s < nunits) {  // weights only: they do not depend on earlier kernels
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        bulk_g2s(st, src_a(u0 + s), a_unit, &full[s]);
      }
      grid_dep_wait();
      if (s < nunits) bulk_g2s(st + a_unit, src_b(u0 + s), b_unit, &full[s]);
      for (int i = s + S; i < nunits; i += S) {
        mbar_wait(&empty[s], (uint32_t)(((i / S) & 1) ^ 1), p.err);
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        bulk_g2s(st, src_a(u0 + i), a_unit, &full[s]);
        bulk_g2s(st + a_unit, src_b(u0 + i), b_unit, &full[s]);
      }
    } else {
      if (lane == 31 && p.pf_bytes > 0) {
        // this CTA's contiguous share of a later projection's weights, in 16 KB blocks;
        // independent of earlier kernels, so issued before the programmatic-launch wait
        const long long nblk = p.pf_bytes / kABytes, per = (nblk + gridDim.x - 1) / gridDim.x;
        const long long b1 = min(nblk, (blockIdx.x + 1) * per);
        for (long long b = blockIdx.x * per; b < b1; ++b) bulk_prefetch_l2(p.pf + b * (kABytes / 2), kABytes);
      }
      grid_dep_wait();
    }
    grid_dep_launch();
    __syncwarp();
    if (C > 1) cluster_wait();
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
          // descriptor of a K-major operand at a_addr + off: its address field is (addr >> 4)
          const uint64_t ad = kmajor_desc(a_addr), bd = kmajor_desc(a_addr + a_unit);
          const uint64_t bd1 = bd + (b_bytes >> 4);  // the unit's second activation block
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(d_taddr, ad + (uint64_t)(kk * 16), bd + (uint64_t)(kk * 16), idesc, (j > 0 || kk > 0) ? 1u : 0u);
          if (kpu == 2) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16(d_taddr, ad + (uint64_t)((kABytes >> 4) + kk * 16), bd1 + (uint64_t)(kk * 16), idesc, 1u);
          }
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[b]);
        u += len;
      }
    }
    __syncwarp();
    if (C > 1) cluster_wait();
  } else {
    // ---------------------------------------------------------------- epilogue
    grid_dep_wait();
    grid_dep_launch();
    if (C > 1) cluster_wait();
    int seg = 0;
    epilogue_range<EPI, kProjEpiWarps>(p, geo, blockIdx.x, u0, u1, seg, acc_full, acc_empty, tmem_base, N, warp, lane, es,
                        [](int) {});
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

size_t tc_proj_smem(int NT, int stages, int cluster, int kpu) {
  const size_t stage_bytes = (size_t)kpu * (kABytes + (size_t)NT * 256);
  const size_t recv = cluster > 1 ? (size_t)(cluster - 1) * 128 * NT * 4 : 0;
  return (size_t)stages * stage_bytes + (size_t)stages * 16 + 48 + 16 + kEpiSmemBytes + recv;
}

cudaError_t launch_tc_proj(const TcParams& p, int ctas, cudaStream_t stream, bool pdl) {
  void (*kern)(TcParams) = nullptr;
  switch (p.epi) {
    case kTcPlain: kern = tc_proj_kernel<kTcPlain>; break;
    case kTcQkvRope: kern = tc_proj_kernel<kTcQkvRope>; break;
    case kTcQkvRopePaged: kern = tc_proj_kernel<kTcQkvRopePaged>; break;
    case kTcResidual: kern = tc_proj_kernel<kTcResidual>; break;
    case kTcSwiglu: kern = tc_proj_kernel<kTcSwiglu>; break;
    case kTcLogits: kern = tc_proj_kernel<kTcLogits>; break;
    default: return cudaErrorInvalidValue;
  }
  cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(kern), 227 * 1024);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, 1, 1);
  cfg.blockDim = dim3(kProjThreads, 1, 1);
  cfg.dynamicSmemBytes = tc_proj_smem(p.NT, p.stages, p.cluster, p.kpu);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n++].val.programmaticStreamSerializationAllowed = 1;
  }
  if (p.cluster > 1) {
    if (ctas % p.cluster != 0 || p.cluster > 8) return cudaErrorInvalidValue;
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)p.cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n++].val.clusterDim.z = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

int tc_proj_max_clusters(int epi, int NT, int stages, int cluster, int kpu) {
  void (*kern)(TcParams) = epi == kTcQkvRope    ? tc_proj_kernel<kTcQkvRope>
                           : epi == kTcQkvRopePaged ? tc_proj_kernel<kTcQkvRopePaged>
                           : epi == kTcResidual ? tc_proj_kernel<kTcResidual>
                           : epi == kTcSwiglu   ? tc_proj_kernel<kTcSwiglu>
                           : epi == kTcLogits   ? tc_proj_kernel<kTcLogits>
                                                : tc_proj_kernel<kTcPlain>;
  if (set_max_dynamic_smem(reinterpret_cast<const void*>(kern), 227 * 1024) != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster, 1, 1);
  cfg.blockDim = dim3(kProjThreads, 1, 1);
  cfg.dynamicSmemBytes = tc_proj_smem(NT, stages, cluster, kpu);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
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
