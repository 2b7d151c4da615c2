// The whole Qwen2 forward of a decode step in ONE cooperative launch (qweninfer/models/
// qwen2.py:263-292 for B tokens at S = 1, or a short prefill).
//
// Why: a decode step is ~120 dependent operations on 0.99 GB of weights. Launched one by
// one, each pays launch, ramp-up, first-byte DRAM latency and drain (~10 us each at
// batch 1), far more than its share of the ~150 us weight stream. Here 148 resident CTAs
// (one per SM) walk a host-built stage table — embed, 24 x {QKV, attention, o, gate/up,
// down}, head — and:
//  * a weight-stream thread per CTA issues the CTA's 16 KB weight blocks for every stage
//    in order, as fast as ring slots free up; weights never depend on activations, so
//    the HBM stream runs ahead across stage boundaries and is never drained;
//  * an activation thread issues each unit's activation tile (the UMMA B operand) only
//    after the previous stage has counted all its completions (acquire on a global
//    counter, bounded wait);
//  * one thread issues tcgen05 UMMAs into double-buffered TMEM accumulators;
//  * four epilogue warps finish tiles (the same fused epilogues as tc_proj: bias/RoPE/KV
//    append, residual + next RMSNorm operands, SwiGLU, logits + argmax), run the
//    attention units of attention stages and the embedding of the first stage, and
//    signal completions.
// Work partition and numerics are exactly those of the per-stage kernels (tc_proj_kernel,
// attention_kernel), so results are identical to the multi-launch path.
//
// Every wait is bounded: on a timeout the kernel records QI_ERR_TIMEOUT and every later
// wait in every CTA returns at once, so a fault ends the launch within ~2 s.
#include "common.cuh"
#include "internal.h"
#include "tc_proj.h"
#include "tc_device.cuh"
#include "attention_device.cuh"
#include "persistent.h"

namespace qi {

namespace {

using namespace tc;
using namespace attn;

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Wait until *ctr >= target (acquire). Bounded; returns at once if another wait failed.
// One thread per CTA and role polls, with a pause between polls: thousands of threads
// spinning on one counter saturate its L2 slice and slow every access that maps there.
__device__ __noinline__ bool wait_count(const unsigned* ctr, unsigned target, int* err) {
  if (ld_acquire(ctr) >= target) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    __nanosleep(100);
    if (ld_acquire(ctr) >= target) return true;
    if (*reinterpret_cast<volatile int*>(err)) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      atomicExch(err, QI_ERR_TIMEOUT);
      return false;
    }
  }
}

// Shared memory: ring slots, their barriers, accumulator barriers, TMEM slot, epilogue
// scratch, embedding reduction, then (128-byte aligned) the attention tiles.
__host__ __device__ inline size_t persistent_attn_offset(int ring, size_t stage_bytes) {
  return ((size_t)ring * stage_bytes + (size_t)ring * 16 + 32 + 16 + kEpiSmemBytes + 16 + 127) & ~(size_t)127;
}

// The 128 epilogue threads wait for a counter: thread 0 polls, then releases the others.
__device__ __forceinline__ void epi_wait(const unsigned* ctr, unsigned target, int* err, int et) {
  if (et == 0) {
    wait_count(ctr, target, err);
    __threadfence();
  }
  epi_bar();
}

// The completion that reaches the stage's target also stamps the stage's finish time
// into the optional trace.
struct Done {
  unsigned* ctr;
  unsigned target;
  unsigned long long* stamp;  // null when not tracing
};

// Signal one completion of a stage. Release pattern: the barrier orders the 128
// threads' writes before thread 0's fence and counter increment.
__device__ __forceinline__ void signal_done(const Done& d, int et) {
  fence_proxy_async_global();  // consumers read these writes with bulk copies
  epi_bar();
  if (et == 0) {
    const unsigned prev = atomic_add_acq_rel(d.ctr, 1u);
    if (d.stamp && prev + 1 == d.target) *d.stamp = global_timer_ns();
  }
}

// Embedding of token t by the 128 epilogue threads (embed_kernel, misc.cu): fp32 stream,
// activation tiles of norm_w * x for the first projection, sum of squares in ss[0][t].
__device__ void embed_token(const PEmbed& e, int t, int NT, int ss_ld, int et, float* red4) {
  const int lane = et & 31, ew = et >> 5;
  int id = e.ids[t];
  if (id < 0 || id >= e.vocab) id = 0;
  float sq = 0.f;
  if (et < kHidden / 8) {
    const int k = et * 8;
    const uint4 w = *reinterpret_cast<const uint4*>(e.table + tiled_offset(id, k, kHidden));
    const float v[8] = {bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y),
                        bf16lo(w.z), bf16hi(w.z), bf16lo(w.w), bf16hi(w.w)};
    float4* o = reinterpret_cast<float4*>(e.x + (long long)t * kHidden + k);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      sq = fmaf(v[i], v[i], sq);
      sq = fmaf(v[i + 1], v[i + 1], sq);
      const float a = v[i] * e.norm_w[k + i], b = v[i + 1] * e.norm_w[k + i + 1];
      const uint16_t ha = f32_to_bf16_rn(a), hb = f32_to_bf16_rn(b);
      hw[i / 2] = (uint32_t)ha | ((uint32_t)hb << 16);
      lw[i / 2] = (uint32_t)f32_to_bf16_rn(a - bf16_to_f32(ha)) | ((uint32_t)f32_to_bf16_rn(b - bf16_to_f32(hb)) << 16);
    }
    *reinterpret_cast<uint4*>(e.act + act_offset(t, k, 0, kHidden, NT)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(e.act + act_offset(t, k, 1, kHidden, NT)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
  if (et == 0 && e.slots && t < e.n_slots) e.slots[t] = 0ull;
  sq = warp_sum(sq);
  if (lane == 0) red4[ew] = sq;
  epi_bar();
  if (et < kHidden / 128) e.ss[(long long)et * ss_ld + t] = et == 0 ? (red4[0] + red4[1]) + (red4[2] + red4[3]) : 0.f;
  epi_bar();
}

__global__ void __launch_bounds__(kThreads, 1) persistent_forward_kernel(const PParams P) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NT = P.NT;
  const int N = 2 * NT;
  const uint32_t b_bytes = (uint32_t)NT * 256;
  const uint32_t stage_bytes = kABytes + b_bytes;
  const int S = P.ring;
  const int G = gridDim.x;
  const int c = blockIdx.x;

  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;      // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  const EpiSmem es = carve_epi(reinterpret_cast<uint8_t*>(tmem_slot + 4));
  float* red4 = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(tmem_slot + 4) + kEpiSmemBytes);  // 4
  AttnSmem& AS = *reinterpret_cast<AttnSmem*>(smem + persistent_attn_offset(S, stage_bytes));

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 2);   // weight and activation copies arrive separately
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_full[1], 1);
    mbar_init(&acc_empty[0], 4);
    mbar_init(&acc_empty[1], 4);
    mbar_init(&AS.bar[0], 1);
    mbar_init(&AS.bar[1], 1);
    fence_barrier_init();
  }
  if (threadIdx.x < 128) es.abest[threadIdx.x] = 0ull;
  if (warp == 1) {
    tmem_alloc(tmem_slot, P.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------- weight stream
      int i = 0;
      for (int s = 0; s < P.n_stages; ++s) {
        const PStage& st = P.stages[s];
        if (st.kind != kPGemm) continue;
        const TcParams& p = st.tc;
        const Geom geo{p.n_mtiles * p.n_ntiles * p.KB, st.ctas};
        const int u0 = c < st.ctas ? geo.start(c) : 0, u1 = c < st.ctas ? geo.start(c + 1) : 0;
        for (int u = u0; u < u1; ++u, ++i) {
          const int slot = i % S;
          if (i >= S) mbar_wait(&empty[slot], (uint32_t)(((i / S) & 1) ^ 1), P.err);
          const int tile = u / p.KB, kb = u - tile * p.KB;
          mbar_arrive_expect_tx(&full[slot], kABytes);
          bulk_g2s(ring + (size_t)slot * stage_bytes, p.w + ((long long)(tile / p.n_ntiles) * p.KB + kb) * (kABytes / 2),
                   kABytes, &full[slot]);
        }
      }
    } else if (lane == 1) {
      // ---------------------------------------------------- activation stream
      int i = 0;
      for (int s = 0; s < P.n_stages; ++s) {
        const PStage& st = P.stages[s];
        if (st.kind != kPGemm) continue;
        const TcParams& p = st.tc;
        const Geom geo{p.n_mtiles * p.n_ntiles * p.KB, st.ctas};
        const int u0 = c < st.ctas ? geo.start(c) : 0, u1 = c < st.ctas ? geo.start(c + 1) : 0;
        if (u0 < u1) {
          wait_count(&P.done[st.dep * kDoneStride], (unsigned)P.stages[st.dep].target, P.err);
          fence_proxy_async_global();
        }
        for (int u = u0; u < u1; ++u, ++i) {
          const int slot = i % S;
          if (i >= S) mbar_wait(&empty[slot], (uint32_t)(((i / S) & 1) ^ 1), P.err);
          const int tile = u / p.KB, kb = u - tile * p.KB;
          const int nt = tile % p.n_ntiles + p.ntile0;
          mbar_arrive_expect_tx(&full[slot], b_bytes);
          bulk_g2s(ring + (size_t)slot * stage_bytes + kABytes, p.act_in + ((long long)nt * p.KB + kb) * (b_bytes / 2),
                   b_bytes, &full[slot]);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(128, N);
      int i = 0, seg = 0;
      for (int s = 0; s < P.n_stages; ++s) {
        const PStage& st = P.stages[s];
        if (st.kind != kPGemm) continue;
        const TcParams& p = st.tc;
        const Geom geo{p.n_mtiles * p.n_ntiles * p.KB, st.ctas};
        const int u0 = c < st.ctas ? geo.start(c) : 0, u1 = c < st.ctas ? geo.start(c + 1) : 0;
        for (int u = u0; u < u1; ++seg) {
          const int kb0 = u % p.KB;
          const int len = min(p.KB - kb0, u1 - u);
          const int b = seg & 1;
          mbar_wait(&acc_empty[b], (uint32_t)(((seg >> 1) & 1) ^ 1), P.err);
          tc_fence_after();
          const uint32_t d_taddr = tmem_base + (uint32_t)(b * N);
          for (int j = 0; j < len; ++j, ++i) {
            const int slot = i % S;
            mbar_wait(&full[slot], (uint32_t)((i / S) & 1), P.err);
            tc_fence_after();
            const uint32_t a_addr = smem_u32(ring + (size_t)slot * stage_bytes);
            const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16(d_taddr, kmajor_desc(a_addr + kk * 256), kmajor_desc(b_addr + kk * 256), idesc,
                        (j > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&empty[slot]);
          }
          umma_commit(&acc_full[b]);
          u += len;
        }
      }
    }
    __syncwarp();
  } else {
    // -------------------------------------------- epilogue, attention, embedding
    const int et = (warp - kEpiWarp0) * 32 + lane;
    int seg = 0;
    uint32_t uses[2] = {0u, 0u};
    if (P.trace && c == 0 && et == 0) P.trace[P.n_stages] = global_timer_ns();
    for (int s = 0; s < P.n_stages; ++s) {
      const PStage& st = P.stages[s];
      const Done dn{&P.done[s * kDoneStride], (unsigned)st.target, P.trace ? P.trace + s : nullptr};
      const unsigned* dep_ctr = st.dep >= 0 ? &P.done[st.dep * kDoneStride] : nullptr;
      const unsigned dep_target = st.dep >= 0 ? (unsigned)P.stages[st.dep].target : 0u;
      if (st.kind == kPEmbed) {
        if (c < P.M && dep_ctr) epi_wait(dep_ctr, dep_target, P.err, et);
        for (int t = c; t < P.M; t += G) {
          embed_token(st.em, t, NT, st.tc.ss_ld, et, red4);
          signal_done(dn, et);
        }
      } else if (st.kind == kPAttn) {
        const AttnParams& a = st.at;
        const int U = a.M * kKvHeads * a.max_splits;
        if (c >= U) continue;  // no unit here: nothing to wait for
        epi_wait(dep_ctr, dep_target, P.err, et);
        fence_proxy_async_global();  // K/V written by the previous stage are read by bulk copies
        for (int u = c; u < U; u += G) {
          const int tok = u % a.M;
          const int g = (u / a.M) % kKvHeads;
          const int split = u / (a.M * kKvHeads);
          if (attention_unit<true, 4>(a, AS, split, g, tok, et, uses)) signal_done(dn, et);
        }
      } else {
        const TcParams& p = st.tc;
        const Geom geo{p.n_mtiles * p.n_ntiles * p.KB, st.ctas};
        const int u0 = c < st.ctas ? geo.start(c) : 0, u1 = c < st.ctas ? geo.start(c + 1) : 0;
        if (u0 >= u1 && p.epi != kTcLogits) continue;  // no unit here
        if (u0 < u1) epi_wait(dep_ctr, dep_target, P.err, et);
        auto on_tile = [&](int e) { signal_done(dn, e); };
        switch (p.epi) {
          case kTcQkvRope:
            epilogue_range<kTcQkvRope, 4>(p, geo, c, u0, u1, seg, acc_full, acc_empty, tmem_base, N, warp, lane, es,
                                       on_tile);
            break;
          case kTcResidual:
            epilogue_range<kTcResidual, 4>(p, geo, c, u0, u1, seg, acc_full, acc_empty, tmem_base, N, warp, lane, es,
                                        on_tile);
            break;
          case kTcSwiglu:
            epilogue_range<kTcSwiglu, 4>(p, geo, c, u0, u1, seg, acc_full, acc_empty, tmem_base, N, warp, lane, es,
                                      on_tile);
            break;
          default:
            epilogue_range<kTcLogits, 4>(p, geo, c, u0, u1, seg, acc_full, acc_empty, tmem_base, N, warp, lane, es,
                                      on_tile);
            break;
        }
      }
    }
  }

  if (*reinterpret_cast<volatile int*>(P.err)) {
    // A wait gave up and the loops above ran on without waiting: let the copies and
    // MMAs already issued land before shared memory and TMEM are released.
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 200000ull) __nanosleep(1000);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, P.tmem_cols);
  }
}

}  // namespace

size_t persistent_smem_bytes(int NT, int ring) {
  return persistent_attn_offset(ring, kABytes + (size_t)NT * 256) + sizeof(AttnSmem);
}

int persistent_ring(int NT) {
  int ring = 12;
  while (ring > 2 && persistent_smem_bytes(NT, ring) > 227 * 1024) --ring;
  return ring;
}

cudaError_t launch_persistent(const PParams& p, int ctas, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e =
        cudaFuncSetAttribute(persistent_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = persistent_smem_bytes(p.NT, p.ring);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: stages wait on each other
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, persistent_forward_kernel, p);
}

}  // namespace qi
