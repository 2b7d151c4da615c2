// Decode projections: skinny GEMMs of M tokens x (N rows of bf16 weights) on CUDA cores,
// with their neighbours fused (RMSNorm prologue; bias/RoPE/KV-append, residual add,
// SwiGLU or logits+argmax epilogue).
//
// Data flow per CTA: the CTA owns a contiguous range of 8-row groups. Each group's
// weights (8 rows x K) sit in the tiled layout as K/64 contiguous 1 KB runs, which one
// warp streams into a shared-memory ring with cp.async.bulk (TMA bulk copies completing
// on an mbarrier). The copies are issued before griddepcontrol.wait, so under
// programmatic dependent launch the weight stream overlaps the previous kernel's tail.
// Activations (fp32) are staged per chunk of MT tokens, RMS-normalised in place when
// the kernel has a norm prologue. Each warp lane owns one row of a group and a stripe
// of 8-column core matrices; lanes and warps reduce with shuffles and shared memory in
// a fixed order, so results do not depend on timing.
#include "common.cuh"
#include "internal.h"

namespace qi {

namespace {

constexpr int kGemvThreads = 256;

template <int MT, bool NORM>
__device__ __forceinline__ void stage_activations(const GemvParams& p, float* abuf, float* rinv,
                                                  int t0, int k0, int kr, int warp, int lane) {
  const int n4 = kr >> 2;
  for (int idx = threadIdx.x; idx < MT * n4; idx += kGemvThreads) {
    const int t = idx / n4;
    const int k4 = idx - t * n4;
    const int tok = t0 + t;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tok < p.M) {
      const long long row = p.act_rows ? (long long)p.act_rows[tok] : (long long)tok;
      v = *reinterpret_cast<const float4*>(p.act + row * p.act_stride + k0 + 4 * k4);
    }
    reinterpret_cast<float4*>(abuf)[idx] = v;
  }
  if constexpr (NORM) {
    __syncthreads();
    if (warp < MT) {
      float ss = 0.f;
      for (int k = lane; k < kr; k += 32) {
        const float a = abuf[warp * kr + k];
        ss = fmaf(a, a, ss);
      }
      ss = warp_sum(ss);
      // RMSNorm.forward (qwen2.py:44-48): x * rsqrt(mean(x^2) + eps) * w
      if (lane == 0) rinv[warp] = 1.0f / sqrtf(ss / (float)kr + p.eps);
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < MT * kr; idx += kGemvThreads) {
      const int t = idx / kr;
      const int k = idx - t * kr;
      abuf[idx] = abuf[idx] * rinv[t] * p.norm_w[k0 + k];
    }
  }
}

template <int MT, int EPI>
__device__ __forceinline__ void epilogue(const GemvParams& p, int group, int r, int lane, int t0,
                                         const float (&acc)[MT], float (&bestv)[MT], int (&besti)[MT]) {
  const int n = group * 8 + r;  // physical output row of this lane
  if constexpr (EPI == kEpiQkvRope) {
    const int head = n >> 6;          // 0..13 q, 14..15 k, 16..17 v
    const int j = (n & 63) >> 1;      // RoPE pair index (dims j and j + 32)
    const int half = n & 1;
    const int d = j + 32 * half;
    const float b = p.bias[n];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int tok = t0 + t;
      float v = acc[t] + b;
      const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
      if (tok >= p.M) continue;
      const int ps = p.pos[tok];
      if (head < kHeads + kKvHeads) {
        // apply_rope (qwen2.py:86-99): x*cos + rotate_half(x)*sin, halves paired.
        const float cs = p.rope_cos[(long long)ps * kHeadDim + j];
        const float sn = p.rope_sin[(long long)ps * kHeadDim + j];
        v = half ? (v * cs + partner * sn) : (v * cs - partner * sn);
      }
      if (lane < 8) {
        if (head < kHeads) {
          p.out[(long long)tok * kHidden + head * kHeadDim + d] = v;
        } else {
          const int row = p.rows[tok];
          const int kvh = (head - kHeads) & 1;
          uint16_t* base = head < kHeads + kKvHeads ? p.kc : p.vc;
          base[(((long long)row * kKvHeads + kvh) * p.max_len + ps) * kHeadDim + d] = f32_to_bf16_rn(v);
        }
      }
    }
  } else if constexpr (EPI == kEpiResidual) {
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int tok = t0 + t;
      if (lane < 8 && tok < p.M) {
        float* o = p.out + (long long)tok * p.out_ld + n;
        if (gridDim.y > 1) atomicAdd(o, acc[t]);
        else *o += acc[t];
      }
    }
  } else if constexpr (EPI == kEpiSwiglu) {
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int tok = t0 + t;
      const float up = __shfl_xor_sync(0xffffffffu, acc[t], 1);
      if (lane < 8 && !(r & 1) && tok < p.M) {
        const float gate = acc[t];
        // F.silu(gate) * up (qwen2.py:114-116)
        p.out[(long long)tok * p.out_ld + (n >> 1)] = gate / (1.0f + expf(-gate)) * up;
      }
    }
  } else {  // kEpiLogits
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int tok = t0 + t;
      if (tok >= p.M) continue;
      const float v = acc[t];
      if (lane < 8 && p.logits) {
        const long long o = (long long)tok * p.logits_ld + n;
        if (p.logits_bf16) reinterpret_cast<uint16_t*>(p.logits)[o] = f32_to_bf16_rn(v);
        else reinterpret_cast<float*>(p.logits)[o] = v;
      }
      if (v > bestv[t]) {  // rows visit in increasing order per lane: keep the first max
        bestv[t] = v;
        besti[t] = n;
      }
    }
  }
}

template <int MT, int EPI, bool NORM>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kr = p.kr;
  const int k0 = blockIdx.y * kr;
  const int kblocks = kr >> 6;
  const uint32_t group_bytes = (uint32_t)kblocks * kGroupChunkBytes;
  const int g_begin = (int)(((long long)blockIdx.x * p.n_groups) / gridDim.x);
  const int g_end = (int)(((long long)(blockIdx.x + 1) * p.n_groups) / gridDim.x);
  const int gc = g_end - g_begin;
  const int wpg = p.wpg;
  const int gpr = 8 / wpg;
  const int slots = p.slots;

  uint8_t* wbuf = smem;
  float* abuf = reinterpret_cast<float*>(smem + (size_t)slots * group_bytes);
  float* red = abuf + MT * kr;
  float* rinv = red + 64 * MT;
  uint64_t* bars = reinterpret_cast<uint64_t*>(rinv + 8);

  if (threadIdx.x == 0) {
    for (int s = 0; s < slots; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncthreads();

  // Warp 0 streams groups [first, first + count) into their ring slots.
  auto issue = [&](int first, int count) {
    if (lane == 0)
      for (int j = 0; j < count; ++j) mbar_arrive_expect_tx(&bars[(first + j) % slots], group_bytes);
    __syncwarp();
    const int kb0 = k0 >> 6;
    for (int idx = lane; idx < count * kblocks; idx += 32) {
      const int gi = first + idx / kblocks;
      const int kb = idx % kblocks;
      uint8_t* dst = wbuf + (size_t)(gi % slots) * group_bytes + (size_t)kb * kGroupChunkBytes;
      bulk_g2s(dst, p.w + tiled_group_offset(g_begin + gi, kb0 + kb, p.K), kGroupChunkBytes,
               &bars[gi % slots]);
    }
  };
  if (warp == 0) issue(0, gc < slots ? gc : slots);

  // Everything above touched only weights; activations come from earlier kernels.
  grid_dep_wait();
  grid_dep_launch();

  float bestv[MT];
  int besti[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    bestv[t] = -INFINITY;
    besti[t] = 0x7fffffff;
  }

  const int nrounds = (gc + gpr - 1) / gpr;
  const int ntchunks = (p.M + MT - 1) / MT;
  const int r = lane & 7;
  const int c = lane >> 3;
  const int kpart = warp % wpg;
  const int nkc = kr >> 3;

  for (int rd = 0; rd < nrounds; ++rd) {
    const int gi = rd * gpr + warp / wpg;
    const bool active = gi < gc;
    if (active) mbar_wait(&bars[gi % slots], (uint32_t)((gi / slots) & 1), p.err);
    const uint8_t* wg = wbuf + (size_t)(gi % slots) * group_bytes + r * 16;

    for (int tc = 0; tc < ntchunks; ++tc) {
      const int t0 = tc * MT;
      if (rd == 0 || ntchunks > 1) {
        __syncthreads();
        stage_activations<MT, NORM>(p, abuf, rinv, t0, k0, kr, warp, lane);
        __syncthreads();
      }
      float acc[MT];
#pragma unroll
      for (int t = 0; t < MT; ++t) acc[t] = 0.f;
      if (active) {
        for (int kc = kpart * 4 + c; kc < nkc; kc += 4 * wpg) {
          const uint4 wv = *reinterpret_cast<const uint4*>(wg + (kc >> 3) * kGroupChunkBytes + (kc & 7) * 128);
          const float w0 = bf16lo(wv.x), w1 = bf16hi(wv.x), w2 = bf16lo(wv.y), w3 = bf16hi(wv.y);
          const float w4 = bf16lo(wv.z), w5 = bf16hi(wv.z), w6 = bf16lo(wv.w), w7 = bf16hi(wv.w);
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const float4* a = reinterpret_cast<const float4*>(abuf + t * kr + kc * 8);
            const float4 a0 = a[0];
            const float4 a1 = a[1];
            float s = acc[t];
            s = fmaf(w0, a0.x, s);
            s = fmaf(w1, a0.y, s);
            s = fmaf(w2, a0.z, s);
            s = fmaf(w3, a0.w, s);
            s = fmaf(w4, a1.x, s);
            s = fmaf(w5, a1.y, s);
            s = fmaf(w6, a1.z, s);
            s = fmaf(w7, a1.w, s);
            acc[t] = s;
          }
        }
      }
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], 8);
        acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], 16);
      }
      if (wpg > 1) {
        if (lane < 8) {
#pragma unroll
          for (int t = 0; t < MT; ++t) red[(warp * 8 + lane) * MT + t] = acc[t];
        }
        __syncthreads();
        if (kpart == 0) {
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            float s = 0.f;
            for (int j = 0; j < wpg; ++j) s += red[((warp + j) * 8 + r) * MT + t];
            acc[t] = s;
          }
        }
      }
      if (active && kpart == 0) epilogue<MT, EPI>(p, g_begin + gi, r, lane, t0, acc, bestv, besti);
      if (wpg > 1) __syncthreads();  // red[] is reused by the next chunk
    }
    __syncthreads();  // this round's slots are free
    if (warp == 0) {
      const int first = rd * gpr + slots;
      int count = gc - first;
      count = count < gpr ? count : gpr;
      if (count > 0) issue(first, count);
    }
  }

  if constexpr (EPI == kEpiLogits) {
    if (kpart == 0) {
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        unsigned long long key = besti[t] == 0x7fffffff ? 0ull : argmax_pack(bestv[t], besti[t]);
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
          key = other > key ? other : key;
        }
        if (lane == 0 && key != 0ull && t < p.M) atomicMax(p.argmax + t, key);
      }
    }
  }
}

template <int MT, int EPI, bool NORM>
cudaError_t launch_one(const GemvParams& p, int ctas, int splits, size_t smem, cudaStream_t stream, bool pdl) {
  auto kern = gemv_kernel<MT, EPI, NORM>;
  if (smem > 48 * 1024) {
    cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(kern), 227 * 1024);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, splits, 1);
  cfg.blockDim = dim3(kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int EPI, bool NORM>
cudaError_t launch_mt(int mt, const GemvParams& p, int ctas, int splits, size_t smem, cudaStream_t s, bool pdl) {
  switch (mt) {
    case 1: return launch_one<1, EPI, NORM>(p, ctas, splits, smem, s, pdl);
    case 2: return launch_one<2, EPI, NORM>(p, ctas, splits, smem, s, pdl);
    case 4: return launch_one<4, EPI, NORM>(p, ctas, splits, smem, s, pdl);
    default: return launch_one<8, EPI, NORM>(p, ctas, splits, smem, s, pdl);
  }
}

}  // namespace

size_t gemv_smem_bytes(int mt, int kr, int slots) {
  const size_t group_bytes = (size_t)(kr / 64) * kGroupChunkBytes;
  return (size_t)slots * group_bytes + (size_t)mt * kr * 4 + 64 * mt * 4 + 8 * 4 + (size_t)slots * 8;
}

cudaError_t launch_gemv(int epi, int mt, GemvParams p, int ctas, int splits, cudaStream_t stream, bool pdl) {
  const size_t smem = gemv_smem_bytes(mt, p.kr, p.slots);
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  const bool norm = p.norm_w != nullptr;
  switch (epi) {
    case kEpiQkvRope:
      return norm ? launch_mt<kEpiQkvRope, true>(mt, p, ctas, splits, smem, stream, pdl)
                  : launch_mt<kEpiQkvRope, false>(mt, p, ctas, splits, smem, stream, pdl);
    case kEpiResidual: return launch_mt<kEpiResidual, false>(mt, p, ctas, splits, smem, stream, pdl);
    case kEpiSwiglu:
      return norm ? launch_mt<kEpiSwiglu, true>(mt, p, ctas, splits, smem, stream, pdl)
                  : launch_mt<kEpiSwiglu, false>(mt, p, ctas, splits, smem, stream, pdl);
    case kEpiLogits: return launch_mt<kEpiLogits, true>(mt, p, ctas, splits, smem, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace qi
