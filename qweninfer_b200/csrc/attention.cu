// Ragged GQA attention for decode and prefill queries (qweninfer/models/qwen2.py:184-199).
//
// One CTA per (key split, KV head, query token). A query at position p reads only keys
// 0..p of its own cache row (the reference reads B x window keys and masks). The CTA's
// key range streams through a two-stage shared-memory ring in 128-key tiles (K and V,
// 16 KB each, bulk-copied from the packed cache, where one head's keys are contiguous).
// The 7 query heads of the KV group share every tile: 4 warps each take 32 keys of a
// tile, compute all 7 scores per key (lane = key), run an fp32 online softmax per warp,
// and accumulate P.V with lane = 2 output dims. Warps and splits are merged with the
// usual max-rescaled sums; the last CTA of a token/head (atomic arrival count) merges
// the splits in split order and resets its counter.
#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "tc_proj.h"

namespace qi {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kTile = 128;  // keys per stage
constexpr int kPartStride = kGqa * (kHeadDim + 2);  // floats per (token, head, split) partial

struct AttnSmem {
  uint16_t k[2][kTile * kHeadDim];
  uint16_t v[2][kTile * kHeadDim];
  float q[kGqa * 2 * 8 * 4];          // per head: [half][chunk][4], scaled by 1/sqrt(64)
  float p[4][32][8];                  // per warp: probabilities of its 32 keys, 7 heads
  float cmb[4][kGqa][kHeadDim + 2];   // per warp: acc[64], m, l
  uint64_t bar[2];
  int last;
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

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem& S = *reinterpret_cast<AttnSmem*>(smem_raw);
  const int split = blockIdx.x;
  const int g = blockIdx.y;
  const int tok = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  grid_dep_wait();
  grid_dep_launch();

  const int ps = p.pos[tok];
  const int nkeys = ps + 1;
  const int nsplit = (nkeys + p.split_keys - 1) / p.split_keys;
  if (split >= nsplit) return;
  const int kbeg = split * p.split_keys;
  const int kend = min(nkeys, kbeg + p.split_keys);
  const int row = p.rows[tok];
  const long long head_base = (((long long)row * kKvHeads + g) * p.max_len) * kHeadDim;
  const uint16_t* kg = p.kc + head_base;
  const uint16_t* vg = p.vc + head_base;

  if (tid == 0) {
    mbar_init(&S.bar[0], 1);
    mbar_init(&S.bar[1], 1);
    fence_barrier_init();
  }
  // q of the 7 heads sharing KV head g, pre-scaled by 1/8 (exact), laid out so that the
  // eight 8-dim chunks' first halves are 16-byte neighbours (conflict-free rotated reads).
  for (int idx = tid; idx < kGqa * kHeadDim; idx += kAttnThreads) {
    const int h = idx >> 6, d = idx & 63;
    const int cc = d >> 3, e = d & 7;
    S.q[((h * 2 + (e >> 2)) * 8 + cc) * 4 + (e & 3)] =
        p.q[(long long)tok * kHidden + (g * kGqa + h) * kHeadDim + d] * 0.125f;
  }
  __syncthreads();

  const int ntiles = (kend - kbeg + kTile - 1) / kTile;
  auto issue = [&](int i) {
    const int k0 = kbeg + i * kTile;
    const int nk = min(kTile, kend - k0);
    const uint32_t bytes = (uint32_t)nk * kHeadDim * 2;
    const int st = i & 1;
    mbar_arrive_expect_tx(&S.bar[st], 2 * bytes);
    bulk_g2s(S.k[st], kg + (long long)k0 * kHeadDim, bytes, &S.bar[st]);
    bulk_g2s(S.v[st], vg + (long long)k0 * kHeadDim, bytes, &S.bar[st]);
  };
  if (tid == 0) {
    issue(0);
    if (ntiles > 1) issue(1);
  }

  float m[kGqa], l[kGqa], acc[kGqa][2];
#pragma unroll
  for (int h = 0; h < kGqa; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
    acc[h][0] = acc[h][1] = 0.f;
  }

  for (int i = 0; i < ntiles; ++i) {
    const int st = i & 1;
    mbar_wait(&S.bar[st], (uint32_t)((i >> 1) & 1), p.err);
    const int k0 = kbeg + i * kTile;
    const int nk = min(kTile, kend - k0);
    const int kw = 32 * warp;
    const int nkw = max(0, min(32, nk - kw));
    if (nkw > 0) {
      const bool valid = lane < nkw;
      float s[kGqa];
#pragma unroll
      for (int h = 0; h < kGqa; ++h) s[h] = 0.f;
      const uint16_t* krow = S.k[st] + (kw + lane) * kHeadDim;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int cc = (c + lane) & 7;
        const uint4 kv = *reinterpret_cast<const uint4*>(krow + cc * 8);
        const float k0f = bf16lo(kv.x), k1f = bf16hi(kv.x), k2f = bf16lo(kv.y), k3f = bf16hi(kv.y);
        const float k4f = bf16lo(kv.z), k5f = bf16hi(kv.z), k6f = bf16lo(kv.w), k7f = bf16hi(kv.w);
#pragma unroll
        for (int h = 0; h < kGqa; ++h) {
          const float4 qa = *reinterpret_cast<const float4*>(&S.q[((h * 2 + 0) * 8 + cc) * 4]);
          const float4 qb = *reinterpret_cast<const float4*>(&S.q[((h * 2 + 1) * 8 + cc) * 4]);
          float a = s[h];
          a = fmaf(qa.x, k0f, a);
          a = fmaf(qa.y, k1f, a);
          a = fmaf(qa.z, k2f, a);
          a = fmaf(qa.w, k3f, a);
          a = fmaf(qb.x, k4f, a);
          a = fmaf(qb.y, k5f, a);
          a = fmaf(qb.z, k6f, a);
          a = fmaf(qb.w, k7f, a);
          s[h] = a;
        }
      }
#pragma unroll
      for (int h = 0; h < kGqa; ++h) {
        const float sv = valid ? s[h] : -INFINITY;
        const float mn = fmaxf(m[h], warp_max(sv));
        const float alpha = expf(m[h] - mn);
        const float pr = valid ? expf(sv - mn) : 0.f;
        l[h] = l[h] * alpha + warp_sum(pr);
        acc[h][0] *= alpha;
        acc[h][1] *= alpha;
        m[h] = mn;
        S.p[warp][lane][h] = pr;
      }
      __syncwarp();
      const uint16_t* vt = S.v[st] + kw * kHeadDim + 2 * lane;
      for (int j = 0; j < nkw; ++j) {
        const uint32_t v2 = *reinterpret_cast<const uint32_t*>(vt + j * kHeadDim);
        const float v0 = bf16lo(v2), v1 = bf16hi(v2);
        const float4 pa = *reinterpret_cast<const float4*>(&S.p[warp][j][0]);
        const float4 pb = *reinterpret_cast<const float4*>(&S.p[warp][j][4]);
        acc[0][0] = fmaf(pa.x, v0, acc[0][0]); acc[0][1] = fmaf(pa.x, v1, acc[0][1]);
        acc[1][0] = fmaf(pa.y, v0, acc[1][0]); acc[1][1] = fmaf(pa.y, v1, acc[1][1]);
        acc[2][0] = fmaf(pa.z, v0, acc[2][0]); acc[2][1] = fmaf(pa.z, v1, acc[2][1]);
        acc[3][0] = fmaf(pa.w, v0, acc[3][0]); acc[3][1] = fmaf(pa.w, v1, acc[3][1]);
        acc[4][0] = fmaf(pb.x, v0, acc[4][0]); acc[4][1] = fmaf(pb.x, v1, acc[4][1]);
        acc[5][0] = fmaf(pb.y, v0, acc[5][0]); acc[5][1] = fmaf(pb.y, v1, acc[5][1]);
        acc[6][0] = fmaf(pb.z, v0, acc[6][0]); acc[6][1] = fmaf(pb.z, v1, acc[6][1]);
      }
      __syncwarp();
    }
    __syncthreads();  // stage st fully consumed
    if (tid == 0 && i + 2 < ntiles) issue(i + 2);
  }

  // Merge the 4 warps.
#pragma unroll
  for (int h = 0; h < kGqa; ++h) {
    S.cmb[warp][h][2 * lane] = acc[h][0];
    S.cmb[warp][h][2 * lane + 1] = acc[h][1];
    if (lane == 0) {
      S.cmb[warp][h][kHeadDim] = m[h];
      S.cmb[warp][h][kHeadDim + 1] = l[h];
    }
  }
  __syncthreads();
  float* part = p.part + (((long long)tok * kKvHeads + g) * p.max_splits + split) * kPartStride;
  for (int idx = tid; idx < kGqa * (kHeadDim + 2); idx += kAttnThreads) {
    const int h = idx / (kHeadDim + 2);
    const int d = idx - h * (kHeadDim + 2);
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) mx = fmaxf(mx, S.cmb[w][h][kHeadDim]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = S.cmb[w][h][kHeadDim];
      if (mw == -INFINITY) continue;
      const float sc = expf(mw - mx);
      L = fmaf(sc, S.cmb[w][h][kHeadDim + 1], L);
      if (d < kHeadDim) A = fmaf(sc, S.cmb[w][h][d], A);
    }
    if (nsplit == 1) {
      if (d < kHeadDim) emit(p, tok, (g * kGqa + h) * kHeadDim + d, A / L);
    } else {
      part[idx] = d < kHeadDim ? A : (d == kHeadDim ? mx : L);
    }
  }
  if (nsplit == 1) return;

  // Split merge by the last-arriving CTA of this (token, head).
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int prev = atomicAdd(&p.counters[tok * kKvHeads + g], 1u);
    S.last = (prev == (unsigned int)(nsplit - 1));
  }
  __syncthreads();
  if (!S.last) return;
  __threadfence();
  const float* base = p.part + (((long long)tok * kKvHeads + g) * p.max_splits) * kPartStride;
  for (int idx = tid; idx < kGqa * kHeadDim; idx += kAttnThreads) {
    const int h = idx >> 6, d = idx & 63;
    float mx = -INFINITY;
    for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, __ldcg(base + s * kPartStride + h * (kHeadDim + 2) + kHeadDim));
    float L = 0.f, A = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float* ph = base + s * kPartStride + h * (kHeadDim + 2);
      const float sc = expf(__ldcg(ph + kHeadDim) - mx);
      L = fmaf(sc, __ldcg(ph + kHeadDim + 1), L);
      A = fmaf(sc, __ldcg(ph + d), A);
    }
    emit(p, tok, (g * kGqa + h) * kHeadDim + d, A / L);
  }
  if (tid == 0) p.counters[tok * kKvHeads + g] = 0u;
}

}  // namespace

cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream, bool pdl) {
  static bool configured = false;
  const size_t smem = sizeof(AttnSmem);
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.max_splits, kKvHeads, p.M);
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, attention_kernel, p);
}


// ---------------------------------------------------------------------------------------
// Attention without caller-provided scratch.
//
// Some callers of this library cannot allocate device memory: a host program that binds
// the C ABI directly (C, Go, Java, ...) and only receives device pointers for the tensors
// it owns, or a serving process whose device memory is reserved once at start-up and must
// not grow afterwards. For them, the split partials and arrival counters of the attention
// kernel live in this file-scope array instead, so the call takes only inputs and outputs.
//
// Capacity: up to kNoAllocMaxTokens query tokens and kNoAllocMaxLen cache slots per row
// (128-key splits). The array (about 3.6 MiB) is part of the library image, so every GPU
// that loads libqi.so holds it until the process exits. All calls share it: two calls whose
// executions overlap on the GPU (other streams, other threads) race on it and give wrong
// results; calls in one stream are ordered and safe.
namespace {
constexpr int kNoAllocMaxTokens = 64;
constexpr int kNoAllocMaxLen = 2048;
constexpr int kNoAllocSplitKeys = 128;
constexpr int kNoAllocMaxSplits = kNoAllocMaxLen / kNoAllocSplitKeys;
constexpr size_t kNoAllocPartWords = (size_t)kNoAllocMaxTokens * kKvHeads * kNoAllocMaxSplits * kPartStride;
constexpr size_t kNoAllocCounterWords = (size_t)kNoAllocMaxTokens * kKvHeads;
}  // namespace

// partials (fp32) followed by the arrival counters (uint32)
static __device__ __align__(256) unsigned int g_attn_noalloc_scratch[kNoAllocPartWords + kNoAllocCounterWords];

namespace {
std::mutex g_noalloc_mutex;
void* g_noalloc_addr[64] = {};  // device address of the array, per device ordinal
}  // namespace

}  // namespace qi

extern "C" int qi_attention_noalloc(const float* q, const uint16_t* k_layer, const uint16_t* v_layer,
                                    const int32_t* pos, const int32_t* rows, int M, int max_len, float* out,
                                    int* err, qi_stream_t stream) {
  using namespace qi;
  if (M > kNoAllocMaxTokens || max_len > kNoAllocMaxLen) return QI_ERR_TOO_LARGE;
  if (M <= 0 || max_len <= 0 || !q || !k_layer || !v_layer || !pos || !rows || !out) return QI_ERR_ARG;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= 64) return QI_ERR_ARG;
  void* base = nullptr;
  {
    // first call on this device: resolve the array's device address (host code must not
    // use the symbol itself, which names a host-side stand-in)
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_addr[dev]) {
      e = cudaGetSymbolAddress(&g_noalloc_addr[dev], g_attn_noalloc_scratch);
      if (e != cudaSuccess) {
        g_noalloc_addr[dev] = nullptr;
        return (int)e;
      }
    }
    base = g_noalloc_addr[dev];
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  unsigned int* counters = static_cast<unsigned int*>(base) + kNoAllocPartWords;
  // the counters must start at zero; the array keeps whatever the previous call left
  e = cudaMemsetAsync(counters, 0, kNoAllocCounterWords * sizeof(unsigned int), s);
  if (e != cudaSuccess) return (int)e;
  AttnParams a = {};
  a.q = q;
  a.kc = k_layer;
  a.vc = v_layer;
  a.pos = pos;
  a.rows = rows;
  a.M = M;
  a.max_len = max_len;
  a.split_keys = kNoAllocSplitKeys;
  a.max_splits = (max_len + kNoAllocSplitKeys - 1) / kNoAllocSplitKeys;
  a.out = out;
  a.part = static_cast<float*>(base);
  a.counters = counters;
  a.err = err;
  e = launch_attention(a, s, false);
  return e == cudaSuccess ? QI_OK : (int)e;
}
