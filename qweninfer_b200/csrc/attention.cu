// Ragged GQA attention for decode and prefill queries (qweninfer/models/qwen2.py:184-199).
//
// One CTA per (key split, KV head, query token). A query at position p reads only keys
// 0..p of its own cache row (the reference reads B x window keys and masks). The CTA's
// key range streams through a two-stage shared-memory ring in 128-key tiles (K and V,
// 16 KB each, cp.async from the packed or paged cache); the 7 query heads of the KV group
// are the rows of warp-level tensor-core MMAs over every tile (attention_device.cuh).
// Splits are merged with the usual max-rescaled sums, in split order: with 2-8 splits
// per launch the splits of a token/head form one thread-block cluster and merge in split
// 0's shared memory; otherwise the last CTA of a token/head (atomic arrival count) merges
// them from global scratch and resets its counter.
#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "tc_proj.h"
#include "attention_device.cuh"

namespace qi {

namespace {

using namespace attn;

constexpr size_t kMergeOffset = (sizeof(AttnSmem) + 15) / 16 * 16;

template <bool kPaged>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem& S = *reinterpret_cast<AttnSmem*>(smem_raw);
  ClusterMerge* cm = p.cluster ? reinterpret_cast<ClusterMerge*>(smem_raw + kMergeOffset) : nullptr;
  // Positions and rows are read before the programmatic-launch wait: they are inputs of the
  // forward, written before its first launch (this kernel is never the first or second
  // launch of a forward; standalone launches do not use programmatic launch). The wait is
  // taken in attention_unit, by splits that have keys.
  const int tok = blockIdx.z;
  const int ps = p.pos[tok], row = p.rows[tok];
  if (cm && threadIdx.x == 0) {
    // split 0 waits for one arrival per thread of each other split of its token
    const int nsplit = (ps >= 0 && ps < p.max_len) ? (ps + p.split_keys) / p.split_keys : 1;
    mbar_init(&cm->bar, (uint32_t)(nsplit > 1 ? (nsplit - 1) * kAttnThreads : 1));
    fence_barrier_init();
  }
  __syncthreads();
  // Cluster handshake: every thread arrives once the barrier is initialised and waits
  // before its first remote access (the splits that push, inside the unit) or before it
  // ends (all others), so no CTA waits for it up front.
  if (cm) cluster_arrive();
  bool waited = false;
  attention_unit<kPaged>(p, S, blockIdx.x, blockIdx.y, tok, ps, row, threadIdx.x, cm, &waited);
  if (cm && !waited) cluster_wait();
}

}  // namespace

cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream, bool pdl) {
  const size_t smem_max = kMergeOffset + sizeof(ClusterMerge);
  const bool paged = p.kv.table != nullptr;
  const void* fn = paged ? reinterpret_cast<const void*>(attention_kernel<true>)
                         : reinterpret_cast<const void*>(attention_kernel<false>);
  cudaError_t e = set_max_dynamic_smem(fn, (int)smem_max);
  if (e != cudaSuccess) return e;
  if (p.cluster && (p.max_splits < 2 || p.max_splits > kMaxClusterSplits)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.max_splits, kKvHeads, p.M);
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = p.cluster ? smem_max : sizeof(AttnSmem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n++].val.programmaticStreamSerializationAllowed = 1;
  }
  if (p.cluster) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)p.max_splits;
    attr[n].val.clusterDim.y = 1;
    attr[n++].val.clusterDim.z = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return paged ? cudaLaunchKernelEx(&cfg, attention_kernel<true>, p) : cudaLaunchKernelEx(&cfg, attention_kernel<false>, p);
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
void* g_noalloc_addr[kMaxDevices] = {};  // device address of the array, per device ordinal
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
  if (dev < 0 || dev >= kMaxDevices) return QI_ERR_ARG;
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
