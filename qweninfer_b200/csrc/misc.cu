// Small kernels: embedding gather into the fp32 residual stream and KV row compaction.
#include "common.cuh"
#include "internal.h"

namespace qi {

namespace {

// One CTA per token; 112 threads each move one 8-element core-matrix row of the tiled
// (vocab, 896) table (qweninfer/models/qwen2.py:273-279: embed lookup, .float()).
__global__ void __launch_bounds__(128) embed_kernel(const uint16_t* __restrict__ embed, int vocab,
                                                     const int32_t* __restrict__ ids, int M, float* __restrict__ x,
                                                     unsigned long long* __restrict__ slots) {
  grid_dep_wait();
  grid_dep_launch();
  const int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= vocab) id = 0;  // ids are validated on the host; stay in bounds regardless
  const int cc = threadIdx.x;
  if (cc < kHidden / 8) {
    const int k = cc * 8;
    const uint4 w = *reinterpret_cast<const uint4*>(embed + tiled_offset(id, k, kHidden));
    float4* o = reinterpret_cast<float4*>(x + (long long)t * kHidden + k);
    o[0] = make_float4(bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y));
    o[1] = make_float4(bf16lo(w.z), bf16hi(w.z), bf16lo(w.w), bf16hi(w.w));
  }
  if (slots && threadIdx.x == 0) slots[t] = 0ull;
}

// KVCache.move_row (qweninfer/engine/kv_cache.py:65-73): for every (layer, K/V, head),
// positions [0, length) of row src are one contiguous run; copy it to row dst.
__global__ void __launch_bounds__(256) move_rows_kernel(uint16_t* __restrict__ k, uint16_t* __restrict__ v,
                                                         int cache_rows, int max_len, int src, int dst,
                                                         int length) {
  const int plane = blockIdx.y;  // layer * 4 + kv * 2 + head
  const int layer = plane >> 2;
  const int which = (plane >> 1) & 1;
  const int head = plane & 1;
  uint16_t* base = which ? v : k;
  const long long src_off = (((long long)layer * cache_rows + src) * kKvHeads + head) * max_len * kHeadDim;
  const long long dst_off = (((long long)layer * cache_rows + dst) * kKvHeads + head) * max_len * kHeadDim;
  const long long n16 = (long long)length * kHeadDim / 8;  // 16-byte units
  const uint4* s = reinterpret_cast<const uint4*>(base + src_off);
  uint4* d = reinterpret_cast<uint4*>(base + dst_off);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (long long)gridDim.x * blockDim.x)
    d[i] = s[i];
}

}  // namespace

cudaError_t launch_embed(const uint16_t* embed, int vocab, const int32_t* ids, int M, float* x,
                         unsigned long long* slots, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M, 1, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, embed_kernel, embed, vocab, ids, M, x, slots);
}

cudaError_t launch_move_rows(uint16_t* k, uint16_t* v, int layers, int cache_rows, int max_len,
                             int src, int dst, int length, cudaStream_t stream) {
  if (length <= 0 || src == dst) return cudaSuccess;
  const long long n16 = (long long)length * kHeadDim / 8;
  int bx = (int)((n16 + 255) / 256);
  bx = bx > 64 ? 64 : bx;
  move_rows_kernel<<<dim3(bx, layers * 4, 1), 256, 0, stream>>>(k, v, cache_rows, max_len, src, dst, length);
  return cudaGetLastError();
}

int sm_count() {
  static int cached_dev = -1, cached = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev != cached_dev) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0) cached = n;
    cached_dev = dev;
  }
  return cached;
}

}  // namespace qi
