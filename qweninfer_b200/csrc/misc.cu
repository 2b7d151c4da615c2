// Small kernels: embedding gather into the fp32 residual stream and KV row compaction;
// per-device launch helpers.
#include <atomic>
#include <map>
#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "tc_proj.h"

namespace qi {

namespace {

// One CTA per token; 112 threads each move one 8-element core-matrix row of the tiled
// (vocab, 896) table (qweninfer/models/qwen2.py:273-279: embed lookup, .float()).
// With `act` set it also writes the first projection's activation tiles of
// norm_w * x and the token's sum of squares into ss[0][t] (ss[1..6][t] = 0).
__global__ void __launch_bounds__(128) embed_kernel(const uint16_t* __restrict__ embed, int vocab,
                                                     const int32_t* __restrict__ ids, int M, float* __restrict__ x,
                                                     unsigned long long* __restrict__ slots, int n_slots,
                                                     const float* __restrict__ norm_w, int NT,
                                                     uint16_t* __restrict__ act, float* __restrict__ ss, int ss_ld) {
  __shared__ float red[4];
  grid_dep_wait();
  grid_dep_launch();
  const int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= vocab) id = 0;  // ids are validated on the host; stay in bounds regardless
  const int cc = threadIdx.x;
  float sq = 0.f;
  if (cc < kHidden / 8) {
    const int k = cc * 8;
    const uint4 w = *reinterpret_cast<const uint4*>(embed + tiled_offset(id, k, kHidden));
    float e[8] = {bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y),
                  bf16lo(w.z), bf16hi(w.z), bf16lo(w.w), bf16hi(w.w)};
    float4* o = reinterpret_cast<float4*>(x + (long long)t * kHidden + k);
    o[0] = make_float4(e[0], e[1], e[2], e[3]);
    o[1] = make_float4(e[4], e[5], e[6], e[7]);
    if (act) {
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        sq = fmaf(e[i], e[i], sq);
        sq = fmaf(e[i + 1], e[i + 1], sq);
        const float v0 = e[i] * norm_w[k + i], v1 = e[i + 1] * norm_w[k + i + 1];
        const uint16_t h0 = f32_to_bf16_rn(v0), h1 = f32_to_bf16_rn(v1);
        const uint16_t l0 = f32_to_bf16_rn(v0 - bf16_to_f32(h0)), l1 = f32_to_bf16_rn(v1 - bf16_to_f32(h1));
        hw[i / 2] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        lw[i / 2] = (uint32_t)l0 | ((uint32_t)l1 << 16);
      }
      // one core-matrix row: 8 consecutive columns, 16 contiguous bytes per half
      *reinterpret_cast<uint4*>(act + act_offset(t, k, 0, kHidden, NT)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(act + act_offset(t, k, 1, kHidden, NT)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
  }
  if (slots && threadIdx.x == 0 && t < n_slots) slots[t] = 0ull;
  if (act && ss) {
    sq = warp_sum(sq);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x < kHidden / 128)
      ss[(long long)threadIdx.x * ss_ld + t] = threadIdx.x == 0 ? (red[0] + red[1]) + (red[2] + red[3]) : 0.f;
  }
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
                         unsigned long long* slots, int n_slots, cudaStream_t stream, bool pdl,
                         const float* norm_w, int NT, uint16_t* act, float* ss, int ss_ld) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M, 1, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, embed_kernel, embed, vocab, ids, M, x, slots, n_slots, norm_w, NT, act, ss,
                            ss_ld);
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
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  static std::atomic<int> cached[kMaxDevices];  // 0: not yet queried
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// Kernel attributes are per device: a process that drives several GPUs sets them once on
// each (the set of (device, kernel) pairs already configured is kept under a mutex).
cudaError_t set_max_dynamic_smem(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  auto it = done.find({dev, kernel});
  if (it != done.end() && it->second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done[{dev, kernel}] = bytes;
  return e;
}

}  // namespace qi
