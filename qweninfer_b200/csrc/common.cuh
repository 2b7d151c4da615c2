// Shared device helpers for the qweninfer_b200 kernels (sm_100a).
//
// Model shape constants are those of Qwen2-0.5B (the block shape the kernels are
// specialised for); layers and vocabulary are runtime values.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qi.h"
#include "kv_layout.h"

namespace qi {

constexpr int kHidden = 896;
constexpr int kHeads = 14;
constexpr int kKvHeads = 2;
constexpr int kHeadDim = 64;
constexpr int kGqa = kHeads / kKvHeads;                         // 7 query heads per KV head
constexpr int kInter = 4864;
constexpr int kQkvRows = (kHeads + 2 * kKvHeads) * kHeadDim;    // 1152
constexpr int kGateUpRows = 2 * kInter;                         // 9728

// Tiled weight layout ("core-matrix tiles"): a row-major (N, K) bf16 matrix is stored
// as 128-row x 64-column blocks of 16 KB, ordered (row tile, k block); inside a block,
// 16 groups of 8 rows at 1 KB stride; inside a group, 8 core matrices of 8 rows x 8
// columns (128 contiguous bytes, row r at byte 16 r). This is the SWIZZLE_NONE K-major
// canonical layout of tcgen05 shared-memory descriptors (LBO = 128 B between core
// matrices along K, SBO = 1024 B between 8-row groups), and every 8-row group's slice
// of one 64-column block is a contiguous 1 KB run that a single bulk copy can move.
constexpr int kTileRows = 128;
constexpr int kTileK = 64;
constexpr int kGroupRows = 8;
constexpr int kBlockElems = kTileRows * kTileK;                 // 8192
constexpr int kGroupChunkBytes = kGroupRows * kTileK * 2;       // 1024

__host__ __device__ __forceinline__ long long tiled_group_offset(int group, int kblock, int K) {
  // element offset of (8-row group `group`, 64-column block `kblock`)
  return ((long long)(group >> 4) * (K / kTileK) + kblock) * kBlockElems + (long long)(group & 15) * 512;
}

__host__ __device__ __forceinline__ long long tiled_offset(int n, int k, int K) {
  return tiled_group_offset(n >> 3, k >> 6, K) + ((k & 63) >> 3) * 64 + (n & 7) * 8 + (k & 7);
}

// Element offset of (row, KV head g, position pos) within one layer's K or V (KvLayout),
// or -1 when the position's page is unmapped.
__device__ __forceinline__ long long kv_offset(const KvLayout& L, int max_len, int row, int g, int pos) {
  if (!L.table) return (((long long)row * kKvHeads + g) * max_len + pos) * kHeadDim;
  const int pg = __ldg(L.table + (long long)row * L.ppr + pos / L.page);
  if (pg < 0 || pg >= L.n_pages) return -1;
  return (((long long)pg * kKvHeads + g) * L.page + pos % L.page) * kHeadDim;
}

// --------------------------------------------------------------- conversions

__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float bf16_to_f32(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_rn(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// Order-preserving map float -> uint32 (larger float => larger code).
__device__ __forceinline__ uint32_t f32_order_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Argmax slot: (value key << 32) | (0xffffffff - index). atomicMax keeps the largest
// value and, among equal values, the lowest index (torch.argmax's first-maximum rule).
__device__ __forceinline__ unsigned long long argmax_pack(float v, int idx) {
  return ((unsigned long long)f32_order_key(v) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}

// ------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Atomic add with acquire-release semantics at GPU scope (returns the old value). After a
// CTA barrier it publishes every participating thread's earlier writes (release is
// cumulative) and, when the caller sees the final count, acquires the other arrivals'.
__device__ __forceinline__ unsigned atomic_add_acq_rel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every wait in these kernels is bounded: after kWaitLimitNs the kernel records
// QI_ERR_TIMEOUT in the caller's error word and gives up instead of hanging.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      if (err) atomicExch(err, QI_ERR_TIMEOUT);
      return false;
    }
  }
}

// ------------------------------------------------------- thread-block clusters
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_rank(const void* p, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_u32(p)), "r"(rank));
  return d;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float a) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(a) : "memory");
}
// arrive (release at cluster scope) on an mbarrier of another CTA of the cluster
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// bounded wait (acquire at cluster scope) on a local mbarrier that other CTAs arrive on
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err) {
  auto try_wait = [&]() {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
  };
  if (try_wait()) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (try_wait()) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      if (err) atomicExch(err, QI_ERR_TIMEOUT);
      return false;
    }
  }
}
// split cluster barrier (every thread of every CTA of the cluster arrives once, then waits)
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Bulk (non-tensor) asynchronous copy global -> shared, completing on `bar`.
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch: wait for the preceding grid (and its memory) before
// touching anything it writes; let the next grid start its own prologue early.
// Bulk prefetch of [src, src + bytes) into L2 (no destination, no completion); src 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace qi
