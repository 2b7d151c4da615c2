// Tensor-core projection kernel (tc_proj.cu) and the activation-tile format it consumes.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "kv_layout.h"

namespace qi {

enum TcEpilogue : int {
  kTcPlain = 0,     // out[t, n] = rinv[t] * D[n, t]
  kTcQkvRope = 1,   // bias + RoPE; q -> fp32, k/v -> bf16 cache
  kTcResidual = 2,  // x[t, n] += D; next activations hi/lo(w_next * x) + sum-of-squares partials
  kTcSwiglu = 3,    // h = silu(gate) * up -> activation tiles of the down projection
  kTcLogits = 4,    // optional logits + packed argmax of the head tokens
  kTcQkvRopePaged = 5,  // kTcQkvRope into a paged cache (TcParams::kv)
};

// the QKV epilogue kinds (packed or paged KV append)
template <int EPI>
constexpr bool kIsQkv = EPI == kTcQkvRope || EPI == kTcQkvRopePaged;

// Activation tiles: for inner size K and token tile NT (8..128, power of two), token t,
// column k, half `part` (0 = hi = bf16(x), 1 = lo = bf16(x - hi)):
//   [t / NT][k / 64][part][(t % NT) / 8][(k % 64) / 8][t % 8][k % 8]   (bf16 elements)
// One (token tile, 64-column block) is NT * 256 contiguous bytes: the B operand of one
// pipeline stage, in the SWIZZLE_NONE K-major canonical layout.
__host__ __device__ __forceinline__ long long act_offset(int t, int k, int part, int K, int NT) {
  const int nt = t / NT, tl = t - nt * NT;
  return ((long long)nt * (K / 64) + (k >> 6)) * (2LL * NT * 64) + (long long)part * NT * 64 +
         (long long)(tl >> 3) * 512 + ((k & 63) >> 3) * 64 + (tl & 7) * 8 + (k & 7);
}

struct TcParams {
  // A: weights (tiled), B: activation tiles
  const uint16_t* w;
  int KB;          // pipeline units per output tile (K / 64 / kpu)
  int kpu;         // 64-column k blocks per pipeline unit (1 or 2)
  int n_mtiles;    // weight rows / 128
  const uint16_t* act_in;
  int NT;          // token tile
  int lg_nt;       // log2(NT)
  int n_ntiles;    // token tiles processed by this launch
  int ntile0;      // first token tile
  int M;           // live tokens (t >= M are padding)
  const float* ss_in;  // (7, ss_ld) per-128-feature partial sums of squares, or null
  int ss_ld;
  float eps;
  int epi;
  // plain
  float* out;
  int out_ld;
  // qkv
  const float* bias;
  const float* rope_cos;
  const float* rope_sin;
  const int32_t* pos;
  const int32_t* rows;
  float* q;
  uint16_t* kc;
  uint16_t* vc;
  int max_len;
  int cache_rows;  // rows of the cache (0: rows are not checked)
  KvLayout kv;     // packed (kv.table == nullptr) or paged cache
  // residual / swiglu
  float* x;
  const float* next_norm_w;
  float* ss_out;
  uint16_t* act_out;
  int out_nt;      // token tile of act_out (the consumer's; run_tc sets 0 to NT)
  int lg_out_nt;   // log2(out_nt)
  // logits: head tokens t = head_lo + i * head_stride (i < ...), t < head_hi
  void* logits;
  int logits_bf16;
  long long logits_ld;
  unsigned long long* argmax;
  int head_lo, head_hi, head_stride;
  // L2 prefetch: bytes from pf (a later projection's weights) spread over the CTAs
  const uint16_t* pf;
  long long pf_bytes;      // multiple of 16 KB, or 0
  // split tiles: cluster > 1 runs each output tile on one thread-block cluster of that
  // many CTAs (k ranges in rank order, partials summed in the rank-0 CTA's shared memory);
  // otherwise stream-K over the grid with partials in `scratch`
  int cluster;
  float* scratch;          // gridDim.x * 2 * 128 * NT floats
  unsigned int* counters;  // one per (m-tile, token tile), zero between launches
  int stages;
  uint32_t tmem_cols;
  int* err;
};

size_t tc_proj_smem(int NT, int stages, int cluster, int kpu);
cudaError_t launch_tc_proj(const TcParams& p, int ctas, cudaStream_t stream, bool pdl);
// clusters of `cluster` tc_proj CTAs that can be resident at once (0: none, or an error)
int tc_proj_max_clusters(int epi, int NT, int stages, int cluster, int kpu);

// x (M, K) fp32 -> activation tiles of (norm_w * x) (norm_w may be null) and, if ss is
// non-null, per-token sums of squares of x in ss[0][t] (ss[1..6][t] = 0; K must be 896).
cudaError_t launch_act_tiles(const float* x, const float* norm_w, int M, int K, int NT, uint16_t* act, float* ss,
                             int ss_ld, cudaStream_t stream, bool pdl);

}  // namespace qi
