// Internal launcher interfaces shared by the .cu files of libqi.so.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "kv_layout.h"

namespace qi {

// Key splits per query token that the attention split merge supports.
constexpr int kMaxAttnSplits = 128;

enum GemvEpilogue : int {
  kEpiQkvRope = 0,   // bias + RoPE; q -> fp32 buffer, k/v -> bf16 cache
  kEpiResidual = 1,  // out[t, n] += value
  kEpiSwiglu = 2,    // h[t, i] = silu(gate) * up (gate/up rows interleaved)
  kEpiLogits = 3,    // optional logits store + packed argmax
};

struct GemvParams {
  const uint16_t* w;       // tiled weights
  int K;                   // full inner dimension
  int kr;                  // inner range per split (multiple of 64)
  int n_groups;            // output rows / 8
  int wpg;                 // warps per 8-row group (1, 2, 4, 8)
  int slots;               // weight slots (in groups) of the shared-memory ring
  int M;                   // tokens
  const float* act;        // (., K) fp32 input rows
  long long act_stride;    // floats between consecutive token rows
  const int32_t* act_rows; // optional token -> input row index (lm_head gather)
  const float* norm_w;     // RMSNorm weight (fp32) for norm-prologue kernels
  float eps;
  // epilogues
  float* out;
  int out_ld;
  const float* bias;
  const float* rope_cos;
  const float* rope_sin;
  const int32_t* pos;
  const int32_t* rows;
  uint16_t* kc;
  uint16_t* vc;
  int max_len;
  void* logits;
  int logits_bf16;
  long long logits_ld;
  unsigned long long* argmax;
  int* err;
};

// Dynamic shared memory of one GEMV CTA (mt tokens per chunk, kr columns, slots groups).
size_t gemv_smem_bytes(int mt, int kr, int slots);

// Launch a GEMV of the given epilogue with mt tokens per chunk (1, 2, 4 or 8);
// splits > 1 only for kEpiResidual. kEpiLogits requires M <= mt.
cudaError_t launch_gemv(int epi, int mt, GemvParams p, int ctas, int splits, cudaStream_t stream, bool pdl);

struct AttnParams {
  const float* q;
  const uint16_t* kc;
  const uint16_t* vc;
  const int32_t* pos;
  const int32_t* rows;
  int M;
  int max_len;
  int cache_rows;  // rows of the cache (0: rows are not checked)
  KvLayout kv;     // packed (kv.table == nullptr) or paged cache
  int split_keys;
  int max_splits;
  float* out;         // fp32 (M, 896), may be null
  uint16_t* out_act;  // activation tiles (K = 896, token tile out_nt) for the o projection, may be null
  int out_nt;
  float* part;
  unsigned int* counters;
  int* err;
  // 1: every query token is the only one of its cache row in this launch's forward and
  // positions, rows and the cached keys below each position were written before it (a
  // decode step): they are read before the programmatic-launch wait
  int decode;
  // 1: the key splits of a (token, KV head) form one thread-block cluster of max_splits
  // CTAs (2..8) and are merged in split 0's shared memory; 0: merged through part/counters
  int cluster;
};

cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream, bool pdl);
// Prefill form (attention_block.cu): one CTA per (16 consecutive query tokens, KV head);
// uses q, kc, vc, pos, rows, M, max_len, cache_rows, out/out_act/out_nt, err.
cudaError_t launch_attention_block(const AttnParams& p, cudaStream_t stream, bool pdl);
// Forwards whose longest prompt has at least kBlockAttnMinRun tokens and is more than half
// of the forward's tokens run attention_block_kernel; the per-token kernel (one key split
// per query up to 4096 cache slots) measured faster below that: time to first token at a
// 4096-slot cache 2.42 vs 2.92 ms at 384 tokens, 2.95 vs 3.42 at 512, 4.45 vs 4.53 at
// 1024, batched prefills of 4 x 1024 and 2 x 2048 tokens 14.7 vs 15.3 and 17.6 vs 18.8 ms;
// single prompts of 1536 and 2048 tokens 6.94 vs 6.71 and 9.30 vs 8.13 ms. With the prompt
// length unknown, forwards of more than kBlockAttnMinTokens tokens run the block kernel.
constexpr int kBlockAttnMinRun = 1536;
constexpr int kBlockAttnMinTokens = 128;

// slots (optional): the first n_slots argmax slots are zeroed. norm_w/NT/act/ss (optional,
// all or none): also emit activation tiles of norm_w * x and per-token sums of squares for
// the tensor-core projections (tc_proj.h).
cudaError_t launch_embed(const uint16_t* embed, int vocab, const int32_t* ids, int M, float* x,
                         unsigned long long* slots, int n_slots, cudaStream_t stream, bool pdl,
                         const float* norm_w = nullptr,
                         int NT = 0, uint16_t* act = nullptr, float* ss = nullptr, int ss_ld = 0);

cudaError_t launch_move_rows(uint16_t* k, uint16_t* v, int layers, int cache_rows, int max_len,
                             int src, int dst, int length, cudaStream_t stream);

cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int M, float* out, cudaStream_t s);

cudaError_t launch_rope(float* q, int hq, float* k, int hk, int B, int S, const int32_t* pos, const float* cos_t,
                        const float* sin_t, cudaStream_t s);

// Device ordinals the per-device caches of this library cover.
constexpr int kMaxDevices = 64;

// Number of SMs of the current device (cached per device).
int sm_count();

// cudaFuncAttributeMaxDynamicSharedMemorySize >= bytes for `kernel` on the current device
// (set once per device and kernel; thread-safe).
cudaError_t set_max_dynamic_smem(const void* kernel, int bytes);

}  // namespace qi
