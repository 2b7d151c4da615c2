// The persistent (single-launch) forward: a stage table built on the host and walked by
// one cooperative kernel (forward_persistent.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"
#include "tc_proj.h"

namespace qi {

enum PStageKind : int {
  kPEmbed = 0,  // embedding gather + first activation tiles (one unit per token)
  kPAttn = 1,   // ragged attention units (split, KV head, token)
  kPGemm = 2,   // tensor-core projection (tc_proj units and epilogue)
};

struct PEmbed {
  const uint16_t* table;  // tiled (vocab, 896)
  int vocab;
  const int32_t* ids;
  const float* norm_w;    // first layer's input RMSNorm weight
  float* x;
  uint16_t* act;
  float* ss;
  unsigned long long* slots;  // argmax slots to zero (may be null)
  int n_slots;                // how many (the head tokens)
};

// One stage of the forward. A stage may start only when stage `dep` has counted
// `target` completions (tiles, finished (token, head) pairs or tokens). A projection
// stage runs on CTAs 0..ctas-1 (its stream-K grid); the others stream later stages.
struct PStage {
  int kind;
  int dep;
  int target;
  int ctas;
  TcParams tc;
  AttnParams at;
  PEmbed em;
};

// Completion counters sit one 128-byte line apart.
constexpr int kDoneStride = 32;

struct PParams {
  const PStage* stages;  // device copy of the table
  int n_stages;
  unsigned int* done;    // counter of stage s at done[s * kDoneStride], zeroed before the launch
  int M;                 // tokens
  int NT;                // token tile (one per launch, <= 128)
  int ring;              // weight/activation pipeline slots
  uint32_t tmem_cols;
  int* err;
  unsigned long long* trace;  // optional: finish time (ns) of each stage, then the start time
};

size_t persistent_smem_bytes(int NT, int ring);
int persistent_ring(int NT);
cudaError_t launch_persistent(const PParams& p, int ctas, cudaStream_t stream);

}  // namespace qi
