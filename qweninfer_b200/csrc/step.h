// The decode-step kernel (step.cu): one cooperative launch runs the whole forward of a
// decode step of up to 32 tokens (embedding, every layer, head + argmax).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "step_plan.h"

namespace qi {

struct StepLayer {
  const uint16_t* w_qkv;  // tiled (1152, 896), RoPE-pair row order
  const uint16_t* w_o;    // tiled (896, 896)
  const uint16_t* w_gu;   // tiled (9728, 896), gate/up interleaved
  const uint16_t* w_down; // tiled (896, 4864)
  const float* b_qkv;
  const float* ln1;
  const float* ln2;
};

struct StepParams {
  StepLayer L[step::kMaxLayers];
  int n_layers;
  const uint16_t* embed;  // tiled (vocab, 896)
  int vocab;
  const float* norm_w;
  float eps;
  const float* rope_cos;
  const float* rope_sin;
  const int32_t* ids;
  const int32_t* pos;
  const int32_t* rows;
  int M;   // tokens (one per cache row)
  int NT;  // token tile: 8, 16 or 32 (>= M)
  uint16_t* kc;
  uint16_t* vc;
  long long layer_elems;  // cache elements per layer (K or V)
  int cache_rows;
  int max_len;
  float* x;            // (NT, 896) residual stream
  float* q;            // (NT, 896) rotated queries
  uint16_t* act_x;     // activation tiles (K = 896, token tile NT)
  uint16_t* act_attn;  // activation tiles (K = 896)
  uint16_t* act_h;     // activation tiles (K = 4864)
  float* ss;           // [7][NT] sums of squares of x per 128-feature tile
  float* ss_o;         // [148][NT] sums of squares of the o projection's finishes
  float* dpart;        // [21][NT][896] down-projection partial sums
  float* apart;        // attention split partials
  unsigned int* acnt;  // attention split arrival counters (zero between launches)
  int split_keys;
  int max_splits;
  unsigned int* ctr;   // phase counters, zeroed before the launch
  void* logits;        // optional (M, logits_ld)
  int logits_bf16;
  long long logits_ld;
  unsigned long long* argmax;  // (M) packed argmax slots
  int* err;
  unsigned long long* trace;  // optional per-CTA phase timestamps (kTraceEvents per phase), or null
  int slots;           // ring slots (step_ring_slots)
  int chains;          // independent accumulators per tile (step_chains, a power of two)
  uint32_t tmem_cols;  // step_tmem_cols
};

// Optional timeline of a launch (StepParams::trace): globaltimer stamps (ns) at
// trace[(cta * kTracePhases + phase) * kTraceEvents + event], phase 0 = embedding,
// 1 + 6 l + {0 qkv, 1 attention, 2 o, 3 gate/up, 4 down, 5 reduce}, 1 + 6 layers = head.
constexpr int kTracePhases = 1 + step::kPhasesPerLayer * step::kMaxLayers + 1;
constexpr int kTraceEvents = 8;
enum StepTraceEvent : int {
  kTrEnter = 0,     // the workers start the phase
  kTrInputs = 1,    // its inputs are complete (phase counter reached)
  kTrAcc = 2,       // the first accumulator is complete (projections)
  kTrDone = 3,      // the phase's outputs are written (before the counter increment)
  kTrMmaB = 4,      // MMA thread: the activation tiles have landed
  kTrMmaLast = 5,   // MMA thread: the first unit's last UMMA is issued
  kTrRecv = 6,      // finishing rank: the peer's partial has arrived
  kTrPushed = 7,    // pushing rank: its partial is pushed
};

// Shared memory of one step CTA for token tile NT, its ring slot count, accumulator chains
// per tile and TMEM columns.
size_t step_smem_bytes(int NT);
int step_ring_slots(int NT);
int step_chains(int NT);
uint32_t step_tmem_cols(int NT);
// Launches the step kernel (cooperative, 148 CTAs); zeroes the phase counters first.
cudaError_t launch_step(const StepParams& p, cudaStream_t stream);
// Whether this device can run it (148 SMs).
bool step_supported();

}  // namespace qi
