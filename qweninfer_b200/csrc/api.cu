// extern "C" entry points of libqi.so (declared in include/qi.h).
//
// Host-side argument checks and launch planning live here; the kernels are in
// gemv.cu, attention.cu and misc.cu. Nothing here allocates device memory.
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "internal.h"
#include "tc_proj.h"

#include <map>
#include <vector>

using namespace qi;

namespace {

constexpr int kVersion = 100;                 // 0.1.0
constexpr size_t kSmemBudget = 200 * 1024;    // per GEMV CTA

inline cudaStream_t as_stream(qi_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }
inline int rc(cudaError_t e) { return e == cudaSuccess ? QI_OK : (int)e; }

// Token-chunk size of a GEMV: the smallest of 1, 2, 4, 8 covering M, capped by mt_max.
inline int pick_mt(int M, int mt_max) {
  int mt = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
  return mt < mt_max ? mt : mt_max;
}

// Plan and launch one CUDA-core GEMV over an (n_rows, K) tiled weight: one CTA per
// SM-sized slice of 8-row groups, all 8 warps on each group, and as many groups resident
// in the shared-memory ring as the budget allows (the rest stream through it).
int run_gemv(int epi, GemvParams p, int n_rows, int K, int ctas, int mt_max, cudaStream_t s, bool pdl) {
  p.K = K;
  p.kr = K;
  p.n_groups = n_rows / kGroupRows;
  p.wpg = 8;
  if (ctas > p.n_groups) ctas = p.n_groups;
  const int gmax = (p.n_groups + ctas - 1) / ctas;
  const int mt = pick_mt(p.M, mt_max);
  const size_t group_bytes = (size_t)(K / kTileK) * kGroupChunkBytes;
  const size_t fixed = gemv_smem_bytes(mt, K, 0);
  if (fixed + group_bytes + 8 > kSmemBudget) return QI_ERR_ARG;
  int fit = (int)((kSmemBudget - fixed) / (group_bytes + 8));
  p.slots = gmax < fit ? gmax : fit;
  return rc(launch_gemv(epi, mt, p, ctas, 1, s, pdl));
}

GemvParams blank_params(int M, int* err) {
  GemvParams p = {};
  p.M = M;
  p.err = err;
  p.eps = 1e-6f;
  return p;
}

int qkv(const float* x, const float* ln_w, float eps, const uint16_t* w_qkv, const float* b_qkv,
        const float* cos_t, const float* sin_t, const int32_t* pos, const int32_t* rows, int M,
        uint16_t* kl, uint16_t* vl, int max_len, float* q_out, int* err, cudaStream_t s, bool pdl) {
  GemvParams p = blank_params(M, err);
  p.act = x;
  p.act_stride = kHidden;
  p.norm_w = ln_w;
  p.eps = eps;
  p.out = q_out;
  p.out_ld = kHidden;
  p.bias = b_qkv;
  p.rope_cos = cos_t;
  p.rope_sin = sin_t;
  p.pos = pos;
  p.rows = rows;
  p.kc = kl;
  p.vc = vl;
  p.max_len = max_len;
  p.w = w_qkv;
  return run_gemv(kEpiQkvRope, p, kQkvRows, kHidden, sm_count(), 8, s, pdl);
}

bool use_tc_clusters();

// QI_BLOCK_ATTN=0 keeps the per-token attention kernel for prefill too, =2 runs the block
// kernel for every forward of more than kBlockAttnMinTokens tokens (comparisons, profiles);
// otherwise the kernel is chosen by the forward's longest prompt
int block_attention_mode() {
  static const int mode = [] {
    const char* v = getenv("QI_BLOCK_ATTN");
    return v && v[0] == '0' ? 0 : (v && v[0] == '2' ? 2 : 1);
  }();
  return mode;
}

int attention(const float* q, const uint16_t* kl, const uint16_t* vl, const int32_t* pos, const int32_t* rows,
              int M, int max_len, int split_keys, int max_splits, float* out, float* part, unsigned int* counters,
              int* err, cudaStream_t s, bool pdl, uint16_t* out_act = nullptr, int out_nt = 0,
              int cache_rows = 0, int query_run = 0, KvLayout kv = KvLayout{}) {
  if (max_splits > kMaxAttnSplits) return QI_ERR_ARG;
  AttnParams a = {};
  a.out_act = out_act;
  a.out_nt = out_nt;
  a.q = q;
  a.kc = kl;
  a.vc = vl;
  a.pos = pos;
  a.rows = rows;
  a.M = M;
  a.max_len = max_len;
  a.cache_rows = cache_rows;
  a.split_keys = split_keys;
  a.max_splits = max_splits;
  a.out = out;
  a.part = part;
  a.counters = counters;
  a.err = err;
  a.kv = kv;
  // query_run 1: a decode step (one query token per cache row, keys below it cached by
  // earlier forwards); the kernel then starts its copies before the previous launch ends
  a.decode = query_run == 1 ? 1 : 0;
  // a prompt of kBlockAttnMinRun tokens or more that is most of the forward (or, length
  // unknown, prefill-sized query counts): blocks of 16 consecutive tokens share K/V tiles
  // on the tensor cores
  const int bm = block_attention_mode();
  if (bm == 2 ? M > kBlockAttnMinTokens
              : bm == 1 && (query_run > 0 ? query_run >= kBlockAttnMinRun && 2LL * query_run > M
                                          : M > kBlockAttnMinTokens))
    return rc(launch_attention_block(a, s, pdl));
  // splits of a token merged inside a cluster when a launch has 2..8 of them
  a.cluster = (use_tc_clusters() && max_splits >= 2 && max_splits <= 8) ? 1 : 0;
  return rc(launch_attention(a, s, pdl));
}

int oproj(const float* attn, const uint16_t* w_o, int M, float* x, int* err, cudaStream_t s, bool pdl) {
  GemvParams p = blank_params(M, err);
  p.act = attn;
  p.act_stride = kHidden;
  p.out = x;
  p.out_ld = kHidden;
  p.w = w_o;
  return run_gemv(kEpiResidual, p, kHidden, kHidden, sm_count(), 8, s, pdl);
}

int gateup(const float* x, const float* ln_w, float eps, const uint16_t* w_gu, int M, float* h, int* err,
           cudaStream_t s, bool pdl) {
  GemvParams p = blank_params(M, err);
  p.act = x;
  p.act_stride = kHidden;
  p.norm_w = ln_w;
  p.eps = eps;
  p.out = h;
  p.out_ld = kInter;
  p.w = w_gu;
  return run_gemv(kEpiSwiglu, p, kGateUpRows, kHidden, sm_count(), 8, s, pdl);
}

int down(const float* h, const uint16_t* w_down, int M, float* x, int* err, cudaStream_t s, bool pdl) {
  GemvParams p = blank_params(M, err);
  p.act = h;
  p.act_stride = kInter;
  p.out = x;
  p.out_ld = kHidden;
  p.w = w_down;
  return run_gemv(kEpiResidual, p, kHidden, kInter, sm_count(), 4, s, pdl);
}

int lm_head(const float* x, long long x_stride, const int32_t* x_rows, const float* norm_w, float eps,
            const uint16_t* embed, int vocab, int M, void* logits, int logits_bf16, long long logits_ld,
            unsigned long long* slots, int* err, cudaStream_t s, bool pdl) {
  for (int t0 = 0; t0 < M; t0 += 8) {
    const int m = M - t0 < 8 ? M - t0 : 8;
    GemvParams p = blank_params(m, err);
    if (x_rows) {
      p.act = x;
      p.act_rows = x_rows + t0;
    } else {
      p.act = x + (long long)t0 * x_stride;
    }
    p.act_stride = x_stride;
    p.norm_w = norm_w;
    p.eps = eps;
    p.w = embed;
    if (logits) {
      const size_t esz = logits_bf16 ? 2 : 4;
      p.logits = static_cast<uint8_t*>(logits) + (size_t)t0 * logits_ld * esz;
    }
    p.logits_bf16 = logits_bf16;
    p.logits_ld = logits_ld;
    p.argmax = slots + t0;
    const int r = run_gemv(kEpiLogits, p, vocab, kHidden, sm_count(), 8, s, pdl && t0 == 0);
    if (r != QI_OK) return r;
  }
  return QI_OK;
}

bool bad_ptr(const void* p) { return p == nullptr; }

inline int round_up(int a, int b) { return (a + b - 1) / b * b; }
inline bool bad_nt(int NT) { return NT < 8 || NT > 128 || (NT & (NT - 1)) != 0; }

// Token tile of a forward over M tokens: 8 up to 8 tokens, 16 up to 96, 32 up to 384,
// 64 beyond (measured on decode batches 22-64 and prefills of 32-512 tokens: about four
// or more token tiles keep more CTAs busy without splitting tiles along K and keep each
// tile's epilogue short). Non-decreasing in M, so a workspace sized for its largest token
// count covers every smaller forward. QI_MAX_TOKEN_TILE (8..128) caps it for tuning.
inline int token_tile(int M) {
  static int cap = -1;
  if (cap < 0) {
    const char* e = getenv("QI_MAX_TOKEN_TILE");
    const int v = e ? atoi(e) : 128;
    cap = (v >= 8 && v <= 128 && (v & (v - 1)) == 0) ? v : 128;
  }
  const int nt = M <= 8 ? 8 : M <= 96 ? 16 : M <= 384 ? 32 : 64;
  return nt < cap ? nt : cap;
}

// Token tiles of the forward's projections over M tokens: {qkv, o, gate/up, down} (the
// head's is chosen from its token range). Each epilogue writes its activation tiles in
// the token tile of the projection that reads them, so the tiles may differ. Gate/up has
// 76 output row tiles, enough to occupy the SMs without splitting tokens, and every
// further token tile re-streams its 17 MB of weights: 8 up to 8 tokens, 32 up to 32, 64
// up to 384, 128 beyond (measured on decode batches 1-128 and prefills of 32-512
// tokens). The others take token_tile(M). QI_TILES="a,b,c,d" (powers of two 8..128, 0 =
// the rule) overrides them for tuning.
void token_tiles(int M, int nt[4]) {
  static int env[4] = {-1, 0, 0, 0};
  if (env[0] < 0) {
    env[0] = 0;
    if (const char* e = getenv("QI_TILES")) {
      if (sscanf(e, "%d,%d,%d,%d", &env[0], &env[1], &env[2], &env[3]) != 4) env[0] = env[1] = env[2] = env[3] = 0;
      for (int i = 0; i < 4; ++i)
        if (env[i] != 0 && bad_nt(env[i])) env[i] = 0;
    }
  }
  const int t = token_tile(M);
  const int gu = M <= 8 ? 8 : M <= 32 ? 32 : M <= 384 ? 64 : 128;
  for (int i = 0; i < 4; ++i) nt[i] = env[i] ? env[i] : (i == 2 ? gu : t);
}

// Shared-memory budget of a tensor-core projection CTA for its pipeline stages, in KB:
// 192 (with two-block pipeline units, against 144: decode step at batch 1 0.792 -> 0.775
// ms, batches 22-64 0.3-0.4 % faster, 208 no better; 1024-token prefill 4.80 -> 4.59 ms).
// QI_TC_SMEM_KB overrides it for tuning experiments.
int tc_smem_budget_kb(int NT) {
  static int kb = -1;
  if (kb < 0) {
    const char* s = getenv("QI_TC_SMEM_KB");
    const int v = s ? atoi(s) : 0;
    kb = (v >= 48 && v <= 220) ? v : 0;
  }
  (void)NT;
  return kb > 0 ? kb : 192;
}

// Stream-K contributor caps of the forward's projections (qkv, o, gate/up, down, head):
// how many CTAs may share one 128-row output tile, by token tile. A shared tile costs a
// partial-sum round trip and a serial fix-up by its last contributor, which outweighs
// the extra SMs streaming its weights except for the long-K down projection (K = 4864)
// and for decode-sized QKV/o tiles; measured on the forward at batch 1-64 and 144-token
// prefill. QI_TC_CAPS="a,b,c,d,e" overrides them for tuning experiments.
void tc_caps(int caps[5], int NT) {
  static int env[5] = {-1, 0, 0, 0, 0};
  if (env[0] < 0) {
    env[0] = 0;
    if (const char* e = getenv("QI_TC_CAPS")) sscanf(e, "%d,%d,%d,%d,%d", &env[0], &env[1], &env[2], &env[3], &env[4]);
  }
  const int small[5] = {4, 4, 1, 8, 148};  // token tile <= 32 (decode)
  const int large[5] = {1, 1, 1, 6, 148};  // token tile 64, 128 (large batches, prefill)
  for (int i = 0; i < 5; ++i) caps[i] = env[0] > 0 ? (env[i] > 0 ? env[i] : 1) : (NT <= 32 ? small[i] : large[i]);
}

// How many projections ahead each projection of the forward prefetches weights into L2
// (0: none). QI_L2_PF overrides it for tuning experiments.
int l2_pf_distance() {
  static int d = -1;
  if (d < 0) {
    const char* e = getenv("QI_L2_PF");
    const int v = e ? atoi(e) : 0;
    d = (v >= 0 && v <= 8) ? v : 0;
  }
  return d;
}

// Split tiles of the per-stage projections, and attention's key splits, reduced inside
// thread-block clusters (QI_TC_CLUSTER=0 turns it off for tuning experiments: partials
// through global scratch and arrival counters everywhere).
// QI_TC_KPU=1 keeps one 64-column k block per pipeline unit (comparisons)
bool tc_units_of_two() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("QI_TC_KPU");
    on = (e && atoi(e) == 1) ? 0 : 1;
  }
  return on != 0;
}

bool use_tc_clusters() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("QI_TC_CLUSTER");
    on = (e && atoi(e) == 0) ? 0 : 1;
  }
  return on != 0;
}

// How many clusters of C projection CTAs with this shared memory can be resident at once
// (cached per configuration).
int max_clusters(int epi, int NT, int stages, int C, int kpu) {
  static std::map<long long, int> known;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const long long key = (((((long long)dev * 8 + epi) * 256 + NT) * 64 + stages) * 16 + C) * 4 + kpu;
  auto it = known.find(key);
  if (it != known.end()) return it->second;
  const int n = tc_proj_max_clusters(epi, NT, stages, C, kpu);
  known[key] = n;
  return n;
}

// Plan and launch one tensor-core projection: grid = min(SMs, units, scratch capacity),
// pipeline stages within the shared-memory budget, TMEM for two accumulators.
int run_tc(TcParams p, float* scratch, long long scratch_floats, unsigned int* counters, int counters_len,
           int ctas, cudaStream_t s, bool pdl) {
  // pipeline units of two 64-column k blocks where K allows: the MMA warp's fixed cost per
  // unit (stage barrier wait ~110 ns after its UMMAs, commit, bookkeeping; measured) is
  // then paid once per 128 columns
  p.kpu = (p.KB % 2 == 0 && tc_units_of_two()) ? 2 : 1;
  p.KB /= p.kpu;
  const long long units = (long long)p.n_mtiles * p.n_ntiles * p.KB;
  if ((long long)p.n_mtiles * p.n_ntiles > counters_len) return QI_ERR_ARG;
  int g = ctas > 0 ? ctas : sm_count();
  if (g > units) g = (int)units;
  const long long per_cta = 2LL * 128 * p.NT;
  if (scratch_floats / per_cta < g) g = (int)(scratch_floats / per_cta);
  if (g < 1) return QI_ERR_ARG;
  // Deep pipelines: a CTA streams at (bytes in flight) / (loaded DRAM latency, ~3 us), so
  // ~130 KB must be in flight per SM to reach the HBM rate.
  const size_t stage = (size_t)p.kpu * (16384 + (size_t)p.NT * 256);
  int stages = (int)((size_t)tc_smem_budget_kb(p.NT) * 1024 / stage);
  stages = stages < 2 ? 2 : (stages > 12 ? 12 : stages);
  // Split tiles on thread-block clusters when every tile has the same number C (2..8) of
  // contributors: the partials then travel through distributed shared memory instead of a
  // global round trip and a counter. The receive buffer comes out of the ring's budget.
  // Only in one wave: the clusters of all tiles resident at once (a cluster's CTAs share a
  // GPC, so fewer CTAs per tile may fit where the stream-K grid would not).
  p.cluster = 0;
  const long long tiles = (long long)p.n_mtiles * p.n_ntiles;
  if (use_tc_clusters() && p.epi != kTcLogits && g >= 2 * tiles) {
    int C = (int)(g / tiles);
    if (C > 8) C = 8;
    if (C > p.KB) C = p.KB;
    for (; C >= 2; --C) {
      const size_t room = 227 * 1024 - tc_proj_smem(p.NT, 0, C, p.kpu);
      int st = (int)(room / (stage + 16));
      if (st > stages) st = stages;
      if (st >= 2 && tiles <= max_clusters(p.epi, p.NT, st, C, p.kpu)) {
        p.cluster = C;
        stages = st;
        g = (int)(tiles * C);
        break;
      }
    }
  }
  uint32_t cols = 32;
  while (cols < (uint32_t)(4 * p.NT)) cols <<= 1;
  p.lg_nt = 0;
  while ((1 << p.lg_nt) < p.NT) ++p.lg_nt;
  if (p.out_nt == 0) p.out_nt = p.NT;
  p.lg_out_nt = 0;
  while ((1 << p.lg_out_nt) < p.out_nt) ++p.lg_out_nt;
  p.scratch = scratch;
  p.counters = counters;
  p.stages = stages;
  p.tmem_cols = cols;
  return rc(launch_tc_proj(p, g, s, pdl));
}

// Stream-K grid of a projection with n_tiles output tiles of KB k-blocks each: enough
// contributors per tile to cover the SMs, but at most max_contrib, because the last
// contributor of a split tile reads every other contributor's partial.
int grid_for(int n_tiles, int KB, int max_contrib) {
  const int sms = sm_count();
  int per = (sms + n_tiles - 1) / n_tiles;
  if (per > max_contrib) per = max_contrib;
  if (per > KB) per = KB;
  const long long g = (long long)n_tiles * per;
  return (int)(g < sms ? g : sms);
}

// qi_forward on the tensor-core path: every projection is a tc_proj launch whose
// epilogue writes the next projection's activation tiles (the RMSNorm weights folded in,
// the per-token RMS applied in the consumer's epilogue from partial sums of squares).
// The cache's KV layout and the elements one layer's K (or V) takes.
KvLayout kv_layout(const qi_cache* c) {
  KvLayout kv = {};
  if (c->page_table) {
    kv.table = c->page_table;
    kv.page = c->page_size;
    kv.ppr = c->pages_per_row;
    kv.n_pages = c->n_pages;
  }
  return kv;
}
long long layer_kv_elems(const qi_cache* c) {
  return c->page_table ? (long long)c->n_pages * kKvHeads * c->page_size * kHeadDim
                       : (long long)c->cache_rows * kKvHeads * c->max_len * kHeadDim;
}
bool bad_paging(const qi_cache* c) {
  return c->page_table && (c->page_size < 128 || c->page_size % 128 != 0 || c->n_pages < 1 ||
                           (long long)c->pages_per_row * c->page_size < c->max_len);
}

// Per-launch device times of one forward: an event recorded before the first launch and
// after every launch (qi_forward_launch_times). The events separate the launches, so each
// time is the launch's own duration without the programmatic-dependent-launch overlap.
struct LaunchTimer {
  cudaStream_t s;
  std::vector<cudaEvent_t> ev;
  std::vector<int> kind;
  int mark(int k) {
    cudaEvent_t e;
    const int r = rc(cudaEventCreate(&e));
    if (r != QI_OK) return r;
    ev.push_back(e);
    kind.push_back(k);
    return rc(cudaEventRecord(e, s));
  }
  ~LaunchTimer() {
    for (cudaEvent_t e : ev) cudaEventDestroy(e);
  }
};

int forward_tc(const qi_model* model, const qi_cache* cache, const qi_workspace* ws, const int32_t* ids,
               const int32_t* pos, const int32_t* rows, int M, int head_lo, int head_stride, int n_head,
               void* logits, int logits_bf16, long long logits_ld, unsigned long long* slots, cudaStream_t s,
               LaunchTimer* lt = nullptr) {
  int tiles[5];
  token_tiles(M, tiles);
  // a workspace padded less than to 128 tokens gets the largest tiles that fit it
  for (int i = 0; i < 4; ++i)
    while (tiles[i] > 8 && (M + tiles[i] - 1) / tiles[i] * tiles[i] > ws->ss_ld) tiles[i] >>= 1;
  const int NT = tiles[0];
  for (int i = 0; i < 4; ++i)
    if ((M + tiles[i] - 1) / tiles[i] * tiles[i] > ws->ss_ld) return QI_ERR_ARG;
  // head token tile: the smallest (from the qkv tile up to 128) that holds all head tokens
  // in one tile, so that the 272 MB head weights are streamed once per forward
  const int head_hi = n_head > 0 ? head_lo + (n_head - 1) * head_stride + 1 : 0;
  tiles[4] = NT;
  while (n_head > 0 && tiles[4] < 128 && head_lo / tiles[4] != (head_hi - 1) / tiles[4] &&
         (M + 2 * tiles[4] - 1) / (2 * tiles[4]) * (2 * tiles[4]) <= ws->ss_ld)
    tiles[4] <<= 1;
  if (!ws->act_x || !ws->act_attn || !ws->act_h || !ws->ss || !ws->tc_scratch || !ws->tc_counters)
    return QI_ERR_ARG;
  const bool pdl = true;
  auto mark = [&](int kind) { return lt ? lt->mark(kind) : QI_OK; };
  int r = mark(-1);
  if (r != QI_OK) return r;
  r = rc(launch_embed(model->embed, model->vocab, ids, M, ws->x, slots, n_head, s, false, model->layers[0].ln1, NT,
                      ws->act_x, ws->ss, ws->ss_ld));
  if (r != QI_OK || (r = mark(QI_LAUNCH_EMBED)) != QI_OK) return r;
  TcParams base = {};
  base.M = M;
  base.ss_ld = ws->ss_ld;
  base.eps = model->eps;
  base.err = ws->err;
  // projection j (0 qkv, 1 o, 2 gate/up, 3 down, 4 head) over token tile tiles[j],
  // writing activation tiles of token tile out_nt
  auto params = [&](int j, int out_nt) {
    TcParams p = base;
    p.NT = tiles[j];
    p.n_ntiles = (M + p.NT - 1) / p.NT;
    p.out_nt = out_nt;
    return p;
  };
  // L2 prefetch: projection i of the forward's sequence (4 per layer) prefetches the
  // weights of projection i + l2_pf_distance()
  auto prefetch = [&](TcParams& p, int i) {
    const int d = l2_pf_distance(), t = i + d;
    if (d <= 0 || t >= 4 * model->num_layers) return;
    const qi_layer& L = model->layers[t / 4];
    const uint16_t* w[4] = {L.w_qkv, L.w_o, L.w_gate_up, L.w_down};
    const long long rows[4] = {kQkvRows, kHidden, kGateUpRows, kHidden};
    const long long K[4] = {kHidden, kHidden, kHidden, kInter};
    p.pf = w[t % 4];
    p.pf_bytes = rows[t % 4] * K[t % 4] * 2;
  };
  auto launch = [&](TcParams& p, int j) {
    int caps[5];
    tc_caps(caps, p.NT);
    const int g = grid_for(p.n_mtiles * p.n_ntiles, p.KB, caps[j]);
    const int kinds[5] = {QI_LAUNCH_QKV, QI_LAUNCH_O, QI_LAUNCH_GATE_UP, QI_LAUNCH_DOWN, QI_LAUNCH_HEAD};
    const int r = run_tc(p, ws->tc_scratch, ws->tc_scratch_floats, ws->tc_counters, ws->tc_counters_len, g, s, pdl);
    return r != QI_OK ? r : mark(kinds[j]);
  };
  const KvLayout kv = kv_layout(cache);
  const long long layer_elems = layer_kv_elems(cache);
  for (int li = 0; li < model->num_layers; ++li) {
    const qi_layer& L = model->layers[li];
    uint16_t* kl = cache->k + li * layer_elems;
    uint16_t* vl = cache->v + li * layer_elems;
    TcParams p = params(0, 0);  // RMSNorm + QKV + bias + RoPE + KV append
    p.kv = kv;
    p.w = L.w_qkv;
    p.KB = kHidden / 64;
    p.n_mtiles = kQkvRows / 128;
    p.act_in = ws->act_x;
    p.ss_in = ws->ss;
    p.epi = cache->page_table ? kTcQkvRopePaged : kTcQkvRope;
    p.bias = L.b_qkv;
    p.rope_cos = model->rope_cos;
    p.rope_sin = model->rope_sin;
    p.pos = pos;
    p.rows = rows;
    p.q = ws->q;
    p.kc = kl;
    p.vc = vl;
    p.max_len = cache->max_len;
    p.cache_rows = cache->cache_rows;
    prefetch(p, 4 * li);
    if ((r = launch(p, 0)) != QI_OK) return r;
    r = attention(ws->q, kl, vl, pos, rows, M, cache->max_len, ws->split_keys, ws->max_splits, nullptr,
                  ws->attn_part, ws->attn_counters, ws->err, s, pdl, ws->act_attn, tiles[1], cache->cache_rows,
                  ws->query_run, kv);
    if (r != QI_OK || (r = mark(QI_LAUNCH_ATTENTION)) != QI_OK) return r;
    p = params(1, tiles[2]);  // o_proj + residual; emits RMSNorm(post_attention) inputs
    p.w = L.w_o;
    p.KB = kHidden / 64;
    p.n_mtiles = kHidden / 128;
    p.act_in = ws->act_attn;
    p.epi = kTcResidual;
    p.x = ws->x;
    p.next_norm_w = L.ln2;
    p.act_out = ws->act_x;
    p.ss_out = ws->ss;
    prefetch(p, 4 * li + 1);
    if ((r = launch(p, 1)) != QI_OK) return r;
    p = params(2, tiles[3]);  // gate/up + SwiGLU
    p.w = L.w_gate_up;
    p.KB = kHidden / 64;
    p.n_mtiles = kGateUpRows / 128;
    p.act_in = ws->act_x;
    p.ss_in = ws->ss;
    p.epi = kTcSwiglu;
    p.act_out = ws->act_h;
    prefetch(p, 4 * li + 2);
    if ((r = launch(p, 2)) != QI_OK) return r;
    p = params(3, tiles[li + 1 < model->num_layers ? 0 : 4]);  // down + residual; emits the next norm's inputs
    p.w = L.w_down;
    p.KB = kInter / 64;
    p.n_mtiles = kHidden / 128;
    p.act_in = ws->act_h;
    p.epi = kTcResidual;
    p.x = ws->x;
    p.next_norm_w = li + 1 < model->num_layers ? model->layers[li + 1].ln1 : model->norm;
    p.act_out = ws->act_x;
    p.ss_out = ws->ss;
    prefetch(p, 4 * li + 3);
    if ((r = launch(p, 3)) != QI_OK) return r;
  }
  if (n_head > 0) {
    for (int nt = head_lo / tiles[4]; nt <= (head_hi - 1) / tiles[4]; ++nt) {
      TcParams p = params(4, 0);  // final RMSNorm + tied head + argmax, one token tile per launch
      p.w = model->embed;
      p.KB = kHidden / 64;
      p.n_mtiles = model->vocab / 128;
      p.act_in = ws->act_x;
      p.ss_in = ws->ss;
      p.n_ntiles = 1;
      p.ntile0 = nt;
      p.epi = kTcLogits;
      p.logits = logits;
      p.logits_bf16 = logits_bf16;
      p.logits_ld = logits_ld;
      p.argmax = slots;
      p.head_lo = head_lo;
      p.head_hi = head_hi;
      p.head_stride = head_stride;
      if ((r = launch(p, 4)) != QI_OK) return r;
    }
  }
  return QI_OK;
}

bool bad_forward_args(const qi_model* model, const qi_cache* cache, const qi_workspace* ws, const int32_t* ids,
                      const int32_t* pos, const int32_t* rows, int M, int head_lo, int head_stride, int n_head,
                      const void* logits, long long logits_ld, const unsigned long long* argmax_slots) {
  return !model || !cache || !ws || !model->layers || M <= 0 || M > ws->max_tokens || n_head < 0 ||
         (n_head > 0 &&
          (head_lo < 0 || head_stride < 1 || (long long)head_lo + (long long)(n_head - 1) * head_stride >= M)) ||
         bad_ptr(ids) || bad_ptr(pos) || bad_ptr(rows) || (n_head > 0 && bad_ptr(argmax_slots)) ||
         (logits && logits_ld < model->vocab) || model->vocab % kTileRows != 0 || model->num_layers <= 0 ||
         ws->split_keys % 128 != 0 || (long long)ws->split_keys * ws->max_splits < cache->max_len ||
         ws->max_splits > kMaxAttnSplits || cache->max_len > model->max_seq;
}

}  // namespace

extern "C" {

int qi_version(void) { return kVersion; }

int qi_init(int device) {
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return (int)e;
  int major = 0;
  e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (e != cudaSuccess) return (int)e;
  if (major != 10) return QI_ERR_DEVICE;
  (void)sm_count();
  return QI_OK;
}

long long qi_tile_offset(int n, int k, int K) { return tiled_offset(n, k, K); }

int qi_embed(const uint16_t* embed, int vocab, const int32_t* ids, int M, float* x,
             unsigned long long* argmax_slots, int* err, qi_stream_t stream) {
  (void)err;
  if (M <= 0 || vocab <= 0 || bad_ptr(embed) || bad_ptr(ids) || bad_ptr(x)) return QI_ERR_ARG;
  return rc(launch_embed(embed, vocab, ids, M, x, argmax_slots, M, as_stream(stream), false));
}

int qi_qkv_rope_append(const float* x, const float* ln_w, float eps, const uint16_t* w_qkv,
                       const float* b_qkv, const float* rope_cos, const float* rope_sin,
                       const int32_t* pos, const int32_t* rows, int M, uint16_t* k_layer,
                       uint16_t* v_layer, int max_len, float* q_out, int* err, qi_stream_t stream) {
  if (M <= 0 || max_len <= 0 || bad_ptr(x) || bad_ptr(w_qkv) || bad_ptr(b_qkv) ||
      bad_ptr(rope_cos) || bad_ptr(rope_sin) || bad_ptr(pos) || bad_ptr(rows) || bad_ptr(k_layer) ||
      bad_ptr(v_layer) || bad_ptr(q_out))
    return QI_ERR_ARG;
  return qkv(x, ln_w, eps, w_qkv, b_qkv, rope_cos, rope_sin, pos, rows, M, k_layer, v_layer, max_len, q_out,
             err, as_stream(stream), false);
}

int qi_attention(const float* q, const uint16_t* k_layer, const uint16_t* v_layer, const int32_t* pos,
                 const int32_t* rows, int M, int max_len, int split_keys, int max_splits, float* out,
                 float* part, unsigned int* counters, int* err, qi_stream_t stream) {
  if (M <= 0 || max_len <= 0 || split_keys <= 0 || split_keys % 128 != 0 || max_splits <= 0 ||
      (long long)split_keys * max_splits < max_len || bad_ptr(q) || bad_ptr(k_layer) || bad_ptr(v_layer) ||
      bad_ptr(pos) || bad_ptr(rows) || bad_ptr(out) || (max_splits > 1 && (bad_ptr(part) || bad_ptr(counters))))
    return QI_ERR_ARG;
  return attention(q, k_layer, v_layer, pos, rows, M, max_len, split_keys, max_splits, out, part, counters, err,
                   as_stream(stream), false);
}

int qi_o_proj_residual(const float* attn, const uint16_t* w_o, int M, float* x, int* err, qi_stream_t stream) {
  if (M <= 0 || bad_ptr(attn) || bad_ptr(w_o) || bad_ptr(x)) return QI_ERR_ARG;
  return oproj(attn, w_o, M, x, err, as_stream(stream), false);
}

int qi_gate_up_swiglu(const float* x, const float* ln_w, float eps, const uint16_t* w_gate_up, int M, float* h,
                      int* err, qi_stream_t stream) {
  if (M <= 0 || bad_ptr(x) || bad_ptr(w_gate_up) || bad_ptr(h)) return QI_ERR_ARG;
  return gateup(x, ln_w, eps, w_gate_up, M, h, err, as_stream(stream), false);
}

int qi_down_residual(const float* h, const uint16_t* w_down, int M, float* x, int* err, qi_stream_t stream) {
  if (M <= 0 || bad_ptr(h) || bad_ptr(w_down) || bad_ptr(x)) return QI_ERR_ARG;
  return down(h, w_down, M, x, err, as_stream(stream), false);
}

int qi_lm_head_argmax(const float* x, long long x_stride, const float* norm_w, float eps, const uint16_t* embed,
                      int vocab, int M, void* logits, int logits_bf16, long long logits_ld,
                      unsigned long long* argmax_slots, int* err, qi_stream_t stream) {
  if (M <= 0 || vocab <= 0 || vocab % kTileRows != 0 || x_stride < kHidden || bad_ptr(x) || bad_ptr(norm_w) ||
      bad_ptr(embed) || bad_ptr(argmax_slots) || (logits && logits_ld < vocab))
    return QI_ERR_ARG;
  return lm_head(x, x_stride, nullptr, norm_w, eps, embed, vocab, M, logits, logits_bf16, logits_ld, argmax_slots,
                 err, as_stream(stream), false);
}

int qi_rmsnorm(const float* x, const float* w, float eps, int M, float* out, qi_stream_t stream) {
  if (M <= 0 || bad_ptr(x) || bad_ptr(w) || bad_ptr(out)) return QI_ERR_ARG;
  return rc(launch_rmsnorm(x, w, eps, M, out, as_stream(stream)));
}

int qi_rope(float* q, int q_heads, float* k, int k_heads, int B, int S, const int32_t* pos, const float* rope_cos,
            const float* rope_sin, qi_stream_t stream) {
  if (B <= 0 || S <= 0 || q_heads < 0 || k_heads < 0 || bad_ptr(pos) || bad_ptr(rope_cos) || bad_ptr(rope_sin) ||
      (q_heads > 0 && bad_ptr(q)) || (k_heads > 0 && bad_ptr(k)))
    return QI_ERR_ARG;
  return rc(launch_rope(q, q_heads, k, k_heads, B, S, pos, rope_cos, rope_sin, as_stream(stream)));
}

int qi_move_rows(uint16_t* k, uint16_t* v, int layers, int cache_rows, int max_len, const int32_t* moves,
                 int n_moves, qi_stream_t stream) {
  if (layers <= 0 || cache_rows <= 0 || max_len <= 0 || n_moves < 0 || bad_ptr(k) || bad_ptr(v) ||
      (n_moves > 0 && bad_ptr(moves)))
    return QI_ERR_ARG;
  for (int i = 0; i < n_moves; ++i) {
    const int src = moves[3 * i], dst = moves[3 * i + 1], len = moves[3 * i + 2];
    if (src < 0 || src >= cache_rows || dst < 0 || dst >= cache_rows || len < 0 || len > max_len) return QI_ERR_ARG;
  }
  for (int i = 0; i < n_moves; ++i) {
    const int r = rc(launch_move_rows(k, v, layers, cache_rows, max_len, moves[3 * i], moves[3 * i + 1],
                                      moves[3 * i + 2], as_stream(stream)));
    if (r != QI_OK) return r;
  }
  return QI_OK;
}

int qi_act_tiles(const float* x, const float* norm_w, int M, int K, int NT, uint16_t* act, float* ss, int ss_ld,
                 qi_stream_t stream) {
  if (M <= 0 || K <= 0 || K % 64 != 0 || bad_nt(NT) || bad_ptr(x) || bad_ptr(act) ||
      (ss && (K != kHidden || ss_ld < round_up(M, NT))))
    return QI_ERR_ARG;
  return rc(launch_act_tiles(x, norm_w, M, K, NT, act, ss, ss_ld, as_stream(stream), false));
}

int qi_tc_linear(const uint16_t* w, int n_rows, int K, const uint16_t* act, int M, int NT, const float* ss, int ss_ld,
                 float eps, float* out, int out_ld, float* scratch, long long scratch_floats, unsigned int* counters,
                 int counters_len, int ctas, int* err, qi_stream_t stream) {
  if (M <= 0 || n_rows <= 0 || n_rows % 128 != 0 || K <= 0 || K % 64 != 0 || bad_nt(NT) || bad_ptr(w) ||
      bad_ptr(act) || bad_ptr(out) || out_ld < n_rows || bad_ptr(scratch) || bad_ptr(counters) ||
      (ss && (K != kHidden || ss_ld < round_up(M, NT))))
    return QI_ERR_ARG;
  TcParams p = {};
  p.w = w;
  p.KB = K / 64;
  p.n_mtiles = n_rows / 128;
  p.act_in = act;
  p.NT = NT;
  p.n_ntiles = (M + NT - 1) / NT;
  p.M = M;
  p.ss_in = ss;
  p.ss_ld = ss_ld;
  p.eps = eps;
  p.epi = kTcPlain;
  p.out = out;
  p.out_ld = out_ld;
  p.err = err;
  return run_tc(p, scratch, scratch_floats, counters, counters_len, ctas, as_stream(stream), false);
}

int qi_tc_gate_up_swiglu(const uint16_t* w_gate_up, const uint16_t* act, int M, int NT, const float* ss, int ss_ld,
                         float eps, uint16_t* act_out, float* scratch, long long scratch_floats,
                         unsigned int* counters, int counters_len, int ctas, int* err, qi_stream_t stream) {
  if (M <= 0 || bad_nt(NT) || bad_ptr(w_gate_up) || bad_ptr(act) || bad_ptr(act_out) || bad_ptr(scratch) ||
      bad_ptr(counters) || (ss && ss_ld < round_up(M, NT)))
    return QI_ERR_ARG;
  TcParams p = {};
  p.w = w_gate_up;
  p.KB = kHidden / 64;
  p.n_mtiles = kGateUpRows / 128;
  p.act_in = act;
  p.NT = NT;
  p.n_ntiles = (M + NT - 1) / NT;
  p.M = M;
  p.ss_in = ss;
  p.ss_ld = ss_ld;
  p.eps = eps;
  p.epi = kTcSwiglu;
  p.act_out = act_out;
  p.err = err;
  if (ctas <= 0) {  // the forward's partition
    int caps[5];
    tc_caps(caps, NT);
    ctas = grid_for(p.n_mtiles * p.n_ntiles, p.KB, caps[2]);
  }
  return run_tc(p, scratch, scratch_floats, counters, counters_len, ctas, as_stream(stream), false);
}

int qi_forward(const qi_model* model, const qi_cache* cache, const qi_workspace* ws, const int32_t* ids,
               const int32_t* pos, const int32_t* rows, int M, int head_lo, int head_stride, int n_head,
               void* logits, int logits_bf16, long long logits_ld, unsigned long long* argmax_slots,
               qi_stream_t stream) {
  if (bad_forward_args(model, cache, ws, ids, pos, rows, M, head_lo, head_stride, n_head, logits, logits_ld,
                       argmax_slots) ||
      bad_paging(cache) || (cache->page_table && !ws->use_tc))
    return QI_ERR_ARG;
  if (ws->use_tc) return forward_tc(model, cache, ws, ids, pos, rows, M, head_lo, head_stride, n_head, logits,
                                    logits_bf16, logits_ld, argmax_slots, as_stream(stream));
  cudaStream_t s = as_stream(stream);
  const bool pdl = true;
  int r = rc(launch_embed(model->embed, model->vocab, ids, M, ws->x, argmax_slots, n_head, s, false));
  if (r != QI_OK) return r;
  const long long layer_elems = (long long)cache->cache_rows * kKvHeads * cache->max_len * kHeadDim;
  for (int li = 0; li < model->num_layers; ++li) {
    const qi_layer& L = model->layers[li];
    uint16_t* kl = cache->k + li * layer_elems;
    uint16_t* vl = cache->v + li * layer_elems;
    r = qkv(ws->x, L.ln1, model->eps, L.w_qkv, L.b_qkv, model->rope_cos, model->rope_sin, pos, rows, M, kl, vl,
            cache->max_len, ws->q, ws->err, s, pdl);
    if (r != QI_OK) return r;
    r = attention(ws->q, kl, vl, pos, rows, M, cache->max_len, ws->split_keys, ws->max_splits, ws->attn,
                  ws->attn_part, ws->attn_counters, ws->err, s, pdl, nullptr, 0, cache->cache_rows);
    if (r != QI_OK) return r;
    r = oproj(ws->attn, L.w_o, M, ws->x, ws->err, s, pdl);
    if (r != QI_OK) return r;
    r = gateup(ws->x, L.ln2, model->eps, L.w_gate_up, M, ws->h, ws->err, s, pdl);
    if (r != QI_OK) return r;
    r = down(ws->h, L.w_down, M, ws->x, ws->err, s, pdl);
    if (r != QI_OK) return r;
  }
  if (n_head > 0)
    r = lm_head(ws->x + (long long)head_lo * kHidden, (long long)head_stride * kHidden, nullptr, model->norm,
                model->eps, model->embed, model->vocab, n_head, logits, logits_bf16, logits_ld, argmax_slots,
                ws->err, s, pdl);
  return r;
}

int qi_forward_launch_times(const qi_model* model, const qi_cache* cache, const qi_workspace* ws,
                            const int32_t* ids, const int32_t* pos, const int32_t* rows, int M, int head_lo,
                            int head_stride, int n_head, void* logits, int logits_bf16, long long logits_ld,
                            unsigned long long* argmax_slots, qi_stream_t stream, int* kinds, float* us,
                            int max_launches, int* n_launches) {
  if (bad_forward_args(model, cache, ws, ids, pos, rows, M, head_lo, head_stride, n_head, logits, logits_ld,
                       argmax_slots) ||
      bad_paging(cache) || !ws->use_tc || !kinds || !us || !n_launches || max_launches <= 0)
    return QI_ERR_ARG;
  LaunchTimer lt;
  lt.s = as_stream(stream);
  int r = forward_tc(model, cache, ws, ids, pos, rows, M, head_lo, head_stride, n_head, logits, logits_bf16,
                     logits_ld, argmax_slots, lt.s, &lt);
  if (r != QI_OK) return r;
  if ((r = rc(cudaStreamSynchronize(lt.s))) != QI_OK) return r;
  const int n = (int)lt.ev.size() - 1;
  if (n > max_launches) return QI_ERR_TOO_LARGE;
  for (int i = 0; i < n; ++i) {
    kinds[i] = lt.kind[i + 1];
    if ((r = rc(cudaEventElapsedTime(&us[i], lt.ev[i], lt.ev[i + 1]))) != QI_OK) return r;
    us[i] *= 1000.f;
  }
  *n_launches = n;
  return QI_OK;
}

}  // extern "C"
