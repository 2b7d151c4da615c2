/*
 * qi.h — C ABI of libqi.so, the sm_100a (B200) kernels behind qweninfer_b200.
 *
 * The library is the device half of a drop-in replacement for the continuous-batching
 * decode path of QwenInfer (qweninfer/models/qwen2.py, qweninfer/engine/*.py). The
 * Python package keeps QwenInfer's API and calls these entry points through ctypes.
 *
 * Conventions
 *   - Every pointer argument except the descriptor structs' host arrays is a DEVICE
 *     pointer owned by the caller (PyTorch tensors). The library never allocates or
 *     frees memory; scratch buffers are passed in.
 *   - `stream` is a cudaStream_t (the caller's current stream). Calls only enqueue work
 *     and never synchronise the host, so they can be captured in a CUDA graph.
 *   - Return value: 0 on success, a cudaError_t code from the launch, or a QI_ERR_*
 *     code for rejected arguments. Argument errors are detected on the host before any
 *     launch.
 *   - `err` is a device int the kernels set to QI_ERR_TIMEOUT if a bounded wait gives
 *     up (they never trap or spin forever); the caller reads it after synchronising.
 *   - Weights are bf16 in the tiled layout produced by qi_tile_offset's mapping
 *     (128x64 blocks of 8x8 core matrices); activations are fp32; the KV cache is bf16
 *     with QwenInfer's packed layout (layers, rows, kv_heads=2, max_len, head_dim=64).
 *   - Compiled for the Qwen2-0.5B block shape: hidden 896, 14 query heads, 2 KV heads,
 *     head_dim 64, intermediate 4864. Layer count and vocabulary are arguments.
 */
#ifndef QI_H_
#define QI_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QI_OK 0
#define QI_ERR_ARG 1001     /* an argument is out of range                          */
#define QI_ERR_TIMEOUT 1002 /* a device-side bounded wait gave up (set in *err)      */
#define QI_ERR_DEVICE 1003  /* the current device is not an sm_100 part              */
#define QI_ERR_TOO_LARGE 1004 /* size beyond a fixed-capacity entry point's maximum  */
#define QI_ERR_INDEX 1005   /* a token's position or cache row lies outside the cache
                               (set in *err by the kernels; the access is skipped)  */

typedef void* qi_stream_t; /* cudaStream_t */

/* Library version (major*10000 + minor*100 + patch). */
int qi_version(void);

/* One-time per-device setup (kernel attributes). Replaces nothing in the reference:
 * the reference calls PyTorch/cuBLAS, which set themselves up. Safe to call again. */
int qi_init(int device);

/* Element offset of W[n][k] in the tiled layout of an (N, K) matrix, N % 128 == 0,
 * K % 64 == 0. The host-side repack (Qwen2.fuse) uses this mapping. */
long long qi_tile_offset(int n, int k, int K);

/* ---------------------------------------------------------------- single ops */

/* Embedding lookup into the fp32 residual stream:
 *   x[t, :] = float(embed[ids[t], :]),  t < M.
 * Replaces the column gather of qweninfer/models/qwen2.py:273-279 (`embed_t[:, ids]`,
 * `.float()`). Also zeroes argmax_slots[0..M) (if non-null) for a following
 * qi_lm_head_argmax. `embed` is the tiled (vocab, 896) table (the tied lm_head). */
int qi_embed(const uint16_t* embed, int vocab, const int32_t* ids, int M, float* x,
             unsigned long long* argmax_slots, int* err, qi_stream_t stream);

/* Input RMSNorm + fused QKV projection + bias + RoPE + KV-cache append:
 *   xn = rmsnorm(x[t]) * ln_w;  qkv = xn @ Wqkv^T + b;  rotate q, k by pos[t];
 *   q_out[t] = q (fp32, 14x64);  K/V cache[row[t], :, pos[t], :] = bf16(k), bf16(v).
 * Replaces qweninfer/models/qwen2.py:44-48 (RMSNorm), 160-171 (QKV + bias, view,
 * apply_rope 86-99) and qweninfer/engine/kv_cache.py:48-60 (KVCache.update scatter).
 * ln_w may be NULL: x is then used as given (no normalisation).
 * w_qkv: tiled (1152, 896) with rows permuted so that RoPE pairs (d, d+32) of each head
 * are adjacent (row 2j <- dim j, row 2j+1 <- dim j+32); b_qkv permuted the same, fp32.
 * rope_cos/rope_sin: (max_seq, 64) fp32 tables of build_rope_cache (qwen2.py:53-73).
 * k_layer/v_layer: this layer's cache base, (cache_rows, 2, max_len, 64) bf16. */
int qi_qkv_rope_append(const float* x, const float* ln_w, float eps, const uint16_t* w_qkv,
                       const float* b_qkv, const float* rope_cos, const float* rope_sin,
                       const int32_t* pos, const int32_t* rows, int M, uint16_t* k_layer,
                       uint16_t* v_layer, int max_len, float* q_out, int* err, qi_stream_t stream);

/* Standalone RMSNorm of M rows of 896 fp32 values (out may alias x):
 *   out[t] = x[t] * rsqrt(mean(x[t]^2) + eps) * w.
 * Replaces RMSNorm.forward, qweninfer/models/qwen2.py:44-48, for direct calls of the
 * module; the model forward fuses the norm into qi_qkv_rope_append /
 * qi_gate_up_swiglu / qi_lm_head_argmax instead. */
int qi_rmsnorm(const float* x, const float* w, float eps, int M, float* out, qi_stream_t stream);

/* Standalone RoPE, in place, on fp32 q (B, q_heads, S, 64) and k (B, k_heads, S, 64)
 * with positions pos (B*S, int32) and the build_rope_cache tables. Replaces apply_rope /
 * _rotate_half, qweninfer/models/qwen2.py:76-99, for direct calls; the model forward
 * fuses RoPE into qi_qkv_rope_append. */
int qi_rope(float* q, int q_heads, float* k, int k_heads, int B, int S, const int32_t* pos,
            const float* rope_cos, const float* rope_sin, qi_stream_t stream);

/* Ragged GQA attention over each query's own live length (keys 0..pos[t]):
 *   out[t, h*64:(h+1)*64] = softmax(q[t,h] . K[row,h/7,0..pos]^T / 8) @ V[...]
 * Replaces the attention core of qweninfer/models/qwen2.py:184-199 (GQA fold, position
 * mask j <= p, fp32 softmax, @ V, head merge). Keys are split into chunks of
 * `split_keys` (multiple of 128); `max_splits` >= ceil((max pos + 1) / split_keys).
 * part: scratch of M*2*max_splits*7*66 floats; counters: M*2 uint32, zero before the
 * first call (the kernel leaves them zero again). */
int qi_attention(const float* q, const uint16_t* k_layer, const uint16_t* v_layer,
                 const int32_t* pos, const int32_t* rows, int M, int max_len, int split_keys,
                 int max_splits, float* out, float* part, unsigned int* counters, int* err,
                 qi_stream_t stream);

/* Attention as qi_attention, for callers that cannot allocate device memory (a host
 * program binding this C ABI directly that only holds device pointers to its own
 * tensors, or a process whose device memory is fixed at start-up): the split partials
 * and arrival counters live in a static array inside the library (~3.6 MiB on every GPU
 * that loads it, held until the process exits) instead of caller-provided scratch. The
 * caller passes only inputs and outputs; `out` is fp32 (M, 896), `err` may be NULL.
 * Limits: M <= 64 query tokens and max_len <= 2048 cache slots per row; larger sizes
 * return QI_ERR_TOO_LARGE before anything is enqueued. The first call on a device looks
 * up the array's device address (cudaGetSymbolAddress) and should come before any stream
 * capture. Calls share the array: calls whose executions overlap on the GPU (different
 * streams or threads) race and give wrong results; calls in one stream are safe.
 * No counterpart in the reference (its attention allocates through PyTorch). */
int qi_attention_noalloc(const float* q, const uint16_t* k_layer, const uint16_t* v_layer,
                         const int32_t* pos, const int32_t* rows, int M, int max_len, float* out,
                         int* err, qi_stream_t stream);

/* o_proj + residual add into the fp32 stream:  x[t] += attn[t] @ Wo^T.
 * Replaces qweninfer/models/qwen2.py:203-204 and the residual add of 237-238.
 * w_o: tiled (896, 896). */
int qi_o_proj_residual(const float* attn, const uint16_t* w_o, int M, float* x, int* err,
                       qi_stream_t stream);

/* Post-attention RMSNorm + fused gate/up projection + SwiGLU:
 *   xn = rmsnorm(x[t]) * ln_w;  h[t, i] = silu(xn . Wg[i]) * (xn . Wu[i]).
 * Replaces qweninfer/models/qwen2.py:44-48 and 113-116 (w_gate_up, chunk, silu * up).
 * w_gate_up: tiled (9728, 896), gate row i at 2i and up row i at 2i+1. ln_w may be
 * NULL: x is then used as given (MLP.forward on an already-normalised input). */
int qi_gate_up_swiglu(const float* x, const float* ln_w, float eps, const uint16_t* w_gate_up,
                      int M, float* h, int* err, qi_stream_t stream);

/* down projection + residual add:  x[t] += h[t] @ Wd^T.
 * Replaces qweninfer/models/qwen2.py:116 (`@ w_down`) and the residual add of 239.
 * w_down: tiled (896, 4864). */
int qi_down_residual(const float* h, const uint16_t* w_down, int M, float* x, int* err,
                     qi_stream_t stream);

/* Final RMSNorm + tied lm_head + greedy argmax:
 *   xn = rmsnorm(x[t]) * norm_w;  logits[t] = xn @ E^T;  slot[t] = argmax (packed).
 * Replaces qweninfer/models/qwen2.py:282-292 (norm, last_only, `@ embed_t`) and the
 * argmax of qweninfer/engine/engine.py:129,155 / generate.py:36,50 (lowest index wins
 * ties). x rows are read at stride x_stride floats. logits may be null; if non-null it
 * receives fp32 (logits_bf16 == 0) or bf16 values at row stride logits_ld elements.
 * argmax_slots (M uint64, zeroed by qi_embed or the caller) receive
 * (order_key(value) << 32) | (0xffffffff - index); the index is 0xffffffff - low32. */
int qi_lm_head_argmax(const float* x, long long x_stride, const float* norm_w, float eps,
                      const uint16_t* embed, int vocab, int M, void* logits, int logits_bf16,
                      long long logits_ld, unsigned long long* argmax_slots, int* err,
                      qi_stream_t stream);

/* Row compaction of the packed KV cache: for each (src, dst, length) triple, copy
 * positions [0, length) of cache row src to row dst in every layer, K and V.
 * Replaces qweninfer/engine/kv_cache.py:65-73 (KVCache.move_row) as driven by
 * qweninfer/engine/engine.py:166-179. `moves` is a HOST array of 3*n_moves ints; the
 * triples are applied in order. */
int qi_move_rows(uint16_t* k, uint16_t* v, int layers, int cache_rows, int max_len,
                 const int32_t* moves, int n_moves, qi_stream_t stream);

/* ------------------------------------------------------------- whole forward */

typedef struct {
  const float* ln1;         /* (896) fp32                               */
  const uint16_t* w_qkv;    /* tiled (1152, 896), RoPE-pair row order   */
  const float* b_qkv;       /* (1152) fp32, same row order              */
  const uint16_t* w_o;      /* tiled (896, 896)                         */
  const float* ln2;         /* (896) fp32                               */
  const uint16_t* w_gate_up;/* tiled (9728, 896), gate/up interleaved   */
  const uint16_t* w_down;   /* tiled (896, 4864)                        */
} qi_layer;

typedef struct {
  int num_layers;
  int vocab;
  int max_seq;              /* rows of the RoPE tables                  */
  float eps;
  const uint16_t* embed;    /* tiled (vocab, 896): lookup and tied head */
  const float* norm;        /* (896) fp32 final norm                    */
  const float* rope_cos;    /* (max_seq, 64) fp32                       */
  const float* rope_sin;
  const qi_layer* layers;   /* HOST array of num_layers entries         */
} qi_model;

typedef struct {
  uint16_t* k;              /* (layers, cache_rows, 2, max_len, 64) bf16, or paged */
  uint16_t* v;
  int cache_rows;
  int max_len;
  /* Paged layout when page_table is not NULL (no reference counterpart: its cache is packed):
   * k and v are pools of n_pages pages per layer, (layers, n_pages, 2, page_size, 64) bf16;
   * page_table[row * pages_per_row + pos / page_size] (device int32, cache_rows x
   * pages_per_row) is the page holding position pos of cache row `row`, -1 if unmapped
   * (reported as QI_ERR_INDEX). page_size is a multiple of 128 and pages_per_row *
   * page_size >= max_len. Only qi_forward with ws->use_tc reads a paged cache. */
  const int32_t* page_table;
  int page_size;
  int pages_per_row;
  int n_pages;
} qi_cache;

typedef struct {
  float* x;                 /* (max_tokens, 896) residual stream         */
  float* q;                 /* (max_tokens, 896)                         */
  float* attn;              /* (max_tokens, 896), CUDA-core path         */
  float* h;                 /* (max_tokens, 4864), CUDA-core path        */
  float* attn_part;         /* max_tokens*2*max_splits*7*66              */
  unsigned int* attn_counters; /* max_tokens*2, zero-initialised         */
  int max_tokens;
  int max_splits;
  int split_keys;
  int* err;                 /* one device int                            */
  /* tensor-core path (use_tc = 1, the default of the Python package) */
  int use_tc;
  uint16_t* act_x;          /* activation tiles, K = 896: ss_ld * 3584 bytes  */
  uint16_t* act_attn;       /* same size                                      */
  uint16_t* act_h;          /* K = 4864: ss_ld * 19456 bytes                  */
  float* ss;                /* 7 * ss_ld floats: per-128-feature sums of squares */
  int ss_ld;                /* >= tokens rounded up to the token tile (8 up to 8
                               tokens, 16 up to 96, 32 up to 384, else 64); padding
                               to 128 lets every projection use its own, larger
                               tile where that measured faster (the Python
                               Workspace pads so)                                */
  float* tc_scratch;        /* stream-K partials, 148*2*128*128 floats covers every
                               token tile (less only lowers the CTAs of a launch) */
  long long tc_scratch_floats;
  unsigned int* tc_counters;/* one per output tile, zero-initialised          */
  int tc_counters_len;
  int query_run;            /* longest run of consecutive query tokens of one cache
                               row in the next forward (a prompt's length), or 0 if
                               unknown. Attention runs the prefill block kernel when
                               it is >= 1536 and more than half of the forward's
                               tokens (0: when the forward has > 128 tokens).
                               1 declares a decode step: every token is the only one
                               of its row and the row's keys below its position are
                               in the cache before the call, so attention copies
                               them while the previous launch still runs          */
} qi_workspace;

/* Full Qwen2 forward of M tokens (qweninfer/models/qwen2.py:263-292 with a cache):
 * embedding, every block (RMSNorm + QKV + bias + RoPE + KV append, ragged attention,
 * o_proj + residual, RMSNorm + gate/up + SwiGLU, down + residual), final RMSNorm, tied
 * head and greedy argmax of the head tokens t = head_lo + i*head_stride, i < n_head
 * (n_head = 0: no head). ids/pos/rows: device int32 (M). logits (optional, row i for head
 * token i) and argmax_slots (n_head) as in qi_lm_head_argmax. Batched decode is M = B
 * tokens at S = 1 (engine.py:140-155); a B = 1 prefill is M = P tokens of one row with
 * head_lo = P-1 (engine.py:115-129, generate.py:33-36).
 * ws->use_tc selects the tcgen05 projections (activation tiles, stream-K) or the
 * CUDA-core GEMV kernels of the single-op entry points above. */
int qi_forward(const qi_model* model, const qi_cache* cache, const qi_workspace* ws,
               const int32_t* ids, const int32_t* pos, const int32_t* rows, int M, int head_lo,
               int head_stride, int n_head, void* logits, int logits_bf16, long long logits_ld,
               unsigned long long* argmax_slots, qi_stream_t stream);

/* Launch kinds reported by qi_forward_launch_times. */
#define QI_LAUNCH_EMBED 0     /* embedding gather + first activation tiles      */
#define QI_LAUNCH_QKV 1       /* RMSNorm + QKV + bias + RoPE + KV append         */
#define QI_LAUNCH_ATTENTION 2 /* ragged GQA attention core                       */
#define QI_LAUNCH_O 3         /* o_proj + residual                               */
#define QI_LAUNCH_GATE_UP 4   /* RMSNorm + gate/up + SwiGLU                      */
#define QI_LAUNCH_DOWN 5      /* down + residual                                 */
#define QI_LAUNCH_HEAD 6      /* final RMSNorm + tied head + argmax              */

/* qi_forward (tensor-core projections, ws->use_tc != 0) with a CUDA event recorded before
 * the first launch and after every launch: kinds[i] (QI_LAUNCH_*) and us[i] (microseconds
 * of device time) of launch i, *n_launches launches (<= max_launches, else
 * QI_ERR_TOO_LARGE). The events serialize the launches, so each time is that launch alone,
 * without the overlap that programmatic dependent launch gives the plain forward.
 * Synchronizes the stream. Instrumentation for per-kernel rooflines; no reference
 * counterpart (the reference's forward is qweninfer/models/qwen2.py:263-292). */
int qi_forward_launch_times(const qi_model* model, const qi_cache* cache, const qi_workspace* ws,
                            const int32_t* ids, const int32_t* pos, const int32_t* rows, int M,
                            int head_lo, int head_stride, int n_head, void* logits, int logits_bf16,
                            long long logits_ld, unsigned long long* argmax_slots,
                            qi_stream_t stream, int* kinds, float* us, int max_launches,
                            int* n_launches);

/* ------------------------------------------------- tensor-core building blocks */

/* fp32 activations x (M, K) -> activation tiles of norm_w * x (norm_w may be NULL) for
 * token tile NT (8..128, power of two): [t/NT][k/64][hi|lo][(t%NT)/8][(k%64)/8][t%8][k%8]
 * bf16, hi = bf16(v), lo = bf16(v - hi). With ss non-NULL (K = 896 only): ss[0][t] =
 * sum_k x[t,k]^2 and ss[1..6][t] = 0, row stride ss_ld. Tokens M..(M rounded up to NT)-1
 * are written as zeros. No reference counterpart: this is the operand format of
 * qi_tc_linear and of the forward's tensor-core projections. */
int qi_act_tiles(const float* x, const float* norm_w, int M, int K, int NT, uint16_t* act,
                 float* ss, int ss_ld, qi_stream_t stream);

/* One tensor-core projection (tcgen05 UMMA, TMEM accumulators, stream-K over `ctas`
 * CTAs; 0 = one per SM):  out[t, n] = r[t] * sum_k W[n, k] * x[t, k]  for the
 * activations encoded in `act` (qi_act_tiles), with r[t] = rsqrt(sum_j ss[j][t] / 896 +
 * eps) when ss is non-NULL (RMSNorm folded as in the forward) and 1 otherwise.
 * W: tiled (n_rows, K), n_rows % 128 == 0, K % 64 == 0. scratch: scratch_floats floats
 * (>= 2*128*NT per CTA); counters: counters_len uint32 >= (n_rows/128)*ceil(M/NT),
 * zero before the call and left zero. The x @ W^T of every projection in
 * qweninfer/models/qwen2.py (160-162, 203-204, 114-116, 291). */
int qi_tc_linear(const uint16_t* w, int n_rows, int K, const uint16_t* act, int M, int NT,
                 const float* ss, int ss_ld, float eps, float* out, int out_ld, float* scratch,
                 long long scratch_floats, unsigned int* counters, int counters_len, int ctas,
                 int* err, qi_stream_t stream);

/* The forward's gate/up projection as one call (the kernel qi_forward launches for it):
 * RMSNorm(post_attention) folded as in qi_tc_linear (ss non-NULL), gate/up rows of the
 * interleaved tiled (9728, 896) weight, SwiGLU silu(gate) * up, written as activation
 * tiles (K = 4864, token tile NT) for the down projection: qwen2.py:114-116 with the
 * norm of qwen2.py:239. Same scratch/counter contract as qi_tc_linear (counters_len >=
 * 76 * ceil(M/NT)); ctas = 0 selects the stream-K partition qi_forward uses for this
 * token tile. act_out: ceil(M/NT) * NT * 4864 * 2 bf16. */
int qi_tc_gate_up_swiglu(const uint16_t* w_gate_up, const uint16_t* act, int M, int NT,
                         const float* ss, int ss_ld, float eps, uint16_t* act_out,
                         float* scratch, long long scratch_floats, unsigned int* counters,
                         int counters_len, int ctas, int* err, qi_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QI_H_ */
