/*
 * jsx.h — C ABI of libjsx.so, the B200 (sm_100a) kernels behind the GLM-4
 * tensor-parallel decoder step of JaxScale (sdh1014/e2e-JaxScale).
 *
 * Conventions
 *  - Every entry point returns an int status (JSX_OK == 0).  Nothing throws
 *    across the ABI; jsx_last_error() returns a thread-local message for the
 *    most recent failing call on the calling thread.
 *  - All tensor arguments are raw device pointers to row-major arrays; sizes
 *    are element counts.  `stream` is a cudaStream_t passed as void* (NULL =
 *    legacy default stream).  Calls are stream-ordered and never synchronise.
 *  - bf16 means IEEE bfloat16 stored as 2 bytes; arithmetic is fp32 inside
 *    the kernels with bf16 rounding (round-to-nearest-even) exactly where the
 *    reference materialises a bf16 array.
 *  - Weights are consumed in PACKED layouts produced once at load time by the
 *    jsx_pack_* entry points from the reference's [in, out] matrices
 *    (layers/linear.py:16 "Weight shape: (input_size, output_size)").
 *  - No entry point allocates device memory except jsx_comm_create.  Scratch
 *    ("workspace") is passed in by the caller, sized by the *_workspace_size
 *    queries, zero-filled once by the caller and left zeroed by every call.
 */
#ifndef JSX_H_
#define JSX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  JSX_OK = 0,
  JSX_EINVAL = 1,    /* bad shape, alignment, pointer or argument */
  JSX_ECUDA = 2,     /* a CUDA runtime call failed */
  JSX_ETIMEDOUT = 3, /* a peer did not arrive within the comm timeout */
  JSX_ENOTSUP = 4,   /* shape outside the compiled kernel set */
  JSX_ENOMEM = 5
};

typedef struct jsx_comm jsx_comm; /* tensor-parallel group state (one per rank) */

/* ---- library ------------------------------------------------------------ */
int jsx_abi_version(void);
const char* jsx_last_error(void);
/* Number of SMs of the current device (grid sizing and tests). */
int jsx_device_sm_count(int* out);
/* Launch flags for every later launch of this process.  JSX_LAUNCH_PDL (1):
 * programmatic dependent launch — each kernel streams its first weight tiles
 * while the previous kernel in the stream drains (default on; the JSX_PDL
 * environment variable "0" turns it off).  No reference counterpart (XLA schedules
 * its own fusions). */
#define JSX_LAUNCH_PDL 1
int jsx_set_launch_flags(int flags);
int jsx_get_launch_flags(void);
/* Reads and clears the device error words of the streaming GEMV, of the
 * whole-step kernel and of the tensor-core projections: a bounded pipeline or
 * grid-barrier wait that gave up (the kernel then finished without its
 * result) reports JSX_ETIMEDOUT.
 * Synchronous (a device copy). */
int jsx_device_error(int* status);

/* ---- packing (load-time, replaces utils/weight_utils.py:248-265 placement) */
/* W[K][N] (reference layout, (in, out)) -> Wt[N][K].  Plain transpose used by
 * jsx_linear, o_proj/down_proj (jsx_row_linear_allreduce) and the router. */
int jsx_pack_transpose(const void* w_kn, void* w_nk, int K, int N, void* stream);
/* q/k/v weights W_q[K][nq*hd], W_k[K][nkv*hd], W_v[K][nkv*hd] -> the fused
 * qkv layout of jsx_qkv_rope_cache: per head, the rotary pairs (d, d+r) for
 * d < r = rotary_dim/2, then the pass-through dims in pairs (d, d+1).
 * layers/attention.py:47-61 (q/k/v projections) + layers/rotary.py:88-91. */
int jsx_pack_qkv(const void* w_q, const void* w_k, const void* w_v, void* w_qkv,
                 int K, int nq, int nkv, int head_dim, int rotary_dim, void* stream);
/* gate W_g[K][I], up W_u[K][I] -> rows interleaved (gate_j, up_j).
 * models/glm4.py:30-39 (gate_proj / up_proj). */
int jsx_pack_gate_up(const void* w_gate, const void* w_up, void* w_gu, int K, int I, void* stream);

/* ---- ops ------------------------------------------------------------------ */
/* layers/normalization.py:31-37 RMSNorm.__call__: y = bf16((f32(x)*rsqrt(mean(x^2)+eps))*f32(g)). */
int jsx_rmsnorm(const void* x, const void* gamma, void* y, int rows, int hidden, float eps,
                void* stream);

/* layers/embedding.py:35-51 Embed.__call__: out[m] = table[ids[m]] (ids device int32[M]). */
int jsx_embed(const int32_t* ids, const void* table, void* out, int M, int hidden, int vocab,
              void* stream);

/* layers/linear.py:57-82 LinearBase.__call__ without a collective (column-
 * parallel or replicated): y = bf16(x @ W) then y = bf16(y + b) when bias is
 * non-NULL.  x[M][K], w_nk[N][K] (jsx_pack_transpose), y[M][N].
 * When gamma is non-NULL the RMSNorm of layers/normalization.py:31-37 is
 * applied to x first (fused prologue).  1 <= M <= 8 per call. */
int jsx_linear(const void* x, const void* gamma, float eps, const void* w_nk, const void* bias,
               void* y, int M, int K, int N, void* stream);

/* Fused input_layernorm + q/k/v projections + bias + partial neox RoPE + KV
 * cache write of one decoder layer (models/glm4.py:118-120,
 * layers/attention.py:104-133, layers/rotary.py:36-93).
 *   h[M][K] bf16, ln_gamma[K] bf16, w_qkv packed ((nq+2*nkv)*hd rows),
 *   b_qkv[(nq+2*nkv)*hd] bf16 in reference order (q | k | v), inv_freq[rotary_dim/2] f32,
 *   positions[M] int32 (RoPE angle and cache slot), token m belongs to
 *   sequence m / tokens_per_seq.
 *   q_out[M][nq*hd] (rotated), k_cache/v_cache [B][max_seq][nkv][hd]. */
int jsx_qkv_rope_cache(const void* h, const void* ln_gamma, float eps, const void* w_qkv,
                       const void* b_qkv, const float* inv_freq, const int32_t* positions,
                       void* q_out, void* k_cache, void* v_cache, int M, int tokens_per_seq,
                       int K, int nq, int nkv, int head_dim, int rotary_dim, int max_seq,
                       void* stream);

/* Fused post_attention_layernorm + gate/up projections + SwiGLU
 * (models/glm4.py:128-129 and :46-49 up to the down_proj input):
 *   act[M][I] = bf16(bf16(silu(bf16(h@Wg))) * bf16(h@Wu)). */
int jsx_gate_up_swiglu(const void* h, const void* ln_gamma, float eps, const void* w_gu,
                       void* act, int M, int K, int I, void* stream);

/* Decode attention over the static KV cache (layers/attention.py:136-153,
 * SDPA with the decode mask of runner.py:49-63): each sequence b attends to
 * cache rows [0, positions[b]] (the masked rows of the reference contribute
 * exactly zero).  q[B][nq][hd] (already rotated), caches [B][max_seq][nkv][hd],
 * out[B][nq*hd].  Split over the context; partial results go to `workspace`. */
int jsx_attn_decode_workspace_size(int B, int nq, int nkv, int head_dim, int max_seq,
                                   size_t* bytes);
/* Causal prefill attention over the static KV cache (layers/attention.py:101-160
 * with the prefill mask of runner.py:26-32, cache_position = start_pos for the
 * whole batch): query token i of sequence b (position start_pos + i) attends to
 * cache rows [0, start_pos + i].  q and out [B * S][nq * head_dim] (q already
 * rotated, rows [start_pos, start_pos + S) of the caches already written),
 * caches [B][max_seq][nkv][head_dim].  head_dim 128 (JSX_ENOTSUP otherwise);
 * fp32 softmax, probabilities rounded to bf16 for the P.V product. */
int jsx_attn_prefill(const void* q, const void* k_cache, const void* v_cache, void* out, int B,
                     int S, int start_pos, int nq, int nkv, int head_dim, int max_seq,
                     float scale, void* stream);
int jsx_attn_decode(const void* q, const void* k_cache, const void* v_cache, void* out,
                    const int32_t* positions, int B, int nq, int nkv, int head_dim,
                    int max_seq, float scale, void* workspace, size_t workspace_bytes,
                    void* stream);
/* Same computation as jsx_attn_decode, for callers that cannot allocate device
 * memory: the split partials live in a 16 MiB static device array of the
 * library instead of a caller workspace.  No counterpart in the reference (XLA
 * allocates its own temporaries).  Shapes whose workspace exceeds 16 MiB get
 * JSX_EINVAL.  The first call on a device looks up the array's address (make
 * it before any stream capture); every call shares the array, so calls that
 * overlap on the GPU race.  Allocates nothing. */
int jsx_attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, void* out,
                            const int32_t* positions, int B, int nq, int nkv, int head_dim,
                            int max_seq, float scale, void* stream);

/* Row-parallel projection (o_proj / down_proj) fused with the tensor-parallel
 * all-reduce and the residual add (layers/linear.py:72-78 row-parallel
 * constraint that makes XLA all-reduce; layers/attention.py:159;
 * models/glm4.py:49,124,130):
 *   h[m] = bf16(h[m] + bf16(sum_ranks x_r[m] @ W_r))
 * x[M][K_local], w_nk[N][K_local] (this rank's input-dim shard, transposed),
 * h[M][N] residual stream (in/out, identical on every rank afterwards).
 * Partials are pushed as fp32 into the peers' buffers over NVLink (P2P
 * stores) and summed in rank order on every rank.  comm may be NULL for a
 * single rank (TP=1). */
int jsx_row_linear_allreduce(jsx_comm* comm, const void* x, const void* w_nk, void* h,
                             int M, int K_local, int N, void* stream);
/* The same with a per-rank addend[M][N] (bf16, may be NULL) summed into this
 * rank's fp32 partial before the all-reduce: h = bf16(h + bf16(sum over ranks
 * of (x_r @ W_r + addend_r))).  The MoE layer passes its routed-expert partial
 * here, so the reference's psum("expert") (layers/moe.py:230) and the shared
 * expert's tensor-parallel all-reduce (layers/moe.py:110-113) are one exchange. */
int jsx_row_linear_allreduce_add(jsx_comm* comm, const void* x, const void* w_nk, const void* addend,
                                 void* h, int M, int K_local, int N, void* stream);

/* Final norm + LM head + greedy argmax (models/glm4.py:193, :251-252,
 * layers/embedding.py:79-92, runner.py:281/:297).  The vocabulary is
 * sharded: this rank holds rows [vocab_offset, vocab_offset+vocab_local) of
 * the [V][H] head.  logits are rounded to bf16 like the reference and the
 * lowest index wins ties (jnp.argmax).  ids_out[M] int32 receives the global
 * argmax on every rank; logits_out[M][vocab_local] bf16 is written when non-NULL. */
int jsx_lmhead_workspace_size(int M, size_t* bytes);
int jsx_lmhead_argmax(jsx_comm* comm, const void* h, const void* norm_gamma, float eps,
                      const void* w_vocab, int vocab_local, int vocab_offset, int M, int hidden,
                      void* logits_out, int32_t* ids_out, void* workspace,
                      size_t workspace_bytes, void* stream);

/* ---- tensor-core projections for 9..32 tokens -------------------------------
 * The same five projections as above (same argument meaning, same packed
 * weights, same epilogues and error behaviour) computed on the tcgen05 tensor
 * cores: weight tiles of 128 rows x 64 K are the MMA's A operand, the M <= 32
 * token rows its B operand, both loaded by TMA, fp32 accumulation in TMEM,
 * K split across CTAs and the split partials summed in split order by a
 * second kernel that runs the epilogue.  They replace the same reference
 * call sites as the GEMV entry points (layers/linear.py:57-82 and :116-145,
 * models/glm4.py:118-120, :47-49, :193, layers/embedding.py:79-92) for
 * batches where one weight element feeds 2*M >= 18 flops.  Sums are fp32
 * like the GEMV path but in a different order, so results agree with it to
 * fp32 rounding, not bitwise.  Across ranks, jsx_tc_row_linear_allreduce
 * rounds each rank's partial to bf16 (the reference's per-rank result) and
 * exchanges in two shots (row pairs to their owner rank, owner sum in rank
 * order + residual, gather), as bf16-pair LL words in the comm buffer.
 * workspace: jsx_tc_workspace_size(M, K, N) bytes, 16-byte aligned; for
 * jsx_tc_lmhead_argmax its first 512 bytes must be zero on the first call
 * (they are left zero). */
int jsx_tc_workspace_size(int M, int K, int N, size_t* bytes);
/* Profiling aid (no reference counterpart): when buf is non-NULL, every later
 * jsx_tc_* launch of this process stamps %globaltimer (ns) per CTA into
 * buf[cta * 8 + k], k = 0 entry, 1 first ring of loads issued, 2 loads done,
 * 3 first stage consumed, 4 last MMA issued, 5 first accumulator read,
 * 6 epilogue done, 7 exit; every jsx_wide_* launch as well, k = 0 entry,
 * 1 first accumulator at the epilogue, 2 epilogue done with the tiles other
 * ranks own, 3 with every tile, 4 finished tiles gathered, 5 last MMA commit,
 * 6 last load issued, 7 exit.  buf holds 8 x (SM count) u64.  NULL turns it
 * off. */
int jsx_tc_set_trace(uint64_t* buf);
int jsx_tc_linear(const void* x, const void* gamma, float eps, const void* w_nk, const void* bias,
                  void* y, int M, int K, int N, void* workspace, size_t workspace_bytes,
                  void* stream);
int jsx_tc_qkv_rope_cache(const void* h, const void* ln_gamma, float eps, const void* w_qkv,
                          const void* b_qkv, const float* inv_freq, const int32_t* positions,
                          void* q_out, void* k_cache, void* v_cache, int M, int tokens_per_seq,
                          int K, int nq, int nkv, int head_dim, int rotary_dim, int max_seq,
                          void* workspace, size_t workspace_bytes, void* stream);
int jsx_tc_gate_up_swiglu(const void* h, const void* ln_gamma, float eps, const void* w_gu,
                          void* act, int M, int K, int I, void* workspace,
                          size_t workspace_bytes, void* stream);
int jsx_tc_row_linear_allreduce(jsx_comm* comm, const void* x, const void* w_nk, void* h, int M,
                                int K_local, int N, void* workspace, size_t workspace_bytes,
                                void* stream);
int jsx_tc_lmhead_argmax(jsx_comm* comm, const void* h, const void* norm_gamma, float eps,
                         const void* w_vocab, int vocab_local, int vocab_offset, int M,
                         int hidden, void* logits_out, int32_t* ids_out, void* workspace,
                         size_t workspace_bytes, void* stream);

/* ---- sampling --------------------------------------------------------------
 * The reference's _jit_sample (runner.py:315-359) for one token per sequence:
 * repetition penalty on the tokens flagged in presence[B][V] (x / rp when x > 0,
 * else x * rp; presence may be NULL), temperature (skipped at 1), the top-k
 * candidates (top_k <= 0 means 200, like the reference; k <= 256), top-p on the
 * k candidates (a candidate whose preceding probability mass reaches top_p is
 * dropped), then the categorical draw argmax(value + gumbel): gumbel[B][k] is
 * the caller's Gumbel noise, one value per candidate in top-k order (values
 * descending, lower index first on ties).  bf16 arithmetic as the reference's,
 * with rp and temperature rounded to bf16.  tokens_out[B] int32. */
int jsx_sample(const void* logits, const uint8_t* presence, const void* gumbel, int32_t* tokens_out,
               int B, int V, float repetition_penalty, float temperature, int top_k, float top_p,
               void* stream);

/* ---- wide tensor-core projections (prefill, many tokens) ---------------------
 * The column-parallel and single-rank row-parallel projections of
 * LinearBase.__call__ (layers/linear.py:57-82) over a whole [B, S] token block
 * (models/glm4.py:97-132 at prefill, runner.py:285-294), for any M >= 1 (tiles
 * of 128 weight rows x 256 tokens on tcgen05 tensor cores, TMA-fed, fp32
 * accumulation in TMEM).  Same packed weights, arguments and results as the
 * jsx_tc_* / GEMV entry points (fp32 accumulation order differs).  gamma /
 * ln_gamma: optional RMSNorm gain applied to the activations first
 * (layers/normalization.py:31-37).
 * workspace: jsx_wide_workspace_size(M, K, N, gamma != NULL) bytes, 16-byte
 * aligned (the normalised activations live there).  Outputs and residuals
 * must be 16-byte aligned. */
int jsx_wide_workspace_size(int M, int K, int N, int has_gamma, size_t* bytes);
int jsx_wide_linear(const void* x, const void* gamma, float eps, const void* w_nk, const void* bias,
                    void* y, int M, int K, int N, void* workspace, size_t workspace_bytes,
                    void* stream);
int jsx_wide_qkv_rope_cache(const void* h, const void* ln_gamma, float eps, const void* w_qkv,
                            const void* b_qkv, const float* inv_freq, const int32_t* positions,
                            void* q_out, void* k_cache, void* v_cache, int M, int tokens_per_seq,
                            int K, int nq, int nkv, int head_dim, int rotary_dim, int max_seq,
                            void* workspace, size_t workspace_bytes, void* stream);
int jsx_wide_gate_up_swiglu(const void* h, const void* ln_gamma, float eps, const void* w_gu,
                            void* act, int M, int K, int I, void* workspace,
                            size_t workspace_bytes, void* stream);
/* Row-parallel projection + TP all-reduce + residual for many tokens
 * (o_proj / down_proj, layers/attention.py:62-66, :159, models/glm4.py:40-44,
 * :49, :124, :130; the psum that layers/linear.py:72-78 leaves to XLA):
 * h[M][N] += bf16(sum over ranks of bf16(x_r[M][K_local] W_r^T)), the ranks'
 * bf16 partials summed in fp32 in rank order (identical h on every rank).
 * comm: NULL or a 1-rank comm (residual add only), or a tile-exchange comm of
 * jsx_comm_create_tiles with max_tokens >= M and hidden >= N: each output tile
 * of 128 rows x 256 tokens is owned by one rank; the others write their
 * partial tile into the owner's buffer over NVLink as soon as it leaves the
 * tensor cores, the owner sums, adds the residual and writes the finished
 * tile to every rank, so the exchange overlaps the GEMM tile by tile.  Every
 * rank calls with the same M, K_local, N; a peer that does not arrive within
 * the comm timeout makes jsx_comm_check report JSX_ETIMEDOUT. */
int jsx_wide_row_linear_allreduce(jsx_comm* comm, const void* x, const void* w_nk, void* h, int M,
                                  int K_local, int N, void* workspace, size_t workspace_bytes,
                                  void* stream);

/* ---- whole decode step ------------------------------------------------------
 * One cooperative kernel runs a full GLM-4 decode step for batch <= 8 on this
 * rank: embedding, every decoder layer (the work of jsx_qkv_rope_cache,
 * jsx_attn_decode, jsx_row_linear_allreduce (o_proj), jsx_gate_up_swiglu,
 * jsx_row_linear_allreduce (down_proj)) and the final norm + LM head +
 * argmax, with grid-wide barriers between the phases instead of kernel
 * launches (models/glm4.py:162-195, :226-260 inside the jit step of
 * runner.py:139-164, greedy argmax runner.py:297).  Results equal the per-op
 * entry points'.  ids are read as the fed tokens and overwritten with the
 * greedy tokens (head != 0); positions are advanced by one when advance != 0. */
typedef struct {
  const void* ln1;    /* [hidden] bf16 */
  const void* w_qkv;  /* jsx_pack_qkv layout, (nq + 2 nkv) * head_dim rows */
  const void* b_qkv;  /* [(nq + 2 nkv) * head_dim] or NULL */
  const void* w_o;    /* [hidden][nq * head_dim] (jsx_pack_transpose of this rank's shard) */
  const void* ln2;    /* [hidden] */
  const void* w_gu;   /* jsx_pack_gate_up layout, 2 * inter rows */
  const void* w_d;    /* [hidden][inter] */
  void* k_cache;      /* [batch][max_seq][nkv][head_dim] */
  void* v_cache;
} jsx_layer_weights;

typedef struct {
  int batch, hidden, n_heads, n_kv_heads, head_dim, rotary_dim, inter;  /* per-rank head/inter counts */
  int vocab, vocab_local, vocab_offset, max_seq, n_layers;
  float eps, scale;
  const jsx_layer_weights* layers; /* DEVICE array of n_layers entries */
  const void* embed;               /* [vocab][hidden] */
  const void* final_norm;          /* [hidden] */
  const void* lm_head;             /* [vocab_local][hidden] */
  const float* inv_freq;           /* [rotary_dim / 2] */
  int32_t* ids;                    /* [batch] */
  int32_t* positions;              /* [batch] */
  int advance, head;
  void* h;                         /* [batch][hidden] residual stream */
  void* q;                         /* [batch][nq * head_dim] */
  void* attn;                      /* [batch][nq * head_dim] */
  void* act;                       /* [batch][inter] */
  void* logits;                    /* [batch][vocab_local] or NULL */
  void* workspace;                 /* jsx_decode_step_workspace_size bytes, zeroed once */
  size_t workspace_bytes;
  uint64_t* trace;                 /* NULL, or [2 + 13 n_layers] u64: %globaltimer (ns) after the
                                      embedding, after each phase of each layer, and at the end;
                                      then per layer 8 attention stamps of head group 0: split 0
                                      started, staged, scored, softmax, P.V done, counted; the
                                      merge done; one spare */
  uint64_t* trace_ar;              /* NULL, or [n_layers][2][2] u64, zero before the call: for each
                                      row-parallel phase (o_proj, down) the latest %globaltimer over
                                      CTAs at which a CTA had pushed its partials to every rank, and
                                      the latest at which a CTA had finished its rank-ordered sums
                                      (the second minus the first is the exchange's exposed time) */
  uint32_t l2_next_bytes;          /* per warp: bytes of its first row pairs of the next projection
                                      requested into L2 (bulk prefetch) once it has read its rows
                                      of the current one; 0 = none */
  uint32_t l2_attn_bytes;          /* per warp: bytes of its first gate/up row pairs requested into
                                      L2 while the attention runs; 0 = none */
  uint64_t* trace_phase;           /* NULL, or [n_layers][5][3] u64, zero before the call: for each
                                      phase (qkv, attention, o_proj, gate/up, down) the latest
                                      %globaltimer over CTAs at which a CTA had (0) staged its input
                                      (attention: begun its items), (1) finished its product and
                                      epilogue (row-parallel: pushed its partials), (2) finished the
                                      phase before its barrier arrival */
} jsx_decode_step_args;

int jsx_decode_step_workspace_size(const jsx_decode_step_args* args, size_t* bytes);
int jsx_decode_step(jsx_comm* comm, const jsx_decode_step_args* args, void* stream);

/* MoE router (layers/moe.py:54-79 MoEGate.__call__): logits = bf16(x @ Wg),
 * softmax in f32, + correction bias (nullable), top-k (ties -> lower index),
 * weights = uncorrected probabilities renormalised (+1e-20) when norm != 0,
 * times scale, rounded to bf16.  x[N][H], w_nk[E][H], topk_w[N][k] bf16,
 * topk_idx[N][k] int32.  E <= 256, k <= 8. */
/* MLA (layers/mla_attention.py:139-172): neox RoPE (rotary_dim = rope) on the
 * rope slice of every query head and on the shared rope key, concatenation
 * [nope | rope], and the expanded per-head cache write.
 *   q_in [M][nh][nope+rope] (q_b output), kv_in [M][nh][nope+vdim] (kv_b
 *   output), k_rope [M][rope] (the rope columns of kv_a_proj_with_mqa),
 *   inv_freq [rope/2], positions [M] (angle and cache slot), token m of
 *   sequence m / tokens_per_seq; q_out [M][nh][nope+rope],
 *   k_cache [B][max_seq][nh][nope+rope], v_cache [B][max_seq][nh][vdim]. */
int jsx_mla_rope_cache(const void* q_in, const void* kv_in, const void* k_rope, const float* inv_freq,
                       const int32_t* positions, void* q_out, void* k_cache, void* v_cache, int M,
                       int tokens_per_seq, int nh, int nope, int rope, int vdim, int max_seq,
                       void* stream);

/* Absorbed-weight MLA decode over a latent cache (the decode form that
 * replaces the expanded per-head cache of layers/mla_attention.py:139-172 and
 * the attention of :174-190; README.md:67 names it as the reference's fix).
 * The cache holds per token the normalised kv latent c and the rotated shared
 * rope key: latent_cache [B][max_seq][kv_lora + rope] bf16.
 * jsx_mla_latent_cache: q_rope [M][nh][rope] = RoPE of the rope slice of q_in
 *   [M][nh][nope + rope]; cache row of token m at positions[m] (sequence
 *   m / tokens_per_seq) = [c[m] | RoPE(k_rope[m])] (rotary.py:56-58, :88-91). */
int jsx_mla_latent_cache(const void* q_in, const void* c, const void* k_rope, const float* inv_freq,
                         const int32_t* positions, void* q_rope, void* latent_cache, int M,
                         int tokens_per_seq, int nh, int nope, int rope, int kv_lora, int max_seq,
                         void* stream);
/* Per-head absorption GEMV: out[m][h][r] = bf16(sum_k w[h][r][k] x[m][h][k]),
 * x of (m, h) at x + m * x_token_stride + h * x_head_stride (elements).  With w
 * = the key columns of kv_b per head ([nh][kv_lora][nope]) it forms q_abs from
 * q_nope; with the value columns ([nh][v][kv_lora]) the head outputs from the
 * latent context.  M <= 32, K <= 512 (multiple of 8). */
int jsx_mla_absorb(const void* x, int x_token_stride, int x_head_stride, const void* w, void* out,
                   int M, int nh, int R, int K, void* stream);
/* Multi-query attention of nh <= 32 heads over the latent cache rows
 * [0, positions[b]]: s = bf16(bf16(q_abs . c + q_rope . kr) * scale) (the
 * reference rounds q.k, then the scaled score, to bf16), fp32 softmax,
 * ctx[b][h] = bf16(P . c) [B][nh][kv_lora].  kv_lora a multiple of 256,
 * kv_lora + rope <= 576.  Split over the context (64 rows) and merged in a
 * second launch; workspace of jsx_mla_decode_workspace_size bytes. */
int jsx_mla_decode_workspace_size(int B, int nh, int kv_lora, int max_seq, size_t* bytes);
int jsx_mla_decode(const void* q_abs, const void* q_rope, const void* latent_cache, void* ctx,
                   const int32_t* positions, int B, int nh, int kv_lora, int rope, int max_seq,
                   float scale, void* workspace, size_t workspace_bytes, void* stream);

/* MoE experts of one rank (layers/moe.py:194-267, _forward_ep / _topk_local_forward):
 * x[N][H] normalised hidden states, topk_w[N][K] bf16 and topk_idx[N][K] from
 * jsx_moe_gate; expert_owner[E] (device int32) names the rank that computes each
 * expert (NULL: this rank computes all).  w_gate_up [E][2I][H] (per expert
 * jsx_pack_gate_up), w_down [E][H][I] (per expert jsx_pack_transpose).
 * out[N][H] = this rank's routed partial: per token, k = 0..K-1 in order over
 * the owned experts, out = bf16(out + bf16(bf16(silu(x Wg) * (x Wu)) Wd * w_k)).
 * N <= 32, K <= 8, E <= 256; workspace of jsx_moe_experts_workspace_size bytes. */
int jsx_moe_experts_workspace_size(int N, int K, int E, int H, int I, size_t* bytes);
int jsx_moe_experts(const void* x, const void* topk_w, const int32_t* topk_idx,
                    const int32_t* expert_owner, int rank, int N, int K, int E, int H, int I,
                    const void* w_gate_up, const void* w_down, void* out, void* workspace,
                    size_t workspace_bytes, void* stream);
int jsx_moe_gate(const void* x, const void* w_nk, const float* correction_bias, void* topk_w,
                 int32_t* topk_idx, int N, int H, int E, int k, float scale, int norm,
                 void* stream);

/* ---- tensor-parallel group (utils/mesh_utils.py:8-45 "tensor" axis) ------- */
/* Allocates this rank's symmetric buffer on the current device: fp32 partial
 * slots for up to max_tokens x hidden, flags and state.  timeout_ns bounds
 * every wait on a peer (0 = 2 s default). */
int jsx_comm_create(int rank, int world, int max_tokens, int hidden, uint64_t timeout_ns,
                    jsx_comm** out);
/* A comm whose symmetric buffer holds the tile exchange of
 * jsx_wide_row_linear_allreduce for up to max_tokens tokens and hidden output
 * rows (partial slots, finished-tile array and flags: about
 * 2 x max_tokens x hidden x 2 bytes per rank).  Peers are opened with
 * jsx_comm_ipc_handle / jsx_comm_open_peers like any comm. */
int jsx_comm_create_tiles(int rank, int world, int max_tokens, int hidden, uint64_t timeout_ns,
                          jsx_comm** out);
/* CUDA IPC handle of the symmetric buffer (64 bytes). */
int jsx_comm_ipc_handle(jsx_comm* comm, void* out64);
/* Opens every peer's handle (handles = world x 64 bytes, in rank order). */
int jsx_comm_open_peers(jsx_comm* comm, const void* handles);
/* Reads and clears the device error word: *status = JSX_OK or JSX_ETIMEDOUT.
 * Synchronises the device. */
int jsx_comm_check(jsx_comm* comm, int* status);
int jsx_comm_destroy(jsx_comm* comm);

#ifdef __cplusplus
}
#endif

#endif /* JSX_H_ */
