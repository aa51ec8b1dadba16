/*
 * libdtree_b200 — C ABI of the B200 (sm_100a) DTree/DFlash speculative-decoding step.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream, allocates
 * nothing, and returns 0 on success or a negative status (see DTREE_*
 * below); dtree_last_error() then describes the failure.  Buffers are owned
 * by the caller.  The reference (DrHB/dtree-mlx, Python/MLX) reaches these
 * operations through the MLXTargetAdapter plugin interface
 * (dtree_mlx/adapters.py:88-213) and the DTree runtime
 * (dtree_mlx/dtree_runtime.py); each declaration names the reference
 * function it replaces.
 *
 * Threading: entry points are reentrant across streams; a model handle must
 * not be used by two streams at once (its activation buffers are shared).
 */
#ifndef DTREE_B200_H_
#define DTREE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DTREE_API __attribute__((visibility("default")))
#else
#define DTREE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
#define DTREE_OK 0
#define DTREE_ERR_INVALID_ARG (-1)
#define DTREE_ERR_CUDA (-2)
#define DTREE_ERR_UNSUPPORTED (-3)
#define DTREE_ERR_CAPACITY (-4)
#define DTREE_ERR_TREE (-5)
#define DTREE_ERR_STATE (-6)

/* Largest tree (root + nodes) one verify step accepts; ancestor masks are
 * DTREE_MASK_WORDS little-endian uint64 words per node. */
#define DTREE_MAX_TREE 128
#define DTREE_MASK_WORDS 2

/* Thread-local description of the last failed call (never NULL). */
DTREE_API const char* dtree_last_error(void);

/* Library ABI version (major*100 + minor). */
DTREE_API int dtree_version(void);

/* Reads the device-side error word (bounded-wait timeouts, invalid device
 * inputs; 0 = none) after synchronizing the device; clears it if clear != 0. */
DTREE_API int dtree_device_error(uint32_t* code_out, int clear);

/* Test support, no counterpart in the reference: stores `value` to the device
 * int at `dst` about delay_ns after launch, while letting the next kernel on
 * the stream start early (programmatic dependent launch).  Used to make a
 * kernel observe a decode-state field change between its early read and its
 * dependency wait. */
DTREE_API int dtree_test_delayed_store(int32_t* dst, int32_t value, int delay_ns, void* stream);

/* ---------------------------------------------------------- decode state
 * Per-sequence decode bookkeeping kept in device memory so that a whole
 * decode step can run (and be graph-replayed) without a host round trip.
 * Mirrors the loop variables of dtree_generate (dtree_runtime.py:351-354,
 * 531-534): `start` is the number of tokens committed to the target KV cache
 * (the reference's `start` / past_length) and `root_token` is
 * output_tokens[start] (sampled but not yet in the cache). */
typedef struct dtree_step_state {
  int32_t start;        /* committed tokens in the target KV cache            */
  int32_t root_token;   /* last posterior token; root of the next tree        */
  int32_t step;         /* decode steps completed                             */
  int32_t n_accepted;   /* accepted inputs of the last step (root included)   */
  int32_t bonus_token;  /* posterior token after the accepted path            */
  int32_t n_output;     /* tokens written to the output buffer                */
  int32_t n_nodes;      /* nodes in the current tree (root included)          */
  int32_t reserved;
} dtree_step_state;

/* --------------------------------------------------------- tree build
 * Replaces build_dtree_tree + compile_dtree_tree (dtree_runtime.py:82-192):
 * per draft row the fp32 top-k (k = min(budget, vocab); equal logits ordered
 * by ascending token id) and log-softmax, then the best-first expansion with
 * the reference's float64 heap key (-logw, ranks, parent, depth, rank, logw)
 * and sibling score logw - lp[r] + lp[r+1].  Outputs (node 0 = root):
 *   tree_tokens[i]  verify input ids (root = state->root_token)
 *   parents[i]      parent index (-1 for the root)
 *   depths[i]       depth (0 for the root)
 *   positions[i]    RoPE position state->start + depth
 *   anc_mask[i][w]  bit j set iff node j is visible to node i (visibility row)
 *   top_ids/top_logprobs (optional, may be NULL) [rows][k] heap inputs
 * state->n_nodes is set to 1 + number of nodes.  rows <= 64, budget <= 127.
 * `workspace` holds per-row partials: dtree_tree_build_workspace_bytes(). */
DTREE_API size_t dtree_tree_build_workspace_bytes(int rows, int vocab, int budget);
DTREE_API int dtree_tree_build(const float* draft_logits, int rows, int vocab, int budget,
                     dtree_step_state* state, void* workspace, size_t workspace_bytes,
                     int32_t* tree_tokens, int32_t* parents, int32_t* depths, int32_t* positions,
                     uint64_t* anc_mask, int32_t* top_ids, float* top_logprobs, void* stream);

/* Same as dtree_tree_build, but allocates nothing and takes no workspace:
 * for callers that cannot allocate device memory while they decode (a
 * serving loop with a fixed memory budget, or a host runtime that only passes
 * buffers it already owns).  No counterpart in the reference, which builds
 * the tree on the host.  The scratch is a fixed 1 MiB device array inside
 * the library (dtree_tree_build_noalloc_max_bytes()), held by every GPU that
 * loads the library until the process exits.  It bounds the vocabulary:
 * dtree_tree_build_noalloc_max_vocab(rows) (about 344k at 64 draft rows,
 * 1.4M at 16); larger sizes are rejected with DTREE_ERR_CAPACITY before any
 * GPU work.  The first call on a device looks up the scratch address for
 * that device and caches it for the life of the process (it does not survive
 * a cudaDeviceReset); make that first call before any stream capture.  All
 * calls share the scratch and it keeps the last call's contents: calls whose
 * GPU work overlaps (other streams or threads) race on it. */
DTREE_API size_t dtree_tree_build_noalloc_max_bytes(void);
DTREE_API int dtree_tree_build_noalloc_max_vocab(int rows);
DTREE_API int dtree_tree_build_noalloc(const float* draft_logits, int rows, int vocab, int budget,
                                       dtree_step_state* state, int32_t* tree_tokens, int32_t* parents,
                                       int32_t* depths, int32_t* positions, uint64_t* anc_mask, void* stream);

/* Heap stage only, from given top-k ids/log-probs (for parity checks against
 * the reference's own heap inputs).  Same outputs as dtree_tree_build. */
DTREE_API int dtree_tree_from_topk(const int32_t* top_ids, const float* top_logprobs, int rows, int topk, int budget,
                         dtree_step_state* state, int32_t* tree_tokens, int32_t* parents, int32_t* depths,
                         int32_t* positions, uint64_t* anc_mask, void* stream);

/* Linear (DFlash) block: the chain tree of dflash_generate's verify block
 * (runtime.py:476-490): node i+1 = argmax of draft row i, parent i, depth i+1.
 * Argmax ties keep the first index (runtime.py:12-19 sample_tokens, T=0). */
DTREE_API int dtree_chain_build(const float* draft_logits, int rows, int vocab, dtree_step_state* state,
                      int32_t* tree_tokens, int32_t* parents, int32_t* depths, int32_t* positions,
                      uint64_t* anc_mask, void* stream);

/* The same chain with the drafted tokens sampled at `temperature`
 * (sample_tokens, runtime.py:12-19, called on the draft logits at
 * runtime.py:486): node i+1 = a draw from softmax(draft row i / T) by the
 * Gumbel-max rule with Philox noise keyed by (seed, state->step, row,
 * token); temperature < 1e-5 is the argmax of dtree_chain_build. */
DTREE_API int dtree_chain_sample(const float* draft_logits, int rows, int vocab, float temperature, uint32_t seed,
                      dtree_step_state* state, int32_t* tree_tokens, int32_t* parents, int32_t* depths,
                      int32_t* positions, uint64_t* anc_mask, void* stream);

/* -------------------------------------------------- planted draft logits
 * Synthetic drafter of the benchmark workloads (stands in for
 * DFlashDraftModel + lm_head_logits, dtree_runtime.py:366-376): row r gets
 * Irwin-Hall(12)-6 noise from Philox4x32-10(seed, state->step, r) and +8 on
 * continuation[state->start + r + 1] with probability p_correct (else on a
 * Philox-chosen random token; also when the position is >= cont_len or the
 * continuation entry is negative, i.e. unknown). */
DTREE_API int dtree_plant_draft_logits(float* logits, int rows, int vocab, uint32_t seed, const dtree_step_state* state,
                             const int32_t* continuation, int cont_len, float p_correct, void* stream);

/* ---------------------------------------------------- acceptance walk
 * Replaces follow_verified_tree (dtree_runtime.py:195-208) and the output
 * commit (dtree_runtime.py:530-537): walks from the root while the posterior
 * token of the current node is the token of one of its children.  Writes
 * accepted[0..n) (node indices, ascending), state->n_accepted,
 * state->bonus_token, appends the accepted tokens and the bonus token to
 * output_tokens at [state->start, ...) (bounded by output_capacity), sets
 * state->n_output, and records n_accepted in accept_history[state->step]
 * (if non-NULL and step < history_capacity). */
DTREE_API int dtree_accept_walk(const int32_t* tree_tokens, const int32_t* parents, const int32_t* posterior,
                      dtree_step_state* state, int32_t* accepted, int32_t* output_tokens, int output_capacity,
                      int32_t* accept_history, int history_capacity, void* stream);

/* ------------------------------------------------------ KV compaction
 * Replaces Qwen3TargetAdapter.compact_kv_caches (adapters.py:635-668) for
 * every layer at once: rows [start + accepted[i]] -> [start + i] of each
 * (layer, K|V, kv-head) plane of a cache laid out
 * [layers][2][kv_heads][capacity][head_dim] (bf16, head_dim*2 bytes a row).
 * All reads of a plane happen before its writes (in-place safe). */
DTREE_API int dtree_kv_compact(void* kv_cache, int layers, int kv_heads, int capacity, int head_dim,
                     const int32_t* accepted, const dtree_step_state* state, void* stream);

/* Hidden select (dtree_runtime.py:519-522): dst[i] = src[accepted[i]] for
 * i < state->n_accepted, rows of row_bytes (multiple of 16). */
DTREE_API int dtree_gather_rows(const void* src, size_t row_bytes, const int32_t* accepted, const dtree_step_state* state,
                      void* dst, int max_rows, void* stream);

/* Advances the decode state after a step: start += n_accepted,
 * root_token = bonus_token, step += 1 (dtree_runtime.py:531-534). */
DTREE_API int dtree_step_commit(dtree_step_state* state, void* stream);

/* ------------------------------------------------------- dense linear
 * y[t, n] = sum_k x[t, k] * w[n, k]  (bf16 in, fp32 accumulate, bf16 out):
 * the projection inside every MLX nn.Linear of the verify forward
 * (qwen3_tree.py:50-52,78,82).  tcgen05 swap-AB GEMM: w streams through
 * TMA into 128-row tiles, x (t_pad rows, multiple of 16, <= 256) is the
 * N side.  k % 64 == 0.  workspace: dtree_linear_workspace_bytes(). */
DTREE_API size_t dtree_linear_workspace_bytes(int t_pad, int n);
DTREE_API int dtree_linear_bf16(const void* x, int t_pad, int k, const void* w, int n, void* y, void* workspace,
                      size_t workspace_bytes, int split_k, void* stream);

/* 4-bit affine linear: y[t, n] = sum_k x[t, k] * (scales[n, k/64] * q[n, k]
 * + biases[n, k/64]), the forward of the MLX QuantizedLinear layers that
 * quantize_model(bits=4, group_size=64) puts in the target (api.py:46-54;
 * mx.quantized_matmul(transpose=True), also adapters.py:63-71).  MLX layout:
 * w_packed uint32 [n][k/8], element 8j+i of a row in bits 4i..4i+3 of word
 * j; scales, biases bf16 [n][k/64].  The weights are dequantized into tensor
 * memory (one bf16 rounding of scale*q + bias) and fed to the same tcgen05
 * GEMM as dtree_linear_bf16.  k % 64 == 0.  workspace:
 * dtree_linear_q4_workspace_bytes(t_pad, n, k) (the GEMM's, plus the scales
 * and biases repacked for this call into 1 KB blocks per 128 rows x 128 K). */
DTREE_API size_t dtree_linear_q4_workspace_bytes(int t_pad, int n, int k);
DTREE_API int dtree_linear_q4(const void* x, int t_pad, int k, const void* w_packed, const void* scales,
                    const void* biases, int n, void* y, void* workspace, size_t workspace_bytes, int split_k,
                    void* stream);

/* LM head fused with argmax (adapters.py:114-118 lm_head_argmax +
 * runtime.py:12-19 at temperature 0): out[t] = argmax_v bf16(h[t]·E[v]),
 * ties to the smallest v; logits never reach HBM.  workspace:
 * dtree_lm_head_workspace_bytes(). */
DTREE_API size_t dtree_lm_head_workspace_bytes(int t_pad);
DTREE_API int dtree_lm_head_argmax(const void* h, int t_pad, int n_rows, int hidden, const void* embed, int vocab,
                         int32_t* out, void* workspace, size_t workspace_bytes, void* stream);

/* LM head fused with sampling at `temperature` (runtime.py:12-19
 * sample_tokens: categorical over logits / T, used by the parallel-replay
 * verify, runtime.py:177 and dtree_runtime.py:460): out[t] = argmax_v
 * (bf16(h[t]·E[v]) / T + G), G standard Gumbel noise from Philox keyed by
 * (seed, state->step, t, v) -- a draw from softmax(logits / T) without
 * writing the logits.  temperature < 1e-5: the argmax above (state may then
 * be NULL). */
DTREE_API int dtree_lm_head_sample(const void* h, int t_pad, int n_rows, int hidden, const void* embed, int vocab,
                         float temperature, uint32_t seed, const dtree_step_state* state, int32_t* out,
                         void* workspace, size_t workspace_bytes, void* stream);

/* ----------------------------------------------------- tree attention
 * softmax(q k^T / sqrt(head_dim) + tree mask) v for the tree rows of one
 * verify forward (replaces the masked scaled_dot_product_attention call of
 * dtree_mlx/qwen3_tree.py:67-76 with the ancestor mask of
 * dtree_mlx/dtree_runtime.py:190-191).  q: [n_nodes][ldq] bf16 (after q-norm
 * and RoPE); k_plane / v_plane: [n_kv_heads][kv_cap][head_dim] bf16 holding
 * the prefix [0, state->start) and the tree keys at slots start..start+n-1;
 * anc_mask: [n_nodes][2] (bit j of node t: tree slot j visible); out:
 * [n_nodes][ldq] bf16.  head_dim 64, 128 (tcgen05) or 256; splits <= 32
 * (0: automatic — one CTA per SM, or for head_dim 64 / 128 with
 * kv_cap <= 1024 ceil(kv_cap / 128) CTAs per KV head as one thread-block
 * cluster that merges its splits in shared memory). */
DTREE_API size_t dtree_tree_attention_workspace_bytes(int n_q_heads, int n_nodes, int head_dim, int splits);
DTREE_API int dtree_tree_attention(const void* q, int ldq, const void* k_plane, const void* v_plane, int kv_cap,
                                   int n_q_heads, int n_kv_heads, int head_dim, int n_nodes,
                                   const dtree_step_state* state, const uint64_t* anc_mask, void* out, int splits,
                                   void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------- Qwen3.5 gated-DeltaNet tree kernels
 * dtype / state_dtype: 0 = f32, 1 = bf16 (the reference's InT / StT).
 * parents[t] < t for t > 0, parents[0] = -1 (the base state).
 *
 * Replaces tree_conv1d_kernel (qwen35_tree_kernels.py:86-134, 180-206): the
 * depthwise causal conv (width keep+1) of every tree node over the `keep`
 * inputs before it on its root path (base_conv_state [keep][conv_dim] when
 * the path is shorter), SiLU, rounded to dtype.  qkv row t starts at
 * qkv + t*ld_qkv; conv_weight is [keep+1][conv_dim] (weight k multiplies
 * the k-th oldest input, the last one the node's own input); conv_out
 * [n_nodes][conv_dim]; conv_states (nullable) [n_nodes][keep][conv_dim]
 * receives each node's window as the reference does. */
DTREE_API int dtree_tree_conv1d(const void* qkv, int ld_qkv, const void* base_conv_state, const void* conv_weight,
                      const int32_t* parents, int n_nodes, int conv_dim, int keep, int dtype, void* conv_out,
                      void* conv_states, void* stream);

/* Replaces tree_gated_delta_kernel (qwen35_tree_kernels.py:8-82, 207-224):
 * per node, S = S_parent * g; kv = S k; delta = (v - kv) * beta;
 * S += k delta; y = S q; the node's state is S rounded to dtype.
 * q, k [n_nodes][n_k_heads][head_k_dim]; v, y [n_nodes][n_v_heads][head_v_dim];
 * g f32 and beta (dtype) [n_nodes][n_v_heads]; state_in (state_dtype)
 * [n_v_heads][head_v_dim][head_k_dim]; node_states (nullable, state_dtype)
 * [n_nodes][n_v_heads][head_v_dim][head_k_dim].  head_k_dim in {32, 64,
 * 128, 256}. */
DTREE_API int dtree_tree_gated_delta(const void* q, const void* k, const void* v, const float* g, const void* beta,
                           const void* state_in, const int32_t* parents, int n_nodes, int n_k_heads, int n_v_heads,
                           int head_k_dim, int head_v_dim, int dtype, int state_dtype, void* y, void* node_states,
                           void* stream);

/* Recurrent half of commit_qwen35_tree_path (qwen35_tree.py:708-732):
 * recurrent_state <- the state of the deepest accepted node, obtained by
 * replaying the accepted path accepted[0 .. state->n_accepted) (root first)
 * from recurrent_state with the per-node arithmetic and rounding of
 * dtree_tree_gated_delta, so per-node states never need to be stored.
 * Inputs as dtree_tree_gated_delta. */
DTREE_API int dtree_gated_delta_commit(const void* q, const void* k, const void* v, const float* g, const void* beta,
                             const int32_t* accepted, const dtree_step_state* state, int n_nodes, int n_k_heads,
                             int n_v_heads, int head_k_dim, int head_v_dim, int dtype, int state_dtype,
                             void* recurrent_state, void* stream);

/* Conv half of commit_qwen35_tree_path: base_conv_state <- the window of the
 * deepest accepted node (its last `keep` inputs), read from the tree's conv
 * inputs qkv (as in dtree_tree_conv1d) and the old base state. */
DTREE_API int dtree_conv_state_commit(const void* qkv, int ld_qkv, const int32_t* parents, const int32_t* accepted,
                            const dtree_step_state* state, int n_nodes, int conv_dim, int keep, int dtype,
                            void* base_conv_state, void* stream);

/* ------------------------------------------------- Qwen3 tree verify
 * A Qwen3 target (mlx-lm qwen3 layer math: RMSNorm, q/k RMSNorm, half-split
 * RoPE, GQA attention, SwiGLU, tied LM head) held as device pointers.
 * Weight layouts (bf16, row-major [out, in]):
 *   qkv      [(n_heads + 2*n_kv_heads)*head_dim, hidden]  rows q | k | v
 *   o_proj   [hidden, n_heads*head_dim]
 *   gate_up  [2*ffn, hidden] in 64-row blocks g0 u0 g1 u1 ... (gate rows
 *            64j..64j+63 then the matching up rows)
 *   down     [hidden, ffn]
 * kv_cache: [layers][2][n_kv_heads][kv_capacity][head_dim] bf16.
 * With quant_bits == 4 the four projection pointers of each layer are MLX
 * packed 4-bit weights (uint32 [rows][in/8], same row order as above) and
 * q4_layer[l] holds their bf16 scales / biases ([rows][in/64]); embedding
 * and norms stay bf16 (the tied LM head is not quantized). */
typedef struct dtree_qwen3_layer {
  const void* input_norm;
  const void* qkv;
  const void* q_norm;
  const void* k_norm;
  const void* o_proj;
  const void* post_norm;
  const void* gate_up;
  const void* down;
} dtree_qwen3_layer;

typedef struct dtree_qwen3_q4_layer {
  const void* qkv_scales;
  const void* qkv_biases;
  const void* o_scales;
  const void* o_biases;
  const void* gate_up_scales;
  const void* gate_up_biases;
  const void* down_scales;
  const void* down_biases;
} dtree_qwen3_q4_layer;

typedef struct dtree_qwen3_desc {
  /* configuration */
  int hidden, layers, n_heads, n_kv_heads, head_dim, ffn, vocab;
  float rope_theta, rms_eps;
  int t_cap;          /* max tree rows per forward (<= DTREE_MAX_TREE), multiple of 16 */
  int kv_capacity;    /* positions per (layer, kv-head) plane */
  int n_capture;      /* hidden-capture layers (verifier_hidden), <= 16 */
  int capture_layers[16];
  /* weights */
  const void* embed;       /* [vocab, hidden], also the tied LM head */
  const void* final_norm;  /* [hidden] */
  const dtree_qwen3_layer* layer;  /* [layers] */
  /* caller-owned buffers (sizes from dtree_qwen3_buffer_bytes) */
  void* kv_cache;
  void* h;            /* [t_cap, hidden] residual stream */
  void* xn;           /* [t_cap, hidden] normalized activations */
  void* q;            /* [t_cap, n_heads*head_dim] */
  void* attn;         /* [t_cap, n_heads*head_dim] */
  void* act;          /* [t_cap, ffn] */
  void* norm_out;     /* [t_cap, hidden] final-norm hidden (norm_hidden_states) */
  void* capture;      /* [t_cap, hidden*n_capture] verifier_hidden */
  void* workspace;    /* fp32 split-K / attention partials + counters */
  size_t workspace_bytes;
  /* weight quantization: 0 / 16 = bf16; 4 = MLX affine 4-bit, group_size 64
   * (api.py:46-54 target_quant_bits / target_quant_group_size) */
  int quant_bits;
  int group_size;
  const dtree_qwen3_q4_layer* q4_layer;  /* [layers] when quant_bits == 4 */
  /* verify forward schedule: 0 = the per-kernel chain (default); 1 = the
   * persistent single-launch forward (one CTA per SM, weights streamed
   * through the glue phases) where the model supports it (bf16 weights,
   * head_dim 128, <= 64 tree rows), else the chain */
  int verify_path;
  /* 4-bit tied LM head: mlx-lm's quantize_model (api.py:46-54) quantizes
   * the embedding too, so the reference's LM head of a 4-bit target is the
   * quantized embedding's as_linear (adapters.py:491).  MLX packed
   * [vocab][hidden/8] and bf16 scales / biases [vocab][hidden/64]; all null:
   * the bf16 `embed` is the LM head.  `embed` stays the table the input rows
   * are gathered from (the dequantized rows for a 4-bit embedding). */
  const void* embed_q4_packed;
  const void* embed_q4_scales;
  const void* embed_q4_biases;
} dtree_qwen3_desc;

typedef struct dtree_qwen3_model dtree_qwen3_model;

/* Bytes each caller buffer must hold: out[0..8] = kv_cache, h, xn, q, attn,
 * act, norm_out, capture, workspace.  With quant_bits == 4 the workspace
 * also holds every projection's scales and biases repacked into 1 KB blocks
 * (128 rows x 128 K); dtree_qwen3_create fills them from q4_layer after a
 * device synchronize, so the weights must be complete when it is called and
 * later changes to the scales / biases need a new model. */
DTREE_API int dtree_qwen3_buffer_bytes(const dtree_qwen3_desc* desc, size_t out[9]);
DTREE_API int dtree_qwen3_create(const dtree_qwen3_desc* desc, dtree_qwen3_model** out);
DTREE_API int dtree_qwen3_destroy(dtree_qwen3_model* model);

/* Replaces Qwen3TargetAdapter.forward_tree_with_hidden_states
 * (adapters.py:568-597, per-layer qwen3_tree.py:39-83) fused with
 * lm_head_argmax: embeds tree_tokens[0..n_nodes), runs every layer with
 * per-node RoPE positions and the ancestor-mask tree attention over the
 * cache prefix [0, state->start) plus the tree, writes the new K/V at cache
 * slots [start, start + n_nodes), leaves norm_hidden in desc.norm_out and
 * verifier_hidden in desc.capture, and writes the greedy posterior token of
 * every node to `posterior` (if non-NULL).  n_nodes <= t_cap. */
DTREE_API int dtree_qwen3_forward_tree(dtree_qwen3_model* model, const int32_t* tree_tokens, const int32_t* positions,
                             const uint64_t* anc_mask, int n_nodes, const dtree_step_state* state,
                             int32_t* posterior, void* stream);

/* Posterior tokens of later forwards are sampled at `temperature`
 * (dtree_lm_head_sample with this seed and the forward's state->step)
 * instead of the greedy argmax; temperature < 1e-5 restores the argmax.
 * Replaces the temperature argument of the parallel-replay verify
 * (runtime.py:160-215, dtree_runtime.py:455-470). */
DTREE_API int dtree_qwen3_set_sampling(dtree_qwen3_model* model, float temperature, uint32_t seed);

/* Bound on prefix + tree keys (state->start + n_nodes) that the following
 * forwards attend over (0: the KV capacity, the default).  A launch-shape
 * hint for the tree attention (the scaled_dot_product_attention step of
 * dtree_mlx/qwen3_tree.py:67-76): while the bound is at most 1024 the KV
 * splits of a head run as one cluster of ceil(bound / 128) CTAs that merge
 * their partials in shared memory, otherwise as ~one CTA per SM merged by a
 * second kernel.  Both shapes split the keys into the same 128-key blocks
 * and merge them in the same order while the keys fit the bound, so the
 * outputs are bit-identical; past the bound the cluster shape stays correct
 * with longer splits (rounded differently).  Forwards captured in a CUDA
 * graph keep the shape that was current at capture. */
DTREE_API int dtree_qwen3_set_attention_keys(dtree_qwen3_model* model, int max_keys);

/* Dense prompt prefill: replaces Qwen3TargetAdapter.forward_with_hidden_states
 * over the prompt (adapters.py:494-533; the prefill at dtree_runtime.py:342-349
 * and runtime.py:459-465).  Rows t < n_rows (tokens[t] at RoPE position
 * positions[t]) run causally after the state->start cached rows; their K/V go
 * to cache slots state->start + t (state->start + n_rows <= kv_capacity).
 * Each projection is one dense tensor-core GEMM over all rows (the weights
 * stream once per call), the attention one launch per layer over the rows'
 * 128-row chunks.  hidden_out [n_rows][ld_hidden_out] bf16 receives the
 * captured layers' hidden states (column block c = capture_layers[c]; may be
 * null when n_capture == 0); norm_out (nullable) [n_rows][hidden] bf16 the
 * final-normed rows; next_token[0] = argmax of the last row's logits
 * (or a sample at the model's temperature, dtree_qwen3_set_sampling, keyed by
 * state->step, row 0).  workspace >= dtree_qwen3_prefill_workspace_bytes(desc,
 * n_rows) device bytes, used by nothing else while the call's kernels run. */
DTREE_API size_t dtree_qwen3_prefill_workspace_bytes(const dtree_qwen3_desc* desc, int n_rows);
DTREE_API int dtree_qwen3_prefill(dtree_qwen3_model* model, const int32_t* tokens, const int32_t* positions,
                                  int n_rows, const dtree_step_state* state, void* hidden_out, int ld_hidden_out,
                                  void* norm_out, int32_t* next_token, void* workspace, size_t workspace_bytes,
                                  void* stream);

/* ----------------------------------------------- DFlash block drafter
 * The drafter (DFlashDraftModel, draft.py:318-367) is a stack of Qwen3
 * decoder layers held as a dtree_qwen3 model whose `embed` is the TARGET's
 * embedding (noise embedding and LM head, dtree_runtime.py:366-375) and
 * whose KV cache is the draft cache.  One draft step:
 *   dtree_dflash_context  -- precompute_context_kv (draft.py:172-187, 329-
 *       336): ctx = RMSNorm(fc(target_hidden), hidden_norm); every layer's
 *       k_norm(k_proj(ctx)) (RoPE at the row's position) and v_proj(ctx) go to
 *       the draft cache.  ctx_base >= 0: rows [0, n_rows) at positions
 *       ctx_base + t (prompt context); ctx_base < 0: the rows the last step
 *       accepted, count state->n_accepted at positions state->start - count + t
 *       (target_hidden row t = accepted node t, as dtree_gather_rows leaves it).
 *       target_hidden is [n_rows][ld_hidden] bf16, the first `width` columns
 *       used (hidden * number of target layers); fc_weight [hidden][width].
 *   dtree_dflash_block    -- block tokens [state->root_token, mask ...] and
 *       positions state->start + i.
 *   dtree_qwen3_forward_logits -- the noise forward (attention to the whole
 *       draft cache plus the block, no mask: anc rows all ones) with the
 *       final RMSNorm and fp32 logits [pad16(n_rows)][vocab] of every row;
 *       rows 1 .. block-1 are the draft logits (dtree_runtime.py:375). */
DTREE_API int dtree_dflash_context(dtree_qwen3_model* model, const void* fc_weight, const void* hidden_norm,
                         const void* target_hidden, int ld_hidden, int width, int n_rows, int ctx_base,
                         const dtree_step_state* state, void* stream);

/* dtree_dflash_context for a context-only draft cache
 * (ContextOnlyDraftKVCache, draft.py:69-112, which the reference uses for
 * Qwen3.5 targets, api.py:62-64): only context rows are cached, the first
 * `sink` of them and a sliding window of the last `window`, as a ring --
 * context row r (counted from the prompt's first row) sits in slot r if
 * r < sink, else sink + (r - sink) % window.  RoPE positions stay the rows'
 * real positions, so the attended set equals the reference's sink + window
 * concatenation.  ring_state (a dtree_step_state the caller owns, zeroed for
 * a new sequence): `reserved` counts the rows appended so far, `start` =
 * min(reserved, sink + window) is the attended context length -- pass
 * ring_state as the state of dtree_qwen3_forward_logits for the block (its
 * rows land in slots start..start+block-1, positions from the positions
 * buffer).  Rows appended: n_rows at positions ctx_base + t when
 * ctx_base >= 0 (prompt), else state->n_accepted rows ending at
 * state->start.  kv_capacity >= sink + window + t_cap. */
DTREE_API int dtree_dflash_context_ring(dtree_qwen3_model* model, const void* fc_weight, const void* hidden_norm,
                                        const void* target_hidden, int ld_hidden, int width, int n_rows,
                                        int ctx_base, const dtree_step_state* state, dtree_step_state* ring_state,
                                        int sink, int window, void* stream);
DTREE_API int dtree_dflash_block(const dtree_step_state* state, int mask_token_id, int block, int32_t* tokens,
                       int32_t* positions, void* stream);
DTREE_API int dtree_qwen3_forward_logits(dtree_qwen3_model* model, const int32_t* tokens, const int32_t* positions,
                               const uint64_t* anc_mask, int n_rows, const dtree_step_state* state, float* logits,
                               void* stream);

/* ------------------------------------------ Qwen3.5 hybrid tree verify
 * A Qwen3.5 text model (custom_qwen35_model.py:777-924): layer l is a gated
 * DeltaNet layer unless (l + 1) % full_attention_interval == 0, then a gated
 * full-attention layer; SwiGLU MLP and RMSNorms around both; tied LM head.
 * Weights bf16, row-major [out, in]:
 *   DeltaNet in_proj  [2*lin_key_dim + lin_value_dim + 2*lin_v_heads, hidden]
 *                     rows: in_proj_qkv | in_proj_z | in_proj_b | in_proj_a
 *            conv_weight [conv_kernel][conv_dim] (conv1d.weight[:, :, 0].T)
 *   attention qkv     [n_heads*2*head_dim + 2*n_kv_heads*head_dim, hidden]:
 *                     q_proj rows (per head [q | gate]), then k_proj, v_proj
 *   gate_up as dtree_qwen3_layer.  lin_key_dim = lin_k_heads*lin_k_dim etc.
 * State (caller-owned, persists across steps):
 *   kv_cache   [n_attn][2][n_kv_heads][kv_capacity][head_dim] bf16
 *   conv_state [n_linear][conv_kernel-1][conv_dim] bf16
 *   rec_state  [n_linear][lin_v_heads][lin_v_dim][lin_k_dim] f32 */
typedef struct dtree_qwen35_linear_layer {
  const void* input_norm;
  const void* in_proj;
  const void* conv_weight;
  const void* norm;      /* [lin_v_dim] RMSNormGated weight */
  const void* out_proj;  /* [hidden, lin_v_heads*lin_v_dim] */
  const void* post_norm;
  const void* gate_up;
  const void* down;
} dtree_qwen35_linear_layer;

typedef struct dtree_qwen35_attn_layer {
  const void* input_norm;
  const void* qkv;
  const void* q_norm;  /* [head_dim] */
  const void* k_norm;
  const void* o_proj;  /* [hidden, n_heads*head_dim] */
  const void* post_norm;
  const void* gate_up;
  const void* down;
} dtree_qwen35_attn_layer;

typedef struct dtree_qwen35_desc {
  int hidden, layers, full_attention_interval, ffn, vocab;
  int n_heads, n_kv_heads, head_dim;
  float rope_theta, partial_rotary_factor, rms_eps;
  int lin_k_heads, lin_v_heads, lin_k_dim, lin_v_dim, conv_kernel;
  int t_cap, kv_capacity, n_capture;
  int capture_layers[16];
  const void* embed;       /* [vocab, hidden], also the tied LM head */
  const void* final_norm;
  const dtree_qwen35_linear_layer* linear_layers;  /* [n_linear], layer order */
  const dtree_qwen35_attn_layer* attn_layers;      /* [n_attn] */
  const float* a_log;      /* [n_linear][lin_v_heads] f32 */
  const void* dt_bias;     /* [n_linear][lin_v_heads] bf16 */
  /* caller-owned state and buffers (sizes from dtree_qwen35_buffer_bytes) */
  void* kv_cache;
  void* conv_state;
  void* rec_state;
  void* h;         /* [t_cap, hidden] residual stream */
  void* xn;        /* [t_cap, hidden] */
  void* q;         /* [t_cap, max(n_heads*head_dim, lin_v_heads*lin_v_dim)] */
  void* gate;      /* [t_cap, n_heads*head_dim] attention output gate */
  void* attn;      /* [t_cap, max(n_heads*head_dim, lin_v_heads*lin_v_dim)] */
  void* act;       /* [t_cap, ffn] */
  void* norm_out;  /* [t_cap, hidden] */
  void* capture;   /* [t_cap, hidden*n_capture] */
  void* lin_proj;  /* [n_linear][t_cap][in_proj rows] DeltaNet projections (kept for commit) */
  void* lin_qkv;   /* [n_linear][t_cap][conv_dim] conv outputs (kept for commit) */
  void* workspace;
  size_t workspace_bytes;
} dtree_qwen35_desc;

typedef struct dtree_qwen35_model dtree_qwen35_model;

/* out[0..13] = kv_cache, conv_state, rec_state, h, xn, q, gate, attn, act,
 * norm_out, capture, lin_proj, lin_qkv, workspace. */
DTREE_API int dtree_qwen35_buffer_bytes(const dtree_qwen35_desc* desc, size_t out[14]);
DTREE_API int dtree_qwen35_create(const dtree_qwen35_desc* desc, dtree_qwen35_model** out);
DTREE_API int dtree_qwen35_destroy(dtree_qwen35_model* model);

/* mode 0 -- tree verify, replaces forward_qwen35_tree_with_hidden_states
 * (qwen35_tree.py:629-705) + lm_head_argmax: DeltaNet layers run the tree
 * conv / gated-delta kernels from the committed conv / recurrent state with
 * per-node rounding (state is not modified); attention layers attend to the
 * cache prefix [0, state->start) plus the tree (ancestor masks) and write
 * the tree's K/V at slots start + t.  parents[t] < t, parents[0] = -1.
 * mode 1 -- sequence (prefill chunk, adapters.py:494-533): parents must be a
 * chain, no per-node rounding, and the conv / recurrent states advance to
 * the last token.  posterior (nullable) receives the greedy token per node. */
DTREE_API int dtree_qwen35_forward(dtree_qwen35_model* model, const int32_t* tokens, const int32_t* positions,
                         const int32_t* parents, const uint64_t* anc_mask, int n_nodes, int mode,
                         const dtree_step_state* state, int32_t* posterior, void* stream);

/* commit_qwen35_tree_path (qwen35_tree.py:708-732) for the accepted path
 * accepted[0 .. state->n_accepted) (root first) of the last tree forward:
 * attention layers keep the accepted K/V rows (moved to start .. start+n-1),
 * DeltaNet layers take the deepest accepted node's conv window and
 * recurrent state (replayed from the committed state).  Call before
 * dtree_step_commit. */
DTREE_API int dtree_qwen35_commit(dtree_qwen35_model* model, const int32_t* parents, const int32_t* accepted,
                        const dtree_step_state* state, void* stream);

/* As dtree_qwen3_set_sampling, for the hybrid model. */
DTREE_API int dtree_qwen35_set_sampling(dtree_qwen35_model* model, float temperature, uint32_t seed);

/* Dense prompt prefill of the hybrid: replaces Qwen35TargetAdapter's
 * forward_with_hidden_states over the prompt (adapters.py:216-450, called by
 * dtree_runtime.py:342-349) with dtree_qwen3_prefill's contract (rows after
 * state->start, K/V of the attention layers to slots state->start + t,
 * hidden_out / norm_out / next_token as there).  Each DeltaNet layer's conv
 * and recurrent state start from the model's current state (zero for a new
 * sequence) and end at the last row: the recurrence runs as one chain in
 * f32, as mlx-lm's sequence kernel does.  workspace >=
 * dtree_qwen35_prefill_workspace_bytes(desc, n_rows). */
DTREE_API size_t dtree_qwen35_prefill_workspace_bytes(const dtree_qwen35_desc* desc, int n_rows);
DTREE_API int dtree_qwen35_prefill(dtree_qwen35_model* model, const int32_t* tokens, const int32_t* positions,
                                   int n_rows, const dtree_step_state* state, void* hidden_out, int ld_hidden_out,
                                   void* norm_out, int32_t* next_token, void* workspace, size_t workspace_bytes,
                                   void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DTREE_B200_H_ */
