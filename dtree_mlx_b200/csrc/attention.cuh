// Tree attention interface (see attention.cu).
#pragma once

#include "common.cuh"
#include "../../include/dtree_b200.h"

namespace dtree {

struct AttnParams {
  const __nv_bfloat16* q;  // [t_pad][n_q_heads*hd]
  int ldq;
  const __nv_bfloat16* k;  // layer K planes [n_kv_heads][cap][hd]
  const __nv_bfloat16* v;
  int cap;
  int n_q_heads, n_kv_heads;
  int n_nodes;
  const dtree_step_state* state;
  const uint64_t* anc;  // [n_nodes][2]
  float scale_log2;     // softmax scale * log2(e)
  int splits;
  float* part_o;        // [splits][n_q_heads*n_nodes][hd]
  float* part_ml;       // [splits][n_q_heads*n_nodes][2]
  __nv_bfloat16* out;   // [t_pad][n_q_heads*hd]
  int causal_prefix;    // unused (0): tree mask only
  const __nv_bfloat16* gate;  // [t_pad][n_q_heads*hd] output gate (nullable)
  int key_align;        // keys per split are a multiple of this (set by attn_launch)
  // prompt mode (chunk_rows > 0, tcgen05 path, one split): the n_nodes rows
  // are causal chunks of chunk_rows; chunk c holds rows [c*chunk_rows, ..)
  // at cache slots start + row, sees every key before its first row and the
  // chain mask `anc` within the chunk, and writes O / l straight to `out`
  int chunk_rows;
  int chunk_rbs;        // 128-row blocks per chunk (set by attn_prefill_launch)
  // tree path, head_dim 64 / 128, no gate: a bound on prefix + tree keys
  // (0: none).  When ceil(bound / 128) <= 8 (and a cluster of that many CTAs
  // for every row block and KV head can be resident at once) the splits are
  // that many CTAs of one
  // thread-block cluster per (row block, KV head) that merge in shared memory
  // (no attn_combine_kernel); keys past the bound stay correct (more passes
  // per CTA)
  int cluster_keys;
};

size_t attn_ws_bytes(int n_q_heads, int t_pad, int head_dim, int splits);
int attn_default_splits(int n_kv_heads, int n_q_heads, int n_nodes);
int attn_launch(const AttnParams& p, int head_dim, void* ws, size_t ws_bytes, cudaStream_t stream);
// kernel attributes and launch queries of the tree attention for head_dim
// (call once, outside stream capture)
int attn_prepare(int head_dim);
// prompt (causal) attention over n_nodes rows in chunks of 128; anc = the
// 128-row chain masks; head_dim 64 or 128; no workspace
int attn_prefill_launch(const AttnParams& p, int head_dim, cudaStream_t stream);

}  // namespace dtree
