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
};

size_t attn_ws_bytes(int n_q_heads, int t_pad, int head_dim, int splits);
int attn_default_splits(int n_kv_heads, int n_q_heads, int n_nodes);
int attn_launch(const AttnParams& p, int head_dim, void* ws, size_t ws_bytes, cudaStream_t stream);

}  // namespace dtree
