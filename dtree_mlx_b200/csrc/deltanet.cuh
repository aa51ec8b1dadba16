// Qwen3.5 gated-DeltaNet kernel interface (see deltanet.cu).
#pragma once

#include "common.cuh"
#include "../../include/dtree_b200.h"

namespace dtree {

struct ConvParams {
  const void* x;          // InT [T][ldx] (first conv_dim columns are the conv channels)
  int ldx;
  const void* base;       // InT [keep][conv_dim] (oldest row first)
  const void* weight;     // InT [keep + 1][conv_dim]
  const int32_t* parents; // [T]
  int n_nodes, conv_dim, keep;
  void* out;              // InT [T][ldo]
  int ldo;
  void* node_states;      // InT [T][keep][conv_dim] (nullable)
  // q / k head normalization of the Qwen3.5 layer (n_norm_heads = 0: off):
  // heads [0, n_q_heads) -> rms_norm(x) / D, heads [n_q_heads, n_norm_heads)
  // -> rms_norm(x) / sqrt(D), each rounded to InT after the norm and after
  // the scale (dtree_mlx/qwen35_tree.py:290-291)
  int n_norm_heads, n_q_heads;
};

struct DeltaParams {
  const void* q;        // InT [T][ldqk]: head h at column h*DK (already normalized)
  const void* k;        // InT [T][ldqk]
  int ldqk;
  const void* v;        // InT [T][ldv]: head h at column h*Dv
  int ldv;
  // gates: either g (f32 [T][Hv]) and beta (InT [T][Hv]) given, or computed
  // from the projections a, b (InT [T][ldab]) with A_log (f32 [Hv]) and
  // dt_bias (InT [Hv]): g = exp(-exp(A_log) softplus(a + dt_bias)),
  // beta = sigmoid(b)  (mlx-lm gated_delta.compute_g / qwen35_tree.py:292-293)
  const float* g;
  const void* beta;
  const void* a;
  const void* b;
  int ldab;
  const float* a_log;
  const void* dt_bias;
  const void* state_in;  // StT [Hv][Dv][DK]
  const int32_t* parents;
  int n_nodes, n_k_heads, n_v_heads, dv;
  void* y;               // InT [T][Hv][Dv] (row stride ldy)
  int ldy;
  void* node_states;     // StT [T][Hv][Dv][DK] (nullable)
  int rows_per_cta;      // warps per CTA (state rows of one head)
  // prefill mode (chain parents only): no per-node rounding (the state stays
  // in f32 registers as in mlx-lm's sequence kernel) and the last node's
  // state is written to final_state (StT [Hv][Dv][DK])
  int no_round;
  void* final_state;
  // commit (replay) mode: the accepted path of length state->n_accepted,
  // node indices in `path`; state_out is advanced in place
  const int32_t* path;
  const dtree_step_state* st;
  void* state_out;
  // multi-layer replay: per-layer strides in elements (0 for a single layer)
  size_t layer_stride_qk, layer_stride_v, layer_stride_ab, layer_stride_state;
  int layer_stride_params;  // elements between layers' a_log / dt_bias
};

int tree_conv1d_launch(const ConvParams& p, int dtype, int block, cudaStream_t st);
// prompt rows as one chain from the base window (parents unused), bf16
int conv1d_seq_launch(const ConvParams& p, int block, cudaStream_t st);
int tree_gated_delta_launch(const DeltaParams& p, int dk, int dtype, int state_dtype, cudaStream_t st);
// prompt rows as one chain, bf16 inputs, f32 state (state_in -> final_state;
// gates from a / b); any n_nodes
int gated_delta_seq_launch(const DeltaParams& p, int dk, cudaStream_t st);
int gated_delta_replay_launch(const DeltaParams& p, int dk, int dtype, int state_dtype, int layers, cudaStream_t st);
int conv_state_commit_launch(const ConvParams& p, int dtype, const int32_t* path, const dtree_step_state* state,
                             int layers, size_t layer_stride_x, size_t layer_stride_base, int fixed_node,
                             cudaStream_t st);
int rmsnorm_gated_launch(const __nv_bfloat16* y, int ldy, const __nv_bfloat16* z, int ldz, const __nv_bfloat16* w,
                         float eps, __nv_bfloat16* out, int ldo, int n_rows, int heads, int head_dim,
                         cudaStream_t st);

}  // namespace dtree
