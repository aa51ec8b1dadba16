// Persistent tree-verify forward (Qwen3, bf16 weights, head_dim 128): the
// whole per-layer chain of model.cu in ONE launch of one CTA per SM.  See
// fused.cu for the design.
#pragma once

#include "common.cuh"
#include "../../include/dtree_b200.h"

namespace dtree {

constexpr int kFusedMaxLayers = 64;
constexpr int kFusedJobs = 4;  // per layer: q|k|v, o_proj, gate|up, down_proj
constexpr int kFusedThreads = 384;

// phase counters per layer (monotone within one forward; zeroed before it)
enum FusedCounter : int {
  kCntN1 = 0,   // input RMSNorm rows done
  kCntQkv,      // q|k|v GEMM epilogues done (per CTA; fp32 split partials written)
  kCntFin,      // q/k norm + RoPE + K/V write done (per CTA)
  kCntAtt,      // attention split partials done (per CTA)
  kCntCmb,      // split merge done (per CTA)
  kCntO,        // o_proj GEMM epilogues done (per CTA)
  kCntN2,       // post-attention RMSNorm rows done
  kCntGu,       // gate|up + SwiGLU done (per CTA)
  kCntDn,       // down_proj GEMM epilogues done (per CTA)
  kCntPerLayer,
};

struct FusedLayerPtrs {
  const __nv_bfloat16* input_norm;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  const __nv_bfloat16* post_norm;
  __nv_bfloat16* capture;  // verifier_hidden block of this layer's output (nullptr: not captured)
};

struct FusedParams {
  // per forward
  const int32_t* tokens;
  const int32_t* positions;
  const uint64_t* anc;
  const dtree_step_state* state;
  int n_rows;
  // model
  int layers, hidden, n_heads, n_kv_heads, ffn, vocab;
  float eps, rope_log2_theta, scale_log2;
  int kv_cap;
  int ldc;  // row stride of the verifier_hidden capture buffer (elements)
  const __nv_bfloat16* embed;
  const __nv_bfloat16* final_norm;
  const CUtensorMap* wmaps;  // [layers][kFusedJobs] weight maps (global memory)
  const FusedLayerPtrs* lp;  // [layers]
  __nv_bfloat16* kv;         // [layers][2][n_kv_heads][kv_cap][128]
  __nv_bfloat16* h;
  __nv_bfloat16* xn;
  __nv_bfloat16* q;
  __nv_bfloat16* attn;
  __nv_bfloat16* act;
  __nv_bfloat16* norm_out;
  // workspace
  float* qkv_part;        // [qkv_split][TPAD][qkv width]
  float* o_part;          // [o_split][TPAD][hidden]
  float* dn_part;         // [dn_split][TPAD][hidden]
  float* gu_ws;           // [grid][2][TPAD][128] stream-K partial tiles
  uint32_t* gu_tile_cnt;  // [gate|up tiles], zero between uses
  float* att_o;           // [att_splits][n_heads * n_rows][128]
  float* att_ml;          // [att_splits][n_heads * n_rows][2]
  uint32_t* cnt;          // [layers][kCntPerLayer], then the abort word
  uint32_t* norm_cnt;     // [2 * layers + 1][64] per-row slice arrivals of each norm step
  float* norm_ss;         // [64][8] per-slice sums of squares of the current norm step
  int qkv_split, o_split, dn_split, att_splits, att_rb;
  int grid;
};

struct FusedPlan {
  CUtensorMap xmap_xn, xmap_attn, xmap_act;
  FusedParams p;
  int t_pad;
  int smem;
};

// host API (fused.cu)
bool fused_supported(const dtree_qwen3_desc& d);
size_t fused_ws_bytes(const dtree_qwen3_desc& d);
int fused_init(const dtree_qwen3_desc& d, void* ws, const std::pair<int, __nv_bfloat16*>* captures, int n_capture);
int fused_plan(const dtree_qwen3_desc& d, void* ws, int t_pad, FusedPlan* plan);
int fused_launch(FusedPlan& plan, const int32_t* tokens, const int32_t* positions, const uint64_t* anc, int n_rows,
                 const dtree_step_state* state, cudaStream_t stream);

}  // namespace dtree
