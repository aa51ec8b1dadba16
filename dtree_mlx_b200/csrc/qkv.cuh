// Finish of a split-K q|k|v projection (see qkv.cu).
#pragma once

#include "common.cuh"
#include "../../include/dtree_b200.h"

namespace dtree {

struct QkvFinishParams {
  const float* partials;  // [split][part_rows][width]
  int split, part_rows, width;
  const __nv_bfloat16* dense;  // non-null: the projection as bf16 [rows][width] instead of partials
  int n_rows;                  // rows (set by qkv_finish_launch)
  int head_dim, n_q_heads, n_kv_heads;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  float eps, rope_log2_theta;
  const int32_t* positions;
  const dtree_step_state* state;
  __nv_bfloat16* q_out;  // [t_pad][n_q_heads*head_dim]
  __nv_bfloat16* k_cache;  // [n_kv_heads][kv_cap][head_dim]
  __nv_bfloat16* v_cache;
  int kv_cap;
  int gated;                // q rows are [q | gate] per head
  __nv_bfloat16* gate_out;  // [t_pad][n_q_heads*head_dim] (gated only)
  int rot_dims;             // rotated features per head (0: all)
  // context rows (DFlash drafter K/V append, n_q_heads = 0): row t goes to
  // slot = position = base + t for t < count, where slot_mode 1 takes
  // count = state->n_accepted, base = state->start - count (the rows the last
  // step accepted) and slot_mode 2 the host values ctx_base / ctx_count
  int slot_mode;
  int ctx_base, ctx_count;
  // context-only draft cache (sink + sliding window, draft.py:69-112): the
  // context row r (r-th row appended since the prompt) goes to slot r for
  // r < ring_sink, else ring_sink + (r - ring_sink) % ring_window; in
  // slot_mode 1 the rows continue at ring_state->reserved (rows appended so
  // far).  ring_window 0: slot = row position.
  const dtree_step_state* ring_state;
  int ring_sink, ring_window;
};

// slot of context row r in a sink + window ring
__device__ __forceinline__ int ring_slot(int r, int sink, int window) {
  return r < sink ? r : sink + (r - sink) % window;
}

int qkv_finish_launch(const QkvFinishParams& p, int n_rows, cudaStream_t stream);
// prompt rows: dense bf16 projection in, slots start + t (slot_mode 0)
int qkv_rows_launch(const QkvFinishParams& p, int n_rows, cudaStream_t stream);

}  // namespace dtree
