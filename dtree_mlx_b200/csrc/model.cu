// Qwen3 tree-verify forward: the whole of
// Qwen3TargetAdapter.forward_tree_with_hidden_states (adapters.py:568-597)
// plus lm_head_argmax (adapters.py:114-118) as one launch sequence.
//
// Per layer (qwen3_tree.py:39-83):
//   xn   = RMSNorm(h, input_norm)                       rmsnorm / residual_rmsnorm
//   p    = xn @ Wqkv^T (split-K fp32 partials)          gemm<kEpiPartial>
//   q,k,v= sum(p); q/k RMSNorm + RoPE; k,v -> cache     qkv_finish_kernel
//   a    = softmax(q k^T / sqrt(d) + tree mask) v       tree_attn (+ combine; merged in-cluster <= 1024 keys)
//   p    = a @ Wo^T  (split-K fp32 partials)           gemm<kEpiPartial>
//   h   += sum(p); xn = RMSNorm(h, post_norm)           residual_rmsnorm_kernel
//   act  = silu(xn Wg^T) * (xn Wu^T)                    gemm<kEpiSwiglu>
//   p    = act @ Wd^T (split-K fp32 partials)           gemm<kEpiPartial>
//   h   += sum(p) (+ copy to verifier_hidden); next layer's RMSNorm
// then norm_out = RMSNorm(h, final_norm) and the fused LM-head argmax.
// The hidden-width projections (N = hidden, 20 tiles at the 4B shape) are
// split along K across ~all SMs; their partials are summed, in split order,
// by the RMSNorm kernel that follows anyway, so the GEMM has no reduction
// tail.
#include <algorithm>
#include <array>
#include <cmath>
#include <vector>

#include "attention.cuh"
#include "fused.cuh"
#include "gemm.cuh"
#include "qkv.cuh"

namespace dtree {

int rmsnorm_launch(const __nv_bfloat16* x, int ldx, const int32_t* tokens, const __nv_bfloat16* embed,
                   __nv_bfloat16* h_out, const __nv_bfloat16* w, __nv_bfloat16* y, int H, int n_rows, int t_pad,
                   float eps, cudaStream_t stream);
int residual_rmsnorm_launch(__nv_bfloat16* h, const float* partials, int n_split, int part_rows,
                            __nv_bfloat16* capture, int ldc, const __nv_bfloat16* w, __nv_bfloat16* xn, int H,
                            int n_rows, int t_pad, float eps, cudaStream_t stream);

// QkvFinishParams, qkv_finish_launch: qkv.cuh

constexpr int kAttnMaxSplits = 32;
constexpr int kMaxProjSplit = 16;  // split-K of the hidden-width projections (o_proj, down_proj)

// tree rows padded to a legal UMMA N (multiple of 16): budget 64 (65 rows)
// pads to 80, not 128
static int pad_rows(int n) {
  if (n <= 16) return 16;
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  if (n <= 80) return 80;
  return 128;
}
static int tpad_index(int t) { return t == 16 ? 0 : t == 32 ? 1 : t == 64 ? 2 : t == 80 ? 3 : 4; }

struct PlanSet {
  bool ready = false;
  std::vector<GemmPlan> qkv, o, gu, down;
  GemmPlan lm;
  GemmPlan lm_logits;  // fp32 logits (kEpiPartial, one split) for drafters
};

}  // namespace dtree

struct dtree_qwen3_model {
  dtree_qwen3_desc d;
  std::vector<dtree_qwen3_layer> layers;
  std::vector<dtree_qwen3_q4_layer> q4_layers;
  // 4-bit: per layer the repacked scale / bias blocks of qkv, o, gate|up,
  // down (in the workspace, filled at creation)
  std::vector<std::array<const void*, 4>> q4_sb;
  const void* embed_sb = nullptr;  // 4-bit LM head: the embedding's blocks
  dtree::PlanSet plans[5];
  void* gemm_ws = nullptr;
  size_t gemm_ws_bytes = 0;
  void* attn_ws = nullptr;
  size_t attn_ws_bytes = 0;
  float* proj_partials = nullptr;  // [kMaxProjSplit][t_pad][hidden] fp32
  void* fused_ws = nullptr;        // persistent-forward region (nullptr: not supported)
  dtree::FusedPlan fused[3];       // t_pad 16 / 32 / 64
  bool fused_ready[3] = {false, false, false};
  float inv_temp = 0.0f;  // posterior sampling (0: greedy argmax)
  uint32_t sample_seed = 0;
  int attn_keys = 0;      // bound on prefix + tree keys of the next forwards (0: the KV capacity)
};

namespace dtree {

static size_t gemm_ws_need(const dtree_qwen3_desc& d) { return gemm_ws_bytes(pad_rows(d.t_cap), 2 * num_sms()); }
static size_t attn_ws_need(const dtree_qwen3_desc& d) {
  return attn_ws_bytes(d.n_heads, d.t_cap, d.head_dim, kAttnMaxSplits);
}
// Split-K of a projection: enough CTAs for two per SM (a CTA's ring fits
// half an SM's shared memory, bf16 and 4-bit alike), so twice the weight
// bytes sit in the rings when the inputs arrive.
static int proj_split(const dtree_qwen3_desc& d, int n_out) {
  const int tiles = (n_out + 127) / 128;
  return std::max(1, std::min(kMaxProjSplit, 2 * num_sms() / tiles));
}
static int qkv_width(const dtree_qwen3_desc& d) { return (d.n_heads + 2 * d.n_kv_heads) * d.head_dim; }
// the four projections of a layer as (rows N, K)
static std::array<std::pair<int, int>, 4> layer_shapes(const dtree_qwen3_desc& d) {
  return {{{qkv_width(d), d.hidden}, {d.hidden, d.n_heads * d.head_dim}, {2 * d.ffn, d.hidden}, {d.hidden, d.ffn}}};
}
static size_t q4_sb_need(const dtree_qwen3_desc& d) {
  size_t b = 0;
  if (d.quant_bits == 4)
    for (const auto& nk : layer_shapes(d)) b += (q4_sb_bytes(nk.first, nk.second) + 255) & ~static_cast<size_t>(255);
  b *= d.layers;
  if (d.embed_q4_packed) b += (q4_sb_bytes(d.vocab, d.hidden) + 255) & ~static_cast<size_t>(255);
  return b;
}
static size_t partials_need(const dtree_qwen3_desc& d) {
  const size_t a = static_cast<size_t>(proj_split(d, d.hidden)) * d.hidden;
  const size_t b = static_cast<size_t>(proj_split(d, qkv_width(d))) * qkv_width(d);
  return std::max(a, b) * pad_rows(d.t_cap) * 4;
}

static int build_plans(dtree_qwen3_model* m, int t_pad) {
  PlanSet& ps = m->plans[tpad_index(t_pad)];
  if (ps.ready) return kOk;
  const dtree_qwen3_desc& d = m->d;
  const int qkv_rows = (d.n_heads + 2 * d.n_kv_heads) * d.head_dim;
  const int qd = d.n_heads * d.head_dim;
  ps.qkv.resize(d.layers);
  ps.o.resize(d.layers);
  ps.gu.resize(d.layers);
  ps.down.resize(d.layers);
  const bool q4 = d.quant_bits == 4;
  for (int l = 0; l < d.layers; ++l) {
    const dtree_qwen3_layer& L = m->layers[l];
    // bf16 or MLX 4-bit weights behind the same plan
    auto plan = [&](GemmPlan* g, const void* w, const void* sb_w, int n, int k, const void* x, int epi, int grid) {
      return q4 ? gemm_plan_q4(g, w, sb_w, n, k, x, t_pad, k, epi, grid)
                : gemm_plan(g, w, n, k, x, t_pad, k, epi, grid);
    };
    const std::array<const void*, 4> sb = q4 ? m->q4_sb[l] : std::array<const void*, 4>{};
    int rc;
    if ((rc = plan(&ps.qkv[l], L.qkv, sb[0], qkv_rows, d.hidden, d.xn, kEpiPartial, proj_split(d, qkv_rows))))
      return rc;
    if ((rc = plan(&ps.o[l], L.o_proj, sb[1], d.hidden, qd, d.attn, kEpiPartial, proj_split(d, d.hidden))))
      return rc;
    if ((rc = plan(&ps.gu[l], L.gate_up, sb[2], 2 * d.ffn, d.hidden, d.xn, kEpiSwiglu, 0))) return rc;
    if ((rc = plan(&ps.down[l], L.down, sb[3], d.hidden, d.ffn, d.act, kEpiPartial, proj_split(d, d.hidden))))
      return rc;
    if (ps.o[l].p.split > kMaxProjSplit || ps.down[l].p.split > kMaxProjSplit || ps.qkv[l].p.split > kMaxProjSplit)
      return fail(kErrUnsupported, "projection split exceeds the partial buffer");
    for (GemmPlan* g : {&ps.qkv[l], &ps.o[l], &ps.gu[l], &ps.down[l]})
      if ((rc = gemm_bind_ws(g, m->gemm_ws, m->gemm_ws_bytes))) return rc;
  }
  // LM head: the bf16 embedding, or the 4-bit one (stream-K over both CTA
  // slots of every SM)
  int rc = m->embed_sb ? gemm_plan_q4(&ps.lm, d.embed_q4_packed, m->embed_sb, d.vocab, d.hidden, d.norm_out, t_pad,
                                      d.hidden, kEpiArgmax, 2 * num_sms())
                       : gemm_plan(&ps.lm, d.embed, d.vocab, d.hidden, d.norm_out, t_pad, d.hidden, kEpiArgmax, 0);
  if (rc) return rc;
  if ((rc = gemm_bind_ws(&ps.lm, m->gemm_ws, m->gemm_ws_bytes))) return rc;
  if ((rc = m->embed_sb ? gemm_plan_q4(&ps.lm_logits, d.embed_q4_packed, m->embed_sb, d.vocab, d.hidden, d.norm_out,
                                       t_pad, d.hidden, kEpiPartial, 1)
                        : gemm_plan(&ps.lm_logits, d.embed, d.vocab, d.hidden, d.norm_out, t_pad, d.hidden, kEpiPartial,
                                    1)))
    return rc;
  if ((rc = gemm_bind_ws(&ps.lm_logits, m->gemm_ws, m->gemm_ws_bytes))) return rc;
  ps.ready = true;
  return kOk;
}

}  // namespace dtree

using namespace dtree;

extern "C" int dtree_qwen3_buffer_bytes(const dtree_qwen3_desc* d, size_t out[9]) {
  DTREE_CHECK_ARG(d && out, "null pointer");
  DTREE_CHECK_ARG(d->t_cap > 0 && d->t_cap <= DTREE_MAX_TREE, "t_cap must be in [1, 128]");
  const size_t tc = static_cast<size_t>(pad_rows(d->t_cap));
  const size_t qd = static_cast<size_t>(d->n_heads) * d->head_dim;
  out[0] = static_cast<size_t>(d->layers) * 2 * d->n_kv_heads * static_cast<size_t>(d->kv_capacity) * d->head_dim * 2;
  out[1] = tc * d->hidden * 2;
  out[2] = tc * d->hidden * 2;
  out[3] = tc * qd * 2;
  out[4] = tc * qd * 2;
  out[5] = tc * d->ffn * 2;
  out[6] = tc * d->hidden * 2;
  out[7] = tc * d->hidden * (d->n_capture > 0 ? d->n_capture : 1) * 2;
  out[8] = ((gemm_ws_need(*d) + 255) & ~static_cast<size_t>(255)) +
           ((attn_ws_need(*d) + 255) & ~static_cast<size_t>(255)) + ((partials_need(*d) + 255) & ~static_cast<size_t>(255)) +
           ((fused_ws_bytes(*d) + 255) & ~static_cast<size_t>(255)) + q4_sb_need(*d);
  return kOk;
}

extern "C" int dtree_qwen3_create(const dtree_qwen3_desc* desc, dtree_qwen3_model** out) {
  DTREE_CHECK_ARG(desc && out, "null pointer");
  const dtree_qwen3_desc& d = *desc;
  DTREE_CHECK_ARG(d.hidden % 64 == 0 && d.ffn % 64 == 0, "hidden and ffn must be multiples of 64");
  DTREE_CHECK_ARG(d.head_dim == 64 || d.head_dim == 128, "head_dim must be 64 or 128");
  DTREE_CHECK_ARG(d.n_heads % d.n_kv_heads == 0, "n_heads must be a multiple of n_kv_heads");
  DTREE_CHECK_ARG((d.n_heads * d.head_dim) % 128 == 0 && (d.n_kv_heads * d.head_dim) % 128 == 0,
                  "q and kv projection widths must be multiples of 128");
  DTREE_CHECK_ARG(d.t_cap > 0 && d.t_cap <= DTREE_MAX_TREE, "t_cap must be in [1, 128]");
  DTREE_CHECK_ARG(d.n_capture >= 0 && d.n_capture <= 16, "n_capture must be in [0, 16]");
  DTREE_CHECK_ARG(d.layer && d.embed && d.final_norm, "null weights");
  DTREE_CHECK_ARG(d.kv_cache && d.h && d.xn && d.q && d.attn && d.act && d.norm_out && d.workspace,
                  "null buffer");
  DTREE_CHECK_ARG(d.n_capture == 0 || d.capture, "null capture buffer");
  size_t need[9];
  dtree_qwen3_buffer_bytes(desc, need);
  DTREE_CHECK_ARG(d.workspace_bytes >= need[8], "workspace too small");
  for (int c = 0; c < d.n_capture; ++c)
    DTREE_CHECK_ARG(d.capture_layers[c] >= 0 && d.capture_layers[c] < d.layers, "capture layer out of range");
  DTREE_CHECK_ARG(d.quant_bits == 0 || d.quant_bits == 16 || d.quant_bits == 4,
                  "quant_bits must be 0/16 (bf16) or 4 (MLX affine)");
  if (d.quant_bits == 4) {
    DTREE_CHECK_ARG(d.group_size == 64, "4-bit weights need group_size 64");
    DTREE_CHECK_ARG(d.q4_layer != nullptr, "null q4_layer");
    for (int l = 0; l < d.layers; ++l) {
      const dtree_qwen3_q4_layer& Q = d.q4_layer[l];
      DTREE_CHECK_ARG(Q.qkv_scales && Q.qkv_biases && Q.o_scales && Q.o_biases && Q.gate_up_scales &&
                          Q.gate_up_biases && Q.down_scales && Q.down_biases,
                      "null q4 scales / biases");
    }
  }
  DTREE_CHECK_ARG(!d.embed_q4_packed || (d.embed_q4_scales && d.embed_q4_biases),
                  "a 4-bit LM head needs embed_q4_scales and embed_q4_biases");
  auto* m = new dtree_qwen3_model();
  m->d = d;
  m->layers.assign(d.layer, d.layer + d.layers);
  m->d.layer = m->layers.data();
  if (d.quant_bits == 4) {
    m->q4_layers.assign(d.q4_layer, d.q4_layer + d.layers);
    m->d.q4_layer = m->q4_layers.data();
  }
  m->gemm_ws = d.workspace;
  m->gemm_ws_bytes = gemm_ws_need(d);
  m->attn_ws = static_cast<char*>(d.workspace) + ((m->gemm_ws_bytes + 255) & ~static_cast<size_t>(255));
  m->attn_ws_bytes = attn_ws_need(d);
  m->proj_partials = reinterpret_cast<float*>(static_cast<char*>(m->attn_ws) +
                                              ((m->attn_ws_bytes + 255) & ~static_cast<size_t>(255)));
  if (int rc = attn_prepare(d.head_dim)) {
    delete m;
    return rc;
  }
  if (d.quant_bits == 4 || d.embed_q4_packed) {
    // the scale / bias blocks of every 4-bit projection (and of a 4-bit LM
    // head), after the other workspace regions (the weights must be
    // complete: wait for the device)
    char* sbp = reinterpret_cast<char*>(m->proj_partials) + ((partials_need(d) + 255) & ~static_cast<size_t>(255)) +
                ((fused_ws_bytes(d) + 255) & ~static_cast<size_t>(255));
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      delete m;
      return fail(kErrCuda, std::string("dtree_qwen3_create (4-bit repack): ") + cudaGetErrorString(e));
    }
    const auto shapes = layer_shapes(d);
    m->q4_sb.resize(d.quant_bits == 4 ? d.layers : 0);
    for (int l = 0; l < static_cast<int>(m->q4_sb.size()); ++l) {
      const dtree_qwen3_q4_layer& Q = m->q4_layers[l];
      const void* sc[4] = {Q.qkv_scales, Q.o_scales, Q.gate_up_scales, Q.down_scales};
      const void* bi[4] = {Q.qkv_biases, Q.o_biases, Q.gate_up_biases, Q.down_biases};
      for (int j = 0; j < 4; ++j) {
        int rc = q4_sb_repack_launch(sc[j], bi[j], shapes[j].first, shapes[j].second, sbp, nullptr);
        if (rc) {
          delete m;
          return rc;
        }
        m->q4_sb[l][j] = sbp;
        sbp += (q4_sb_bytes(shapes[j].first, shapes[j].second) + 255) & ~static_cast<size_t>(255);
      }
    }
    if (d.embed_q4_packed) {
      int rc = q4_sb_repack_launch(d.embed_q4_scales, d.embed_q4_biases, d.vocab, d.hidden, sbp, nullptr);
      if (rc) {
        delete m;
        return rc;
      }
      m->embed_sb = sbp;
    }
    e = cudaStreamSynchronize(nullptr);
    if (e != cudaSuccess) {
      delete m;
      return fail(kErrCuda, std::string("dtree_qwen3_create (4-bit repack): ") + cudaGetErrorString(e));
    }
  }
  if (d.verify_path == 1 && fused_supported(d)) {
    m->fused_ws = reinterpret_cast<char*>(m->proj_partials) + ((partials_need(d) + 255) & ~static_cast<size_t>(255));
    std::vector<std::pair<int, __nv_bfloat16*>> caps;
    for (int c = 0; c < d.n_capture; ++c)
      caps.emplace_back(d.capture_layers[c], static_cast<__nv_bfloat16*>(d.capture) + static_cast<size_t>(c) * d.hidden);
    int rc = fused_init(d, m->fused_ws, caps.data(), static_cast<int>(caps.size()));
    if (rc) {
      delete m;
      return rc;
    }
  }
  *out = m;
  return kOk;
}

extern "C" int dtree_qwen3_destroy(dtree_qwen3_model* m) {
  delete m;
  return kOk;
}

static int forward_impl(dtree_qwen3_model* m, const int32_t* tree_tokens, const int32_t* positions,
                        const uint64_t* anc_mask, int n_nodes, const dtree_step_state* state, int32_t* posterior,
                        float* logits, void* stream_);

extern "C" int dtree_qwen3_forward_tree(dtree_qwen3_model* m, const int32_t* tree_tokens, const int32_t* positions,
                                        const uint64_t* anc_mask, int n_nodes, const dtree_step_state* state,
                                        int32_t* posterior, void* stream_) {
  return forward_impl(m, tree_tokens, positions, anc_mask, n_nodes, state, posterior, nullptr, stream_);
}

extern "C" int dtree_qwen3_forward_logits(dtree_qwen3_model* m, const int32_t* tokens, const int32_t* positions,
                                          const uint64_t* anc_mask, int n_rows, const dtree_step_state* state,
                                          float* logits, void* stream_) {
  DTREE_CHECK_ARG(logits, "null logits");
  return forward_impl(m, tokens, positions, anc_mask, n_rows, state, nullptr, logits, stream_);
}

// context-only draft cache bookkeeping after an append of `host_count` rows
// (>= 0) or of state->n_accepted rows (host_count < 0): reserved (rows
// appended so far) grows by that count, start (the attended context
// length) = min(reserved, sink + window)
__global__ void ring_advance_kernel(dtree_step_state* ring, const dtree_step_state* state, int host_count, int sink,
                                    int window) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const int n = host_count >= 0 ? host_count : state->n_accepted;
    const int total = ring->reserved + n;
    ring->reserved = total;
    ring->start = total < sink + window ? total : sink + window;
  }
}

static int dflash_context_impl(dtree_qwen3_model* m, const void* fc_weight, const void* hidden_norm,
                               const void* target_hidden, int ld_hidden, int width, int n_rows, int ctx_base,
                               const dtree_step_state* state, dtree_step_state* ring_state, int sink, int window,
                               void* stream_);

extern "C" int dtree_dflash_context_ring(dtree_qwen3_model* m, const void* fc_weight, const void* hidden_norm,
                                         const void* target_hidden, int ld_hidden, int width, int n_rows,
                                         int ctx_base, const dtree_step_state* state, dtree_step_state* ring_state,
                                         int sink, int window, void* stream_) {
  DTREE_CHECK_ARG(ring_state, "null ring state");
  DTREE_CHECK_ARG(sink >= 0 && window > 0, "sink must be >= 0 and window > 0");
  DTREE_CHECK_ARG(m && sink + window + m->d.t_cap <= m->d.kv_capacity,
                  "draft cache capacity below sink + window + block rows");
  return dflash_context_impl(m, fc_weight, hidden_norm, target_hidden, ld_hidden, width, n_rows, ctx_base, state,
                             ring_state, sink, window, stream_);
}

extern "C" int dtree_dflash_context(dtree_qwen3_model* m, const void* fc_weight, const void* hidden_norm,
                                    const void* target_hidden, int ld_hidden, int width, int n_rows, int ctx_base,
                                    const dtree_step_state* state, void* stream_) {
  return dflash_context_impl(m, fc_weight, hidden_norm, target_hidden, ld_hidden, width, n_rows, ctx_base, state,
                             nullptr, 0, 0, stream_);
}

static int dflash_context_impl(dtree_qwen3_model* m, const void* fc_weight, const void* hidden_norm,
                               const void* target_hidden, int ld_hidden, int width, int n_rows, int ctx_base,
                               const dtree_step_state* state, dtree_step_state* ring_state, int sink, int window,
                               void* stream_) {
  DTREE_CHECK_ARG(m && fc_weight && hidden_norm && target_hidden && state, "null pointer");
  const dtree_qwen3_desc& d = m->d;
  DTREE_CHECK_ARG(n_rows > 0 && n_rows <= d.t_cap, "n_rows must be in [1, t_cap]");
  DTREE_CHECK_ARG(width % 64 == 0 && ld_hidden >= width, "context width must be a multiple of 64 <= ld_hidden");
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  const int t_pad = pad_rows(n_rows);
  auto bw = [](void* p) { return static_cast<__nv_bfloat16*>(p); };
  // ctx = RMSNorm(fc(target_hidden), hidden_norm)   (draft.py:329-330)
  GemmPlan fc;
  int rc = gemm_plan(&fc, fc_weight, d.hidden, width, target_hidden, t_pad, ld_hidden, kEpiStore, 0);
  if (rc) return rc;
  if ((rc = gemm_bind_ws(&fc, m->gemm_ws, m->gemm_ws_bytes))) return rc;
  fc.p.n_rows = n_rows;
  fc.p.out = bw(d.norm_out);
  fc.p.ldo = d.hidden;
  if ((rc = gemm_launch(fc, st))) return rc;
  if ((rc = rmsnorm_launch(static_cast<const __nv_bfloat16*>(d.norm_out), d.hidden, nullptr, nullptr, nullptr,
                           static_cast<const __nv_bfloat16*>(hidden_norm), bw(d.xn), d.hidden, n_rows, t_pad,
                           d.rms_eps, st)))
    return rc;
  // per layer: k_norm(k_proj(ctx)) with RoPE at the rows' positions, v_proj(ctx)
  // -> draft cache slots (DFlashAttention.precompute_context_kv, draft.py:172-187)
  const int kvw = 2 * d.n_kv_heads * d.head_dim;
  const int qd = d.n_heads * d.head_dim;
  const size_t plane = static_cast<size_t>(d.n_kv_heads) * d.kv_capacity * d.head_dim;
  for (int l = 0; l < d.layers; ++l) {
    const dtree_qwen3_layer& L = m->layers[l];
    GemmPlan g;
    const void* wkv = static_cast<const __nv_bfloat16*>(L.qkv) + static_cast<size_t>(qd) * d.hidden;
    if ((rc = gemm_plan(&g, wkv, kvw, d.hidden, d.xn, t_pad, d.hidden, kEpiPartial, proj_split(d, kvw)))) return rc;
    DTREE_CHECK_ARG(static_cast<size_t>(g.p.split) * kvw * t_pad * 4 <= partials_need(d),
                    "context K/V partials exceed the workspace");
    if ((rc = gemm_bind_ws(&g, m->gemm_ws, m->gemm_ws_bytes))) return rc;
    g.p.n_rows = n_rows;
    g.p.out_f32 = m->proj_partials;
    g.p.ldo = kvw;
    if ((rc = gemm_launch(g, st))) return rc;
    QkvFinishParams f{};
    f.partials = m->proj_partials;
    f.split = g.p.split;
    f.part_rows = t_pad;
    f.width = kvw;
    f.head_dim = d.head_dim;
    f.n_q_heads = 0;
    f.n_kv_heads = d.n_kv_heads;
    f.q_norm = static_cast<const __nv_bfloat16*>(L.q_norm);
    f.k_norm = static_cast<const __nv_bfloat16*>(L.k_norm);
    f.eps = d.rms_eps;
    f.rope_log2_theta = std::log2(d.rope_theta);
    f.state = state;
    f.k_cache = bw(d.kv_cache) + (static_cast<size_t>(l) * 2 + 0) * plane;
    f.v_cache = bw(d.kv_cache) + (static_cast<size_t>(l) * 2 + 1) * plane;
    f.kv_cap = d.kv_capacity;
    f.slot_mode = ctx_base >= 0 ? 2 : 1;
    f.ctx_base = ctx_base;
    f.ctx_count = n_rows;
    f.ring_state = ring_state;
    f.ring_sink = ring_state ? sink : 0;
    f.ring_window = ring_state ? window : 0;
    if ((rc = qkv_finish_launch(f, n_rows, st))) return rc;
  }
  if (ring_state)
    DTREE_CUDA_RET(launch_pdl(ring_advance_kernel, dim3(1), dim3(32), 0, st, ring_state, state,
                              ctx_base >= 0 ? n_rows : -1, sink, window));
  return kOk;
}

static int forward_impl(dtree_qwen3_model* m, const int32_t* tree_tokens, const int32_t* positions,
                        const uint64_t* anc_mask, int n_nodes, const dtree_step_state* state, int32_t* posterior,
                        float* logits, void* stream_) {
  DTREE_CHECK_ARG(m && tree_tokens && positions && anc_mask && state, "null pointer");
  const dtree_qwen3_desc& d = m->d;
  DTREE_CHECK_ARG(n_nodes > 0 && n_nodes <= d.t_cap, "n_nodes must be in [1, t_cap]");
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  const int t_pad = pad_rows(n_nodes);
  int rc = build_plans(m, t_pad);
  if (rc) return rc;
  PlanSet& ps = m->plans[tpad_index(t_pad)];
  auto bf = [](const void* p) { return static_cast<const __nv_bfloat16*>(p); };
  auto bw = [](void* p) { return static_cast<__nv_bfloat16*>(p); };
  const size_t plane = static_cast<size_t>(d.n_kv_heads) * d.kv_capacity * d.head_dim;
  const int qd = d.n_heads * d.head_dim;
  const float log2_theta = std::log2(d.rope_theta);
  const int qkv_rows_all = qkv_width(d);
  const int splits = std::min(kAttnMaxSplits, attn_default_splits(d.n_kv_heads, d.n_heads, n_nodes));
  // verifier_hidden column block of layer l (nullptr if l is not captured)
  const int ldc = d.hidden * (d.n_capture > 0 ? d.n_capture : 1);
  auto capture_ptr = [&](int l) -> __nv_bfloat16* {
    for (int c = 0; c < d.n_capture; ++c)
      if (d.capture_layers[c] == l) return bw(d.capture) + static_cast<size_t>(c) * d.hidden;
    return nullptr;
  };

  if (m->fused_ws && !logits && t_pad <= 64) {
    // the whole layer stack in one persistent launch, then the LM head
    const int fi = t_pad == 16 ? 0 : (t_pad == 32 ? 1 : 2);
    if (!m->fused_ready[fi]) {
      if ((rc = fused_plan(d, m->fused_ws, t_pad, &m->fused[fi]))) return rc;
      m->fused_ready[fi] = true;
    }
    if ((rc = fused_launch(m->fused[fi], tree_tokens, positions, anc_mask, n_nodes, state, st))) return rc;
    if (posterior) {
      GemmPlan g = ps.lm;
      g.p.n_rows = n_nodes;
      g.p.vocab = d.vocab;
      g.p.argmax_out = posterior;
      g.p.inv_temp = m->inv_temp;
      g.p.sample_seed = m->sample_seed;
      g.p.sample_state = state;
      if ((rc = gemm_launch(g, st))) return rc;
    }
    return kOk;
  }
  // embedding gather + first input norm
  if ((rc = rmsnorm_launch(nullptr, 0, tree_tokens, bf(d.embed), bw(d.h), bf(m->layers[0].input_norm), bw(d.xn),
                           d.hidden, n_nodes, t_pad, d.rms_eps, st)))
    return rc;
  for (int l = 0; l < d.layers; ++l) {
    const dtree_qwen3_layer& L = m->layers[l];
    __nv_bfloat16* kc = bw(d.kv_cache) + (static_cast<size_t>(l) * 2 + 0) * plane;
    __nv_bfloat16* vc = bw(d.kv_cache) + (static_cast<size_t>(l) * 2 + 1) * plane;
    if (l > 0) {  // h += down_proj(l-1) (+ capture), xn = RMSNorm(h, input_norm[l])
      if ((rc = residual_rmsnorm_launch(bw(d.h), m->proj_partials, ps.down[l - 1].p.split, t_pad,
                                        capture_ptr(l - 1), ldc, bf(L.input_norm), bw(d.xn), d.hidden, n_nodes,
                                        t_pad, d.rms_eps, st)))
        return rc;
    }
    {  // q | k | v projection: split-K fp32 partials
      GemmPlan g = ps.qkv[l];
      g.p.n_rows = n_nodes;
      g.p.out_f32 = m->proj_partials;
      g.p.ldo = qkv_rows_all;
      if ((rc = gemm_launch(g, st))) return rc;
    }
    {  // sum partials, q/k RMSNorm + RoPE, q -> buffer, k/v -> cache slots start + t
      QkvFinishParams f{};
      f.partials = m->proj_partials;
      f.split = ps.qkv[l].p.split;
      f.part_rows = t_pad;
      f.width = qkv_rows_all;
      f.head_dim = d.head_dim;
      f.n_q_heads = d.n_heads;
      f.n_kv_heads = d.n_kv_heads;
      f.q_norm = bf(L.q_norm);
      f.k_norm = bf(L.k_norm);
      f.eps = d.rms_eps;
      f.rope_log2_theta = log2_theta;
      f.positions = positions;
      f.state = state;
      f.q_out = bw(d.q);
      f.k_cache = kc;
      f.v_cache = vc;
      f.kv_cap = d.kv_capacity;
      if ((rc = qkv_finish_launch(f, n_nodes, st))) return rc;
    }
    {  // tree attention
      AttnParams a{};
      a.q = bf(d.q);
      a.ldq = qd;
      a.k = kc;
      a.v = vc;
      a.cap = d.kv_capacity;
      a.n_q_heads = d.n_heads;
      a.n_kv_heads = d.n_kv_heads;
      a.n_nodes = n_nodes;
      a.state = state;
      a.anc = anc_mask;
      a.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(d.head_dim)));
      a.splits = splits;
      a.cluster_keys = m->attn_keys > 0 ? std::min(m->attn_keys, d.kv_capacity) : d.kv_capacity;
      a.out = bw(d.attn);
      if ((rc = attn_launch(a, d.head_dim, m->attn_ws, m->attn_ws_bytes, st))) return rc;
    }
    {  // o_proj split-K partials
      GemmPlan g = ps.o[l];
      g.p.n_rows = n_nodes;
      g.p.out_f32 = m->proj_partials;
      g.p.ldo = d.hidden;
      if ((rc = gemm_launch(g, st))) return rc;
    }
    // h += o_proj, xn = RMSNorm(h, post_norm)
    if ((rc = residual_rmsnorm_launch(bw(d.h), m->proj_partials, ps.o[l].p.split, t_pad, nullptr, 0,
                                      bf(L.post_norm), bw(d.xn), d.hidden, n_nodes, t_pad, d.rms_eps, st)))
      return rc;
    {  // gate | up + SwiGLU
      GemmPlan g = ps.gu[l];
      g.p.n_rows = n_nodes;
      g.p.out = bw(d.act);
      g.p.ldo = d.ffn;
      if ((rc = gemm_launch(g, st))) return rc;
    }
    {  // down_proj split-K partials (added by the next residual_rmsnorm)
      GemmPlan g = ps.down[l];
      g.p.n_rows = n_nodes;
      g.p.out_f32 = m->proj_partials;
      g.p.ldo = d.hidden;
      if ((rc = gemm_launch(g, st))) return rc;
    }
  }
  // h += down_proj(L-1) (+ capture), norm_out = RMSNorm(h, final_norm)
  if ((rc = residual_rmsnorm_launch(bw(d.h), m->proj_partials, ps.down[d.layers - 1].p.split, t_pad,
                                    capture_ptr(d.layers - 1), ldc, bf(d.final_norm), bw(d.norm_out), d.hidden,
                                    n_nodes, t_pad, d.rms_eps, st)))
    return rc;
  if (logits) {  // full fp32 logits [t_pad][vocab]
    GemmPlan g = ps.lm_logits;
    g.p.n_rows = n_nodes;
    g.p.out_f32 = logits;
    g.p.ldo = d.vocab;
    if ((rc = gemm_launch(g, st))) return rc;
  }
  if (posterior) {
    GemmPlan g = ps.lm;
    g.p.n_rows = n_nodes;
    g.p.vocab = d.vocab;
    g.p.argmax_out = posterior;
    g.p.inv_temp = m->inv_temp;
    g.p.sample_seed = m->sample_seed;
    g.p.sample_state = state;
    if ((rc = gemm_launch(g, st))) return rc;
  }
  return kOk;
}

// ------------------------------------------------------------ prompt prefill
// Dense causal forward of the prompt (Qwen3TargetAdapter._forward_states over
// the prompt, adapters.py:494-533, as called by dtree_runtime.py:342-349):
// every projection is one dense tcgen05 GEMM over all prompt rows (tiles of
// 128 weight rows x 256 tokens), so the weights stream once per prompt
// instead of once per 128 rows, and the attention runs the prompt's 128-row
// chunks in one launch per layer.  Same bf16 rounding points as the verify
// forward: projections are bf16, residual adds round once, RMSNorm in fp32.
namespace dtree {

__global__ void chain_masks_kernel(uint64_t* anc) {
  const int i = threadIdx.x;  // row i of a 128-row chain sees rows 0..i
  anc[2 * i] = i >= 63 ? ~0ull : ((1ull << (i + 1)) - 1ull);
  anc[2 * i + 1] = i < 64 ? 0ull : (i >= 127 ? ~0ull : ((1ull << (i - 63)) - 1ull));
}

struct PrefillLayout {
  size_t h, xn, big, q, attn, lm_in, anc, wdq, gemm, total;
  int n_pad;
};

static PrefillLayout prefill_layout(const dtree_qwen3_desc& d, int n_rows) {
  PrefillLayout L{};
  L.n_pad = ((n_rows + kDenseRows - 1) / kDenseRows) * kDenseRows;
  const size_t np = static_cast<size_t>(L.n_pad);
  const size_t qd = static_cast<size_t>(d.n_heads) * d.head_dim;
  const size_t wide = std::max<size_t>(qkv_width(d), d.ffn);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~static_cast<size_t>(255);
    return o;
  };
  L.h = take(np * d.hidden * 2);
  L.xn = take(np * d.hidden * 2);
  L.big = take(np * wide * 2);
  L.q = take(np * qd * 2);
  L.attn = take(np * qd * 2);
  L.lm_in = take(static_cast<size_t>(16) * d.hidden * 2);
  L.anc = take(128 * 16);
  // 4-bit weights: the largest matrix dequantized to bf16 ahead of its GEMM
  const size_t wmax = std::max({static_cast<size_t>(qkv_width(d)) * d.hidden, static_cast<size_t>(d.hidden) * qd,
                                static_cast<size_t>(2) * d.ffn * d.hidden, static_cast<size_t>(d.hidden) * d.ffn});
  L.wdq = d.quant_bits == 4 ? take(wmax * 2) : off;
  L.gemm = take(gemm_ws_bytes(kDenseRows, num_sms()));
  L.total = off;
  return L;
}

}  // namespace dtree

extern "C" size_t dtree_qwen3_prefill_workspace_bytes(const dtree_qwen3_desc* d, int n_rows) {
  if (!d || n_rows <= 0) return 0;
  return prefill_layout(*d, n_rows).total;
}

extern "C" int dtree_qwen3_prefill(dtree_qwen3_model* m, const int32_t* tokens, const int32_t* positions, int n_rows,
                                   const dtree_step_state* state, void* hidden_out, int ld_hidden_out,
                                   void* norm_out, int32_t* next_token, void* workspace, size_t workspace_bytes,
                                   void* stream_) {
  DTREE_CHECK_ARG(m && tokens && positions && state && next_token && workspace, "null pointer");
  const dtree_qwen3_desc& d = m->d;
  DTREE_CHECK_ARG(n_rows > 0 && n_rows <= d.kv_capacity, "n_rows must be in [1, kv_capacity]");
  DTREE_CHECK_ARG(d.n_capture == 0 || hidden_out, "null hidden_out with captured layers");
  DTREE_CHECK_ARG(!hidden_out || ld_hidden_out >= d.hidden * d.n_capture, "ld_hidden_out below n_capture * hidden");
  const PrefillLayout Lo = prefill_layout(d, n_rows);
  DTREE_CHECK_ARG(workspace_bytes >= Lo.total, "prefill workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  char* ws = static_cast<char*>(workspace);
  auto at = [&](size_t off) { return reinterpret_cast<__nv_bfloat16*>(ws + off); };
  auto bf = [](const void* p) { return static_cast<const __nv_bfloat16*>(p); };
  __nv_bfloat16 *h = at(Lo.h), *xn = at(Lo.xn), *big = at(Lo.big), *q = at(Lo.q), *attn = at(Lo.attn);
  __nv_bfloat16* wdq = at(Lo.wdq);
  uint64_t* anc = reinterpret_cast<uint64_t*>(ws + Lo.anc);
  void* gws = ws + Lo.gemm;
  const size_t gws_bytes = Lo.total - Lo.gemm;
  const int np = Lo.n_pad;
  const int qd = d.n_heads * d.head_dim;
  const int qkvw = qkv_width(d);
  const size_t plane = static_cast<size_t>(d.n_kv_heads) * d.kv_capacity * d.head_dim;
  const bool q4 = d.quant_bits == 4;
  DTREE_CUDA_RET(cudaMemsetAsync(gws, 0, gemm_ws_counter_bytes(), st));
  DTREE_CUDA_RET(launch_pdl(chain_masks_kernel, dim3(1), dim3(128), 0, st, anc));
  int rc;
  // dense GEMM out = x @ W^T with W bf16, or dequantized from 4 bits first
  auto dense = [&](const void* w, const void* sc, const void* bi, int n_out, int k, const __nv_bfloat16* x, int epi,
                   __nv_bfloat16* out, int ldo, __nv_bfloat16* capture, int ldc) -> int {
    const void* wb = w;
    if (q4) {
      int r = dequant_q4_launch(w, sc, bi, n_out, k, wdq, st);
      if (r) return r;
      wb = wdq;
    }
    GemmPlan g;
    int r = gemm_plan_dense(&g, wb, n_out, k, x, n_rows, np, k, epi);
    if (r) return r;
    if ((r = gemm_bind_ws(&g, gws, gws_bytes))) return r;
    g.p.out = out;
    g.p.ldo = ldo;
    g.p.capture = capture;
    g.p.ldc = ldc;
    g.p.w_dep = q4 ? 1 : 0;  // the dequant kernel just before writes W
    return gemm_launch(g, st);
  };
  auto capture_ptr = [&](int l) -> __nv_bfloat16* {
    for (int c = 0; c < d.n_capture; ++c)
      if (d.capture_layers[c] == l) return static_cast<__nv_bfloat16*>(hidden_out) + static_cast<size_t>(c) * d.hidden;
    return nullptr;
  };
  // embedding gather + first input norm (rows n_rows..n_pad-1 zero)
  if ((rc = rmsnorm_launch(nullptr, 0, tokens, bf(d.embed), h, bf(m->layers[0].input_norm), xn, d.hidden, n_rows, np,
                           d.rms_eps, st)))
    return rc;
  for (int l = 0; l < d.layers; ++l) {
    const dtree_qwen3_layer& L = m->layers[l];
    const dtree_qwen3_q4_layer Q = q4 ? m->q4_layers[l] : dtree_qwen3_q4_layer{};
    __nv_bfloat16* kc = static_cast<__nv_bfloat16*>(d.kv_cache) + (static_cast<size_t>(l) * 2 + 0) * plane;
    __nv_bfloat16* vc = static_cast<__nv_bfloat16*>(d.kv_cache) + (static_cast<size_t>(l) * 2 + 1) * plane;
    if ((rc = dense(L.qkv, Q.qkv_scales, Q.qkv_biases, qkvw, d.hidden, xn, kEpiStore, big, qkvw, nullptr, 0)))
      return rc;
    {  // q/k RMSNorm + RoPE, q -> buffer, k/v -> cache slots start + t
      QkvFinishParams f{};
      f.dense = big;
      f.width = qkvw;
      f.head_dim = d.head_dim;
      f.n_q_heads = d.n_heads;
      f.n_kv_heads = d.n_kv_heads;
      f.q_norm = bf(L.q_norm);
      f.k_norm = bf(L.k_norm);
      f.eps = d.rms_eps;
      f.rope_log2_theta = std::log2(d.rope_theta);
      f.positions = positions;
      f.state = state;
      f.q_out = q;
      f.k_cache = kc;
      f.v_cache = vc;
      f.kv_cap = d.kv_capacity;
      if ((rc = qkv_rows_launch(f, n_rows, st))) return rc;
    }
    {  // causal attention, 128-row chunks
      AttnParams a{};
      a.q = q;
      a.ldq = qd;
      a.k = kc;
      a.v = vc;
      a.cap = d.kv_capacity;
      a.n_q_heads = d.n_heads;
      a.n_kv_heads = d.n_kv_heads;
      a.n_nodes = n_rows;
      a.state = state;
      a.anc = anc;
      a.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(d.head_dim)));
      a.out = attn;
      if ((rc = attn_prefill_launch(a, d.head_dim, st))) return rc;
    }
    // h += attn @ Wo^T; xn = RMSNorm(h, post_norm)
    if ((rc = dense(L.o_proj, Q.o_scales, Q.o_biases, d.hidden, qd, attn, kEpiResidual, h, d.hidden, nullptr, 0)))
      return rc;
    if ((rc = rmsnorm_launch(h, d.hidden, nullptr, nullptr, nullptr, bf(L.post_norm), xn, d.hidden, n_rows, np,
                             d.rms_eps, st)))
      return rc;
    if ((rc = dense(L.gate_up, Q.gate_up_scales, Q.gate_up_biases, 2 * d.ffn, d.hidden, xn, kEpiSwiglu, big, d.ffn,
                    nullptr, 0)))
      return rc;
    // h += act @ Wd^T (+ the captured layer's hidden rows)
    if ((rc = dense(L.down, Q.down_scales, Q.down_biases, d.hidden, d.ffn, big, kEpiResidual, h, d.hidden,
                    capture_ptr(l), ld_hidden_out)))
      return rc;
    if (l + 1 < d.layers &&
        (rc = rmsnorm_launch(h, d.hidden, nullptr, nullptr, nullptr, bf(m->layers[l + 1].input_norm), xn, d.hidden,
                             n_rows, np, d.rms_eps, st)))
      return rc;
  }
  if (norm_out &&  // RMSNorm(h, final_norm) of every row
      (rc = rmsnorm_launch(h, d.hidden, nullptr, nullptr, nullptr, bf(d.final_norm),
                           static_cast<__nv_bfloat16*>(norm_out), d.hidden, n_rows, n_rows, d.rms_eps, st)))
    return rc;
  // the next token from the last prompt row only
  __nv_bfloat16* lm_in = at(Lo.lm_in);
  if ((rc = rmsnorm_launch(h + static_cast<size_t>(n_rows - 1) * d.hidden, d.hidden, nullptr, nullptr, nullptr,
                           bf(d.final_norm), lm_in, d.hidden, 1, 16, d.rms_eps, st)))
    return rc;
  GemmPlan g;
  if ((rc = m->embed_sb ? gemm_plan_q4(&g, d.embed_q4_packed, m->embed_sb, d.vocab, d.hidden, lm_in, 16, d.hidden,
                                      kEpiArgmax, 0)
                        : gemm_plan(&g, d.embed, d.vocab, d.hidden, lm_in, 16, d.hidden, kEpiArgmax, 0)))
    return rc;
  if ((rc = gemm_bind_ws(&g, gws, gws_bytes))) return rc;
  g.p.n_rows = 1;
  g.p.vocab = d.vocab;
  g.p.argmax_out = next_token;
  g.p.inv_temp = m->inv_temp;
  g.p.sample_seed = m->sample_seed;
  g.p.sample_state = state;
  return gemm_launch(g, st);
}

extern "C" int dtree_qwen3_set_attention_keys(dtree_qwen3_model* m, int max_keys) {
  DTREE_CHECK_ARG(m, "null model");
  DTREE_CHECK_ARG(max_keys >= 0, "max_keys must be >= 0");
  m->attn_keys = max_keys;
  return kOk;
}

extern "C" int dtree_qwen3_set_sampling(dtree_qwen3_model* m, float temperature, uint32_t seed) {
  DTREE_CHECK_ARG(m, "null model");
  DTREE_CHECK_ARG(temperature >= 0.0f, "temperature must be >= 0");
  m->inv_temp = temperature < 1e-5f ? 0.0f : 1.0f / temperature;
  m->sample_seed = seed;
  return kOk;
}
