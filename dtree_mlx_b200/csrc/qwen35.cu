// Qwen3.5 hybrid tree-verify forward and accepted-path commit.
//
// forward_qwen35_tree_with_hidden_states (dtree_mlx/qwen35_tree.py:629-705)
// with lm_head_argmax, as one launch sequence per call:
//   DeltaNet layer (qwen35_tree.py:362-480, custom_qwen35_model.py:777-891):
//     xn = RMSNorm(h)                                   (residual_)rmsnorm
//     proj = xn @ [Wqkv | Wz | Wb | Wa]^T  (bf16)       gemm<kEpiStore>
//     qkv' = silu(tree conv1d(proj_qkv)); q, k RMSNorm  tree_conv1d (norm heads)
//     y = tree gated delta(q, k, v, g(a), beta(b))     tree_gated_delta
//     o = RMSNormGated(y, z)                            rmsnorm_gated
//     h += o @ Wout^T; xn = RMSNorm(h); MLP             gemm<kEpiPartial> ...
//   gated attention layer (qwen35_tree.py:483-626):
//     q | gate, k, v projection (split-K partials)      gemm<kEpiPartial>
//     q / k RMSNorm, partial RoPE, gate, K/V -> cache   qkv_finish (gated)
//     a = tree attention (head_dim 256) * sigmoid(gate) tree_attn + combine
//     h += a @ Wo^T; MLP
// The DeltaNet projections and conv outputs of every layer stay in per-layer
// buffers so that dtree_qwen35_commit can derive the accepted node's conv
// window and replay its recurrent state without per-node state storage.
#include <algorithm>
#include <cmath>
#include <vector>

#include "attention.cuh"
#include "deltanet.cuh"
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

namespace {

constexpr int kAttnSplitsMax = 32;
constexpr int kProjSplitMax = 16;

int pad_rows35(int n) { return n <= 16 ? 16 : n <= 32 ? 32 : n <= 64 ? 64 : n <= 80 ? 80 : 128; }
int tpad_idx(int t) { return t == 16 ? 0 : t == 32 ? 1 : t == 64 ? 2 : t == 80 ? 3 : 4; }

struct Dims {
  int n_attn, n_lin, key_dim, value_dim, conv_dim, proj_w, qkv_w, q_dim, keep, wide;
};

Dims dims_of(const dtree_qwen35_desc& d) {
  Dims x{};
  x.n_attn = d.layers / d.full_attention_interval;
  x.n_lin = d.layers - x.n_attn;
  x.key_dim = d.lin_k_heads * d.lin_k_dim;
  x.value_dim = d.lin_v_heads * d.lin_v_dim;
  x.conv_dim = 2 * x.key_dim + x.value_dim;
  x.proj_w = x.conv_dim + x.value_dim + 2 * d.lin_v_heads;
  x.q_dim = d.n_heads * d.head_dim;
  x.qkv_w = 2 * x.q_dim + 2 * d.n_kv_heads * d.head_dim;
  x.keep = d.conv_kernel - 1;
  x.wide = std::max(x.q_dim, x.value_dim);
  return x;
}

bool is_attn_layer(const dtree_qwen35_desc& d, int l) { return (l + 1) % d.full_attention_interval == 0; }

// split-K of a projection: two CTAs per SM (see the Qwen3 model)
int proj_split(int n_out) {
  const int tiles = (n_out + 127) / 128;
  return std::max(1, std::min(kProjSplitMax, 2 * num_sms() / tiles));
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

}  // namespace

struct Qwen35Plans {
  bool ready = false;
  std::vector<GemmPlan> in_proj, out_proj, qkv, o, gu, down;  // per layer (unused slots stay empty)
  GemmPlan lm;
};

}  // namespace dtree

struct dtree_qwen35_model {
  dtree_qwen35_desc d;
  dtree::Dims x;
  std::vector<dtree_qwen35_linear_layer> lin;
  std::vector<dtree_qwen35_attn_layer> att;
  std::vector<int> slot;  // layer -> index among its kind
  dtree::Qwen35Plans plans[5];
  void* gemm_ws = nullptr;
  size_t gemm_ws_bytes = 0;
  void* attn_ws = nullptr;
  size_t attn_ws_bytes = 0;
  float* partials = nullptr;
  float inv_temp = 0.0f;  // posterior sampling (0: greedy argmax)
  uint32_t sample_seed = 0;
};

namespace dtree {

static size_t gemm_need(const dtree_qwen35_desc& d) { return gemm_ws_bytes(pad_rows35(d.t_cap), 2 * num_sms()); }
static size_t attn_need(const dtree_qwen35_desc& d) {
  return attn_ws_bytes(d.n_heads, d.t_cap, d.head_dim, kAttnSplitsMax);
}
static size_t partials_need(const dtree_qwen35_desc& d, const Dims& x) {
  size_t w = static_cast<size_t>(proj_split(d.hidden)) * d.hidden;
  w = std::max(w, static_cast<size_t>(proj_split(x.qkv_w)) * x.qkv_w);
  return w * pad_rows35(d.t_cap) * 4;
}

static int build_plans(dtree_qwen35_model* m, int t_pad) {
  Qwen35Plans& ps = m->plans[tpad_idx(t_pad)];
  if (ps.ready) return kOk;
  const dtree_qwen35_desc& d = m->d;
  const Dims& x = m->x;
  ps.in_proj.resize(d.layers);
  ps.out_proj.resize(d.layers);
  ps.qkv.resize(d.layers);
  ps.o.resize(d.layers);
  ps.gu.resize(d.layers);
  ps.down.resize(d.layers);
  for (int l = 0; l < d.layers; ++l) {
    const int s = m->slot[l];
    int rc;
    const void *gate_up, *down;
    if (is_attn_layer(d, l)) {
      const dtree_qwen35_attn_layer& A = m->att[s];
      if ((rc = gemm_plan(&ps.qkv[l], A.qkv, x.qkv_w, d.hidden, d.xn, t_pad, d.hidden, kEpiPartial,
                          proj_split(x.qkv_w))))
        return rc;
      if ((rc = gemm_plan(&ps.o[l], A.o_proj, d.hidden, x.q_dim, d.attn, t_pad, x.q_dim, kEpiPartial,
                          proj_split(d.hidden))))
        return rc;
      gate_up = A.gate_up;
      down = A.down;
    } else {
      const dtree_qwen35_linear_layer& L = m->lin[s];
      if ((rc = gemm_plan(&ps.in_proj[l], L.in_proj, x.proj_w, d.hidden, d.xn, t_pad, d.hidden, kEpiStore, 0)))
        return rc;
      if ((rc = gemm_plan(&ps.out_proj[l], L.out_proj, d.hidden, x.value_dim, d.q, t_pad, x.wide, kEpiPartial,
                          proj_split(d.hidden))))
        return rc;
      gate_up = L.gate_up;
      down = L.down;
    }
    if ((rc = gemm_plan(&ps.gu[l], gate_up, 2 * d.ffn, d.hidden, d.xn, t_pad, d.hidden, kEpiSwiglu, 0))) return rc;
    if ((rc = gemm_plan(&ps.down[l], down, d.hidden, d.ffn, d.act, t_pad, d.ffn, kEpiPartial, proj_split(d.hidden))))
      return rc;
    for (GemmPlan* g : {&ps.in_proj[l], &ps.out_proj[l], &ps.qkv[l], &ps.o[l], &ps.gu[l], &ps.down[l]})
      if (g->p.n_out > 0 && (rc = gemm_bind_ws(g, m->gemm_ws, m->gemm_ws_bytes))) return rc;
  }
  int rc = gemm_plan(&ps.lm, d.embed, d.vocab, d.hidden, d.norm_out, t_pad, d.hidden, kEpiArgmax, 0);
  if (rc) return rc;
  if ((rc = gemm_bind_ws(&ps.lm, m->gemm_ws, m->gemm_ws_bytes))) return rc;
  ps.ready = true;
  return kOk;
}

}  // namespace dtree

using namespace dtree;

extern "C" int dtree_qwen35_buffer_bytes(const dtree_qwen35_desc* dp, size_t out[14]) {
  DTREE_CHECK_ARG(dp && out, "null pointer");
  const dtree_qwen35_desc& d = *dp;
  DTREE_CHECK_ARG(d.t_cap > 0 && d.t_cap <= DTREE_MAX_TREE, "t_cap must be in [1, 128]");
  DTREE_CHECK_ARG(d.full_attention_interval > 0 && d.layers > 0, "bad layer pattern");
  const Dims x = dims_of(d);
  const size_t tc = static_cast<size_t>(pad_rows35(d.t_cap));
  out[0] = static_cast<size_t>(x.n_attn) * 2 * d.n_kv_heads * static_cast<size_t>(d.kv_capacity) * d.head_dim * 2;
  out[1] = static_cast<size_t>(x.n_lin) * x.keep * x.conv_dim * 2;
  out[2] = static_cast<size_t>(x.n_lin) * d.lin_v_heads * d.lin_v_dim * d.lin_k_dim * 4;
  out[3] = tc * d.hidden * 2;
  out[4] = tc * d.hidden * 2;
  out[5] = tc * x.wide * 2;
  out[6] = tc * x.q_dim * 2;
  out[7] = tc * x.wide * 2;
  out[8] = tc * d.ffn * 2;
  out[9] = tc * d.hidden * 2;
  out[10] = tc * d.hidden * (d.n_capture > 0 ? d.n_capture : 1) * 2;
  out[11] = static_cast<size_t>(x.n_lin) * tc * x.proj_w * 2;
  out[12] = static_cast<size_t>(x.n_lin) * tc * x.conv_dim * 2;
  out[13] = align256(gemm_need(d)) + align256(attn_need(d)) + partials_need(d, x);
  return kOk;
}

extern "C" int dtree_qwen35_create(const dtree_qwen35_desc* dp, dtree_qwen35_model** out) {
  DTREE_CHECK_ARG(dp && out, "null pointer");
  const dtree_qwen35_desc& d = *dp;
  size_t need[14];
  int rc = dtree_qwen35_buffer_bytes(dp, need);
  if (rc) return rc;
  const Dims x = dims_of(d);
  DTREE_CHECK_ARG(d.hidden % 64 == 0 && d.ffn % 64 == 0 && d.hidden <= 4096, "hidden (<= 4096) and ffn must be multiples of 64");
  DTREE_CHECK_ARG(d.head_dim == 64 || d.head_dim == 128 || d.head_dim == 256, "head_dim must be 64, 128 or 256");
  DTREE_CHECK_ARG(d.n_heads % d.n_kv_heads == 0, "n_heads must be a multiple of n_kv_heads");
  DTREE_CHECK_ARG(d.lin_k_dim == d.lin_v_dim && (d.lin_k_dim == 64 || d.lin_k_dim == 128),
                  "DeltaNet key and value head dims must be equal, 64 or 128");
  DTREE_CHECK_ARG(d.lin_v_heads % d.lin_k_heads == 0, "lin_v_heads must be a multiple of lin_k_heads");
  DTREE_CHECK_ARG(d.conv_kernel >= 2 && d.conv_kernel <= 9, "conv_kernel must be in [2, 9]");
  DTREE_CHECK_ARG(x.q_dim % 128 == 0 && x.value_dim % 64 == 0, "projection widths must be multiples of 128 / 64");
  const int rot = static_cast<int>(std::lround(d.head_dim * d.partial_rotary_factor));
  DTREE_CHECK_ARG(rot >= 2 && rot <= d.head_dim && rot % 2 == 0, "partial_rotary_factor gives an odd or empty rotation");
  DTREE_CHECK_ARG(d.n_capture >= 0 && d.n_capture <= 16, "n_capture must be in [0, 16]");
  for (int c = 0; c < d.n_capture; ++c)
    DTREE_CHECK_ARG(d.capture_layers[c] >= 0 && d.capture_layers[c] < d.layers, "capture layer out of range");
  DTREE_CHECK_ARG(d.embed && d.final_norm && d.a_log && d.dt_bias && (x.n_attn == 0 || d.attn_layers) &&
                      (x.n_lin == 0 || d.linear_layers),
                  "null weights");
  DTREE_CHECK_ARG(d.kv_cache && d.conv_state && d.rec_state && d.h && d.xn && d.q && d.gate && d.attn && d.act &&
                      d.norm_out && d.lin_proj && d.lin_qkv && d.workspace,
                  "null buffer");
  DTREE_CHECK_ARG(d.n_capture == 0 || d.capture, "null capture buffer");
  DTREE_CHECK_ARG(d.workspace_bytes >= need[13], "workspace too small");
  auto* m = new dtree_qwen35_model();
  m->d = d;
  m->x = x;
  m->lin.assign(d.linear_layers, d.linear_layers + x.n_lin);
  m->att.assign(d.attn_layers, d.attn_layers + x.n_attn);
  int li = 0, ai = 0;
  for (int l = 0; l < d.layers; ++l) m->slot.push_back(is_attn_layer(d, l) ? ai++ : li++);
  m->gemm_ws = d.workspace;
  m->gemm_ws_bytes = gemm_need(d);
  m->attn_ws = static_cast<char*>(d.workspace) + align256(m->gemm_ws_bytes);
  m->attn_ws_bytes = attn_need(d);
  m->partials = reinterpret_cast<float*>(static_cast<char*>(m->attn_ws) + align256(m->attn_ws_bytes));
  *out = m;
  return kOk;
}

extern "C" int dtree_qwen35_destroy(dtree_qwen35_model* m) {
  delete m;
  return kOk;
}

extern "C" int dtree_qwen35_forward(dtree_qwen35_model* m, const int32_t* tokens, const int32_t* positions,
                                    const int32_t* parents, const uint64_t* anc_mask, int n, int mode,
                                    const dtree_step_state* state, int32_t* posterior, void* stream_) {
  DTREE_CHECK_ARG(m && tokens && positions && parents && anc_mask && state, "null pointer");
  const dtree_qwen35_desc& d = m->d;
  const Dims& x = m->x;
  DTREE_CHECK_ARG(n > 0 && n <= d.t_cap, "n_nodes must be in [1, t_cap]");
  DTREE_CHECK_ARG(mode == 0 || mode == 1, "mode must be 0 (tree) or 1 (sequence)");
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  const int t_pad = pad_rows35(n);
  int rc = build_plans(m, t_pad);
  if (rc) return rc;
  Qwen35Plans& ps = m->plans[tpad_idx(t_pad)];
  auto bf = [](const void* p) { return static_cast<const __nv_bfloat16*>(p); };
  auto bw = [](void* p) { return static_cast<__nv_bfloat16*>(p); };
  const size_t plane = static_cast<size_t>(d.n_kv_heads) * d.kv_capacity * d.head_dim;
  const size_t tc = static_cast<size_t>(pad_rows35(d.t_cap));
  const int ldc = d.hidden * (d.n_capture > 0 ? d.n_capture : 1);
  auto capture_ptr = [&](int l) -> __nv_bfloat16* {
    for (int c = 0; c < d.n_capture; ++c)
      if (d.capture_layers[c] == l) return bw(d.capture) + static_cast<size_t>(c) * d.hidden;
    return nullptr;
  };
  const int G = d.n_heads / d.n_kv_heads;
  const int rb = (G * n + 127) / 128;
  const int nvh = d.head_dim > 128 ? 2 : 1;
  const int splits = std::max(1, std::min(kAttnSplitsMax, num_sms() / (d.n_kv_heads * rb * nvh)));
  const int rot = static_cast<int>(std::lround(d.head_dim * d.partial_rotary_factor));

  // embedding gather + first input norm
  const void* norm0 = is_attn_layer(d, 0) ? m->att[0].input_norm : m->lin[0].input_norm;
  if ((rc = rmsnorm_launch(nullptr, 0, tokens, bf(d.embed), bw(d.h), bf(norm0), bw(d.xn), d.hidden, n, t_pad,
                           d.rms_eps, st)))
    return rc;
  int prev_split = 0;
  for (int l = 0; l < d.layers; ++l) {
    const int s = m->slot[l];
    const bool attn = is_attn_layer(d, l);
    const void* in_norm = attn ? m->att[s].input_norm : m->lin[s].input_norm;
    const void* post_norm = attn ? m->att[s].post_norm : m->lin[s].post_norm;
    if (l > 0 && (rc = residual_rmsnorm_launch(bw(d.h), m->partials, prev_split, t_pad, capture_ptr(l - 1), ldc,
                                               bf(in_norm), bw(d.xn), d.hidden, n, t_pad, d.rms_eps, st)))
      return rc;
    int mix_split;
    if (attn) {
      const dtree_qwen35_attn_layer& A = m->att[s];
      __nv_bfloat16* kc = bw(d.kv_cache) + (static_cast<size_t>(s) * 2 + 0) * plane;
      __nv_bfloat16* vc = bw(d.kv_cache) + (static_cast<size_t>(s) * 2 + 1) * plane;
      GemmPlan g = ps.qkv[l];
      g.p.n_rows = n;
      g.p.out_f32 = m->partials;
      g.p.ldo = x.qkv_w;
      if ((rc = gemm_launch(g, st))) return rc;
      QkvFinishParams f{};
      f.partials = m->partials;
      f.split = g.p.split;
      f.part_rows = t_pad;
      f.width = x.qkv_w;
      f.head_dim = d.head_dim;
      f.n_q_heads = d.n_heads;
      f.n_kv_heads = d.n_kv_heads;
      f.q_norm = bf(A.q_norm);
      f.k_norm = bf(A.k_norm);
      f.eps = d.rms_eps;
      f.rope_log2_theta = std::log2(d.rope_theta);
      f.positions = positions;
      f.state = state;
      f.q_out = bw(d.q);
      f.k_cache = kc;
      f.v_cache = vc;
      f.kv_cap = d.kv_capacity;
      f.gated = 1;
      f.gate_out = bw(d.gate);
      f.rot_dims = rot;
      if ((rc = qkv_finish_launch(f, n, st))) return rc;
      AttnParams a{};
      a.q = bf(d.q);
      a.ldq = x.q_dim;
      a.k = kc;
      a.v = vc;
      a.cap = d.kv_capacity;
      a.n_q_heads = d.n_heads;
      a.n_kv_heads = d.n_kv_heads;
      a.n_nodes = n;
      a.state = state;
      a.anc = anc_mask;
      a.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(d.head_dim)));
      a.splits = splits;
      a.out = bw(d.attn);
      a.gate = bf(d.gate);
      if ((rc = attn_launch(a, d.head_dim, m->attn_ws, m->attn_ws_bytes, st))) return rc;
      GemmPlan o = ps.o[l];
      o.p.n_rows = n;
      o.p.out_f32 = m->partials;
      o.p.ldo = d.hidden;
      if ((rc = gemm_launch(o, st))) return rc;
      mix_split = o.p.split;
    } else {
      const dtree_qwen35_linear_layer& L = m->lin[s];
      __nv_bfloat16* proj = bw(d.lin_proj) + static_cast<size_t>(s) * tc * x.proj_w;
      __nv_bfloat16* qkvn = bw(d.lin_qkv) + static_cast<size_t>(s) * tc * x.conv_dim;
      __nv_bfloat16* cst = bw(d.conv_state) + static_cast<size_t>(s) * x.keep * x.conv_dim;
      float* rst = static_cast<float*>(d.rec_state) + static_cast<size_t>(s) * d.lin_v_heads * d.lin_v_dim * d.lin_k_dim;
      GemmPlan g = ps.in_proj[l];
      g.p.n_rows = n;
      g.p.out = proj;
      g.p.ldo = x.proj_w;
      if ((rc = gemm_launch(g, st))) return rc;
      ConvParams c{};
      c.x = proj;
      c.ldx = x.proj_w;
      c.base = cst;
      c.weight = L.conv_weight;
      c.parents = parents;
      c.n_nodes = n;
      c.conv_dim = x.conv_dim;
      c.keep = x.keep;
      c.out = qkvn;
      c.ldo = x.conv_dim;
      c.n_norm_heads = 2 * d.lin_k_heads;
      c.n_q_heads = d.lin_k_heads;
      if ((rc = tree_conv1d_launch(c, 1, d.lin_k_dim, st))) return rc;
      DeltaParams dp{};
      dp.q = qkvn;
      dp.k = qkvn + x.key_dim;
      dp.ldqk = x.conv_dim;
      dp.v = qkvn + 2 * x.key_dim;
      dp.ldv = x.conv_dim;
      dp.b = proj + x.conv_dim + x.value_dim;
      dp.a = proj + x.conv_dim + x.value_dim + d.lin_v_heads;
      dp.ldab = x.proj_w;
      dp.a_log = d.a_log + static_cast<size_t>(s) * d.lin_v_heads;
      dp.dt_bias = bf(d.dt_bias) + static_cast<size_t>(s) * d.lin_v_heads;
      dp.state_in = rst;
      dp.parents = parents;
      dp.n_nodes = n;
      dp.n_k_heads = d.lin_k_heads;
      dp.n_v_heads = d.lin_v_heads;
      dp.dv = d.lin_v_dim;
      dp.y = d.attn;
      dp.ldy = x.wide;
      dp.no_round = mode == 1;
      dp.final_state = mode == 1 ? rst : nullptr;
      if ((rc = tree_gated_delta_launch(dp, d.lin_k_dim, 1, 0, st))) return rc;
      if ((rc = rmsnorm_gated_launch(bf(d.attn), x.wide, proj + x.conv_dim, x.proj_w, bf(L.norm), d.rms_eps,
                                     bw(d.q), x.wide, n, d.lin_v_heads, d.lin_v_dim, st)))
        return rc;
      if (mode == 1) {  // sequence: the conv window advances to the last token
        if ((rc = conv_state_commit_launch(c, 1, nullptr, nullptr, 1, 0, 0, n - 1, st))) return rc;
      }
      GemmPlan o = ps.out_proj[l];
      o.p.n_rows = n;
      o.p.out_f32 = m->partials;
      o.p.ldo = d.hidden;
      if ((rc = gemm_launch(o, st))) return rc;
      mix_split = o.p.split;
    }
    if ((rc = residual_rmsnorm_launch(bw(d.h), m->partials, mix_split, t_pad, nullptr, 0, bf(post_norm), bw(d.xn),
                                      d.hidden, n, t_pad, d.rms_eps, st)))
      return rc;
    GemmPlan gu = ps.gu[l];
    gu.p.n_rows = n;
    gu.p.out = bw(d.act);
    gu.p.ldo = d.ffn;
    if ((rc = gemm_launch(gu, st))) return rc;
    GemmPlan dn = ps.down[l];
    dn.p.n_rows = n;
    dn.p.out_f32 = m->partials;
    dn.p.ldo = d.hidden;
    if ((rc = gemm_launch(dn, st))) return rc;
    prev_split = dn.p.split;
  }
  if ((rc = residual_rmsnorm_launch(bw(d.h), m->partials, prev_split, t_pad, capture_ptr(d.layers - 1), ldc,
                                    bf(d.final_norm), bw(d.norm_out), d.hidden, n, t_pad, d.rms_eps, st)))
    return rc;
  if (posterior) {
    GemmPlan g = ps.lm;
    g.p.n_rows = n;
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
// Dense causal forward of the prompt for the hybrid (Qwen35TargetAdapter's
// forward_with_hidden_states over the prompt, adapters.py:216-450 with the
// prefill of dtree_runtime.py:342-349): every projection is one dense
// tcgen05 GEMM over all rows; a DeltaNet layer runs its causal conv over all
// rows in one launch (chain parents), the recurrence as one sequence kernel
// (state in f32 registers from the first row to the last, as mlx-lm's
// sequence kernel) and advances the layer's conv / recurrent state to the
// last row; a gated attention layer attends per 128-row chunk.
namespace dtree {
namespace {

__global__ void prefill35_init_kernel(int32_t* parents, int n, uint64_t* anc, dtree_step_state* chunk_states,
                                      int chunks, const dtree_step_state* state) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) parents[i] = i - 1;
  if (i < 128) {  // row i of a 128-row chain sees rows 0..i
    anc[2 * i] = i >= 63 ? ~0ull : ((1ull << (i + 1)) - 1ull);
    anc[2 * i + 1] = i < 64 ? 0ull : (i >= 127 ? ~0ull : ((1ull << (i - 63)) - 1ull));
  }
  if (i < chunks) {  // attention chunk i: rows from i*128 at slots start + i*128
    dtree_step_state s = *state;
    s.start += i * 128;
    chunk_states[i] = s;
  }
}

struct Prefill35Layout {
  size_t h, xn, big, qkvn, mix, q, gate, parents, anc, states, lm_in, gemm, total;
  int n_pad, chunks;
};

Prefill35Layout prefill35_layout(const dtree_qwen35_desc& d, const Dims& x, int n_rows) {
  Prefill35Layout L{};
  L.n_pad = ((n_rows + kDenseRows - 1) / kDenseRows) * kDenseRows;
  L.chunks = (n_rows + 127) / 128;
  const size_t np = static_cast<size_t>(L.n_pad);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += align256(bytes);
    return o;
  };
  L.h = take(np * d.hidden * 2);
  L.xn = take(np * d.hidden * 2);
  L.big = take(np * std::max({x.proj_w, x.qkv_w, d.ffn}) * 2);
  L.qkvn = take(np * x.conv_dim * 2);
  L.mix = take(np * x.wide * 2);
  L.q = take(np * x.wide * 2);
  L.gate = take(np * x.q_dim * 2);
  L.parents = take(np * 4);
  L.anc = take(128 * 16);
  L.states = take(static_cast<size_t>(L.chunks) * sizeof(dtree_step_state));
  L.lm_in = take(static_cast<size_t>(16) * d.hidden * 2);
  L.gemm = take(gemm_ws_bytes(kDenseRows, num_sms()));
  L.total = off;
  return L;
}

}  // namespace
}  // namespace dtree

extern "C" size_t dtree_qwen35_prefill_workspace_bytes(const dtree_qwen35_desc* d, int n_rows) {
  if (!d || n_rows <= 0 || d->full_attention_interval <= 0) return 0;
  return prefill35_layout(*d, dims_of(*d), n_rows).total;
}

extern "C" int dtree_qwen35_prefill(dtree_qwen35_model* m, const int32_t* tokens, const int32_t* positions,
                                    int n_rows, const dtree_step_state* state, void* hidden_out, int ld_hidden_out,
                                    void* norm_out, int32_t* next_token, void* workspace, size_t workspace_bytes,
                                    void* stream_) {
  DTREE_CHECK_ARG(m && tokens && positions && state && next_token && workspace, "null pointer");
  const dtree_qwen35_desc& d = m->d;
  const Dims& x = m->x;
  DTREE_CHECK_ARG(n_rows > 0 && n_rows <= d.kv_capacity, "n_rows must be in [1, kv_capacity]");
  DTREE_CHECK_ARG(d.n_capture == 0 || hidden_out, "null hidden_out with captured layers");
  DTREE_CHECK_ARG(!hidden_out || ld_hidden_out >= d.hidden * d.n_capture, "ld_hidden_out below n_capture * hidden");
  const Prefill35Layout Lo = prefill35_layout(d, x, n_rows);
  DTREE_CHECK_ARG(workspace_bytes >= Lo.total, "prefill workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  char* ws = static_cast<char*>(workspace);
  auto at = [&](size_t off) { return reinterpret_cast<__nv_bfloat16*>(ws + off); };
  auto bf = [](const void* p) { return static_cast<const __nv_bfloat16*>(p); };
  __nv_bfloat16 *h = at(Lo.h), *xn = at(Lo.xn), *big = at(Lo.big), *qkvn = at(Lo.qkvn), *mix = at(Lo.mix);
  __nv_bfloat16 *q = at(Lo.q), *gate = at(Lo.gate);
  int32_t* parents = reinterpret_cast<int32_t*>(ws + Lo.parents);
  uint64_t* anc = reinterpret_cast<uint64_t*>(ws + Lo.anc);
  dtree_step_state* cstates = reinterpret_cast<dtree_step_state*>(ws + Lo.states);
  void* gws = ws + Lo.gemm;
  const size_t gws_bytes = Lo.total - Lo.gemm;
  const int np = Lo.n_pad;
  const size_t plane = static_cast<size_t>(d.n_kv_heads) * d.kv_capacity * d.head_dim;
  const int rot = static_cast<int>(std::lround(d.head_dim * d.partial_rotary_factor));
  DTREE_CUDA_RET(cudaMemsetAsync(gws, 0, gemm_ws_counter_bytes(), st));
  const int init_n = std::max({n_rows, 128, Lo.chunks});
  DTREE_CUDA_RET(launch_pdl(prefill35_init_kernel, dim3((init_n + 255) / 256), dim3(256), 0, st, parents, n_rows, anc,
                            cstates, Lo.chunks, state));
  int rc;
  auto dense = [&](const void* w, int n_out, int k, const __nv_bfloat16* xin, int ldx, int epi, __nv_bfloat16* out,
                   int ldo, __nv_bfloat16* capture, int ldc) -> int {
    GemmPlan g;
    int r = gemm_plan_dense(&g, w, n_out, k, xin, n_rows, np, ldx, epi);
    if (r) return r;
    if ((r = gemm_bind_ws(&g, gws, gws_bytes))) return r;
    g.p.out = out;
    g.p.ldo = ldo;
    g.p.capture = capture;
    g.p.ldc = ldc;
    return gemm_launch(g, st);
  };
  auto capture_ptr = [&](int l) -> __nv_bfloat16* {
    for (int c = 0; c < d.n_capture; ++c)
      if (d.capture_layers[c] == l) return static_cast<__nv_bfloat16*>(hidden_out) + static_cast<size_t>(c) * d.hidden;
    return nullptr;
  };
  const void* norm0 = is_attn_layer(d, 0) ? m->att[0].input_norm : m->lin[0].input_norm;
  if ((rc = rmsnorm_launch(nullptr, 0, tokens, bf(d.embed), h, bf(norm0), xn, d.hidden, n_rows, np, d.rms_eps, st)))
    return rc;
  const int G = d.n_heads / d.n_kv_heads;
  const int nvh = d.head_dim > 128 ? 2 : 1;
  for (int l = 0; l < d.layers; ++l) {
    const int s = m->slot[l];
    const bool attn = is_attn_layer(d, l);
    const void* post_norm = attn ? m->att[s].post_norm : m->lin[s].post_norm;
    const void *gate_up, *down;
    if (attn) {
      const dtree_qwen35_attn_layer& A = m->att[s];
      gate_up = A.gate_up;
      down = A.down;
      __nv_bfloat16* kc = static_cast<__nv_bfloat16*>(d.kv_cache) + (static_cast<size_t>(s) * 2 + 0) * plane;
      __nv_bfloat16* vc = static_cast<__nv_bfloat16*>(d.kv_cache) + (static_cast<size_t>(s) * 2 + 1) * plane;
      if ((rc = dense(A.qkv, x.qkv_w, d.hidden, xn, d.hidden, kEpiStore, big, x.qkv_w, nullptr, 0))) return rc;
      QkvFinishParams f{};
      f.dense = big;
      f.width = x.qkv_w;
      f.head_dim = d.head_dim;
      f.n_q_heads = d.n_heads;
      f.n_kv_heads = d.n_kv_heads;
      f.q_norm = bf(A.q_norm);
      f.k_norm = bf(A.k_norm);
      f.eps = d.rms_eps;
      f.rope_log2_theta = std::log2(d.rope_theta);
      f.positions = positions;
      f.state = state;
      f.q_out = q;
      f.k_cache = kc;
      f.v_cache = vc;
      f.kv_cap = d.kv_capacity;
      f.gated = 1;
      f.gate_out = gate;
      f.rot_dims = rot;
      if ((rc = qkv_rows_launch(f, n_rows, st))) return rc;
      for (int c = 0; c < Lo.chunks; ++c) {  // causal attention, one 128-row chunk per launch
        const int t = std::min(128, n_rows - c * 128);
        const size_t off = static_cast<size_t>(c) * 128 * x.q_dim;
        AttnParams a{};
        a.q = q + off;
        a.ldq = x.q_dim;
        a.k = kc;
        a.v = vc;
        a.cap = d.kv_capacity;
        a.n_q_heads = d.n_heads;
        a.n_kv_heads = d.n_kv_heads;
        a.n_nodes = t;
        a.state = cstates + c;
        a.anc = anc;
        a.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(d.head_dim)));
        a.splits = std::max(1, std::min(kAttnSplitsMax, num_sms() / (d.n_kv_heads * ((G * t + 127) / 128) * nvh)));
        a.out = mix + off;
        a.gate = gate + off;
        if ((rc = attn_launch(a, d.head_dim, m->attn_ws, m->attn_ws_bytes, st))) return rc;
      }
      if ((rc = dense(A.o_proj, d.hidden, x.q_dim, mix, x.q_dim, kEpiResidual, h, d.hidden, nullptr, 0))) return rc;
    } else {
      const dtree_qwen35_linear_layer& L = m->lin[s];
      gate_up = L.gate_up;
      down = L.down;
      __nv_bfloat16* cst = static_cast<__nv_bfloat16*>(d.conv_state) + static_cast<size_t>(s) * x.keep * x.conv_dim;
      float* rst = static_cast<float*>(d.rec_state) + static_cast<size_t>(s) * d.lin_v_heads * d.lin_v_dim * d.lin_k_dim;
      if ((rc = dense(L.in_proj, x.proj_w, d.hidden, xn, d.hidden, kEpiStore, big, x.proj_w, nullptr, 0))) return rc;
      ConvParams c{};
      c.x = big;
      c.ldx = x.proj_w;
      c.base = cst;
      c.weight = L.conv_weight;
      c.parents = parents;
      c.n_nodes = n_rows;
      c.conv_dim = x.conv_dim;
      c.keep = x.keep;
      c.out = qkvn;
      c.ldo = x.conv_dim;
      c.n_norm_heads = 2 * d.lin_k_heads;
      c.n_q_heads = d.lin_k_heads;
      if ((rc = conv1d_seq_launch(c, d.lin_k_dim, st))) return rc;
      DeltaParams dp{};
      dp.q = qkvn;
      dp.k = qkvn + x.key_dim;
      dp.ldqk = x.conv_dim;
      dp.v = qkvn + 2 * x.key_dim;
      dp.ldv = x.conv_dim;
      dp.b = big + x.conv_dim + x.value_dim;
      dp.a = big + x.conv_dim + x.value_dim + d.lin_v_heads;
      dp.ldab = x.proj_w;
      dp.a_log = d.a_log + static_cast<size_t>(s) * d.lin_v_heads;
      dp.dt_bias = bf(d.dt_bias) + static_cast<size_t>(s) * d.lin_v_heads;
      dp.state_in = rst;
      dp.final_state = rst;
      dp.n_nodes = n_rows;
      dp.n_k_heads = d.lin_k_heads;
      dp.n_v_heads = d.lin_v_heads;
      dp.dv = d.lin_v_dim;
      dp.y = mix;
      dp.ldy = x.wide;
      if ((rc = gated_delta_seq_launch(dp, d.lin_k_dim, st))) return rc;
      // the conv window advances to the last prompt row (before `big` is reused)
      if ((rc = conv_state_commit_launch(c, 1, nullptr, nullptr, 1, 0, 0, n_rows - 1, st))) return rc;
      if ((rc = rmsnorm_gated_launch(mix, x.wide, big + x.conv_dim, x.proj_w, bf(L.norm), d.rms_eps, q, x.wide, n_rows,
                                     d.lin_v_heads, d.lin_v_dim, st)))
        return rc;
      if ((rc = dense(L.out_proj, d.hidden, x.value_dim, q, x.wide, kEpiResidual, h, d.hidden, nullptr, 0))) return rc;
    }
    if ((rc = rmsnorm_launch(h, d.hidden, nullptr, nullptr, nullptr, bf(post_norm), xn, d.hidden, n_rows, np,
                             d.rms_eps, st)))
      return rc;
    if ((rc = dense(gate_up, 2 * d.ffn, d.hidden, xn, d.hidden, kEpiSwiglu, big, d.ffn, nullptr, 0))) return rc;
    if ((rc = dense(down, d.hidden, d.ffn, big, d.ffn, kEpiResidual, h, d.hidden, capture_ptr(l), ld_hidden_out)))
      return rc;
    if (l + 1 < d.layers) {
      const void* nn = is_attn_layer(d, l + 1) ? m->att[m->slot[l + 1]].input_norm : m->lin[m->slot[l + 1]].input_norm;
      if ((rc = rmsnorm_launch(h, d.hidden, nullptr, nullptr, nullptr, bf(nn), xn, d.hidden, n_rows, np, d.rms_eps,
                               st)))
        return rc;
    }
  }
  if (norm_out && (rc = rmsnorm_launch(h, d.hidden, nullptr, nullptr, nullptr, bf(d.final_norm),
                                       static_cast<__nv_bfloat16*>(norm_out), d.hidden, n_rows, n_rows, d.rms_eps, st)))
    return rc;
  __nv_bfloat16* lm_in = at(Lo.lm_in);
  if ((rc = rmsnorm_launch(h + static_cast<size_t>(n_rows - 1) * d.hidden, d.hidden, nullptr, nullptr, nullptr,
                           bf(d.final_norm), lm_in, d.hidden, 1, 16, d.rms_eps, st)))
    return rc;
  GemmPlan g;
  if ((rc = gemm_plan(&g, d.embed, d.vocab, d.hidden, lm_in, 16, d.hidden, kEpiArgmax, 0))) return rc;
  if ((rc = gemm_bind_ws(&g, gws, gws_bytes))) return rc;
  g.p.n_rows = 1;
  g.p.vocab = d.vocab;
  g.p.argmax_out = next_token;
  g.p.inv_temp = m->inv_temp;
  g.p.sample_seed = m->sample_seed;
  g.p.sample_state = state;
  return gemm_launch(g, st);
}

extern "C" int dtree_qwen35_set_sampling(dtree_qwen35_model* m, float temperature, uint32_t seed) {
  DTREE_CHECK_ARG(m, "null model");
  DTREE_CHECK_ARG(temperature >= 0.0f, "temperature must be >= 0");
  m->inv_temp = temperature < 1e-5f ? 0.0f : 1.0f / temperature;
  m->sample_seed = seed;
  return kOk;
}

extern "C" int dtree_kv_compact(void* kv_cache, int layers, int kv_heads, int capacity, int head_dim,
                                const int32_t* accepted, const dtree_step_state* state, void* stream);

extern "C" int dtree_qwen35_commit(dtree_qwen35_model* m, const int32_t* parents, const int32_t* accepted,
                                   const dtree_step_state* state, void* stream_) {
  DTREE_CHECK_ARG(m && parents && accepted && state, "null pointer");
  const dtree_qwen35_desc& d = m->d;
  const Dims& x = m->x;
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  int rc;
  if (x.n_attn > 0 &&
      (rc = dtree_kv_compact(d.kv_cache, x.n_attn, d.n_kv_heads, d.kv_capacity, d.head_dim, accepted, state, st)))
    return rc;
  if (x.n_lin == 0) return kOk;
  const size_t tc = static_cast<size_t>(pad_rows35(d.t_cap));
  DeltaParams p{};
  p.q = d.lin_qkv;
  p.k = static_cast<const __nv_bfloat16*>(d.lin_qkv) + x.key_dim;
  p.ldqk = x.conv_dim;
  p.v = static_cast<const __nv_bfloat16*>(d.lin_qkv) + 2 * x.key_dim;
  p.ldv = x.conv_dim;
  p.b = static_cast<const __nv_bfloat16*>(d.lin_proj) + x.conv_dim + x.value_dim;
  p.a = static_cast<const __nv_bfloat16*>(d.lin_proj) + x.conv_dim + x.value_dim + d.lin_v_heads;
  p.ldab = x.proj_w;
  p.a_log = d.a_log;
  p.dt_bias = d.dt_bias;
  p.n_nodes = d.t_cap;
  p.n_k_heads = d.lin_k_heads;
  p.n_v_heads = d.lin_v_heads;
  p.dv = d.lin_v_dim;
  p.path = accepted;
  p.st = state;
  p.state_out = d.rec_state;
  p.layer_stride_qk = tc * x.conv_dim;
  p.layer_stride_v = tc * x.conv_dim;
  p.layer_stride_ab = tc * x.proj_w;
  p.layer_stride_state = static_cast<size_t>(d.lin_v_heads) * d.lin_v_dim * d.lin_k_dim;
  p.layer_stride_params = d.lin_v_heads;
  if ((rc = gated_delta_replay_launch(p, d.lin_k_dim, 1, 0, x.n_lin, st))) return rc;
  ConvParams c{};
  c.x = d.lin_proj;
  c.ldx = x.proj_w;
  c.base = d.conv_state;
  c.parents = parents;
  c.n_nodes = d.t_cap;
  c.conv_dim = x.conv_dim;
  c.keep = x.keep;
  return conv_state_commit_launch(c, 1, accepted, state, x.n_lin, tc * x.proj_w,
                                  static_cast<size_t>(x.keep) * x.conv_dim, -1, st);
}
