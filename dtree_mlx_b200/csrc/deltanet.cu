// Qwen3.5 gated-DeltaNet tree kernels: the causal conv1d and the gated delta
// recurrence evaluated along every root->node path of a verify tree, and the
// commit of the accepted path into the layer's conv / recurrent state.
//
// Reference semantics: tree_conv1d_kernel and tree_gated_delta_kernel
// (dtree_mlx/qwen35_tree_kernels.py:8-224), commit_qwen35_tree_path
// (dtree_mlx/qwen35_tree.py:708-732).  Per node t with parent p (p < 0: the
// layer's base state):
//   conv:   window = last `keep` inputs on the path to p (or the base conv
//           state), out = silu(sum_k window[k] w[k] + x_t w[keep]) -> InT
//   delta:  S = S_p * g_t;  kv = S k_t;  delta = (v_t - kv) beta_t;
//           S += k_t delta^T;  y_t = S q_t -> InT;  S_t = InT(S)   (rounded)
//
// B200 layout choices:
// * conv: a node's window is the inputs of its ancestors, so each (node,
//   channel) is computed independently by walking `keep` parent links;
//   no per-node conv state is materialized (commit derives the accepted
//   node's window the same way).
// * delta: one warp per state row (hv, dv), Dk/32 elements per lane; the CTA
//   stages its head's q / k / g / beta for all nodes in shared memory and
//   keeps every node's rounded state row there (InT-exact, so storing it as
//   InT loses nothing) for its children.  Per-node states are not written to
//   HBM unless asked: commit replays the accepted path from the base state
//   with the identical per-node arithmetic, which reproduces the deepest
//   accepted node's state bit for bit.
#include <cmath>

#include "deltanet.cuh"

namespace dtree {

template <typename T>
__device__ __forceinline__ float ld_f(const T* p) {
  if constexpr (std::is_same<T, float>::value) return *p;
  else return __bfloat162float(*p);
}
template <typename T>
__device__ __forceinline__ void st_f(T* p, float v) {
  if constexpr (std::is_same<T, float>::value) *p = v;
  else *p = __float2bfloat16_rn(v);
}
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  if constexpr (std::is_same<T, float>::value) return v;
  else return __bfloat162float(__float2bfloat16_rn(v));
}

constexpr int kMaxKeep = 8;

// ------------------------------------------------------------------ conv1d
// ConvParams / DeltaParams: deltanet.cuh

// input `m` steps up the path of node t (m = 0: the node itself), or the
// base conv state once the path runs out
template <typename InT>
__device__ __forceinline__ void conv_window(const ConvParams& p, int t, int c, float* win) {
  const InT* x = static_cast<const InT*>(p.x);
  const InT* base = static_cast<const InT*>(p.base);
  win[p.keep] = ld_f(x + static_cast<size_t>(t) * p.ldx + c);
  int prev = t;
  int cur = p.parents[t];
  int bi = p.keep - 1;
  for (int m = 1; m <= p.keep; ++m) {
    if (cur >= prev) {  // parents must precede their children
      dev_error(0x2004u);
      cur = -1;
    }
    if (cur >= 0) {
      win[p.keep - m] = ld_f(x + static_cast<size_t>(cur) * p.ldx + c);
      prev = cur;
      cur = p.parents[cur];
    } else {
      win[p.keep - m] = ld_f(base + static_cast<size_t>(bi) * p.conv_dim + c);
      --bi;
    }
  }
}

// grid (n_nodes, ceil(conv_dim / blockDim)); with head normalization the
// block is exactly one head (blockDim = head dim)
template <typename InT>
__global__ void tree_conv1d_kernel(ConvParams p) {
  pdl_trigger();
  __shared__ float s_red[32];
  const int t = blockIdx.x;
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  pdl_wait();
  const bool ok = c < p.conv_dim;
  float win[kMaxKeep + 1];
  float y = 0.0f;
  if (ok) {
    conv_window<InT>(p, t, c, win);
    const InT* w = static_cast<const InT*>(p.weight);
    float acc = 0.0f;
    for (int k = 0; k < p.keep; ++k) acc = fmaf(win[k], ld_f(w + static_cast<size_t>(k) * p.conv_dim + c), acc);
    acc = fmaf(win[p.keep], ld_f(w + static_cast<size_t>(p.keep) * p.conv_dim + c), acc);
    y = round_to<InT>(acc / (1.0f + expf(-acc)));
    if (p.node_states) {
      InT* ns = static_cast<InT*>(p.node_states);
      for (int k = 0; k < p.keep; ++k)
        st_f(ns + (static_cast<size_t>(t) * p.keep + k) * p.conv_dim + c, win[k + 1]);
    }
  }
  const int head = blockIdx.y;
  if (head < p.n_norm_heads) {  // uniform per block
    const int D = blockDim.x;
    float ss = y * y;
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int w = 0; w < (D + 31) / 32; ++w) tot += s_red[w];
    const float r = round_to<InT>(y * rsqrtf(tot / static_cast<float>(D) + 1e-6f));
    const float scale = head < p.n_q_heads ? 1.0f / static_cast<float>(D) : rsqrtf(static_cast<float>(D));
    y = round_to<InT>(r * scale);
  }
  if (ok) st_f(static_cast<InT*>(p.out) + static_cast<size_t>(t) * p.ldo + c, y);
}

// ------------------------------------------------------------ gated delta


template <typename InT>
__device__ __forceinline__ void node_gates(const DeltaParams& p, int t, int hv, float& g, float& beta) {
  if (p.g) {
    g = p.g[static_cast<size_t>(t) * p.n_v_heads + hv];
    beta = ld_f(static_cast<const InT*>(p.beta) + static_cast<size_t>(t) * p.n_v_heads + hv);
  } else {
    const float a = ld_f(static_cast<const InT*>(p.a) + static_cast<size_t>(t) * p.ldab + hv);
    const float bb = ld_f(static_cast<const InT*>(p.b) + static_cast<size_t>(t) * p.ldab + hv);
    const float x = round_to<InT>(a + ld_f(static_cast<const InT*>(p.dt_bias) + hv));
    const float sp = round_to<InT>(x > 20.0f ? x : log1pf(expf(x)));
    g = expf(-expf(p.a_log[hv]) * sp);
    beta = round_to<InT>(1.0f / (1.0f + expf(-bb)));
  }
}

// One node of the recurrence on a state row held as NP floats per lane.
template <typename InT, int NP>
__device__ __forceinline__ float delta_step(float (&s)[NP], const float (&kk)[NP], const float (&qq)[NP], float v,
                                            float g, float beta, bool rnd = true) {
  float kv = 0.0f;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    s[i] = s[i] * g;
    kv = fmaf(s[i], kk[i], kv);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) kv += __shfl_xor_sync(0xffffffffu, kv, o);
  const float delta = (v - kv) * beta;
  float out = 0.0f;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    s[i] = fmaf(kk[i], delta, s[i]);
    out = fmaf(s[i], qq[i], out);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) out += __shfl_xor_sync(0xffffffffu, out, o);
  if (rnd) {
#pragma unroll
    for (int i = 0; i < NP; ++i) s[i] = round_to<InT>(s[i]);
  }
  return out;
}

// grid (Hv * Dv / rows_per_cta), block rows_per_cta warps.  Lane l of a warp
// holds state elements l*NP .. l*NP+NP-1 of its row (the reference's
// n_per_t split).  Shared memory: q/k of the head for every node (f32),
// v / g / beta per node and row, and the rounded node states (InT).
template <typename InT, typename StT, int DK>
__global__ void tree_gated_delta_kernel(DeltaParams p) {
  constexpr int NP = DK / 32;
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int T = p.n_nodes;
  const int R = p.rows_per_cta;
  float* s_q = reinterpret_cast<float*>(smem_raw);           // [T][DK]
  float* s_k = s_q + T * DK;                                  // [T][DK]
  float* s_g = s_k + T * DK;                                  // [T]
  float* s_b = s_g + T;                                       // [T]
  float* s_v = s_b + T;                                       // [T][R]
  InT* s_state = reinterpret_cast<InT*>(s_v + T * R);         // [R][T][DK]

  const int rows_per_head = p.dv / R;
  const int hv = blockIdx.x / rows_per_head;
  const int dv0 = (blockIdx.x % rows_per_head) * R;
  const int hk = hv / (p.n_v_heads / p.n_k_heads);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dv = dv0 + warp;
  pdl_wait();

  const InT* q = static_cast<const InT*>(p.q);
  const InT* k = static_cast<const InT*>(p.k);
  const InT* v = static_cast<const InT*>(p.v);
  for (int e = threadIdx.x; e < T * DK; e += blockDim.x) {
    const int t = e / DK, d = e % DK;
    s_q[e] = ld_f(q + static_cast<size_t>(t) * p.ldqk + hk * DK + d);
    s_k[e] = ld_f(k + static_cast<size_t>(t) * p.ldqk + hk * DK + d);
  }
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    float g, beta;
    node_gates<InT>(p, t, hv, g, beta);
    s_g[t] = g;
    s_b[t] = beta;
  }
  for (int e = threadIdx.x; e < T * R; e += blockDim.x) {
    const int t = e / R, r = e % R;
    s_v[e] = ld_f(v + static_cast<size_t>(t) * p.ldv + hv * p.dv + dv0 + r);
  }
  __syncthreads();

  const StT* st_in = static_cast<const StT*>(p.state_in) + (static_cast<size_t>(hv) * p.dv + dv) * DK;
  float base[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) base[i] = ld_f(st_in + lane * NP + i);
  InT* my_states = s_state + static_cast<size_t>(warp) * T * DK;
  InT* y = static_cast<InT*>(p.y);
  StT* ns = static_cast<StT*>(p.node_states);

  float s[NP];
  for (int t = 0; t < T; ++t) {
    int par = p.parents[t];
    if (par >= t || (p.no_round && par != t - 1)) {  // malformed tree / prefill needs a chain
      dev_error(0x2004u);
      par = -1;
    }
    if (par < 0) {
#pragma unroll
      for (int i = 0; i < NP; ++i) s[i] = base[i];
    } else if (par != t - 1) {
#pragma unroll
      for (int i = 0; i < NP; ++i) s[i] = ld_f(my_states + static_cast<size_t>(par) * DK + lane * NP + i);
    }  // par == t - 1: the previous node's state is still in registers
    float kk[NP], qq[NP];
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      kk[i] = s_k[t * DK + lane * NP + i];
      qq[i] = s_q[t * DK + lane * NP + i];
    }
    const float out = delta_step<InT, NP>(s, kk, qq, s_v[t * R + warp], s_g[t], s_b[t], !p.no_round);
    if (lane == 0) st_f(y + static_cast<size_t>(t) * p.ldy + hv * p.dv + dv, out);
#pragma unroll
    for (int i = 0; i < NP; ++i) st_f(my_states + static_cast<size_t>(t) * DK + lane * NP + i, s[i]);
    if (ns) {
#pragma unroll
      for (int i = 0; i < NP; ++i)
        st_f(ns + ((static_cast<size_t>(t) * p.n_v_heads + hv) * p.dv + dv) * DK + lane * NP + i, s[i]);
    }
    __syncwarp();
  }
  if (p.final_state) {
    StT* fs = static_cast<StT*>(p.final_state) + (static_cast<size_t>(hv) * p.dv + dv) * DK;
#pragma unroll
    for (int i = 0; i < NP; ++i) st_f(fs + lane * NP + i, s[i]);
  }
}

// Prompt (sequence) recurrence: rows 0..n_nodes-1 form one chain from
// state_in, the state stays in f32 registers from the first row to the last
// (mlx-lm's sequence kernel; no per-row rounding) and is written to
// final_state.  One warp per state row (hv, dv), Dk/32 elements per lane,
// every warp independent (no shared memory, no block barrier); each row's
// q / k / v / a / b are loaded kPf rows ahead into registers.  Per row
//   S' = S g;  kv = S' k;  delta = (v - kv) beta;  S'' = S' + k delta;
//   y = S'' q = g (S q) + delta (k q)
// so the two reductions of a row (S k and S q of the incoming state, plus
// the state-free k q) run side by side instead of one after the other.
constexpr int kSeqPf = 4;

template <typename InT, typename StT, int DK>
__global__ void __launch_bounds__(256) gated_delta_seq_kernel(DeltaParams p) {
  constexpr int NP = DK / 32;
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const bool live = row < p.n_v_heads * p.dv;
  const int hv = live ? row / p.dv : 0, dv = live ? row % p.dv : 0;
  const int hk = hv / (p.n_v_heads / p.n_k_heads);
  pdl_wait();
  if (!live) return;  // (whole warps)
  const InT* q = static_cast<const InT*>(p.q) + hk * DK + lane * NP;
  const InT* k = static_cast<const InT*>(p.k) + hk * DK + lane * NP;
  const InT* v = static_cast<const InT*>(p.v) + hv * p.dv + dv;
  const InT* a = static_cast<const InT*>(p.a) + hv;
  const InT* b = static_cast<const InT*>(p.b) + hv;
  const float dt_b = ld_f(static_cast<const InT*>(p.dt_bias) + hv);
  const float ea = expf(p.a_log[hv]);
  const StT* st_in = static_cast<const StT*>(p.state_in) + (static_cast<size_t>(hv) * p.dv + dv) * DK + lane * NP;
  float s[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) s[i] = ld_f(st_in + i);
  InT* y = static_cast<InT*>(p.y) + hv * p.dv + dv;
  const int T = p.n_nodes;
  // register ring of the next kPf rows' inputs
  InT rq[kSeqPf][NP], rk[kSeqPf][NP];
  float rv[kSeqPf], ra[kSeqPf], rb[kSeqPf];
  auto fetch = [&](int j, int t) {
    if (t < T) {
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        rq[j][i] = q[static_cast<size_t>(t) * p.ldqk + i];
        rk[j][i] = k[static_cast<size_t>(t) * p.ldqk + i];
      }
      rv[j] = ld_f(v + static_cast<size_t>(t) * p.ldv);
      ra[j] = ld_f(a + static_cast<size_t>(t) * p.ldab);
      rb[j] = ld_f(b + static_cast<size_t>(t) * p.ldab);
    }
  };
#pragma unroll
  for (int j = 0; j < kSeqPf; ++j) fetch(j, j);
  for (int t0 = 0; t0 < T; t0 += kSeqPf) {
#pragma unroll
    for (int j = 0; j < kSeqPf; ++j) {
      const int t = t0 + j;
      if (t >= T) break;
      float kk[NP], qq[NP];
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        kk[i] = ld_f(&rk[j][i]);
        qq[i] = ld_f(&rq[j][i]);
      }
      const float vv = rv[j];
      // gates (node_gates with a, b): g = exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b)
      const float x = round_to<InT>(ra[j] + dt_b);
      const float sp = round_to<InT>(x > 20.0f ? x : log1pf(expf(x)));
      const float g = expf(-ea * sp);
      const float beta = round_to<InT>(1.0f / (1.0f + expf(-rb[j])));
      fetch(j, t + kSeqPf);
      float sk = 0.0f, sq = 0.0f, kq = 0.0f;
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        sk = fmaf(s[i], kk[i], sk);
        sq = fmaf(s[i], qq[i], sq);
        kq = fmaf(kk[i], qq[i], kq);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        kq += __shfl_xor_sync(0xffffffffu, kq, o);
      }
      const float delta = (vv - g * sk) * beta;
#pragma unroll
      for (int i = 0; i < NP; ++i) s[i] = fmaf(kk[i], delta, s[i] * g);
      if (lane == 0) st_f(y + static_cast<size_t>(t) * p.ldy, fmaf(g, sq, delta * kq));
    }
  }
  StT* fs = static_cast<StT*>(p.final_state) + (static_cast<size_t>(hv) * p.dv + dv) * DK + lane * NP;
#pragma unroll
  for (int i = 0; i < NP; ++i) st_f(fs + i, s[i]);
}

// Commit: advance each layer's recurrent state along the accepted path with
// the tree kernel's per-node arithmetic.  grid (Hv*Dv/4, layers), 4 warps.
template <typename InT, typename StT, int DK>
__global__ void gated_delta_replay_kernel(DeltaParams p) {
  constexpr int NP = DK / 32;
  pdl_trigger();
  const int layer = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_per_head = p.dv / 4;
  const int hv = blockIdx.x / rows_per_head;
  const int dv = (blockIdx.x % rows_per_head) * 4 + warp;
  const int hk = hv / (p.n_v_heads / p.n_k_heads);
  pdl_wait();
  const int n = p.st->n_accepted;
  if (n <= 0) return;
  DeltaParams L = p;
  L.q = static_cast<const InT*>(p.q) + layer * p.layer_stride_qk;
  L.k = static_cast<const InT*>(p.k) + layer * p.layer_stride_qk;
  L.a = p.a ? static_cast<const InT*>(p.a) + layer * p.layer_stride_ab : nullptr;
  L.b = p.b ? static_cast<const InT*>(p.b) + layer * p.layer_stride_ab : nullptr;
  L.a_log = p.a_log ? p.a_log + layer * p.layer_stride_params : nullptr;
  L.dt_bias = p.dt_bias ? static_cast<const InT*>(p.dt_bias) + layer * p.layer_stride_params : nullptr;
  const InT* q = static_cast<const InT*>(L.q);
  const InT* k = static_cast<const InT*>(L.k);
  const InT* v = static_cast<const InT*>(p.v) + layer * p.layer_stride_v;
  StT* state = static_cast<StT*>(p.state_out) + layer * p.layer_stride_state +
               (static_cast<size_t>(hv) * p.dv + dv) * DK;
  float s[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) s[i] = ld_f(state + lane * NP + i);
  for (int j = 0; j < n; ++j) {
    const int t = p.path[j];
    if (t < 0 || t >= p.n_nodes) {
      dev_error(0x2003u);
      return;
    }
    float kk[NP], qq[NP];
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      kk[i] = ld_f(k + static_cast<size_t>(t) * p.ldqk + hk * DK + lane * NP + i);
      qq[i] = ld_f(q + static_cast<size_t>(t) * p.ldqk + hk * DK + lane * NP + i);
    }
    float g, beta;
    node_gates<InT>(L, t, hv, g, beta);
    const float vv = ld_f(v + static_cast<size_t>(t) * p.ldv + hv * p.dv + dv);
    delta_step<InT, NP>(s, kk, qq, vv, g, beta);
  }
#pragma unroll
  for (int i = 0; i < NP; ++i) st_f(state + lane * NP + i, s[i]);
}

// Conv-state commit: base[k][c] <- window row k of the deepest accepted node
// (grid (ceil(conv_dim/256), layers), 256 threads).  The window is read from
// the layer's pre-conv inputs before any base row is overwritten.
// fixed_node >= 0 takes that node instead of the accepted path (the last
// node of a prefill chain).
template <typename InT>
__global__ void conv_state_commit_kernel(ConvParams p, const int32_t* path, const dtree_step_state* st,
                                         size_t layer_stride_x, size_t layer_stride_base, int fixed_node) {
  pdl_trigger();
  const int layer = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();
  const int n = fixed_node >= 0 ? 1 : st->n_accepted;
  if (n <= 0 || c >= p.conv_dim) return;
  const int d = fixed_node >= 0 ? fixed_node : path[n - 1];
  if (d < 0 || d >= p.n_nodes) {
    dev_error(0x2003u);
    return;
  }
  ConvParams L = p;
  L.x = static_cast<const InT*>(p.x) + layer * layer_stride_x;
  L.base = static_cast<const InT*>(p.base) + layer * layer_stride_base;
  float win[kMaxKeep + 1];
  conv_window<InT>(L, d, c, win);
  InT* base = const_cast<InT*>(static_cast<const InT*>(L.base));
  for (int kk = 0; kk < p.keep; ++kk) st_f(base + static_cast<size_t>(kk) * p.conv_dim + c, win[kk + 1]);
}

// ------------------------------------------------------------ gated norm
// out[t][h*D + d] = InT(rms_norm(y[t][h], w)[d]) * silu(z[t][h*D + d])
// (mlx-lm Qwen3NextRMSNormGated: rms_norm then swiglu(gate, x)), rounded to
// InT after the norm, after silu and after the product.  grid (T, H), block D.
template <typename InT>
__global__ void rmsnorm_gated_kernel(const InT* __restrict__ y, int ldy, const InT* __restrict__ z, int ldz,
                                     const InT* __restrict__ w, float eps, InT* __restrict__ out, int ldo) {
  pdl_trigger();
  __shared__ float s_red[32];
  const int t = blockIdx.x, h = blockIdx.y, d = threadIdx.x, D = blockDim.x;
  pdl_wait();
  const float x = ld_f(y + static_cast<size_t>(t) * ldy + h * D + d);
  float ss = x * x;
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((d & 31) == 0) s_red[d >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int i = 0; i < (D + 31) / 32; ++i) tot += s_red[i];
  const float n = round_to<InT>(x * rsqrtf(tot / static_cast<float>(D) + eps) * ld_f(w + d));
  const float zz = ld_f(z + static_cast<size_t>(t) * ldz + h * D + d);
  const float sz = round_to<InT>(zz / (1.0f + expf(-zz)));
  st_f(out + static_cast<size_t>(t) * ldo + h * D + d, n * sz);
}

// ------------------------------------------------------------ launchers
static size_t delta_smem(int T, int R, int dk, int in_bytes) {
  return static_cast<size_t>(2 * T * dk + 2 * T + T * R) * 4 + static_cast<size_t>(R) * T * dk * in_bytes;
}

int tree_conv1d_launch(const ConvParams& p, int dtype, int block, cudaStream_t st) {
  dim3 grid(p.n_nodes, (p.conv_dim + block - 1) / block);
  if (dtype == 0) DTREE_CUDA_RET(launch_pdl(tree_conv1d_kernel<float>, grid, dim3(block), 0, st, p));
  else DTREE_CUDA_RET(launch_pdl(tree_conv1d_kernel<__nv_bfloat16>, grid, dim3(block), 0, st, p));
  return kOk;
}

template <typename InT, typename StT>
static int delta_launch_t(DeltaParams p, int dk, cudaStream_t st) {
  const int in_bytes = static_cast<int>(sizeof(InT));
  int R = 8;
  while (R > 1 && (p.dv % R != 0 || delta_smem(p.n_nodes, R, dk, in_bytes) > 200 * 1024)) R >>= 1;
  DTREE_CHECK_ARG(delta_smem(p.n_nodes, R, dk, in_bytes) <= 200 * 1024, "gated delta: tree too large for shared memory");
  p.rows_per_cta = R;
  const int smem = static_cast<int>(delta_smem(p.n_nodes, R, dk, in_bytes));
  dim3 grid(p.n_v_heads * p.dv / R);
  auto go = [&](auto kern) -> int {
    DTREE_CUDA_RET(ensure_smem_attr(kern, smem));
    DTREE_CUDA_RET(launch_pdl(kern, grid, dim3(R * 32), static_cast<size_t>(smem), st, p));
    return kOk;
  };
  switch (dk) {
    case 32: return go(tree_gated_delta_kernel<InT, StT, 32>);
    case 64: return go(tree_gated_delta_kernel<InT, StT, 64>);
    case 128: return go(tree_gated_delta_kernel<InT, StT, 128>);
    case 256: return go(tree_gated_delta_kernel<InT, StT, 256>);
  }
  return fail(kErrInvalidArg, "head_k_dim must be 32, 64, 128 or 256");
}

int gated_delta_seq_launch(const DeltaParams& p, int dk, cudaStream_t st) {
  DTREE_CHECK_ARG(p.q && p.k && p.v && p.a && p.b && p.a_log && p.dt_bias && p.state_in && p.final_state && p.y,
                  "sequence gated delta: null pointer (gates come from a / b)");
  DTREE_CHECK_ARG(p.n_nodes > 0 && p.n_v_heads % p.n_k_heads == 0, "bad sequence gated delta shape");
  const int rows = p.n_v_heads * p.dv;
  const dim3 grid((rows + 7) / 8), block(256);
  using B = __nv_bfloat16;
  switch (dk) {
    case 64: DTREE_CUDA_RET(launch_pdl(gated_delta_seq_kernel<B, float, 64>, grid, block, 0, st, p)); return kOk;
    case 128: DTREE_CUDA_RET(launch_pdl(gated_delta_seq_kernel<B, float, 128>, grid, block, 0, st, p)); return kOk;
  }
  return fail(kErrInvalidArg, "sequence gated delta: head_k_dim must be 64 or 128");
}

int tree_gated_delta_launch(const DeltaParams& p, int dk, int dtype, int state_dtype, cudaStream_t st) {
  if (dtype == 0 && state_dtype == 0) return delta_launch_t<float, float>(p, dk, st);
  if (dtype == 1 && state_dtype == 0) return delta_launch_t<__nv_bfloat16, float>(p, dk, st);
  if (dtype == 1 && state_dtype == 1) return delta_launch_t<__nv_bfloat16, __nv_bfloat16>(p, dk, st);
  return fail(kErrInvalidArg, "unsupported dtype / state dtype combination");
}

template <typename InT, typename StT>
static int replay_launch_t(const DeltaParams& p, int dk, int layers, cudaStream_t st) {
  dim3 grid(p.n_v_heads * p.dv / 4, layers);
  switch (dk) {
    case 32: DTREE_CUDA_RET(launch_pdl(gated_delta_replay_kernel<InT, StT, 32>, grid, dim3(128), 0, st, p)); return kOk;
    case 64: DTREE_CUDA_RET(launch_pdl(gated_delta_replay_kernel<InT, StT, 64>, grid, dim3(128), 0, st, p)); return kOk;
    case 128: DTREE_CUDA_RET(launch_pdl(gated_delta_replay_kernel<InT, StT, 128>, grid, dim3(128), 0, st, p)); return kOk;
    case 256: DTREE_CUDA_RET(launch_pdl(gated_delta_replay_kernel<InT, StT, 256>, grid, dim3(128), 0, st, p)); return kOk;
  }
  return fail(kErrInvalidArg, "head_k_dim must be 32, 64, 128 or 256");
}

int gated_delta_replay_launch(const DeltaParams& p, int dk, int dtype, int state_dtype, int layers, cudaStream_t st) {
  DTREE_CHECK_ARG(p.dv % 4 == 0, "head_v_dim must be a multiple of 4");
  if (dtype == 0 && state_dtype == 0) return replay_launch_t<float, float>(p, dk, layers, st);
  if (dtype == 1 && state_dtype == 0) return replay_launch_t<__nv_bfloat16, float>(p, dk, layers, st);
  if (dtype == 1 && state_dtype == 1) return replay_launch_t<__nv_bfloat16, __nv_bfloat16>(p, dk, layers, st);
  return fail(kErrInvalidArg, "unsupported dtype / state dtype combination");
}

int conv_state_commit_launch(const ConvParams& p, int dtype, const int32_t* path, const dtree_step_state* state,
                             int layers, size_t layer_stride_x, size_t layer_stride_base, int fixed_node,
                             cudaStream_t st) {
  dim3 grid((p.conv_dim + 255) / 256, layers);
  if (dtype == 0)
    DTREE_CUDA_RET(launch_pdl(conv_state_commit_kernel<float>, grid, dim3(256), 0, st, p, path, state, layer_stride_x,
                              layer_stride_base, fixed_node));
  else
    DTREE_CUDA_RET(launch_pdl(conv_state_commit_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, p, path, state,
                              layer_stride_x, layer_stride_base, fixed_node));
  return kOk;
}

int rmsnorm_gated_launch(const __nv_bfloat16* y, int ldy, const __nv_bfloat16* z, int ldz, const __nv_bfloat16* w,
                         float eps, __nv_bfloat16* out, int ldo, int n_rows, int heads, int head_dim,
                         cudaStream_t st) {
  DTREE_CUDA_RET(launch_pdl(rmsnorm_gated_kernel<__nv_bfloat16>, dim3(n_rows, heads), dim3(head_dim), 0, st, y, ldy,
                            z, ldz, w, eps, out, ldo));
  return kOk;
}

}  // namespace dtree

using namespace dtree;

static bool valid_dtype(int d) { return d == 0 || d == 1; }

extern "C" int dtree_tree_conv1d(const void* qkv, int ld_qkv, const void* base_conv_state, const void* conv_weight,
                                 const int32_t* parents, int n_nodes, int conv_dim, int keep, int dtype,
                                 void* conv_out, void* conv_states, void* stream) {
  DTREE_CHECK_ARG(qkv && base_conv_state && conv_weight && parents && conv_out, "null pointer");
  DTREE_CHECK_ARG(n_nodes > 0 && n_nodes <= DTREE_MAX_TREE, "n_nodes must be in [1, 128]");
  DTREE_CHECK_ARG(keep >= 1 && keep <= kMaxKeep, "keep (conv kernel size - 1) must be in [1, 8]");
  DTREE_CHECK_ARG(conv_dim > 0 && ld_qkv >= conv_dim, "bad conv_dim / ld_qkv");
  DTREE_CHECK_ARG(valid_dtype(dtype), "dtype must be 0 (f32) or 1 (bf16)");
  ConvParams p{};
  p.x = qkv;
  p.ldx = ld_qkv;
  p.base = base_conv_state;
  p.weight = conv_weight;
  p.parents = parents;
  p.n_nodes = n_nodes;
  p.conv_dim = conv_dim;
  p.keep = keep;
  p.out = conv_out;
  p.ldo = conv_dim;
  p.node_states = conv_states;
  return tree_conv1d_launch(p, dtype, 128, static_cast<cudaStream_t>(stream));
}

extern "C" int dtree_tree_gated_delta(const void* q, const void* k, const void* v, const float* g, const void* beta,
                                      const void* state_in, const int32_t* parents, int n_nodes, int n_k_heads,
                                      int n_v_heads, int head_k_dim, int head_v_dim, int dtype, int state_dtype,
                                      void* y, void* node_states, void* stream) {
  DTREE_CHECK_ARG(q && k && v && g && beta && state_in && parents && y, "null pointer");
  DTREE_CHECK_ARG(n_nodes > 0 && n_nodes <= DTREE_MAX_TREE, "n_nodes must be in [1, 128]");
  DTREE_CHECK_ARG(n_k_heads > 0 && n_v_heads % n_k_heads == 0, "n_v_heads must be a multiple of n_k_heads");
  DTREE_CHECK_ARG(head_v_dim > 0, "head_v_dim must be positive");
  DTREE_CHECK_ARG(valid_dtype(dtype) && valid_dtype(state_dtype), "dtype must be 0 (f32) or 1 (bf16)");
  DeltaParams p{};
  p.q = q;
  p.k = k;
  p.ldqk = n_k_heads * head_k_dim;
  p.v = v;
  p.ldv = n_v_heads * head_v_dim;
  p.g = g;
  p.beta = beta;
  p.state_in = state_in;
  p.parents = parents;
  p.n_nodes = n_nodes;
  p.n_k_heads = n_k_heads;
  p.n_v_heads = n_v_heads;
  p.dv = head_v_dim;
  p.y = y;
  p.ldy = n_v_heads * head_v_dim;
  p.node_states = node_states;
  return tree_gated_delta_launch(p, head_k_dim, dtype, state_dtype, static_cast<cudaStream_t>(stream));
}

extern "C" int dtree_gated_delta_commit(const void* q, const void* k, const void* v, const float* g, const void* beta,
                                        const int32_t* accepted, const dtree_step_state* state, int n_nodes,
                                        int n_k_heads, int n_v_heads, int head_k_dim, int head_v_dim, int dtype,
                                        int state_dtype, void* recurrent_state, void* stream) {
  DTREE_CHECK_ARG(q && k && v && g && beta && accepted && state && recurrent_state, "null pointer");
  DTREE_CHECK_ARG(n_nodes > 0 && n_nodes <= DTREE_MAX_TREE, "n_nodes must be in [1, 128]");
  DTREE_CHECK_ARG(n_k_heads > 0 && n_v_heads % n_k_heads == 0, "n_v_heads must be a multiple of n_k_heads");
  DTREE_CHECK_ARG(valid_dtype(dtype) && valid_dtype(state_dtype), "dtype must be 0 (f32) or 1 (bf16)");
  DeltaParams p{};
  p.q = q;
  p.k = k;
  p.ldqk = n_k_heads * head_k_dim;
  p.v = v;
  p.ldv = n_v_heads * head_v_dim;
  p.g = g;
  p.beta = beta;
  p.n_nodes = n_nodes;
  p.n_k_heads = n_k_heads;
  p.n_v_heads = n_v_heads;
  p.dv = head_v_dim;
  p.path = accepted;
  p.st = state;
  p.state_out = recurrent_state;
  return gated_delta_replay_launch(p, head_k_dim, dtype, state_dtype, 1, static_cast<cudaStream_t>(stream));
}

extern "C" int dtree_conv_state_commit(const void* qkv, int ld_qkv, const int32_t* parents, const int32_t* accepted,
                                       const dtree_step_state* state, int n_nodes, int conv_dim, int keep, int dtype,
                                       void* base_conv_state, void* stream) {
  DTREE_CHECK_ARG(qkv && parents && accepted && state && base_conv_state, "null pointer");
  DTREE_CHECK_ARG(n_nodes > 0 && n_nodes <= DTREE_MAX_TREE, "n_nodes must be in [1, 128]");
  DTREE_CHECK_ARG(keep >= 1 && keep <= kMaxKeep, "keep must be in [1, 8]");
  DTREE_CHECK_ARG(valid_dtype(dtype), "dtype must be 0 (f32) or 1 (bf16)");
  ConvParams p{};
  p.x = qkv;
  p.ldx = ld_qkv;
  p.base = base_conv_state;
  p.parents = parents;
  p.n_nodes = n_nodes;
  p.conv_dim = conv_dim;
  p.keep = keep;
  return conv_state_commit_launch(p, dtype, accepted, state, 1, 0, 0, -1, static_cast<cudaStream_t>(stream));
}
