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

// 4 consecutive elements as one 8-byte (bf16) or 16-byte (float) access;
// the address must be aligned to that size
template <typename T>
__device__ __forceinline__ void ld4_f(const T* p, float (&v)[4]) {
  if constexpr (std::is_same<T, float>::value) {
    const float4 x = *reinterpret_cast<const float4*>(p);
    v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w;
  } else {
    const uint2 x = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&x.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&x.y);
    v[0] = __low2float(a), v[1] = __high2float(a), v[2] = __low2float(b), v[3] = __high2float(b);
  }
}
template <typename T>
__device__ __forceinline__ void st4_f(T* p, const float (&v)[4]) {
  if constexpr (std::is_same<T, float>::value) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 x;
    x.x = *reinterpret_cast<const uint32_t*>(&a);
    x.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = x;
  }
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

// Prompt rows as one chain (row t's predecessors t-1, t-2, .. then the base
// window: position j < 0 is base row keep + j): block = kConvSeqRows rows x
// one channel block (one head with head normalization); each thread slides
// its channel's window through the rows in registers, one load per row.
// Same arithmetic, order and rounding as tree_conv1d_kernel.
constexpr int kConvSeqRows = 16;

// KEEP > 0: the window length at compile time (registers); 0: keep
template <typename InT, int KEEP>
__global__ void conv1d_seq_kernel(ConvParams p) {
  const int keep = KEEP > 0 ? KEEP : p.keep;
  pdl_trigger();
  __shared__ float s_red[32];
  const int t0 = blockIdx.x * kConvSeqRows;
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  const int head = blockIdx.y;
  const bool ok = c < p.conv_dim;
  const InT* x = static_cast<const InT*>(p.x);
  const InT* base = static_cast<const InT*>(p.base);
  const InT* w = static_cast<const InT*>(p.weight);
  float wk[kMaxKeep + 1];
#pragma unroll
  for (int k = 0; k <= keep; ++k) wk[k] = ok ? ld_f(w + static_cast<size_t>(k) * p.conv_dim + c) : 0.0f;
  pdl_wait();
  // win[k] = the input at position t - keep + k, k < keep
  float win[kMaxKeep];
#pragma unroll
  for (int k = 0; k < keep; ++k) {
    const int j = t0 - keep + k;
    win[k] = !ok ? 0.0f
                 : (j >= 0 ? ld_f(x + static_cast<size_t>(j) * p.ldx + c)
                           : ld_f(base + static_cast<size_t>(keep + j) * p.conv_dim + c));
  }
  const int t1 = min(t0 + kConvSeqRows, p.n_nodes);
  // the block's rows of this channel, all loads in flight at once
  float xs[kConvSeqRows];
#pragma unroll
  for (int i = 0; i < kConvSeqRows; ++i)
    xs[i] = (ok && t0 + i < t1) ? ld_f(x + static_cast<size_t>(t0 + i) * p.ldx + c) : 0.0f;
#pragma unroll
  for (int i = 0; i < kConvSeqRows; ++i) {
    const int t = t0 + i;
    if (t >= t1) break;  // (uniform per block)
    const float xt = xs[i];
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < keep; ++k) acc = fmaf(win[k], wk[k], acc);
    acc = fmaf(xt, wk[keep], acc);
#pragma unroll
    for (int k = 0; k + 1 < keep; ++k) win[k] = win[k + 1];
    win[keep - 1] = xt;
    float y = round_to<InT>(acc / (1.0f + expf(-acc)));
    if (head < p.n_norm_heads) {
      const int D = blockDim.x;
      float ss = y * y;
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
      __syncthreads();
      float tot = 0.0f;
      for (int i = 0; i < (D + 31) / 32; ++i) tot += s_red[i];
      __syncthreads();  // s_red is rewritten by the next row
      const float r = round_to<InT>(y * rsqrtf(tot / static_cast<float>(D) + 1e-6f));
      const float scale = head < p.n_q_heads ? 1.0f / static_cast<float>(D) : rsqrtf(static_cast<float>(D));
      y = round_to<InT>(r * scale);
    }
    if (ok) st_f(static_cast<InT*>(p.out) + static_cast<size_t>(t) * p.ldo + c, y);
  }
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

// One node of the recurrence on a state row held as NP floats per lane:
//   S' = S g;  kv = S' k;  delta = (v - kv) beta;  S'' = S' + k delta;
//   y = S'' q = g (S q) + delta (k q)
// The three reductions (S k, S q, k q) of the incoming state run side by
// side, one butterfly deep instead of two after each other.  The tree
// kernel and the commit replay share this step, so a replayed node state
// equals the tree kernel's bit for bit.
// k·q of a node: the same per-lane chain and butterfly as delta_step's, so
// a value computed once per node (the tree kernel) equals the one each
// row's step would reduce (the replay) bit for bit
template <int NP>
__device__ __forceinline__ float node_kq(const float (&kk)[NP], const float (&qq)[NP]) {
  float kq = 0.0f;
#pragma unroll
  for (int i = 0; i < NP; ++i) kq = fmaf(kk[i], qq[i], kq);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) kq += __shfl_xor_sync(0xffffffffu, kq, o);
  return kq;
}
// the step given k·q: S k and S q reduced side by side, the update (the
// state left unrounded: the caller rounds)
template <int NP>
__device__ __forceinline__ float delta_update(float (&s)[NP], const float (&kk)[NP], const float (&qq)[NP], float kq,
                                              float v, float g, float beta) {
  float sk = 0.0f, sq = 0.0f;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    sk = fmaf(s[i], kk[i], sk);
    sq = fmaf(s[i], qq[i], sq);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sk += __shfl_xor_sync(0xffffffffu, sk, o);
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
  }
  const float delta = (v - g * sk) * beta;
#pragma unroll
  for (int i = 0; i < NP; ++i) s[i] = fmaf(kk[i], delta, s[i] * g);
  return fmaf(g, sq, delta * kq);
}
template <typename InT, int NP>
__device__ __forceinline__ float delta_step(float (&s)[NP], const float (&kk)[NP], const float (&qq)[NP], float v,
                                            float g, float beta, bool rnd = true) {
  const float kq = node_kq(kk, qq);
  const float out = delta_update(s, kk, qq, kq, v, g, beta);
  if (rnd) {
#pragma unroll
    for (int i = 0; i < NP; ++i) s[i] = round_to<InT>(s[i]);
  }
  return out;
}

// grid (Hv * Dv / rows_per_cta), block rows_per_cta warps.  Lane l of a warp
// holds state elements l*NP .. l*NP+NP-1 of its row (the reference's
// n_per_t split).  Shared memory: q/k of the head for every node (InT, as
// they arrive), v / g / beta per node and row, and the rounded states of
// nodes 0 .. T-2 (InT; a node's state is reloaded only by a child that is
// not the next node, and the last node has none).  At 25 nodes 16 rows per
// CTA take 110 KB, so two CTAs share an SM and the verify's 256 CTAs run in
// one wave.
template <typename InT, typename StT, int DK>
__global__ void tree_gated_delta_kernel(DeltaParams p) {
  constexpr int NP = DK / 32;
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int T = p.n_nodes;
  const int R = p.rows_per_cta;
  InT* s_q = reinterpret_cast<InT*>(smem_raw);               // [T][DK]
  InT* s_k = s_q + T * DK;                                    // [T][DK]
  float* s_g = reinterpret_cast<float*>(s_k + T * DK);        // [T]
  float* s_b = s_g + T;                                       // [T]
  float* s_v = s_b + T;                                       // [T][R]
  float* s_kq = s_v + T * R;                                  // [T]: k·q per node
  int* s_par = reinterpret_cast<int*>(s_kq + T);              // [T]: validated parents
  // [R][T - 1][DK], 16-byte aligned for the 4-element accesses
  InT* s_state = reinterpret_cast<InT*>((reinterpret_cast<uintptr_t>(s_par + T) + 15) & ~static_cast<uintptr_t>(15));

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
  // q / k of the head for every node: 16-byte copies (all issued before the
  // first lands) when the rows allow, else element by element
  constexpr int VE = 16 / static_cast<int>(sizeof(InT));  // elements per 16 bytes
  const bool vec = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k)) & 15) == 0 &&
                   (static_cast<size_t>(p.ldqk) * sizeof(InT)) % 16 == 0;
  if (vec) {
    constexpr int kPer = 4;  // 16-byte chunks in flight per thread and matrix
    for (int e0 = threadIdx.x * kPer; e0 < T * DK / VE; e0 += blockDim.x * kPer) {
      uint4 aq[kPer], ak[kPer];
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int e = e0 + j;
        if (e < T * DK / VE) {
          const int t = e / (DK / VE), c = e % (DK / VE);
          const size_t off = static_cast<size_t>(t) * p.ldqk + hk * DK + c * VE;
          aq[j] = *reinterpret_cast<const uint4*>(q + off);
          ak[j] = *reinterpret_cast<const uint4*>(k + off);
        }
      }
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int e = e0 + j;
        if (e < T * DK / VE) {
          reinterpret_cast<uint4*>(s_q)[e] = aq[j];
          reinterpret_cast<uint4*>(s_k)[e] = ak[j];
        }
      }
    }
  } else {
    for (int e = threadIdx.x; e < T * DK; e += blockDim.x) {
      const int t = e / DK, d = e % DK;
      s_q[e] = q[static_cast<size_t>(t) * p.ldqk + hk * DK + d];
      s_k[e] = k[static_cast<size_t>(t) * p.ldqk + hk * DK + d];
    }
  }
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    float g, beta;
    node_gates<InT>(p, t, hv, g, beta);
    s_g[t] = g;
    s_b[t] = beta;
    int par = p.parents[t];
    if (par >= t || (p.no_round && par != t - 1)) {  // malformed tree / prefill needs a chain
      dev_error(0x2004u);
      par = -1;
    }
    s_par[t] = par;
  }
  for (int e = threadIdx.x; e < T * R; e += blockDim.x) {
    const int t = e / R, r = e % R;
    s_v[e] = ld_f(v + static_cast<size_t>(t) * p.ldv + hv * p.dv + dv0 + r);
  }
  __syncthreads();
  // k·q of every node once per CTA (the same chain and butterfly as each
  // row's step would run): warp w takes nodes w, w + warps, ...
  for (int t = warp; t < T; t += static_cast<int>(blockDim.x >> 5)) {
    float kk[NP], qq[NP];
    if constexpr (NP == 4) {
      ld4_f(s_k + t * DK + lane * NP, kk);
      ld4_f(s_q + t * DK + lane * NP, qq);
    } else {
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        kk[i] = ld_f(s_k + t * DK + lane * NP + i);
        qq[i] = ld_f(s_q + t * DK + lane * NP + i);
      }
    }
    const float kq = node_kq(kk, qq);
    if (lane == 0) s_kq[t] = kq;
  }
  __syncthreads();

  const StT* st_in = static_cast<const StT*>(p.state_in) + (static_cast<size_t>(hv) * p.dv + dv) * DK;
  float base[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) base[i] = ld_f(st_in + lane * NP + i);
  // node states a later node may branch from (the last node has no child)
  InT* my_states = s_state + static_cast<size_t>(warp) * (T - 1) * DK;
  InT* y = static_cast<InT*>(p.y);
  StT* ns = static_cast<StT*>(p.node_states);

  float s[NP];
  for (int t = 0; t < T; ++t) {
    const int par = s_par[t];
    if (par < 0) {
#pragma unroll
      for (int i = 0; i < NP; ++i) s[i] = base[i];
    } else if (par != t - 1) {
      if constexpr (NP == 4) {
        ld4_f(my_states + static_cast<size_t>(par) * DK + lane * NP, s);
      } else {
#pragma unroll
        for (int i = 0; i < NP; ++i) s[i] = ld_f(my_states + static_cast<size_t>(par) * DK + lane * NP + i);
      }
    }  // par == t - 1: the previous node's state is still in registers
    float kk[NP], qq[NP];
    if constexpr (NP == 4) {
      ld4_f(s_k + t * DK + lane * NP, kk);
      ld4_f(s_q + t * DK + lane * NP, qq);
    } else {
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        kk[i] = ld_f(s_k + t * DK + lane * NP + i);
        qq[i] = ld_f(s_q + t * DK + lane * NP + i);
      }
    }
    const float out = delta_update(s, kk, qq, s_kq[t], s_v[t * R + warp], s_g[t], s_b[t]);
    if (lane == 0) st_f(y + static_cast<size_t>(t) * p.ldy + hv * p.dv + dv, out);
    InT* row = my_states + static_cast<size_t>(t) * DK + lane * NP;
    if constexpr (std::is_same<InT, __nv_bfloat16>::value && NP == 4) {
      // round to bf16 once: the packed pairs are the stored row and, read
      // back, the state the children continue from (delta_step's rounding)
      const __nv_bfloat162 a = __floats2bfloat162_rn(s[0], s[1]), b = __floats2bfloat162_rn(s[2], s[3]);
      if (!p.no_round) s[0] = __low2float(a), s[1] = __high2float(a), s[2] = __low2float(b), s[3] = __high2float(b);
      if (t < T - 1)
        *reinterpret_cast<uint2*>(row) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
    } else {
      if (!p.no_round) {
#pragma unroll
        for (int i = 0; i < NP; ++i) s[i] = round_to<InT>(s[i]);
      }
      if (t < T - 1) {
        if constexpr (NP == 4) {
          st4_f(row, s);
        } else {
#pragma unroll
          for (int i = 0; i < NP; ++i) st_f(row + i, s[i]);
        }
      }
    }
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
// final_state.  CTA = kSeqWarps warps x 2 state rows = 16 consecutive state
// rows of one value head (they share the head's q / k); a half-warp holds a
// state row, Dk/16 elements per lane.  The rows' inputs arrive in blocks of
// kSeqRows in shared memory by cp.async, double buffered (block b + 2 is
// fetched while block b + 1 lands and block b is computed): per row the
// head's q and k (Dk bf16 each), the CTA's 16 v values and the a / b gate
// inputs, from which the rows' gates are computed once per CTA.  Per row
//   S' = S g;  kv = S' k;  delta = (v - kv) beta;  S'' = S' + k delta;
//   y = S'' q = g (S q) + delta (k q)
// so the three reductions (S k, S q, k q) run side by side.
constexpr int kSeqWarps = 8;
constexpr int kSeqCtaRows = 2 * kSeqWarps;  // state rows per CTA
constexpr int kSeqRows = 32;                // prompt rows per staged block

__device__ __forceinline__ void seq_cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void seq_cp4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

template <int DK>
struct SeqBuf {
  __nv_bfloat16 q[kSeqRows][DK];
  __nv_bfloat16 k[kSeqRows][DK];
  __nv_bfloat16 v[kSeqRows][kSeqCtaRows];
  uint32_t a[kSeqRows];  // the bf16 pair holding this head's a (hv & ~1, hv | 1)
  uint32_t b[kSeqRows];
  float g[kSeqRows];     // the rows' gates, computed once per CTA from a / b
  float beta[kSeqRows];
};

template <int DK>
__global__ void __launch_bounds__(kSeqWarps * 32) gated_delta_seq_kernel(DeltaParams p) {
  constexpr int NP = DK / 16;
  static_assert(NP == 4 || NP == 8, "sequence gated delta: head_k_dim 64 or 128");
  pdl_trigger();
  __shared__ __align__(16) SeqBuf<DK> buf[2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane >> 4, l16 = lane & 15;  // state row of the half-warp, lane within it
  const int rows_per_head = p.dv / kSeqCtaRows;
  const int hv = blockIdx.x / rows_per_head;
  const int dv0 = (blockIdx.x % rows_per_head) * kSeqCtaRows;
  const int rl = warp * 2 + sub;  // state row within the CTA
  const int dv = dv0 + rl;
  const int hk = hv / (p.n_v_heads / p.n_k_heads);
  const int T = p.n_nodes;
  const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(p.q) + hk * DK;
  const __nv_bfloat16* k = static_cast<const __nv_bfloat16*>(p.k) + hk * DK;
  const __nv_bfloat16* v = static_cast<const __nv_bfloat16*>(p.v) + hv * p.dv + dv0;
  const __nv_bfloat16* a = static_cast<const __nv_bfloat16*>(p.a) + (hv & ~1);
  const __nv_bfloat16* b = static_cast<const __nv_bfloat16*>(p.b) + (hv & ~1);
  const float dt_b = __bfloat162float(static_cast<const __nv_bfloat16*>(p.dt_bias)[hv]);
  const float ea = expf(p.a_log[hv]);
  pdl_wait();
  // copies of row block blk into buffer blk % 2: q / k rows in 16-byte
  // chunks, then per row v (two 16-byte chunks) and the a / b pairs
  auto issue = [&](int blk) {
    SeqBuf<DK>& B = buf[blk & 1];
    const int r0 = blk * kSeqRows;
    constexpr int CPR = DK * 2 / 16;  // 16-byte chunks per q (or k) row
    for (int c = threadIdx.x; c < kSeqRows * CPR * 2; c += blockDim.x) {
      const int which = c / (kSeqRows * CPR), rem = c % (kSeqRows * CPR);
      const int r = rem / CPR, ch = rem % CPR;
      if (r0 + r < T) {
        const __nv_bfloat16* src = (which ? k : q) + static_cast<size_t>(r0 + r) * p.ldqk + ch * 8;
        seq_cp16((which ? &B.k[r][0] : &B.q[r][0]) + ch * 8, src);
      }
    }
    for (int c = threadIdx.x; c < kSeqRows * 2; c += blockDim.x) {
      const int r = c >> 1, half = c & 1;
      if (r0 + r < T) seq_cp16(&B.v[r][half * 8], v + static_cast<size_t>(r0 + r) * p.ldv + half * 8);
    }
    for (int r = threadIdx.x; r < kSeqRows; r += blockDim.x) {
      if (r0 + r < T) {
        seq_cp4(&B.a[r], a + static_cast<size_t>(r0 + r) * p.ldab);
        seq_cp4(&B.b[r], b + static_cast<size_t>(r0 + r) * p.ldab);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  const float* st_in = static_cast<const float*>(p.state_in) + (static_cast<size_t>(hv) * p.dv + dv) * DK + l16 * NP;
  float s[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) s[i] = st_in[i];
  __nv_bfloat16* y = static_cast<__nv_bfloat16*>(p.y) + hv * p.dv + dv;
  const int nblk = (T + kSeqRows - 1) / kSeqRows;
  issue(0);
  if (nblk > 1) issue(1);
  else asm volatile("cp.async.commit_group;" ::: "memory");
  const bool hi = (hv & 1) != 0;
  for (int blk = 0; blk < nblk; ++blk) {
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // block blk landed (this thread's copies)
    __syncthreads();                                       // ... and everyone's
    SeqBuf<DK>& B = buf[blk & 1];
    const int rn = min(kSeqRows, T - blk * kSeqRows);
    // the rows' gates, once per CTA (node_gates with a, b):
    // g = exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b)
    if (threadIdx.x < rn) {
      const int r = threadIdx.x;
      const __nv_bfloat162 a2 = *reinterpret_cast<const __nv_bfloat162*>(&B.a[r]);
      const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&B.b[r]);
      const float x = round_to<__nv_bfloat16>(__bfloat162float(hi ? a2.y : a2.x) + dt_b);
      const float sp = round_to<__nv_bfloat16>(x > 20.0f ? x : log1pf(expf(x)));
      B.g[r] = expf(-ea * sp);
      B.beta[r] = round_to<__nv_bfloat16>(1.0f / (1.0f + expf(-__bfloat162float(hi ? b2.y : b2.x))));
    }
    __syncthreads();
    for (int r = 0; r < rn; ++r) {
      float kk[NP], qq[NP];
#pragma unroll
      for (int c = 0; c < NP / 4; ++c) {
        const uint2 kw = *reinterpret_cast<const uint2*>(&B.k[r][l16 * NP + c * 4]);
        const uint2 qw = *reinterpret_cast<const uint2*>(&B.q[r][l16 * NP + c * 4]);
        const float2 k0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kw.x));
        const float2 k1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kw.y));
        const float2 q0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qw.x));
        const float2 q1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qw.y));
        kk[c * 4] = k0.x; kk[c * 4 + 1] = k0.y; kk[c * 4 + 2] = k1.x; kk[c * 4 + 3] = k1.y;
        qq[c * 4] = q0.x; qq[c * 4 + 1] = q0.y; qq[c * 4 + 2] = q1.x; qq[c * 4 + 3] = q1.y;
      }
      const float vv = __bfloat162float(B.v[r][rl]);
      const float g = B.g[r], beta = B.beta[r];
      float sk = 0.0f, sq = 0.0f, kq = 0.0f;
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        sk = fmaf(s[i], kk[i], sk);
        sq = fmaf(s[i], qq[i], sq);
        kq = fmaf(kk[i], qq[i], kq);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {  // within the half-warp
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        kq += __shfl_xor_sync(0xffffffffu, kq, o);
      }
      const float delta = (vv - g * sk) * beta;
#pragma unroll
      for (int i = 0; i < NP; ++i) s[i] = fmaf(kk[i], delta, s[i] * g);
      if (l16 == 0) y[static_cast<size_t>(blk * kSeqRows + r) * p.ldy] = __float2bfloat16_rn(fmaf(g, sq, delta * kq));
    }
    __syncthreads();  // buffer blk % 2 is refilled next
    if (blk + 2 < nblk) issue(blk + 2);
    else asm volatile("cp.async.commit_group;" ::: "memory");
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  float* fs = static_cast<float*>(p.final_state) + (static_cast<size_t>(hv) * p.dv + dv) * DK + l16 * NP;
#pragma unroll
  for (int i = 0; i < NP; ++i) fs[i] = s[i];
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
  const size_t qk = (static_cast<size_t>(2) * T * dk * in_bytes + 15) & ~static_cast<size_t>(15);
  return qk + static_cast<size_t>(4 * T + T * R) * 4 + 16 /* state alignment */ +
         static_cast<size_t>(R) * (T > 1 ? T - 1 : 1) * dk * in_bytes;
}

int conv1d_seq_launch(const ConvParams& p, int block, cudaStream_t st) {
  DTREE_CHECK_ARG(p.keep >= 1 && p.keep <= kMaxKeep && p.n_nodes > 0, "sequence conv: bad shape");
  DTREE_CHECK_ARG(p.n_norm_heads == 0 || block % 32 == 0, "sequence conv: head blocks of whole warps");
  dim3 grid((p.n_nodes + kConvSeqRows - 1) / kConvSeqRows, (p.conv_dim + block - 1) / block);
  if (p.keep == 3) DTREE_CUDA_RET(launch_pdl(conv1d_seq_kernel<__nv_bfloat16, 3>, grid, dim3(block), 0, st, p));
  else DTREE_CUDA_RET(launch_pdl(conv1d_seq_kernel<__nv_bfloat16, 0>, grid, dim3(block), 0, st, p));
  return kOk;
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
  int R = 16;
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
  DTREE_CHECK_ARG(p.n_nodes > 0 && p.n_v_heads % p.n_k_heads == 0 && p.dv % kSeqCtaRows == 0,
                  "sequence gated delta: bad shape (head_v_dim a multiple of 16)");
  auto al = [](const void* x, uintptr_t m) { return (reinterpret_cast<uintptr_t>(x) & (m - 1)) == 0; };
  DTREE_CHECK_ARG(al(p.q, 16) && al(p.k, 16) && al(p.v, 16) && p.ldqk % 8 == 0 && p.ldv % 8 == 0,
                  "sequence gated delta: q / k / v rows must be 16-byte aligned");
  DTREE_CHECK_ARG(al(p.a, 4) && al(p.b, 4) && p.ldab % 2 == 0, "sequence gated delta: a / b must be 4-byte aligned");
  const dim3 grid(p.n_v_heads * p.dv / kSeqCtaRows), block(kSeqWarps * 32);
  switch (dk) {
    case 64: DTREE_CUDA_RET(launch_pdl(gated_delta_seq_kernel<64>, grid, block, 0, st, p)); return kOk;
    case 128: DTREE_CUDA_RET(launch_pdl(gated_delta_seq_kernel<128>, grid, block, 0, st, p)); return kOk;
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
