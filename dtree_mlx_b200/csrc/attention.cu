// Tree attention: softmax(Q K^T * scale + mask) V for the tree rows of one
// verify forward, GQA (n_q_heads / n_kv_heads query heads share a K/V head).
//
// Keys are the cache prefix [0, start) (all visible) followed by the tree's
// own slots [start, start + n_nodes) written by this layer's QKV epilogue;
// tree slot j is visible to node t iff bit j of anc_mask[t] is set -- the
// bool mask of dtree_runtime.py:190-191 / qwen3_tree.py:69-76, stored as bits.
//
// Split-KV (flash-decoding): grid (splits, row_blocks, n_kv_heads); a CTA of
// 8 warps owns 128 query rows of one KV head (row r -> query head
// kvh*G + r / n_nodes, node r % n_nodes) and a contiguous key range, streams
// 64-key K/V chunks through shared memory with cp.async double buffering, and
// runs bf16 mma.sync with an fp32 online softmax.  Partial (m, l, O) go to a
// workspace; attn_combine_kernel merges the splits (log-sum-exp) into bf16.
//
// head_dim 256 (Qwen3.5 full attention): a CTA computes QK^T over all 256
// features but only one 128-wide half of V / O (grid z = kv head x half),
// which keeps the per-thread accumulators within the register file.  The
// combine optionally applies the Qwen3.5 output gate: out =
// bf16(bf16(o) * bf16(sigmoid(gate))) (qwen35_tree.py:537-538).
#include "attention.cuh"

namespace dtree {



constexpr int kAttnWarps = 8;
constexpr int kAttnRows = kAttnWarps * 16;
constexpr int kChunk = 64;

template <int HD, int HDV = HD>
struct AttnCfg {
  static constexpr int kLd = HD + 8;    // padded smem row (bank-conflict free ldmatrix)
  static constexpr int kLdV = HDV + 8;
  static constexpr int kQBytes = kAttnRows * kLd * 2;
  static constexpr int kKBytes = kChunk * kLd * 2;
  static constexpr int kVBytes = kChunk * kLdV * 2;
  static constexpr int kSmem = kQBytes + 2 * (kKBytes + kVBytes);  // Q + 2 x (K, V)
  static constexpr bool kQInRegs = HD <= 128;  // else Q fragments are re-read from smem
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const uint32_t s = smem_u32(smem);
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// keys per split for a live key count L: at least 2 chunks, multiple of kChunk
__device__ __forceinline__ int attn_keys_per_split(int L, int splits) {
  int kps = (L + splits - 1) / splits;
  if (kps < 2 * kChunk) kps = 2 * kChunk;
  return ((kps + kChunk - 1) / kChunk) * kChunk;
}

template <int HD, int HDV>
__global__ void __launch_bounds__(kAttnWarps * 32) tree_attn_kernel(AttnParams p) {
  using C = AttnCfg<HD, HDV>;
  constexpr int LD = C::kLd;
  constexpr int LDV = C::kLdV;
  constexpr int NVH = HD / HDV;  // V halves
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  uint8_t* skv = smem_raw + C::kQBytes;  // [2][K (kChunk x LD) | V (kChunk x LDV)]

  const int split = blockIdx.x, rb = blockIdx.y, kvh = blockIdx.z / NVH;
  const int v_off = (blockIdx.z % NVH) * HDV;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.n_q_heads / p.n_kv_heads;
  const int T = p.n_nodes;
  const int rows_kv = G * T;

  pdl_wait();
  const int P = p.state->start;
  const int L = P + T;
  const int kps = attn_keys_per_split(L, p.splits);
  const int k_begin = split * kps;
  if (k_begin >= L) return;  // idle split (short prefix)
  const int k_end = min(L, k_begin + kps);
  const int n_chunks = k_end > k_begin ? (k_end - k_begin + kChunk - 1) / kChunk : 0;

  // ---- stage Q rows of this block
  constexpr int VPR = HD / 8;  // 16-byte vectors per row
  for (int e = threadIdx.x; e < kAttnRows * VPR; e += blockDim.x) {
    const int r = e / VPR, v = e % VPR;
    const int rg = rb * kAttnRows + r;
    const bool ok = rg < rows_kv;
    const int g = ok ? rg / T : 0, t = ok ? rg % T : 0;
    const __nv_bfloat16* src = p.q + static_cast<size_t>(t) * p.ldq + (kvh * G + g) * HD + v * 8;
    cp_async16(sq + r * LD + v * 8, src, ok);
  }
  cp_async_commit();

  const __nv_bfloat16* kplane = p.k + static_cast<size_t>(kvh) * p.cap * HD;
  const __nv_bfloat16* vplane = p.v + static_cast<size_t>(kvh) * p.cap * HD;
  constexpr int VPRV = HDV / 8;
  auto sk_of = [&](int buf) {
    return reinterpret_cast<__nv_bfloat16*>(skv + buf * (C::kKBytes + C::kVBytes));
  };
  auto sv_of = [&](int buf) {
    return reinterpret_cast<__nv_bfloat16*>(skv + buf * (C::kKBytes + C::kVBytes) + C::kKBytes);
  };
  auto load_chunk = [&](int c, int buf) {
    const int key0 = k_begin + c * kChunk;
    __nv_bfloat16* sk = sk_of(buf);
    __nv_bfloat16* sv = sv_of(buf);
    for (int e = threadIdx.x; e < kChunk * VPR; e += blockDim.x) {
      const int r = e / VPR, v = e % VPR;
      const int key = key0 + r;
      const bool ok = key < k_end;
      const size_t off = static_cast<size_t>(ok ? key : 0) * HD + v * 8;
      cp_async16(sk + r * LD + v * 8, kplane + off, ok);
    }
    for (int e = threadIdx.x; e < kChunk * VPRV; e += blockDim.x) {
      const int r = e / VPRV, v = e % VPRV;
      const int key = key0 + r;
      const bool ok = key < k_end;
      const size_t off = static_cast<size_t>(ok ? key : 0) * HD + v_off + v * 8;
      cp_async16(sv + r * LDV + v * 8, vplane + off, ok);
    }
  };
  if (n_chunks > 0) load_chunk(0, 0);
  cp_async_commit();

  // ---- per-thread rows: lane/4 and lane/4 + 8 of this warp's 16
  int row_g[2], node[2];
  bool row_ok[2];
  uint64_t anc0[2], anc1[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    row_g[h] = rb * kAttnRows + warp * 16 + (lane >> 2) + h * 8;
    row_ok[h] = row_g[h] < rows_kv;
    node[h] = row_ok[h] ? row_g[h] % T : 0;
    anc0[h] = row_ok[h] ? p.anc[2 * node[h]] : 0ull;
    anc1[h] = row_ok[h] ? p.anc[2 * node[h] + 1] : 0ull;
  }

  cp_async_wait<1>();  // Q landed
  __syncthreads();
  auto load_qf = [&](int kk, uint32_t (&f)[4]) {
    const int mi = lane >> 3, i = lane & 7;
    const int r = warp * 16 + i + 8 * (mi & 1);
    const int col = kk * 16 + 8 * (mi >> 1);
    ldmatrix_x4(f, sq + r * LD + col);
  };
  constexpr int QF = C::kQInRegs ? HD / 16 : 1;
  uint32_t qf[QF][4];
  if constexpr (C::kQInRegs) {
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) load_qf(kk, qf[kk]);
  }

  float o[HDV / 8][4];
#pragma unroll
  for (int j = 0; j < HDV / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};

  for (int c = 0; c < n_chunks; ++c) {
    const int buf = c & 1;
    if (c + 1 < n_chunks) load_chunk(c + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const __nv_bfloat16* sk = sk_of(buf);
    const __nv_bfloat16* sv = sv_of(buf);
    const int key0 = k_begin + c * kChunk;

    // S = Q K^T  (16 rows x 64 keys per warp)
    float s[kChunk / 8][4];
#pragma unroll
    for (int nt = 0; nt < kChunk / 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
    if constexpr (C::kQInRegs) {
#pragma unroll
      for (int nt = 0; nt < kChunk / 8; ++nt) {
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk += 2) {
          uint32_t b[4];
          const int mi = lane >> 3, i = lane & 7;
          ldmatrix_x4(b, sk + (nt * 8 + i) * LD + kk * 16 + 8 * mi);
          mma_bf16_16816(s[nt], qf[kk], b[0], b[1]);
          mma_bf16_16816(s[nt], qf[kk + 1], b[2], b[3]);
        }
      }
    } else {
#pragma unroll 1
      for (int kk = 0; kk < HD / 16; kk += 2) {
        uint32_t qa[4], qb[4];
        load_qf(kk, qa);
        load_qf(kk + 1, qb);
#pragma unroll
        for (int nt = 0; nt < kChunk / 8; ++nt) {
          uint32_t b[4];
          const int mi = lane >> 3, i = lane & 7;
          ldmatrix_x4(b, sk + (nt * 8 + i) * LD + kk * 16 + 8 * mi);
          mma_bf16_16816(s[nt], qa, b[0], b[1]);
          mma_bf16_16816(s[nt], qb, b[2], b[3]);
        }
      }
    }
    // mask + online softmax (log2 domain)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < kChunk / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const int key = key0 + nt * 8 + 2 * (lane & 3) + (e & 1);
        bool vis = row_ok[h] && key < k_end;
        if (vis && key >= P) {
          const int j = key - P;
          vis = ((j < 64 ? (anc0[h] >> j) : (anc1[h] >> (j - 64))) & 1ull) != 0ull;
        }
        const float x = vis ? s[nt][e] * p.scale_log2 : -INFINITY;
        s[nt][e] = x;
        mx[h] = fmaxf(mx[h], x);
      }
    }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      const float m_new = fmaxf(m_run[h], mx[h]);
      const float m_use = (m_new == -INFINITY) ? 0.0f : m_new;
      alpha[h] = exp2f(m_run[h] - m_use);
      m_run[h] = m_new;
      mx[h] = m_use;
    }
    float rs[2] = {0.0f, 0.0f};
    uint32_t pf[kChunk / 16][4];
#pragma unroll
    for (int nt = 0; nt < kChunk / 8; ++nt) {
      const float p0 = exp2f(s[nt][0] - mx[0]), p1 = exp2f(s[nt][1] - mx[0]);
      const float p2 = exp2f(s[nt][2] - mx[1]), p3 = exp2f(s[nt][3] - mx[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      const int kt = nt >> 1, half = nt & 1;
      pf[kt][half * 2 + 0] = pack_bf16(p0, p1);
      pf[kt][half * 2 + 1] = pack_bf16(p2, p3);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
      l_run[h] = l_run[h] * alpha[h] + rs[h];
    }
#pragma unroll
    for (int j = 0; j < HDV / 8; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }
    // O += P V
#pragma unroll
    for (int kt = 0; kt < kChunk / 16; ++kt) {
      const uint32_t a[4] = {pf[kt][0], pf[kt][1], pf[kt][2], pf[kt][3]};
#pragma unroll
      for (int nt = 0; nt < HDV / 8; nt += 2) {
        uint32_t b[4];
        const int mi = lane >> 3, i = lane & 7;
        ldmatrix_x4_trans(b, sv + (kt * 16 + i + 8 * (mi & 1)) * LDV + nt * 8 + 8 * (mi >> 1));
        mma_bf16_16816(o[nt], a, b[0], b[1]);
        mma_bf16_16816(o[nt + 1], a, b[2], b[3]);
      }
    }
    __syncthreads();  // buffer `buf` is refilled by the next iteration's prefetch
  }

  // ---- write split partials
  const int rows_total = p.n_q_heads * T;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (!row_ok[h]) continue;
    const int g = row_g[h] / T, t = node[h];
    const int qrow = (kvh * G + g) * T + t;  // [head][node]
    float* po = p.part_o + (static_cast<size_t>(split) * rows_total + qrow) * HD + v_off;
#pragma unroll
    for (int j = 0; j < HDV / 8; ++j) {
      const int d = j * 8 + 2 * (lane & 3);
      *reinterpret_cast<float2*>(po + d) = make_float2(o[j][2 * h], o[j][2 * h + 1]);
    }
    if ((lane & 3) == 0 && v_off == 0) {
      float* pml = p.part_ml + (static_cast<size_t>(split) * rows_total + qrow) * 2;
      pml[0] = m_run[h];
      pml[1] = l_run[h];
    }
  }
}

// grid = n_q_heads * n_nodes rows, block = HD threads.  The per-split (m, l)
// are loaded by one thread each, the O partials with several splits in flight.
template <int HD>
__global__ void attn_combine_kernel(AttnParams p) {
  pdl_trigger();
  __shared__ float s_w[64];
  __shared__ float s_inv_l;
  const int qrow = blockIdx.x;  // head * T + t
  const int d = threadIdx.x;
  const int T = p.n_nodes;
  const int head = qrow / T, t = qrow % T;
  pdl_wait();
  const int P = p.state->start;
  const int L = P + T;
  const int kps = attn_keys_per_split(L, p.splits);
  const int active = min(p.splits, (L + kps - 1) / kps);
  const int rows_total = p.n_q_heads * T;
  // this thread's O partials of every split: loaded before the weights are
  // known so the two reads overlap (splits <= 32)
  float ov[32];
#pragma unroll
  for (int s = 0; s < 32; ++s)
    ov[s] = s < active ? p.part_o[(static_cast<size_t>(s) * rows_total + qrow) * HD + d] : 0.0f;
  if (d < 32) {
    float m = -INFINITY, l = 0.0f;
    if (d < active) {
      const size_t r = static_cast<size_t>(d) * rows_total + qrow;
      m = p.part_ml[r * 2];
      l = p.part_ml[r * 2 + 1];
    }
    float M = m;
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float m_use = (M == -INFINITY) ? 0.0f : M;
    const float w = (d < active) ? exp2f(m - m_use) : 0.0f;
    float wl = w * l;
    // fixed-order (split 0, 1, ...) sum of the weights: deterministic
    float Ls = 0.0f;
    for (int s = 0; s < active; ++s) Ls += __shfl_sync(0xffffffffu, wl, s);
    s_w[d] = w;
    if (d == 0) s_inv_l = Ls > 0.0f ? 1.0f / Ls : 0.0f;
  }
  __syncthreads();
  float acc = 0.0f;
#pragma unroll
  for (int s = 0; s < 32; ++s)
    if (s < active) acc += s_w[s] * ov[s];
  float o = acc * s_inv_l;
  if (p.gate) {
    const float gt = __bfloat162float(p.gate[static_cast<size_t>(t) * p.ldq + head * HD + d]);
    o = bf16_round(o) * bf16_round(1.0f / (1.0f + expf(-gt)));
  }
  p.out[static_cast<size_t>(t) * p.ldq + head * HD + d] = __float2bfloat16_rn(o);
}

size_t attn_ws_bytes(int n_q_heads, int t_pad, int head_dim, int splits) {
  const size_t rows = static_cast<size_t>(n_q_heads) * t_pad;
  return ((static_cast<size_t>(splits) * rows * head_dim * 4 + 255) & ~static_cast<size_t>(255)) +
         ((static_cast<size_t>(splits) * rows * 2 * 4 + 255) & ~static_cast<size_t>(255));
}

int attn_default_splits(int n_kv_heads, int n_q_heads, int n_nodes) {
  const int G = n_q_heads / n_kv_heads;
  const int rb = (G * n_nodes + kAttnRows - 1) / kAttnRows;
  int s = num_sms() / (n_kv_heads * rb);
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  return s;
}

template <int HD, int HDV>
static int attn_launch_t(const AttnParams& p, int rb, cudaStream_t stream) {
  const int smem = AttnCfg<HD, HDV>::kSmem;
  auto kern = tree_attn_kernel<HD, HDV>;
  DTREE_CUDA_RET(ensure_smem_attr(kern, smem));
  dim3 grid(p.splits, rb, p.n_kv_heads * (HD / HDV));
  DTREE_CUDA_RET(launch_pdl(kern, grid, dim3(kAttnWarps * 32), static_cast<size_t>(smem), stream, p));
  DTREE_CUDA_RET(launch_pdl(attn_combine_kernel<HD>, dim3(p.n_q_heads * p.n_nodes), dim3(HD), 0, stream, p));
  return kOk;
}

int attn_launch(const AttnParams& p0, int head_dim, void* ws, size_t ws_bytes, cudaStream_t stream) {
  AttnParams p = p0;
  DTREE_CHECK_ARG(head_dim == 64 || head_dim == 128 || head_dim == 256,
                  "tree attention supports head_dim 64, 128 or 256");
  DTREE_CHECK_ARG(p.n_nodes > 0 && p.n_nodes <= DTREE_MAX_TREE, "n_nodes out of range");
  DTREE_CHECK_ARG(p.splits >= 1 && p.splits <= 32, "attention splits must be in [1, 32]");
  DTREE_CHECK_ARG(p.n_q_heads % p.n_kv_heads == 0, "n_q_heads must be a multiple of n_kv_heads");
  const size_t need = attn_ws_bytes(p.n_q_heads, p.n_nodes, head_dim, p.splits);
  DTREE_CHECK_ARG(ws && ws_bytes >= need, "attention workspace too small");
  const size_t rows = static_cast<size_t>(p.n_q_heads) * p.n_nodes;
  p.part_o = static_cast<float*>(ws);
  p.part_ml = reinterpret_cast<float*>(static_cast<char*>(ws) +
                                       ((static_cast<size_t>(p.splits) * rows * head_dim * 4 + 255) & ~static_cast<size_t>(255)));
  const int G = p.n_q_heads / p.n_kv_heads;
  const int rb = (G * p.n_nodes + kAttnRows - 1) / kAttnRows;
  if (head_dim == 256) return attn_launch_t<256, 128>(p, rb, stream);
  if (head_dim == 128) return attn_launch_t<128, 128>(p, rb, stream);
  return attn_launch_t<64, 64>(p, rb, stream);
}

}  // namespace dtree
