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
#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <tuple>

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

// keys per split for a live key count L: at least 128, a multiple of `align`
// (64: the mma.sync kernel's chunk; 128: one tcgen05 pass)
__device__ __forceinline__ int attn_keys_per_split(int L, int splits, int align) {
  int kps = (L + splits - 1) / splits;
  if (kps < 2 * kChunk) kps = 2 * kChunk;
  return ((kps + align - 1) / align) * align;
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

  if (threadIdx.x == 0) {
    // The cache prefix [0, start) is not written by this forward: pull this
    // CTA's prefix keys into L2 while the upstream kernels finish.  `start`
    // read before the dependency wait only steers this hint (never the
    // result); the range is clamped to the cache.
    const int P0 = p.state->start;
    const int kps0 = attn_keys_per_split(P0 + T, p.splits, p.key_align);
    const int lo = split * kps0;
    const int hi = min(min(P0, lo + kps0), p.cap);
    if (lo >= 0 && hi > lo) {
      const size_t off = static_cast<size_t>(kvh) * p.cap * HD + static_cast<size_t>(lo) * HD;
      const uint32_t bytes = static_cast<uint32_t>(hi - lo) * HD * 2;
      l2_prefetch_bulk(p.k + off, bytes);
      l2_prefetch_bulk(p.v + off, bytes);
    }
  }
  pdl_wait();
  const int P = p.state->start;
  const int L = P + T;
  const int kps = attn_keys_per_split(L, p.splits, p.key_align);
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

// ------------------------------------------------------------ tcgen05 path
// head_dim 64 / 128.  One CTA = 128 query rows (row r -> query head
// kvh*G + r / n_nodes, node r % n_nodes) x the split's keys, taken 128 keys
// per pass:
//   TMA      K, V rows [kvh*cap + k0, +128) -> smem (128-byte swizzle, two
//            64-feature boxes when head_dim = 128)
//   tcgen05  S[128 x 128] = Q K^T -> TMEM columns [0, 128)
//   softmax  8 warps: warp w reads TMEM lanes 32*(w%4).. (its rows) and key
//            half w/4 of each row; row max / sum meet in shared memory;
//            P = bf16(p) -> smem (K-major, 128-byte swizzle)
//   tcgen05  O[128 x HD] (+)= P V -> TMEM columns [128, 128 + HD); V is the
//            MN-major operand straight from its TMA boxes
// Passes after the first rescale O in TMEM by exp2(m_old - m_new).  Output
// is the same (m, l, unnormalised O) split partial as the mma.sync kernel,
// merged by attn_combine_kernel.
constexpr int kTcThreads = 256;
constexpr int kTcKeys = 128;
constexpr uint32_t kTcBlock = 128 * 128;  // one [128 rows x 128 B] swizzled block

template <int HD>
struct TcCfg {
  static constexpr int kNA = HD / 64;  // 64-feature blocks
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kK = kQ + kNA * kTcBlock;
  static constexpr uint32_t kV = kK + kNA * kTcBlock;
  // P (128 rows x 128 keys = 2 blocks) reuses K's space when it is as large
  static constexpr uint32_t kP = kNA == 2 ? kK : kV + kNA * kTcBlock;
  static constexpr uint32_t kBar = (kNA == 2 ? kV + kNA * kTcBlock : kP + 2 * kTcBlock);
  static constexpr uint32_t kRed = kBar + 64;  // [2 halves][128 rows] max, then sum
  static constexpr int kSmem = 1024 + kRed + 2 * 2 * 128 * 4;
  static constexpr uint32_t kIdescS = idesc_bf16_f32(128, kTcKeys);
  static constexpr uint32_t kIdescO = idesc_bf16_f32(128, HD) | (1u << 16);  // B (V) MN-major
  static constexpr uint32_t kTmemCols = 256;
};

__device__ __forceinline__ uint32_t sw128_off(int row, int chunk16) {
  return static_cast<uint32_t>(row * 128 + ((chunk16 ^ (row & 7)) << 4));
}

// PROMPT: the prompt (prefill) instantiation, causal 128-row chunks
// (AttnParams::chunk_rows); the tree-verify one has none of its code.
// CL: the splits of one (row block, KV head) form one thread-block cluster
// (cluster size = gridDim.x = splits <= 8) and merge their partials through
// distributed shared memory instead of the global workspace and
// attn_combine_kernel: each CTA stages its unnormalised O and (m, l) in its
// own shared memory, and after a cluster barrier CTA c merges rows
// c, c + splits, ... of the block with the combine kernel's arithmetic in the
// same order (bit-identical output).  Any prefix is covered (keys per split
// grow with it); the launch pays off while 8 x 128 keys cover the prefix and
// the tree (one pass per CTA, 8 CTAs per KV head instead of ~18).
template <int HD, bool PROMPT = false, bool CL = false>
__global__ void __launch_bounds__(kTcThreads) tree_attn_tc_kernel(const __grid_constant__ CUtensorMap tmap_k,
                                                                   const __grid_constant__ CUtensorMap tmap_v,
                                                                   AttnParams p) {
  using C = TcCfg<HD>;
  constexpr int NA = C::kNA;
  constexpr int KH = kTcKeys / 2;  // keys per thread and pass
  constexpr int OH = HD / 2;       // O columns per thread
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = sm + C::kQ;
  uint8_t* sk = sm + C::kK;
  uint8_t* sv = sm + C::kV;
  uint8_t* sp = sm + C::kP;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + C::kBar);  // [0] K/V landed, [1] S done, [2] O done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 4);
  int* s_p0 = reinterpret_cast<int*>(tmem_slot + 1);        // `start` as read before the wait
  float* red_max = reinterpret_cast<float*>(sm + C::kRed);  // [2][128]
  float* red_sum = red_max + 2 * 128;                       // [2][128]

  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int r = (warp & 3) * 32 + lane;  // softmax / output row (TMEM lane)
  const int h = warp >> 2;               // key half (S) and column half (O)
  const int G = p.n_q_heads / p.n_kv_heads;
  // prompt mode: blockIdx.x = kv head * chunk_rbs + row block, blockIdx.y
  // counts chunks from the last (chunk c takes c + 1 passes, so the longest
  // CTAs launch first); the chunk's rows are queries row0 .. row0 + T - 1
  // at slots start + row0 ..
  constexpr bool chunked = PROMPT;
  const int split = chunked ? 0 : static_cast<int>(blockIdx.x);
  const int kvh = chunked ? static_cast<int>(blockIdx.x) / p.chunk_rbs : static_cast<int>(blockIdx.z);
  const int chunk = chunked ? static_cast<int>(gridDim.y - 1 - blockIdx.y) : 0;
  const int rb = chunked ? static_cast<int>(blockIdx.x) % p.chunk_rbs : static_cast<int>(blockIdx.y);
  const int row0 = chunk * p.chunk_rows;
  const int T = chunked ? min(p.chunk_rows, p.n_nodes - row0) : p.n_nodes;
  const int rows_kv = G * T;
  if (chunked && rb * 128 >= rows_kv) return;  // row block past a ragged last chunk (CTA-uniform)

  if (t == 0) {
    // prefix keys into L2 while the upstream kernels finish.  `start` read
    // before the dependency wait only steers this hint and the speculative
    // first K/V load below (re-read and checked after the wait)
    const int P0 = p.state->start + row0;
    *s_p0 = P0;
    const int kps0 = attn_keys_per_split(P0 + T, p.splits, p.key_align);
    const int lo = split * kps0;
    const int hi = min(min(P0, lo + kps0), p.cap);
    if (lo >= 0 && hi > lo) {
      const size_t off = static_cast<size_t>(kvh) * p.cap * HD + static_cast<size_t>(lo) * HD;
      const uint32_t bytes = static_cast<uint32_t>(hi - lo) * HD * 2;
      l2_prefetch_bulk(p.k + off, bytes);
      l2_prefetch_bulk(p.v + off, bytes);
    }
    for (int i = 0; i < 3; ++i) mbar_init(&bar[i], 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_lane = static_cast<uint32_t>((warp & 3) * 32) << 16;

  auto issue_kv = [&](int k0) {
    const uint64_t pol = l2_policy_evict_first();
    mbar_arrive_expect_tx(&bar[0], 2u * NA * kTcBlock);
    const int y = kvh * p.cap + k0;
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      tma_load_2d(sk + a * kTcBlock, &tmap_k, &bar[0], a * 64, y, pol);
      tma_load_2d(sv + a * kTcBlock, &tmap_v, &bar[0], a * 64, y, pol);
    }
  };
  // this split's first pass as implied by the early `start` (a sane one only)
  const int P0 = *s_p0;
  const bool p0_ok = P0 >= 0 && P0 + T <= p.cap;
  const int kps0 = p0_ok ? attn_keys_per_split(P0 + T, p.splits, p.key_align) : 0;
  const int k_begin0 = split * kps0;
  const bool spec = p0_ok && k_begin0 < min(P0 + T, k_begin0 + kps0);

  pdl_wait();
  // the K/V tiles (written upstream) go first; Q is loaded while `start` is
  // re-read; thread t stages half t/128 of row t%128
  if (t == 0 && spec) issue_kv(k_begin0);
  const int qr = t & 127, qh = t >> 7;
  const int qrg = rb * 128 + qr;
  const bool q_ok = qrg < rows_kv;
  uint4 qv[HD / 16];
  {
    const int qg = q_ok ? qrg / T : 0, qn = q_ok ? qrg % T : 0;
    const uint4* src =
        reinterpret_cast<const uint4*>(p.q + static_cast<size_t>(row0 + qn) * p.ldq + (kvh * G + qg) * HD) +
        qh * (HD / 16);
#pragma unroll
    for (int c = 0; c < HD / 16; ++c) qv[c] = q_ok ? __ldg(src + c) : make_uint4(0, 0, 0, 0);
  }
  const int rg = rb * 128 + r;
  const bool row_ok = rg < rows_kv;
  const int g = row_ok ? rg / T : 0, node = row_ok ? rg % T : 0;
  const uint64_t anc0 = row_ok ? p.anc[2 * node] : 0ull;
  const uint64_t anc1 = row_ok ? p.anc[2 * node + 1] : 0ull;
  const int P = p.state->start + row0;
  const int L = P + T;
  const int kps = attn_keys_per_split(L, p.splits, p.key_align);
  const int k_begin = split * kps;
  const int k_end = min(L, k_begin + kps);
  const int n_pass = k_begin < k_end ? (k_end - k_begin + kTcKeys - 1) / kTcKeys : 0;
  // `start` is the same before and after the wait unless a kernel that had
  // not completed when this one started changed it: then the speculative
  // load lands unused (phase 0 of bar[0]) and the right one follows.  Every
  // thread waits for that phase: a thread that went on to the pass-0 wait
  // (parity 1) while phase 0 is still open would return at once and zero the
  // V tail rows that the two loads in flight can still overwrite.
  uint32_t ph_kv = 0;
  if (!(spec && P == P0 && k_begin == k_begin0)) {
    if (spec) {
      ph_kv = 1;
      mbar_wait(&bar[0], 0, 0x35);
    }
    if (t == 0 && n_pass > 0) issue_kv(k_begin);
  }
  if (n_pass > 0) {
#pragma unroll
    for (int c = 0; c < HD / 16; ++c) {
      const int cc = qh * (HD / 16) + c;  // 16-byte chunk of the row
      *reinterpret_cast<uint4*>(sq + (cc >> 3) * kTcBlock + sw128_off(qr, cc & 7)) = qv[c];
    }
    fence_proxy_async_smem();
  }

  float m_run = -INFINITY, l_run = 0.0f;
  bool ok = true;
  int fail_bar = 0;
  uint32_t ph = 0;
  for (int j = 0; j < n_pass && ok; ++j, ph ^= 1u, ph_kv ^= 1u) {
    const int k0 = k_begin + j * kTcKeys;
    if (t == 0 && j > 0) issue_kv(k0);
    ok = mbar_wait(&bar[0], ph_kv, 0x31);
    // V rows past the live keys may hold anything (NaN included): zero them so
    // that P = 0 there contributes exactly 0
    if (ok && qh < NA && k0 + qr >= k_end) {
      uint4* row = reinterpret_cast<uint4*>(sv + qh * kTcBlock + qr * 128);
#pragma unroll
      for (int c = 0; c < 8; ++c) row[c] = make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async_smem();
    // every wait's outcome is made CTA-uniform so all threads take the same path
    if (!__syncthreads_and(ok)) {
      ok = false;
      fail_bar = 0;
      break;
    }
    if (t == 0) {
      tc_fence_after();
#pragma unroll
      for (int s = 0; s < HD / 16; ++s) {
        const uint32_t off = (s >> 2) * kTcBlock + (s & 3) * 32;
        umma_bf16(tmem, sw128_kmajor_desc(smem_u32(sq) + off), sw128_kmajor_desc(smem_u32(sk) + off), C::kIdescS,
                  s > 0 ? 1u : 0u);
      }
      umma_commit(&bar[1]);
    }
    if (!__syncthreads_and(mbar_wait(&bar[1], ph, 0x32))) {
      ok = false;
      fail_bar = 1;
      break;
    }
    tc_fence_after();

    // ---- softmax: row r, keys k0 + h*64 .. +63 of this pass
    float x[KH];
#pragma unroll
    for (int c = 0; c < KH / 32; ++c) {
      uint32_t v[32];
      tmem_ld_x32(tmem + t_lane + h * KH + c * 32, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) x[c * 32 + i] = __uint_as_float(v[i]);
    }
    tmem_wait_ld();
    // visibility of keys kb + i (i < 64) as one bitmask: prefix keys, then
    // the tree slots' ancestor bits, cut at the split's end
    const int kb = k0 + h * KH;
    uint64_t vis = 0ull;
    if (row_ok) {
      const int np = P - kb;  // prefix keys among the 64
      const uint64_t pre = np >= 64 ? ~0ull : (np <= 0 ? 0ull : (1ull << np) - 1ull);
      uint64_t tree = 0ull;
      if (np < 64) {
        const int sh = -np;  // tree slot of key kb (negative: slot 0 sits at bit np)
        if (sh >= 128) tree = 0ull;
        else if (sh >= 64) tree = anc1 >> (sh - 64);
        else if (sh > 0) tree = (anc0 >> sh) | (anc1 << (64 - sh));
        else if (sh == 0) tree = anc0;
        else tree = anc0 << np;  // np in (0, 64)
      }
      const int ne = k_end - kb;  // live keys among the 64
      const uint64_t live = ne >= 64 ? ~0ull : (ne <= 0 ? 0ull : (1ull << ne) - 1ull);
      vis = (pre | (tree & ~pre)) & live;
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < KH; ++i) {
      x[i] = ((vis >> i) & 1ull) ? x[i] * p.scale_log2 : -INFINITY;
      mx = fmaxf(mx, x[i]);
    }
    red_max[h * 128 + r] = mx;
    __syncthreads();
    const float m_new = fmaxf(m_run, fmaxf(red_max[r], red_max[128 + r]));
    const float m_use = (m_new == -INFINITY) ? 0.0f : m_new;
    const float alpha = exp2f(m_run - m_use);
    float rs = 0.0f;
#pragma unroll
    for (int c = 0; c < KH / 8; ++c) {
      uint4 pk;
      uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float p0 = exp2f(x[c * 8 + 2 * i] - m_use), p1 = exp2f(x[c * 8 + 2 * i + 1] - m_use);
        rs += p0 + p1;
        pw[i] = pack_bf16(p0, p1);
      }
      *reinterpret_cast<uint4*>(sp + h * kTcBlock + sw128_off(r, c)) = pk;
    }
    red_sum[h * 128 + r] = rs;
    if (j > 0) {  // rescale this thread's half of the running O of row r
#pragma unroll 1
      for (int c = 0; c < OH / 32; ++c) {
        uint32_t v[32];
        tmem_ld_x32(tmem + t_lane + kTcKeys + h * OH + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
        tmem_st_x32(tmem + t_lane + kTcKeys + h * OH + c * 32, v);
      }
      tmem_wait_st();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    l_run = l_run * alpha + (red_sum[r] + red_sum[128 + r]);
    m_run = m_new;
    if (t == 0) {
      tc_fence_after();
#pragma unroll
      for (int s = 0; s < kTcKeys / 16; ++s) {
        const uint32_t a_off = (s >> 2) * kTcBlock + (s & 3) * 32;
        umma_bf16(tmem + kTcKeys, sw128_kmajor_desc(smem_u32(sp) + a_off),
                  sw128_mnmajor_desc(smem_u32(sv) + s * 2048, kTcBlock, 1024), C::kIdescO,
                  (j > 0 || s > 0) ? 1u : 0u);
      }
      umma_commit(&bar[2]);
    }
    ok = __syncthreads_and(mbar_wait(&bar[2], ph, 0x33)) != 0;
    if (!ok) {
      fail_bar = 2;
      break;
    }
    tc_fence_after();
  }
  if (!ok && t == 0) mbar_wait(&bar[fail_bar], fail_bar == 0 ? ph_kv : ph, 0x34);  // let the async op in flight land

  // ---- split partials (unnormalised O, m, l).  Each warp stages its 32 rows x
  // OH columns in the (now idle) Q/K/V space, then writes whole row segments.
  if (ok && n_pass > 0) {
    constexpr int LDS = OH + 4;  // padded row (floats): conflict-free 16-byte stores
    static_assert(8 * 32 * LDS * 4 <= C::kBar, "staging exceeds the operand space");
    float* stage = reinterpret_cast<float*>(sq) + warp * 32 * LDS;
#pragma unroll 1
    for (int c = 0; c < OH / 32; ++c) {
      uint32_t v[32];
      tmem_ld_x32(tmem + t_lane + kTcKeys + h * OH + c * 32, v);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 8; ++i)
        *reinterpret_cast<float4*>(stage + lane * LDS + c * 32 + 4 * i) =
            make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]), __uint_as_float(v[4 * i + 2]),
                        __uint_as_float(v[4 * i + 3]));
    }
    const int rows_total = p.n_q_heads * T;
    constexpr int VPR = OH / 4;       // float4 per staged row
    constexpr int RPI = 32 / VPR;     // rows per warp instruction
    const int sub = lane / VPR, vi = lane % VPR;
    if (chunked) {
      // O / l as bf16 straight into the output rows (one split holds every key)
      stage[lane * LDS + OH] = l_run > 0.0f ? 1.0f / l_run : 0.0f;
      __syncwarp();
#pragma unroll 4
      for (int rr = sub; rr < 32; rr += RPI) {
        const int rg2 = rb * 128 + (warp & 3) * 32 + rr;
        if (rg2 < rows_kv) {
          const float il = stage[rr * LDS + OH];
          const float4 o4 = *reinterpret_cast<const float4*>(stage + rr * LDS + vi * 4);
          uint2 pk;
          pk.x = pack_bf16(o4.x * il, o4.y * il);
          pk.y = pack_bf16(o4.z * il, o4.w * il);
          __nv_bfloat16* dst =
              p.out + static_cast<size_t>(row0 + rg2 % T) * p.ldq + (kvh * G + rg2 / T) * HD + h * OH;
          *reinterpret_cast<uint2*>(dst + vi * 4) = pk;
        }
      }
    }
    if (row_ok && h == 0 && !chunked && !CL) {
      const int qrow = (kvh * G + g) * T + node;  // [head][node]
      float* pml = p.part_ml + (static_cast<size_t>(split) * rows_total + qrow) * 2;
      pml[0] = m_run;
      pml[1] = l_run;
    }
    __syncwarp();
    if (!chunked && !CL) {
#pragma unroll 4
    for (int rr = sub; rr < 32; rr += RPI) {
      const int rg2 = rb * 128 + (warp & 3) * 32 + rr;
      if (rg2 < rows_kv) {
        const int qrow = (kvh * G + rg2 / T) * T + rg2 % T;
        float4* dst = reinterpret_cast<float4*>(p.part_o + (static_cast<size_t>(split) * rows_total + qrow) * HD + h * OH);
        dst[vi] = *reinterpret_cast<const float4*>(stage + rr * LDS + vi * 4);
      }
    }
    }
  }
  if constexpr (CL) {
    // ---- merge of the cluster's splits.  Staged O of split s, row q, column
    // d: CTA s's `stage` of warp (d / OH) * 4 + q / 32, row q % 32, column
    // d % OH; its (m, l) in red_max[q], red_sum[q] (-inf / 0: no keys)
    constexpr int LDS = OH + 4;
    float* const stage0 = reinterpret_cast<float*>(sq);
    float* const s_w = stage0 + 8 * 32 * LDS;  // [my rows][splits] weights (my rows * splits <= 128 + 7)
    float* const s_il = s_w + 136;             // [my rows] 1 / sum of weights
    static_assert((8 * 32 * LDS + 136 + 128) * 4 <= C::kBar, "merge scratch exceeds the operand space");
    const bool live = ok && n_pass > 0;
    if (h == 0) {
      red_max[r] = live ? m_run : -INFINITY;
      red_sum[r] = live ? l_run : 0.0f;
    }
    cluster_arrive();  // staged O and (m, l) of every split are published
    cluster_wait();
    const int S = p.splits;  // == cluster size <= 8
    const int active = min(S, (L + kps - 1) / kps);  // splits holding keys: 0 .. active-1
    const int rows_here = min(128, rows_kv - rb * 128);
    const int n_mine = split < rows_here ? (rows_here - split + S - 1) / S : 0;
    // weights of my rows (split, split + S, ...): warp per row, lane s =
    // split s, attn_combine_kernel's arithmetic in its order
    for (int i = warp; i < n_mine; i += kTcThreads / 32) {
      const int q = split + i * S;
      float m = -INFINITY, l = 0.0f;
      if (lane < active) {
        m = ld_dsmem_f32(red_max + q, static_cast<uint32_t>(lane));
        l = ld_dsmem_f32(red_sum + q, static_cast<uint32_t>(lane));
      }
      float M = m;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
      const float m_use = (M == -INFINITY) ? 0.0f : M;
      const float w = (lane < active) ? exp2f(m - m_use) : 0.0f;
      const float wl = w * l;
      float Ls = 0.0f;  // fixed order (split 0, 1, ...)
      for (int s2 = 0; s2 < active; ++s2) Ls += __shfl_sync(0xffffffffu, wl, s2);
      if (lane < S) s_w[i * S + lane] = w;
      if (lane == 0) s_il[i] = Ls > 0.0f ? 1.0f / Ls : 0.0f;
    }
    __syncthreads();
    // O: one 4-column group of one of my rows per thread and round, every
    // split's 16 bytes loaded before the ordered sum; O / l in bf16 to `out`
    constexpr int G4 = HD / 4;
    for (int slot = t; slot < n_mine * G4; slot += kTcThreads) {
      const int i = slot / G4, d = (slot % G4) * 4;
      const int q = split + i * S;
      const float* src = stage0 + ((d / OH) * 4 + q / 32) * 32 * LDS + (q % 32) * LDS + (d % OH);
      float4 v[8];
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2)
        v[s2] = s2 < active ? ld_dsmem_f32x4(src, static_cast<uint32_t>(s2)) : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2) {
        if (s2 < active) {
          const float w = s_w[i * S + s2];
          acc.x += w * v[s2].x;
          acc.y += w * v[s2].y;
          acc.z += w * v[s2].z;
          acc.w += w * v[s2].w;
        }
      }
      const float il = s_il[i];
      const int rg2 = rb * 128 + q;
      uint2 pk;
      pk.x = pack_bf16(acc.x * il, acc.y * il);
      pk.y = pack_bf16(acc.z * il, acc.w * il);
      *reinterpret_cast<uint2*>(p.out + static_cast<size_t>(rg2 % T) * p.ldq + (kvh * G + rg2 / T) * HD + d) = pk;
    }
    cluster_arrive();  // no CTA leaves while another reads its shared memory
    cluster_wait();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
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
  const int rows_total = p.n_q_heads * T;
  // this thread's O partials of every launched split (splits <= 32, all in
  // the workspace) and the splits' (m, l), loaded together with `start`:
  // which splits hold keys is known only from `start`, so it selects among
  // the loaded values instead of gating the loads
  float ov[32];
#pragma unroll
  for (int s = 0; s < 32; ++s)
    ov[s] = s < p.splits ? p.part_o[(static_cast<size_t>(s) * rows_total + qrow) * HD + d] : 0.0f;
  float m_ld = -INFINITY, l_ld = 0.0f;
  if (d < p.splits) {
    const size_t r = static_cast<size_t>(d) * rows_total + qrow;
    m_ld = p.part_ml[r * 2];
    l_ld = p.part_ml[r * 2 + 1];
  }
  const int P = p.state->start;
  const int L = P + T;
  const int kps = attn_keys_per_split(L, p.splits, p.key_align);
  const int active = min(p.splits, (L + kps - 1) / kps);
  if (d < 32) {
    float m = -INFINITY, l = 0.0f;
    if (d < active) {
      m = m_ld;
      l = l_ld;
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

// K / V plane tensor maps ([n_kv_heads * cap] rows x HD, boxes of 64 features
// x 128 keys), encoded once per (plane, rows, HD)
static int plane_tmap(CUtensorMap* out, const void* plane, int rows, int hd) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, int>, CUtensorMap> cache;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(plane, rows, hd);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return kOk;
  }
  if (cache.size() > 4096) cache.clear();
  CUtensorMap m;
  int rc = make_tmap_2d_bf16(&m, plane, static_cast<uint64_t>(hd), static_cast<uint64_t>(rows),
                             static_cast<uint64_t>(hd) * 2, 64, kTcKeys, true);
  if (rc) return rc;
  cache.emplace(key, m);
  *out = m;
  return kOk;
}

// How many clusters of `size` CTAs of the cluster-merge kernel can be resident
// at once (the driver's occupancy query with its shared memory; asked once per
// kernel and size, 0 on error).  Also opts the kernel into its shared memory.
template <typename K>
static int attn_cluster_capacity(K kern, int smem, int size) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> known;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(reinterpret_cast<const void*>(kern), size);
  auto it = known.find(key);
  if (it != known.end()) return it->second;
  if (ensure_smem_attr(kern, smem) != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(size, 1, 1);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(size);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  known.emplace(key, n);
  return n;
}

template <int HD>
static int attn_launch_tc(const AttnParams& p, int rb, cudaStream_t stream) {
  using C = TcCfg<HD>;
  CUtensorMap tk, tv;
  const int rows = p.n_kv_heads * p.cap;
  int rc = plane_tmap(&tk, p.k, rows, HD);
  if (rc) return rc;
  if ((rc = plane_tmap(&tv, p.v, rows, HD))) return rc;
  const int want = p.cluster_keys > 0 ? (p.cluster_keys + kTcKeys - 1) / kTcKeys : 0;
  if (p.gate == nullptr && want >= 1 && want <= 8) {
    // every split of a (row block, KV head) in one cluster, merged in
    // shared memory, when all the clusters can be resident at once (whole
    // clusters are placed within one GPC: a cluster that waits for room
    // would run as a second wave)
    auto kern = tree_attn_tc_kernel<HD, false, true>;
    if (attn_cluster_capacity(kern, C::kSmem, want) >= rb * p.n_kv_heads) {
      AttnParams pc = p;
      pc.splits = want;
      DTREE_CUDA_RET(launch_pdl_cluster(kern, dim3(want, rb, p.n_kv_heads), dim3(kTcThreads),
                                        static_cast<size_t>(C::kSmem), stream, want, tk, tv, pc));
      return kOk;
    }
  }
  auto kern = tree_attn_tc_kernel<HD>;
  DTREE_CUDA_RET(ensure_smem_attr(kern, C::kSmem));
  DTREE_CUDA_RET(launch_pdl(kern, dim3(p.splits, rb, p.n_kv_heads), dim3(kTcThreads), static_cast<size_t>(C::kSmem),
                            stream, tk, tv, p));
  DTREE_CUDA_RET(launch_pdl(attn_combine_kernel<HD>, dim3(p.n_q_heads * p.n_nodes), dim3(HD), 0, stream, p));
  return kOk;
}

int attn_prepare(int head_dim) {
  // shared-memory opt-ins and the cluster query of both tree-attention
  // shapes, outside any stream capture
  if (head_dim == 128) {
    DTREE_CUDA_RET(ensure_smem_attr(tree_attn_tc_kernel<128>, TcCfg<128>::kSmem));
    for (int c = 1; c <= 8; ++c) attn_cluster_capacity(tree_attn_tc_kernel<128, false, true>, TcCfg<128>::kSmem, c);
  } else if (head_dim == 64) {
    DTREE_CUDA_RET(ensure_smem_attr(tree_attn_tc_kernel<64>, TcCfg<64>::kSmem));
    for (int c = 1; c <= 8; ++c) attn_cluster_capacity(tree_attn_tc_kernel<64, false, true>, TcCfg<64>::kSmem, c);
  }
  return kOk;
}

int attn_prefill_launch(const AttnParams& p0, int head_dim, cudaStream_t stream) {
  AttnParams p = p0;
  DTREE_CHECK_ARG(head_dim == 64 || head_dim == 128, "prompt attention supports head_dim 64 or 128");
  DTREE_CHECK_ARG(p.n_nodes > 0 && p.n_q_heads % p.n_kv_heads == 0 && p.q && p.out && p.anc && p.state,
                  "bad prompt attention arguments");
  DTREE_CHECK_ARG(p.gate == nullptr, "prompt attention has no output gate");
  p.chunk_rows = kTcKeys;
  const int G = p.n_q_heads / p.n_kv_heads;
  p.chunk_rbs = (G * p.chunk_rows + 127) / 128;
  const int chunks = (p.n_nodes + p.chunk_rows - 1) / p.chunk_rows;
  DTREE_CHECK_ARG(chunks < 65536, "prompt too long for one launch");
  p.splits = 1;
  p.key_align = kTcKeys;
  p.part_o = nullptr;
  p.part_ml = nullptr;
  CUtensorMap tk, tv;
  const int rows = p.n_kv_heads * p.cap;
  int rc = plane_tmap(&tk, p.k, rows, head_dim);
  if (rc) return rc;
  if ((rc = plane_tmap(&tv, p.v, rows, head_dim))) return rc;
  const dim3 grid(p.n_kv_heads * p.chunk_rbs, chunks, 1);
  if (head_dim == 128) {
    DTREE_CUDA_RET(ensure_smem_attr(tree_attn_tc_kernel<128, true>, TcCfg<128>::kSmem));
    DTREE_CUDA_RET(launch_pdl(tree_attn_tc_kernel<128, true>, grid, dim3(kTcThreads),
                              static_cast<size_t>(TcCfg<128>::kSmem), stream, tk, tv, p));
  } else {
    DTREE_CUDA_RET(ensure_smem_attr(tree_attn_tc_kernel<64, true>, TcCfg<64>::kSmem));
    DTREE_CUDA_RET(launch_pdl(tree_attn_tc_kernel<64, true>, grid, dim3(kTcThreads),
                              static_cast<size_t>(TcCfg<64>::kSmem), stream, tk, tv, p));
  }
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
  if (head_dim == 256) {
    p.key_align = kChunk;
    return attn_launch_t<256, 128>(p, rb, stream);
  }
  p.key_align = kTcKeys;
  if (head_dim == 128) return attn_launch_tc<128>(p, rb, stream);
  return attn_launch_tc<64>(p, rb, stream);
}

}  // namespace dtree

using namespace dtree;

// Standalone tree attention (the attention step of qwen3_tree.py:67-76:
// softmax(q k^T * scale + tree mask) v over the cache prefix and the tree's
// own slots): q [n_nodes][ldq] bf16 (post q-norm / RoPE), K / V planes
// [n_kv_heads][kv_cap][head_dim] bf16 with the tree keys already at slots
// start..start+n_nodes-1, anc_mask [n_nodes][2]; out [n_nodes][ldq] bf16.
extern "C" size_t dtree_tree_attention_workspace_bytes(int n_q_heads, int n_nodes, int head_dim, int splits) {
  if (n_q_heads <= 0 || n_nodes <= 0 || head_dim <= 0) return 0;
  if (splits <= 0) splits = 32;
  return attn_ws_bytes(n_q_heads, n_nodes, head_dim, splits);
}

extern "C" int dtree_tree_attention(const void* q, int ldq, const void* k_plane, const void* v_plane, int kv_cap,
                                    int n_q_heads, int n_kv_heads, int head_dim, int n_nodes,
                                    const dtree_step_state* state, const uint64_t* anc_mask, void* out, int splits,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  DTREE_CHECK_ARG(q && k_plane && v_plane && state && anc_mask && out, "null pointer");
  DTREE_CHECK_ARG(n_q_heads > 0 && n_kv_heads > 0, "head counts must be positive");
  DTREE_CHECK_ARG(ldq >= n_q_heads * head_dim && ldq % 8 == 0, "ldq must be >= n_q_heads * head_dim, multiple of 8");
  DTREE_CHECK_ARG(kv_cap > 0, "kv_cap must be positive");
  AttnParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.ldq = ldq;
  p.k = static_cast<const __nv_bfloat16*>(k_plane);
  p.v = static_cast<const __nv_bfloat16*>(v_plane);
  p.cap = kv_cap;
  p.n_q_heads = n_q_heads;
  p.n_kv_heads = n_kv_heads;
  p.n_nodes = n_nodes;
  p.state = state;
  p.anc = anc_mask;
  p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(head_dim)));
  p.splits = splits > 0 ? splits : std::min(32, attn_default_splits(n_kv_heads, n_q_heads, n_nodes));
  p.cluster_keys = splits > 0 ? 0 : kv_cap;  // automatic splits: merged in a cluster when the cache is short
  p.out = static_cast<__nv_bfloat16*>(out);
  return attn_launch(p, head_dim, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

