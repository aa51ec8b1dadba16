// Stream-K, warp-specialized tcgen05 GEMM for the skinny verify projections.
//
//   out[t, n] = sum_k X[t, k] * W[n, k]      t < TPAD (tree rows), n < N
//
// Dense mode (prompt prefill, n_tiles > 1): the token rows are cut into
// n_tiles tiles of TPAD = 256 (the largest UMMA N at M = 128); tile index
// = m_tile * n_tiles + token_tile, so the CTAs working at one time share
// weight tiles (read from HBM once, the rest from L2) and the activations
// (rows x K bf16, tens of MB) stay L2 resident.  The stream-K split is the
// same over (tile, k_block) units.
//
// Swap-AB: W (weights, streamed once from HBM) is the MMA's M=128 A operand,
// X (the tree's activations, L2 resident) the N=TPAD B operand; both K-major
// bf16 tiles of 64 elements (128 B, one swizzle atom) per stage, brought in
// by TMA with 128-byte swizzle.  The accumulator D[128 x TPAD] fp32 lives in
// TMEM (two buffers, so the MMA of the next segment overlaps the epilogue).
//
// Work split: the (m_tile, k_block) units are linearized and cut into
// `grid` equal contiguous ranges (stream-K), so every shape keeps all SMs
// streaming weights.  A range covers whole tiles plus at most two partial
// tiles; partial tiles are written as fp32 partials and the last CTA to
// finish a tile sums them in CTA order (deterministic) before the epilogue.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = MMA issuer,
// warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4)..+31).
//
// Q4 variant (4-bit affine weights, group 64 along K, MLX layout: packed
// uint32 [N][K/8] with element 8j+i in bits 4i..4i+3 of word j, bf16 scales
// and biases [N][K/64]): a stream-K unit is 128 wide in K (2 groups); TMA
// brings the packed 128x128 tile (8 KB, 64-byte swizzled) and the two
// 64-wide X blocks; 4 more warps (6..9, 320 threads, two CTAs per SM)
// dequantize it, w = scale*q + bias rounded once to bf16 (fma.rn.bf16x2),
// into a TMEM buffer that the MMA reads as its A operand (8 MMAs of K 16
// per unit).
#pragma once

#include "common.cuh"
#include "../../include/dtree_b200.h"

namespace dtree {

enum Epi : int {
  kEpiStore = 0,     // out[t*ldo + n] = bf16(acc)
  kEpiResidual = 1,  // resid[t*ldo + n] = bf16(resid + bf16(acc)); optional capture copy
  kEpiSwiglu = 2,    // rows g(64) | u(64) per tile -> act[t*ldo + j] = silu(g)*u
  kEpiQkv = 3,       // q/k RMSNorm + RoPE -> q buffer / K cache; v -> V cache
  kEpiArgmax = 4,    // per-row argmax over n (LM head), ties -> smallest n
  kEpiPartial = 5,   // split-K: fp32 partial of split s -> out_f32[(s*TPAD + t)*ldo + n]
};

struct GemmParams {
  int n_out;   // rows of W
  int kb;      // K / 64
  int m_tiles; // ceil(n_out / 128)
  int n_rows;  // valid tree rows (<= TPAD; dense mode: token rows, <= n_tiles * TPAD)
  int n_tiles; // token tiles of TPAD rows (1: tree verify)
  int w_dep;   // weights written by the upstream kernel (dequantized): load them after the dependency wait
  int grid;    // CTAs (stream-K ranges, or m_tiles * split)
  int split;   // > 0: tile-aligned split-K (CTA c -> tile c / split, split c % split); 0: stream-K
  float* out_f32;  // kEpiPartial output [split][TPAD][ldo]
  float* ws;            // [grid][2][128][TPAD] fp32 partial tiles (row-major per slot)
  uint32_t* tile_cnt;   // [m_tiles] arrival counters (zero between launches)
  // store / residual / swiglu
  __nv_bfloat16* out;
  int ldo;
  __nv_bfloat16* capture;  // residual copy for verifier_hidden (nullable)
  int ldc;
  // qkv
  __nv_bfloat16* q_out;
  int ldq;
  __nv_bfloat16* k_cache;  // this layer's K planes [n_kv_heads][kv_cap][head_dim]
  __nv_bfloat16* v_cache;
  int kv_cap, head_dim, n_q_heads, n_kv_heads;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  float eps;
  float rope_log2_theta;
  const int32_t* positions;
  const dtree_step_state* state;
  // argmax
  int vocab;
  unsigned long long* argmax_keys;  // [TPAD], zero between launches
  uint32_t* done_cnt;               // zero between launches
  int32_t* argmax_out;              // [n_rows]
  // sampling (inv_temp > 0): argmax of logit * inv_temp + Gumbel noise keyed
  // by (sample_seed, sample_state->step, row, column) = a draw from
  // softmax(logits / T); 0: greedy argmax
  float inv_temp;
  uint32_t sample_seed;
  const dtree_step_state* sample_state;
  // q4 scales and biases, repacked once per weight (q4_sb_repack_launch):
  // per (m tile, unit) one 1 KB block of 128 rows x (s0, s1, b0, b1) bf16
  // for the unit's two groups of 64; rows past N and groups past K are zero
  const uint8_t* q_sb;
};

// bytes of a weight's repacked q4 scale / bias blocks
constexpr int kQ4SbBlock = 128 * 4 * 2;

constexpr int kGemmThreads = 192;
constexpr int kDeqWarps = 4;                             // q4 dequant warps (one per TMEM lane quarter)
constexpr int kQ4BudgetKB = 110;                         // q4 CTA shared memory (two CTAs per SM)
constexpr int kGemmThreadsQ4 = 192 + kDeqWarps * 32;
constexpr int kWTileBytes = 128 * 64 * 2;
constexpr int kPkTileBytes = 128 * 64 / 2;  // packed 4-bit tile of one 64-wide K block
constexpr int kQ4Kb = 2;                    // q4: 64-wide K blocks per stream-K unit (64-byte packed rows)

template <int TPAD, int EPI, bool Q4 = false>
struct GemmCfg {
  // 64-wide K blocks per stream-K unit: 1 (bf16) or kQ4Kb (q4: the MMA
  // thread waits and commits once per 4 * kQ4Kb MMAs)
  static constexpr int kKb = Q4 ? kQ4Kb : 1;
  static constexpr int kXBlock = TPAD * 64 * 2;  // X of one K block (128-byte swizzled rows)
  static constexpr int kXBytes = kXBlock * kKb;
  // bf16 stage: [W 16 KB][X]; q4 stage: [X blocks][packed tile][scale /
  // bias block 1 KB] (X stays 1024-aligned)
  static constexpr int kStageBytes = (Q4 ? kPkTileBytes * kKb + kQ4SbBlock : kWTileBytes) + kXBytes;
  static constexpr int kXOff = Q4 ? 0 : kWTileBytes;
  static constexpr int kWOff = Q4 ? kXBytes : 0;
  static constexpr int kSbOff = kWOff + kPkTileBytes * kKb;  // q4 only
  static constexpr int kBarBytes = Q4 ? 512 : 256;
  static constexpr int kXchBytes = (EPI == kEpiQkv || EPI == kEpiSwiglu) ? 128 * 8 * 4 : 0;
  // [0,256): per-warp reductions of one 8-row chunk; then s_best / s_pos
  // [TPAD] (8 B each) and the argmax chunk keys [4][8] (8 B each)
  static constexpr int kRedBytes = 256 + TPAD * 8 + 4 * 8 * 8;
  // keep a CTA within ~half an SM's shared memory so the next kernel's CTA
  // (launched early by PDL) can be resident and prefetch its weights
  // (q4 stages are a quarter as large; a deeper ring keeps enough packed
  // bytes in flight)
  // (TPAD 256, dense prefill: one CTA per SM with a 4-stage ring)
  static constexpr int kBudget = (Q4 ? kQ4BudgetKB : (TPAD >= 256 ? 200 : 110)) * 1024;
  static constexpr int kFixed = 1024 /*align*/ + kBarBytes + kXchBytes + kRedBytes;
  static constexpr int kStagesRaw = (kBudget - kFixed) / kStageBytes;
  static constexpr int kMaxStages = Q4 ? 16 : 8;
  static constexpr int kStagesFit = kStagesRaw < 2 ? 2 : (kStagesRaw > kMaxStages ? kMaxStages : kStagesRaw);
  // TMEM: accumulator buffers (two, so a segment's MMAs overlap the previous
  // segment's epilogue; one for q4 from TPAD 80) and, for q4, kDeq buffers
  // of dequantized W units (the MMA's A operand: 128 lanes x 32 * kKb
  // columns of bf16 pairs); the dequant warps refill buffer i % kDeq once
  // the MMA of unit i - kDeq has committed it free.  A q4 CTA holds at most
  // 256 columns, so two CTAs share an SM (the next GEMM's CTA streams its
  // weights while this one drains)
  static constexpr int kAccBufs = (Q4 && TPAD >= 80) ? 1 : 2;
  static constexpr int kTmemAcc = kAccBufs * TPAD;
  static constexpr int kDeq = Q4 ? (256 - kTmemAcc) / (32 * kKb) : 0;
  static constexpr int kTmemNeed = kTmemAcc + (Q4 ? kDeq * 32 * kKb : 0);
  // q4 with at least 3 dequant buffers: a ring of exactly kDeq stages, so a
  // stage's arrival (its refill waited for the MMAs of the unit kDeq back)
  // also proves that unit's TMEM buffer free (the dequant warps skip that
  // wait); the TMA copies land well within 3 units' time
  static constexpr int kStages = (Q4 && kDeq >= 3 && kDeq <= kStagesFit) ? kDeq : kStagesFit;
  static constexpr int kSmem = kFixed + kStages * kStageBytes;
  static constexpr int kTmemCols =
      kTmemNeed <= 32 ? 32 : (kTmemNeed <= 64 ? 64 : (kTmemNeed <= 128 ? 128 : (kTmemNeed <= 256 ? 256 : 512)));
  static constexpr uint32_t kIdesc = idesc_bf16_f32(128, TPAD);
};

// first unit of CTA c (floor(c * U / G))
__device__ __forceinline__ long long sk_u0(int c, long long U, int G) {
  return static_cast<long long>((static_cast<unsigned>(c) * static_cast<unsigned>(U)) / static_cast<unsigned>(G));
}
// CTA containing unit u
__device__ __forceinline__ int sk_cta_of(long long u, long long U, int G) {
  return static_cast<int>((static_cast<unsigned>(u + 1) * static_cast<unsigned>(G) - 1u) / static_cast<unsigned>(U));
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// CW (16 or 32) consecutive accumulator columns of this thread's TMEM lane
template <int CW>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&g)[CW]) {
  if constexpr (CW == 32) {
    uint32_t r[32];
    tmem_ld_x32(taddr, r);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) g[j] = __uint_as_float(r[j]);
  } else {
    static_assert(CW == 16, "column group of 16 or 32");
    uint32_t r0[8], r1[8];
    tmem_ld_x8(taddr, r0);
    tmem_ld_x8(taddr + 8, r1);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      g[j] = __uint_as_float(r0[j]);
      g[8 + j] = __uint_as_float(r1[j]);
    }
  }
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ __nv_bfloat162 u32_as_bf162(uint32_t v) { return *reinterpret_cast<__nv_bfloat162*>(&v); }
__device__ __forceinline__ uint32_t bf162_as_u32(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }

// 8 packed 4-bit weights (one uint32, element i in bits 4i..4i+3) -> 8 bf16
// scale*q + bias as 4 bf16x2 words in element order.  (0x43 << 8 | q) is the
// bf16 of 128 + q exactly, so (128 + q) - 128 = q exactly and the fma rounds
// once.
__device__ __forceinline__ uint4 dequant8(uint32_t x, __nv_bfloat162 s2, __nv_bfloat162 b2) {
  const uint32_t lo = x & 0x0F0F0F0Fu;         // elements 0,2,4,6 (one per byte)
  const uint32_t hi = (x >> 4) & 0x0F0F0F0Fu;  // elements 1,3,5,7
  const uint32_t a = prmt(lo, hi, 0x5140u);    // bytes q0 q1 q2 q3
  const uint32_t b = prmt(lo, hi, 0x7362u);    // bytes q4 q5 q6 q7
  const uint32_t c43 = 0x43434343u;
  const __nv_bfloat162 k128 = u32_as_bf162(0x43004300u);
  uint4 o;
  o.x = bf162_as_u32(__hfma2(__hsub2(u32_as_bf162(prmt(a, c43, 0x4140u)), k128), s2, b2));
  o.y = bf162_as_u32(__hfma2(__hsub2(u32_as_bf162(prmt(a, c43, 0x4342u)), k128), s2, b2));
  o.z = bf162_as_u32(__hfma2(__hsub2(u32_as_bf162(prmt(b, c43, 0x4140u)), k128), s2, b2));
  o.w = bf162_as_u32(__hfma2(__hsub2(u32_as_bf162(prmt(b, c43, 0x4342u)), k128), s2, b2));
  return o;
}

template <int TPAD, int EPI, bool Q4>
__global__ void __launch_bounds__(Q4 ? kGemmThreadsQ4 : kGemmThreads, Q4 ? 2 : 1)
    gemm_streamk_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                        GemmParams p) {
  using C = GemmCfg<TPAD, EPI, Q4>;
  constexpr int S = C::kStages;
  constexpr int D = C::kDeq > 0 ? C::kDeq : 1;  // (bf16: deq barriers unused)
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_base = smem;
  uint8_t* bar_base = smem + S * C::kStageBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(bar_base);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* tfull_bar = empty_bar + S;
  uint64_t* tempty_bar = tfull_bar + 2;
  // q4: deq_full[d] completes when the dequant warps have written TMEM
  // buffer d (and, through their own wait, the stage's X blocks landed);
  // tfree[d] when the MMAs that read buffer d completed.
  uint64_t* deq_full = tempty_bar + 2;   // [D] (q4 only)
  uint64_t* tfree = deq_full + D;        // [D] (q4 only)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(deq_full + 2 * D);
  int* s_flag = reinterpret_cast<int*>(tmem_slot + 1);
  float* xch = reinterpret_cast<float*>(bar_base + C::kBarBytes);
  uint8_t* red_raw = bar_base + C::kBarBytes + C::kXchBytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.grid;
  // token tiles: dense (prefill) tiles only; a tree verify has one
  constexpr bool kDense = TPAD >= 256;
  const int NT = kDense ? p.n_tiles : 1;
  const long long U = static_cast<long long>(p.m_tiles) * NT * p.kb;
  const int cta = blockIdx.x;
  long long u0, u1;
  if (p.split > 0) {  // tile-aligned split-K: one segment per CTA
    const int tile = cta / p.split, sp = cta % p.split;
    u0 = static_cast<long long>(tile) * p.kb + (sp * p.kb) / p.split;
    u1 = static_cast<long long>(tile) * p.kb + ((sp + 1) * p.kb) / p.split;
  } else {
    u0 = sk_u0(cta, U, G);
    u1 = sk_u0(cta + 1, U, G);
  }
  const int n_units = static_cast<int>(u1 - u0);

  if (warp == 0) {
    if (lane == 0) {
      for (int s = 0; s < S; ++s) {
        mbar_init(&full_bar[s], 1);
        mbar_init(&empty_bar[s], 1);
      }
      for (int b = 0; b < 2; ++b) {
        mbar_init(&tfull_bar[b], 1);
        mbar_init(&tempty_bar[b], 4);
      }
      for (int b = 0; b < D; ++b) {
        mbar_init(&deq_full[b], kDeqWarps);  // one arrival per dequant warp and unit
        mbar_init(&tfree[b], 1);
      }
      fence_barrier_init();
      tma_prefetch_desc(&tmap_w);
      tma_prefetch_desc(&tmap_x);
    }
    __syncwarp();
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      // weights stream once per verify (evict first); a dense tile's weights
      // are re-read by every token tile (keep them)
      const uint64_t pol_w = kDense ? l2_policy_evict_last() : l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      constexpr int LA = S;  // units in flight: the whole ring
      const int pre = n_units < LA ? n_units : LA;
      // weights do not depend on the upstream kernel (unless w_dep): start
      // streaming now
      if (p.w_dep) pdl_wait();
      // the prefetched units' X coordinates are computed here, before the
      // dependency wait: after it only the TMA issues remain
      int xk[S], xr[S];
      {
        int tile = static_cast<int>(u0 / p.kb), kblk = static_cast<int>(u0 % p.kb);
        int mt = tile / NT, nt = tile % NT;
#pragma unroll
        for (int i = 0; i < S; ++i) {
          if (i < pre) {
            mbar_arrive_expect_tx(&full_bar[i], C::kStageBytes);
            tma_load_2d(stage_base + i * C::kStageBytes + C::kWOff, &tmap_w, &full_bar[i],
                        kblk * (Q4 ? 8 * C::kKb : 64), mt * 128, pol_w);
            if constexpr (Q4)
              bulk_load_1d(stage_base + i * C::kStageBytes + C::kSbOff,
                           p.q_sb + (static_cast<size_t>(mt) * p.kb + kblk) * kQ4SbBlock, kQ4SbBlock, &full_bar[i],
                           pol_w);
          }
          xk[i] = kblk * C::kKb * 64;
          xr[i] = nt * TPAD;
          if (++kblk == p.kb) {
            kblk = 0;
            if (++nt == NT) {
              nt = 0;
              ++mt;
            }
          }
        }
      }
      pdl_wait();
#pragma unroll
      for (int i = 0; i < S; ++i) {
        if (i < pre) {
#pragma unroll
          for (int k2 = 0; k2 < C::kKb; ++k2)
            tma_load_2d(stage_base + i * C::kStageBytes + C::kXOff + k2 * C::kXBlock, &tmap_x, &full_bar[i],
                        xk[i] + k2 * 64, xr[i], pol_x);
        }
      }
      bool ok = true;
      // (tile, kblk) of unit `pre`, advanced incrementally (no 64-bit division per unit)
      int tile = static_cast<int>((u0 + pre) / p.kb), kblk = static_cast<int>((u0 + pre) % p.kb);
      int mt = tile / NT, nt = tile % NT;  // weight tile, token tile
      int s = pre % S;
      for (int i = pre; i < n_units && ok; ++i) {
        // the MMA of unit i - S released this stage
        ok = mbar_wait(&empty_bar[s], static_cast<uint32_t>((i - S) / S) & 1u, 1);
        if (!ok) break;
        mbar_arrive_expect_tx(&full_bar[s], C::kStageBytes);
        uint8_t* st = stage_base + s * C::kStageBytes;
        tma_load_2d(st + C::kWOff, &tmap_w, &full_bar[s], kblk * (Q4 ? 8 * C::kKb : 64), mt * 128, pol_w);
        if constexpr (Q4)
          bulk_load_1d(st + C::kSbOff, p.q_sb + (static_cast<size_t>(mt) * p.kb + kblk) * kQ4SbBlock, kQ4SbBlock,
                       &full_bar[s], pol_w);
#pragma unroll
        for (int k2 = 0; k2 < C::kKb; ++k2)
          tma_load_2d(st + C::kXOff + k2 * C::kXBlock, &tmap_x, &full_bar[s], (kblk * C::kKb + k2) * 64, nt * TPAD,
                      pol_x);
        if (++kblk == p.kb) {
          kblk = 0;
          if (++nt == NT) {
            nt = 0;
            ++mt;
          }
        }
        if (++s == S) s = 0;
      }
      // drain: every issued load must land before the CTA can retire
      const int first_undrained = n_units > S ? n_units - S : 0;
      for (int i = first_undrained; i < n_units; ++i)
        mbar_wait(&full_bar[i % S], static_cast<uint32_t>(i / S) & 1u, 2);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // Lean per-unit loop (this thread's issue rate bounds the unit rate):
      // descriptors are a base plus a 16-byte-unit offset, ring slots and
      // phases advance incrementally.
      const uint64_t a_base = sw128_kmajor_desc(smem_u32(stage_base));
      const uint64_t b_base = sw128_kmajor_desc(smem_u32(stage_base + C::kXOff));
      long long u = u0;
      int i = 0, seg = 0;
      int s = 0, d = 0;  // stage, dequant buffer
      uint32_t ph = 0, phd = 0;
      bool ok = true;
      while (u < u1) {
        const int kblk0 = static_cast<int>(u % p.kb);
        const int len = static_cast<int>(min(static_cast<long long>(p.kb - kblk0), u1 - u));
        const int b = seg % C::kAccBufs;
        const int use = seg / C::kAccBufs;
        if (use >= 1 && ok) ok = mbar_wait(&tempty_bar[b], static_cast<uint32_t>(use - 1) & 1u, 3);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * TPAD);
        for (int j = 0; j < len; ++j, ++i) {
          if constexpr (Q4) {
            if (ok) ok = mbar_wait(&deq_full[d], phd, 8);
          } else {
            if (ok) ok = mbar_wait(&full_bar[s], ph, 4);
          }
          tc_fence_after();
          if (ok) {
            const uint64_t b0 = b_base + ((s * C::kStageBytes) >> 4);
            if constexpr (Q4) {  // A = the dequantized unit in TMEM, 8 columns per K step of 16
              const uint32_t a_tmem = tmem_base + static_cast<uint32_t>(C::kTmemAcc + d * 32 * C::kKb);
#pragma unroll
              for (int k2 = 0; k2 < C::kKb; ++k2)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                  umma_bf16_ts(d_tmem, a_tmem + k2 * 32 + kk * 8, b0 + ((k2 * C::kXBlock) >> 4) + kk * 2, C::kIdesc,
                               (j > 0 || k2 > 0 || kk > 0) ? 1u : 0u);
            } else {
              const uint64_t a0 = a_base + ((s * C::kStageBytes) >> 4);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                umma_bf16(d_tmem, a0 + kk * 2, b0 + kk * 2, C::kIdesc, (j > 0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(&empty_bar[s]);
          if constexpr (Q4) umma_commit(&tfree[d]);
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
          if constexpr (Q4) {
            if (++d == D) {
              d = 0;
              phd ^= 1u;
            }
          }
        }
        umma_commit(&tfull_bar[b]);
        u += len;
        ++seg;
      }
    }
  } else if (Q4 && warp >= 6) {
    // ------------------------------------------------------------ dequant (q4)
    // All 4 warps work on one unit at a time: thread = tile row r, each warp
    // on the TMEM lane quarter it may write (lanes 32 * (warp % 4) ..).  A
    // thread turns its row's 16 packed words (two groups of 64) into 64 TMEM
    // columns of bf16 pairs.  The packed tile arrives 64-byte swizzled
    // (16-byte chunk c of the 64-byte row r at chunk c ^ ((r / 2) % 4)), so
    // a quarter-warp's chunk reads hit 8 different bank groups; the row's
    // scales and biases come with the stage (its 1 KB block, 8 B a row).
    static_assert(kDeqWarps == 4, "one dequant thread per tile row");
    const int r = 32 * (warp & 3) + lane;
    constexpr int h = 0;
    const uint32_t t_lane = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    bool ok = true;
    for (int i = 0; i < n_units && ok; ++i) {
      const int s = i % S, d = i % D;
      ok = mbar_wait(&full_bar[s], static_cast<uint32_t>(i / S) & 1u, 6);
      // (a ring of S <= D stages: the stage's arrival already proves the
      // MMAs of unit i - D, and with them TMEM buffer d, done)
      if constexpr (S > D)
        if (ok && i >= D) ok = mbar_wait(&tfree[d], static_cast<uint32_t>(i / D - 1) & 1u, 9);
      ok = __all_sync(0xffffffffu, ok);  // the TMEM stores below are warp-wide
      if (!ok) break;
      tc_fence_after();
      const uint8_t* stg = stage_base + s * C::kStageBytes;
      const uint8_t* rowp = stg + C::kWOff + r * 64;
      const int sw = (r >> 1) & 3;
      // this row's scale pair and bias pair, and all four packed chunks,
      // loaded before the first TMEM store
      const uint2 sbv = *reinterpret_cast<const uint2*>(stg + C::kSbOff + r * 8);
      const __nv_bfloat162 sc2 = u32_as_bf162(sbv.x), bi2 = u32_as_bf162(sbv.y);
      uint4 pc[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) pc[c] = *reinterpret_cast<const uint4*>(rowp + (((4 * h + c) ^ sw) << 4));
#pragma unroll
      for (int gq = 0; gq < 2; ++gq) {  // group 2h + gq: 8 words, 32 TMEM columns
        const uint4 pa = pc[2 * gq], pb = pc[2 * gq + 1];
        const __nv_bfloat16 sc = gq ? __high2bfloat16(sc2) : __low2bfloat16(sc2);
        const __nv_bfloat16 bi = gq ? __high2bfloat16(bi2) : __low2bfloat16(bi2);
        const __nv_bfloat162 s2 = __halves2bfloat162(sc, sc), b2 = __halves2bfloat162(bi, bi);
        const uint32_t pk[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
        uint32_t v[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint4 q = dequant8(pk[j], s2, b2);
          v[4 * j] = q.x;
          v[4 * j + 1] = q.y;
          v[4 * j + 2] = q.z;
          v[4 * j + 3] = q.w;
        }
        tmem_st_x32(tmem_base + t_lane + static_cast<uint32_t>(C::kTmemAcc + d * 32 * C::kKb + h * 64 + gq * 32), v);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&deq_full[d]);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Processes the 128 x TPAD accumulator in chunks of 8 tree rows (TMEM
    // columns) in a rolled loop: the code stays small and hot in the
    // instruction cache although it runs only once or twice per tile.
    const int q = warp & 3;            // TMEM lane quarter
    const int row = q * 32 + lane;     // row of the 128-row tile
    const int et = threadIdx.x - 64;   // 0..127 epilogue thread id
    // accumulator columns per group (the q4 kernel's 448 threads leave 128
    // registers a thread) and contributing CTAs' partial rows in flight
    constexpr int CW = (TPAD % 32 == 0 && !Q4) ? 32 : 16;
    constexpr int NV = Q4 ? 1 : 2;
    pdl_wait();
    float* red = reinterpret_cast<float*>(red_raw);                                   // [4][8]
    unsigned long long* s_best = reinterpret_cast<unsigned long long*>(red_raw + 256);  // argmax [TPAD]
    float* s_pos = reinterpret_cast<float*>(red_raw + 256);                           // qkv    [TPAD]
    int start = 0;
    uint32_t sample_step = 0;
    if constexpr (EPI == kEpiArgmax) {
      for (int t = et; t < TPAD; t += 128) s_best[t] = 0ull;
      if (p.sample_state) sample_step = static_cast<uint32_t>(p.sample_state->step);
    }
    if constexpr (EPI == kEpiQkv) {
      start = p.state ? p.state->start : 0;
      for (int t = et; t < TPAD; t += 128) s_pos[t] = t < p.n_rows ? static_cast<float>(p.positions[t]) : 0.0f;
    }
    epi_bar();
    long long u = u0;
    int seg = 0;
    const int first_tile = static_cast<int>(u0 / p.kb);
    while (u < u1) {
      const int tile = static_cast<int>(u / p.kb);
      const int kblk0 = static_cast<int>(u % p.kb);
      const int len = static_cast<int>(min(static_cast<long long>(p.kb - kblk0), u1 - u));
      const bool full = (kblk0 == 0 && len == p.kb) || EPI == kEpiPartial;
      const int b = seg % C::kAccBufs;
      const int use = seg / C::kAccBufs;
      mbar_wait(&tfull_bar[b], static_cast<uint32_t>(use) & 1u, 5);
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * TPAD);

      bool have = true;
      int c_first = cta, c_last = cta;
      if (!full) {
        // this CTA holds part of the tile's K range: publish the partial
        // (TPAD < 256: [TPAD][128] fp32, thread = row; 256: [128][TPAD],
        // each thread its own row, 16-byte stores)
        const int which = (tile == first_tile) ? 0 : 1;
        float* slot = p.ws + (static_cast<size_t>(cta) * 2 + which) * TPAD * 128;
        if constexpr (TPAD >= 256) {
          float* srow = slot + static_cast<size_t>(row) * TPAD;
#pragma unroll 1
          for (int cg = 0; cg < TPAD; cg += CW) {
            float g[CW];
            tmem_ld_cols<CW>(taddr + cg, g);
#pragma unroll
            for (int j = 0; j < CW; j += 4)
              *reinterpret_cast<float4*>(srow + cg + j) = make_float4(g[j], g[j + 1], g[j + 2], g[j + 3]);
          }
        } else {
#pragma unroll 1
          for (int c0 = 0; c0 < TPAD; c0 += 8) {
            uint32_t r[8];
            tmem_ld_x8(taddr + c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 8; ++j) slot[(c0 + j) * 128 + row] = __uint_as_float(r[j]);
          }
        }
        __threadfence();
        epi_bar();
        const long long tu0 = static_cast<long long>(tile) * p.kb, tu1 = tu0 + p.kb - 1;
        c_first = sk_cta_of(tu0, U, G);
        c_last = sk_cta_of(tu1, U, G);
        if (et == 0) {
          const uint32_t prev = atomicAdd(&p.tile_cnt[tile], 1u);
          *s_flag = (prev == static_cast<uint32_t>(c_last - c_first)) ? 1 : 0;
        }
        epi_bar();
        have = (*s_flag != 0);
        if (have) {
          __threadfence();
          if (et == 0) p.tile_cnt[tile] = 0u;
        }
      }
      if (have) {
        const int mt = tile / NT;         // weight tile
        const int tb = (tile % NT) * TPAD;  // first token row of the tile
        const int n = mt * 128 + row;
        // the epilogue of accumulator columns c0 .. c0 + 7 (values a)
        // (hv_in, have_h: the residual rows, already loaded by a dense
        // tile's group prefetch)
        auto body = [&](const int c0, float (&a)[8], const __nv_bfloat16 (&hv_in)[8], const bool have_h) {
            if constexpr (EPI == kEpiPartial) {
              if (n < p.n_out) {
                float* o = p.out_f32 + static_cast<size_t>(cta % p.split) * TPAD * p.ldo + n;
#pragma unroll
                for (int j = 0; j < 8; ++j) o[static_cast<size_t>(c0 + j) * p.ldo] = a[j];
              }
            } else if constexpr (EPI == kEpiStore) {
              if (n < p.n_out) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const int t = tb + c0 + j;
                  p.out[static_cast<size_t>(t) * p.ldo + n] = __float2bfloat16_rn(t < p.n_rows ? a[j] : 0.0f);
                }
              }
            } else if constexpr (EPI == kEpiResidual) {
              if (n < p.n_out) {
                __nv_bfloat16 hv[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const int t = tb + c0 + j;
                  hv[j] = have_h ? hv_in[j]
                                 : (t < p.n_rows ? p.out[static_cast<size_t>(t) * p.ldo + n] : __float2bfloat16_rn(0.0f));
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const int t = tb + c0 + j;
                  __nv_bfloat16 hn = __float2bfloat16_rn(0.0f);
                  if (t < p.n_rows) hn = __float2bfloat16_rn(__bfloat162float(hv[j]) + bf16_round(a[j]));
                  p.out[static_cast<size_t>(t) * p.ldo + n] = hn;
                  if (p.capture && t < p.n_rows) p.capture[static_cast<size_t>(t) * p.ldc + n] = hn;
                }
              }
            } else if constexpr (EPI == kEpiSwiglu) {
              if (row >= 64) {
#pragma unroll
                for (int j = 0; j < 8; ++j) xch[j * 128 + row] = a[j];
              }
              epi_bar();
              if (row < 64) {
                const int jf = mt * 64 + row;
                // every exchange load, then every column's arithmetic, then
                // every store: a store may alias the (generic) exchange
                // pointer, so a load after it could not be hoisted and the
                // eight expf / divide chains would run one after another
                float uu[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) uu[j] = bf16_round(xch[j * 128 + row + 64]);
                __nv_bfloat16 o[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const int t = tb + c0 + j;
                  const float g = bf16_round(a[j]);
                  // branch-free approximate exp / divide: their few-ulp fp32
                  // error is far below the bf16 rounding that follows, and
                  // the IEEE divide's guarded slow path kept the eight
                  // columns' chains from overlapping
                  const float sg = bf16_round(__fdividef(1.0f, 1.0f + __expf(-g)));
                  const float sl = bf16_round(g * sg);
                  o[j] = __float2bfloat16_rn(t < p.n_rows ? sl * uu[j] : 0.0f);
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) p.out[static_cast<size_t>(tb + c0 + j) * p.ldo + jf] = o[j];
              }
              epi_bar();
            } else if constexpr (EPI == kEpiQkv) {
              const int hd = p.head_dim;
              const int gh = n / hd;  // global head index across q | k | v
              const int d = n % hd;
              if (gh >= p.n_q_heads + p.n_kv_heads) {
                const int kvh = gh - p.n_q_heads - p.n_kv_heads;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const int t = c0 + j;
                  if (t < p.n_rows) {
                    const int slot = start + t;
                    if (slot < p.kv_cap)
                      p.v_cache[(static_cast<size_t>(kvh) * p.kv_cap + slot) * hd + d] = __float2bfloat16_rn(a[j]);
                    else
                      dev_error(0x2001u);
                  }
                }
              } else {
                // RMSNorm over the head (hd rows = hd/32 warps), then RoPE
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  a[j] = bf16_round(a[j]);
                  float v = a[j] * a[j];
                  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                  if (lane == 0) red[q * 8 + j] = v;
                }
                epi_bar();
                const int wph = hd / 32;
                const int w0 = (q / wph) * wph;
                const float nw = __bfloat162float((gh < p.n_q_heads ? p.q_norm : p.k_norm)[d]);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  float ss = 0.0f;
                  for (int w = w0; w < w0 + wph; ++w) ss += red[w * 8 + j];
                  const float rms = rsqrtf(ss / static_cast<float>(hd) + p.eps);
                  a[j] = bf16_round(a[j] * rms * nw);
                  xch[j * 128 + row] = a[j];
                }
                epi_bar();
                const int half = hd / 2;
                const int i_f = d % half;
                const float inv_freq =
                    exp2f(-(2.0f * static_cast<float>(i_f) / static_cast<float>(hd)) * p.rope_log2_theta);
                const int partner = (d < half) ? row + half : row - half;
                const bool is_q = gh < p.n_q_heads;
                const int kvh = gh - p.n_q_heads;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const int t = c0 + j;
                  float outv = 0.0f;
                  if (t < p.n_rows) {
                    float sn, cs;
                    sincosf(s_pos[t] * inv_freq, &sn, &cs);
                    const float y = a[j], yp = xch[j * 128 + partner];
                    outv = (d < half) ? (y * cs - yp * sn) : (y * cs + yp * sn);
                  }
                  if (is_q) {
                    p.q_out[static_cast<size_t>(t) * p.ldq + gh * hd + d] = __float2bfloat16_rn(outv);
                  } else if (t < p.n_rows) {
                    const int slot = start + t;
                    if (slot < p.kv_cap)
                      p.k_cache[(static_cast<size_t>(kvh) * p.kv_cap + slot) * hd + d] = __float2bfloat16_rn(outv);
                    else
                      dev_error(0x2001u);
                  }
                }
                epi_bar();
              }
            } else if constexpr (EPI == kEpiArgmax) {
              // per tree row: max over this tile's 128 vocab rows (ties -> smallest id)
              const bool valid = n < p.vocab;
              unsigned long long* rk = reinterpret_cast<unsigned long long*>(red_raw + 256 + TPAD * 8);  // [4][8]
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                unsigned long long key = 0ull;
                if (valid) {
                  float v = bf16_round(a[j]);
                  if (p.inv_temp > 0.0f)
                    v = v * p.inv_temp + gumbel_noise(p.sample_seed, kSampleTagVerify, sample_step,
                                                      static_cast<uint32_t>(c0 + j), static_cast<uint32_t>(n));
                  key = (static_cast<unsigned long long>(float_order_key(v)) << 32) |
                        static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(n));
                }
                for (int o = 16; o > 0; o >>= 1) {
                  const unsigned long long ok2 = __shfl_xor_sync(0xffffffffu, key, o);
                  key = ok2 > key ? ok2 : key;
                }
                if (lane == 0) rk[q * 8 + j] = key;
              }
              epi_bar();
              if (et < 8) {
                unsigned long long bk = s_best[c0 + et];
                for (int w = 0; w < 4; ++w) bk = rk[w * 8 + et] > bk ? rk[w * 8 + et] : bk;
                s_best[c0 + et] = bk;
              }
              epi_bar();
            }
        };
        if constexpr (TPAD >= 256) {
          // column groups of CW: one TMEM load, or one round of 16-byte
          // partial loads per NV contributing CTAs, per group; the body then
          // runs on 8 columns at a time (rolled, the group shifted down)
#pragma unroll 1
          for (int cg = 0; cg < TPAD; cg += CW) {
            float g[CW];
            if (full) {
              tmem_ld_cols<CW>(taddr + cg, g);
            } else {
              // sum the partials in CTA order (deterministic)
#pragma unroll
              for (int j = 0; j < CW; ++j) g[j] = 0.0f;
              for (int c = c_first; c <= c_last; c += NV) {
                float4 v[NV][CW / 4];
#pragma unroll
                for (int i = 0; i < NV; ++i) {
                  if (c + i <= c_last) {
                    const int w2 = (tile == static_cast<int>(sk_u0(c + i, U, G) / p.kb)) ? 0 : 1;
                    const float4* sl = reinterpret_cast<const float4*>(
                        p.ws + (static_cast<size_t>(c + i) * 2 + w2) * TPAD * 128 + static_cast<size_t>(row) * TPAD +
                        cg);
#pragma unroll
                    for (int j = 0; j < CW / 4; ++j) v[i][j] = __ldcg(sl + j);
                  }
                }
#pragma unroll
                for (int i = 0; i < NV; ++i)
                  if (c + i <= c_last) {
#pragma unroll
                    for (int j = 0; j < CW / 4; ++j) {
                      g[4 * j] += v[i][j].x;
                      g[4 * j + 1] += v[i][j].y;
                      g[4 * j + 2] += v[i][j].z;
                      g[4 * j + 3] += v[i][j].w;
                    }
                  }
              }
            }
            // the residual rows of the whole group, all loads in flight at once
            __nv_bfloat16 hg[CW];
            if constexpr (EPI == kEpiResidual) {
#pragma unroll
              for (int j = 0; j < CW; ++j) {
                const int t = tb + cg + j;
                hg[j] = (n < p.n_out && t < p.n_rows) ? p.out[static_cast<size_t>(t) * p.ldo + n]
                                                      : __float2bfloat16_rn(0.0f);
              }
            }
#pragma unroll 1
            for (int sub = 0; sub < CW / 8; ++sub) {
              float a[8];
              __nv_bfloat16 h8[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) a[j] = g[j];
#pragma unroll
              for (int j = 0; j < CW - 8; ++j) g[j] = g[j + 8];
              if constexpr (EPI == kEpiResidual) {
#pragma unroll
                for (int j = 0; j < 8; ++j) h8[j] = hg[j];
#pragma unroll
                for (int j = 0; j < CW - 8; ++j) hg[j] = hg[j + 8];
              }
              body(cg + sub * 8, a, h8, EPI == kEpiResidual);
            }
          }
        } else {
          // Processes the 128 x TPAD accumulator in chunks of 8 tree rows
          // (TMEM columns) in a rolled loop: the code stays small and hot in
          // the instruction cache although it runs only once or twice per tile.
#pragma unroll 1
          for (int c0 = 0; c0 < TPAD; c0 += 8) {
            float a[8];
            if (full) {
              uint32_t r[8];
              tmem_ld_x8(taddr + c0, r);
              tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < 8; ++j) a[j] = __uint_as_float(r[j]);
            } else {
              // sum the partials in CTA order (deterministic), 8 in flight
#pragma unroll
              for (int j = 0; j < 8; ++j) a[j] = 0.0f;
              for (int c = c_first; c <= c_last; c += 8) {
                float v[8][8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  if (c + i <= c_last) {
                    const int w2 = (tile == static_cast<int>(sk_u0(c + i, U, G) / p.kb)) ? 0 : 1;
                    const float* sl = p.ws + (static_cast<size_t>(c + i) * 2 + w2) * TPAD * 128 + c0 * 128 + row;
#pragma unroll
                    for (int j = 0; j < 8; ++j) v[i][j] = __ldcg(sl + j * 128);
                  }
                }
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  if (c + i <= c_last) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) a[j] += v[i][j];
                  }
              }
            }
            const __nv_bfloat16 h8[8] = {};
            body(c0, a, h8, false);
          }
        }
      }
      // the accumulator buffer is free once every partial / epilogue read it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[b]);
      u += len;
      ++seg;
    }
    if constexpr (EPI == kEpiArgmax) {
      for (int t = et; t < p.n_rows; t += 128)
        if (s_best[t]) atomicMax(&p.argmax_keys[t], s_best[t]);
      __threadfence();
      epi_bar();
      if (et == 0) {
        const uint32_t prev = atomicAdd(p.done_cnt, 1u);
        *s_flag = (prev == static_cast<uint32_t>(G - 1)) ? 1 : 0;
      }
      epi_bar();
      if (*s_flag) {
        __threadfence();
        for (int t = et; t < TPAD; t += 128) {
          const unsigned long long k = atomicExch(&p.argmax_keys[t], 0ull);
          if (t < p.n_rows) p.argmax_out[t] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
        }
        if (et == 0) *p.done_cnt = 0u;
      }
    }
  }
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ------------------------------------------------------------ host launcher
struct GemmPlan {
  CUtensorMap tmap_w;
  CUtensorMap tmap_x;
  GemmParams p;
  int t_pad;
  int epi;
  bool q4;
};

size_t gemm_ws_bytes(int t_pad, int grid);  // fp32 partials
// Dense (prompt) GEMM: out[t, n] for t < n_rows token rows, cut into tiles of
// kDenseRows; x holds x_rows >= the rows padded to kDenseRows (the padding
// rows are read, their outputs skipped or written as zero rows).  Workspace:
// gemm_ws_bytes(kDenseRows, num_sms()).
constexpr int kDenseRows = 256;
int gemm_plan_dense(GemmPlan* plan, const void* w, int n_out, int k, const void* x, int n_rows, int x_rows,
                    int x_row_stride_elems, int epi);
int gemm_plan(GemmPlan* plan, const void* w, int n_out, int k, const void* x, int t_pad, int x_row_stride_elems,
              int epi, int grid);
// 4-bit affine weights (MLX layout): packed uint32 [n_out][k/8], bf16
// scales / biases [n_out][k/64]; epilogues kEpiStore, kEpiPartial, kEpiSwiglu
// q4 plan: sb = the weight's scale / bias blocks from q4_sb_repack_launch
int gemm_plan_q4(GemmPlan* plan, const void* w_packed, const void* sb, int n_out, int k, const void* x, int t_pad,
                 int x_row_stride_elems, int epi, int grid);
// bytes of a [n_out][k] weight's repacked scale / bias blocks, and the
// repack of MLX scales / biases bf16 [n_out][k/64] into them
size_t q4_sb_bytes(int n_out, int k);
int q4_sb_repack_launch(const void* scales, const void* biases, int n_out, int k, void* sb, cudaStream_t stream);
size_t gemm_ws_counter_bytes();  // the counter block at the start of a workspace (zero between launches)
// 4-bit affine weights (MLX layout) -> bf16 [n_out][k]
int dequant_q4_launch(const void* packed, const void* scales, const void* biases, int n_out, int k, void* out,
                      cudaStream_t st);
int gemm_bind_ws(GemmPlan* plan, void* ws, size_t ws_bytes);
int gemm_launch(const GemmPlan& plan, cudaStream_t stream);

}  // namespace dtree
