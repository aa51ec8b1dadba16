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
// and biases [N][K/64]): TMA brings the packed 128x64 tile (4 KB) instead of
// the bf16 one, and 8 more warps (6..13) dequantize it, w = scale*q + bias
// rounded once to bf16 (fma.rn.bf16x2), straight into the 128-byte-swizzled
// K-major layout the MMA reads.  One K block of 64 is exactly one group.
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
  float* ws;            // [grid][2][TPAD][128] fp32 partial tiles
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
  // q4 weights: bf16 scale / bias per (row, group of 64); row stride = kb
  const __nv_bfloat16* q_scales;
  const __nv_bfloat16* q_biases;
};

constexpr int kGemmThreads = 192;
constexpr int kDeqWarps = 8;                             // q4 dequant warps
constexpr int kQ4BudgetKB = 150;                         // q4 CTA shared memory (one CTA per SM)
constexpr int kDeqGroups = 2;                            // units dequantized concurrently
constexpr int kDeqGroupWarps = kDeqWarps / kDeqGroups;
constexpr int kGemmThreadsQ4 = 192 + kDeqWarps * 32;
constexpr int kDeqTpr = kDeqGroupWarps * 32 / 128;       // threads per tile row (within a group)
constexpr int kDeqWpt = 8 / kDeqTpr;                     // packed words (8 weights) per thread
constexpr int kWTileBytes = 128 * 64 * 2;
constexpr int kPkTileBytes = 128 * 64 / 2;  // packed 4-bit tile

template <int TPAD, int EPI, bool Q4 = false>
struct GemmCfg {
  static constexpr int kXBytes = TPAD * 64 * 2;
  // bf16 stage: [W 16 KB][X]; q4 stage: [X][packed 4 KB] (X stays 1024-aligned)
  static constexpr int kStageBytes = (Q4 ? kPkTileBytes : kWTileBytes) + kXBytes;
  static constexpr int kXOff = Q4 ? 0 : kWTileBytes;
  static constexpr int kWOff = Q4 ? kXBytes : 0;
  // dequantized W units in TMEM (32 columns each, beside the accumulators).
  // The producer loads unit i only once the MMA of unit i - kDeq is done, so
  // a landed stage also means a free buffer: kDeq is the q4 load lookahead.
  static constexpr int kDeq = Q4 ? (TPAD >= 128 ? 4 : (TPAD >= 64 ? 8 : 12)) : 0;
  static constexpr int kLookahead = Q4 ? kDeq : 0;  // 0: the whole ring
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
  // units per empty / deq_full barrier phase: the MMA thread's mbarrier
  // operations (a few hundred cycles each next to in-flight MMAs) are paid
  // once per group of kUpb q4 units
  static constexpr int kUpb = Q4 ? (TPAD >= 64 ? 2 : 4) : 1;
  static constexpr int kStages0 = kStagesRaw < 2 ? 2 : (kStagesRaw > kMaxStages ? kMaxStages : kStagesRaw);
  static constexpr int kStages = (kStages0 / kUpb) * kUpb;
  static constexpr int kSmem = kFixed + kStages * kStageBytes;
  // TMEM: accumulator buffers (two, so a segment's MMAs overlap the previous
  // segment's epilogue; one for q4 at TPAD 128) and, for q4, the dequantized
  // W units (the MMA's A operand: 128 lanes x 32 columns of bf16 pairs each)
  static constexpr int kAccBufs = (Q4 && TPAD >= 128) ? 1 : 2;
  static constexpr int kTmemAcc = kAccBufs * TPAD;
  static constexpr int kTmemNeed = kTmemAcc + (Q4 ? kDeq * 32 : 0);
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
__global__ void __launch_bounds__(Q4 ? kGemmThreadsQ4 : kGemmThreads, 1)
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
  // q4: deq_full[d] completes when the dequant warps have written buffer d
  // (and, through their own wait, the stage's X tile has landed).  Buffer d
  // of unit i is free again once the MMA of unit i - D completed, which the
  // dequant warps read off that unit's empty_bar phase: one commit per unit.
  uint64_t* deq_full = tempty_bar + 2;   // [D] (q4 only)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(deq_full + 2 * D);
  int* s_flag = reinterpret_cast<int*>(tmem_slot + 1);
  float* xch = reinterpret_cast<float*>(bar_base + C::kBarBytes);
  uint8_t* red_raw = bar_base + C::kBarBytes + C::kXchBytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.grid;
  const long long U = static_cast<long long>(p.m_tiles) * p.n_tiles * p.kb;
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
        mbar_init(&deq_full[b], kDeqWarps * (C::kUpb / kDeqGroups));  // one arrival per dequant warp and unit
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
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      constexpr int LA = C::kLookahead > 0 ? C::kLookahead : S;  // units in flight
      const int pre = n_units < LA ? n_units : LA;
      // weights do not depend on the upstream kernel (unless w_dep): start
      // streaming now
      if (p.w_dep) pdl_wait();
      for (int i = 0; i < pre; ++i) {
        const long long u = u0 + i;
        const int tile = static_cast<int>(u / p.kb), kblk = static_cast<int>(u % p.kb);
        mbar_arrive_expect_tx(&full_bar[i], C::kStageBytes);
        tma_load_2d(stage_base + i * C::kStageBytes + C::kWOff, &tmap_w, &full_bar[i], kblk * (Q4 ? 8 : 64),
                    (tile / p.n_tiles) * 128, pol_w);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) {
        const long long u = u0 + i;
        const int tile = static_cast<int>(u / p.kb), kblk = static_cast<int>(u % p.kb);
        tma_load_2d(stage_base + i * C::kStageBytes + C::kXOff, &tmap_x, &full_bar[i], kblk * 64,
                    (tile % p.n_tiles) * TPAD, pol_x);
      }
      bool ok = true;
      // (tile, kblk) of unit `pre`, advanced incrementally (no 64-bit division per unit)
      int tile = static_cast<int>((u0 + pre) / p.kb), kblk = static_cast<int>((u0 + pre) % p.kb);
      int mt = tile / p.n_tiles, nt = tile % p.n_tiles;  // weight tile, token tile
      int s = pre % S;
      for (int i = pre; i < n_units && ok; ++i) {
        if ((i - LA) % C::kUpb == 0) {  // the MMA of units i - LA .. (their phase's commit)
          // released this stage and the next kUpb - 1 (and, for q4, their TMEM buffers)
          const int jp = (i - LA) / C::kUpb;
          ok = mbar_wait(&empty_bar[jp % (S / C::kUpb)], static_cast<uint32_t>(jp / (S / C::kUpb)) & 1u, 1);
        }
        if (!ok) break;
        mbar_arrive_expect_tx(&full_bar[s], C::kStageBytes);
        uint8_t* st = stage_base + s * C::kStageBytes;
        tma_load_2d(st + C::kWOff, &tmap_w, &full_bar[s], kblk * (Q4 ? 8 : 64), mt * 128, pol_w);
        tma_load_2d(st + C::kXOff, &tmap_x, &full_bar[s], kblk * 64, nt * TPAD, pol_x);
        if (++kblk == p.kb) {
          kblk = 0;
          if (++nt == p.n_tiles) {
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
      int s = 0, d = 0, dp = 0;  // stage, dequant buffer, deq_full phase slot
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
          if (i % C::kUpb == 0) {  // first unit of a barrier phase
            if constexpr (Q4) {
              if (ok) ok = mbar_wait(&deq_full[dp], phd, 8);
            } else {
              if (ok) ok = mbar_wait(&full_bar[s], ph, 4);
            }
            tc_fence_after();
          }
          if (ok) {
            const uint64_t b0 = b_base + ((s * C::kStageBytes) >> 4);
            if constexpr (Q4) {  // A = the dequantized unit in TMEM, 8 columns per K step of 16
              const uint32_t a_tmem = tmem_base + static_cast<uint32_t>(C::kTmemAcc + d * 32);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                umma_bf16_ts(d_tmem, a_tmem + kk * 8, b0 + kk * 2, C::kIdesc, (j > 0 || kk > 0) ? 1u : 0u);
            } else {
              const uint64_t a0 = a_base + ((s * C::kStageBytes) >> 4);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                umma_bf16(d_tmem, a0 + kk * 2, b0 + kk * 2, C::kIdesc, (j > 0 || kk > 0) ? 1u : 0u);
            }
          }
          if (i % C::kUpb == C::kUpb - 1 || i == n_units - 1) {
            umma_commit(&empty_bar[(i / C::kUpb) % (S / C::kUpb)]);
            if constexpr (Q4) {
              if (++dp == D / C::kUpb) {
                dp = 0;
                phd ^= 1u;
              }
            }
          }
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
          if constexpr (Q4) {
            if (++d == D) d = 0;
          }
        }
        umma_commit(&tfull_bar[b]);
        u += len;
        ++seg;
      }
    }
  } else if (Q4 && warp >= 6) {
    // ------------------------------------------------------------ dequant (q4)
    // kDeqGroups groups of warps work on different units at once (group g:
    // units i = g, g + kDeqGroups, ...), so the per-unit chain of waits,
    // shared-memory round trips and arrivals of one unit overlaps the
    // others'.  Within a group, thread tt dequantizes row tt / kDeqTpr, part
    // tt % kDeqTpr of the unit (kDeqWpt packed words -> kDeqWpt 16-byte
    // chunks of the 128-byte-swizzled bf16 row).
    // Scales / biases (no upstream dependency) come 8 groups per 16-byte
    // load when rows are 16-byte aligned (kb % 8 == 0): `cur` holds the
    // 8-group block of the current unit, `nxt` the following block.
    const int t = threadIdx.x - kGemmThreads;
    const int grp = t / (kDeqGroupWarps * 32), tt = t % (kDeqGroupWarps * 32);
    // one tile row per thread: the TMEM lane this warp may write (lanes
    // 32 * (warp % 4) ..), which the group's four warps cover once
    static_assert(kDeqTpr == 1 && kDeqWpt == 8, "q4 dequant: one thread per tile row");
    const int r = 32 * (warp & 3) + lane;
    const uint32_t t_lane = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    (void)tt;
    const bool vec = (p.kb & 7) == 0 &&
                     ((reinterpret_cast<uintptr_t>(p.q_scales) | reinterpret_cast<uintptr_t>(p.q_biases)) & 15u) == 0;
    const long long ug = u0 + grp;
    int tile = static_cast<int>(ug / p.kb), kblk = static_cast<int>(ug % p.kb);
    int cur_t = -1, cur_k = -1, nxt_t = -1, nxt_k = -1;  // 8-group blocks held in cur / nxt
    uint4 cur_s = make_uint4(0, 0, 0, 0), cur_b = cur_s, nxt_s = cur_s, nxt_b = cur_s;
    auto load_block = [&](int tl, int kb0, uint4& vs, uint4& vb) {
      const int nn = tl * 128 + r;
      if (nn < p.n_out) {
        const size_t off = static_cast<size_t>(nn) * p.kb + kb0;
        vs = __ldg(reinterpret_cast<const uint4*>(p.q_scales + off));
        vb = __ldg(reinterpret_cast<const uint4*>(p.q_biases + off));
      } else {
        vs = make_uint4(0, 0, 0, 0);
        vb = vs;
      }
    };
    static_assert(!Q4 || S >= D, "q4 needs at least as many stages as dequant buffers");
    static_assert(!Q4 || D % kDeqGroups == 0, "dequant buffers per group must be whole");
    static_assert(!Q4 || (C::kUpb % kDeqGroups == 0 && D % C::kUpb == 0 && S >= C::kLookahead + C::kUpb),
                  "q4 barrier phases: whole units per group, whole phases of buffers, stages ahead of buffers");
    constexpr int NS = D / C::kUpb;  // deq_full slots
    bool ok = true;
    // every unit of a phase gets one arrival per warp of its group on the
    // phase's deq_full barrier, also the units past the CTA's last one that
    // fill its last phase
    const int n_pairs_units = ((n_units + C::kUpb - 1) / C::kUpb) * C::kUpb;
    for (int i = grp; i < n_pairs_units && ok; i += kDeqGroups) {
      if (i >= n_units) {
        // no load orders this arrival after the slot's previous phase
        // (phase jp - NS): wait for that phase to complete first
        const int jp = i / C::kUpb;
        if (jp >= NS) ok = mbar_wait(&deq_full[jp % NS], static_cast<uint32_t>((jp - NS) / NS) & 1u, 9);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
      }
      if (i < n_units) {
        const int n = tile * 128 + r;
        __nv_bfloat16 sc = __float2bfloat16_rn(0.0f), bi = sc;
        if (vec) {
          const int k8 = kblk & ~7;
          if (tile != cur_t || k8 != cur_k) {
            if (tile == nxt_t && k8 == nxt_k) {
              cur_s = nxt_s;
              cur_b = nxt_b;
            } else {
              load_block(tile, k8, cur_s, cur_b);
            }
            cur_t = tile;
            cur_k = k8;
            // prefetch the following block if this CTA's range reaches it
            if (n_units - i > 8 - (kblk & 7)) {
              nxt_t = k8 + 8 < p.kb ? tile : tile + 1;
              nxt_k = k8 + 8 < p.kb ? k8 + 8 : 0;
              load_block(nxt_t, nxt_k, nxt_s, nxt_b);
            }
          }
          const int g = kblk & 7, wi = g >> 1;
          const uint32_t ws = wi == 0 ? cur_s.x : wi == 1 ? cur_s.y : wi == 2 ? cur_s.z : cur_s.w;
          const uint32_t wb = wi == 0 ? cur_b.x : wi == 1 ? cur_b.y : wi == 2 ? cur_b.z : cur_b.w;
          const int sh = (g & 1) * 16;
          sc = __ushort_as_bfloat16(static_cast<unsigned short>((ws >> sh) & 0xFFFFu));
          bi = __ushort_as_bfloat16(static_cast<unsigned short>((wb >> sh) & 0xFFFFu));
        } else if (n < p.n_out) {
          sc = p.q_scales[static_cast<size_t>(n) * p.kb + kblk];
          bi = p.q_biases[static_cast<size_t>(n) * p.kb + kblk];
        }
        const int s = i % S, d = i % D;
        ok = mbar_wait(&full_bar[s], static_cast<uint32_t>(i / S) & 1u, 6);
        // (the producer loaded unit i after the MMA of unit i - D, the last
        // reader of buffer d, completed)
        ok = __all_sync(0xffffffffu, ok);  // the TMEM store below is warp-wide
        if (!ok) break;
        tc_fence_after();
        // the row's 64 packed weights -> 32 columns of bf16 pairs (K order) in
        // the unit's TMEM buffer
        const uint4* src = reinterpret_cast<const uint4*>(stage_base + s * C::kStageBytes + C::kWOff + r * 32);
        const uint4 pa = src[0], pb = src[1];
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
        tmem_st_x32(tmem_base + t_lane + static_cast<uint32_t>(C::kTmemAcc + d * 32), v);
        tmem_wait_st();
        tc_fence_before();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&deq_full[(i / C::kUpb) % NS]);
      kblk += kDeqGroups;
      while (kblk >= p.kb) {
        kblk -= p.kb;
        ++tile;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Processes the 128 x TPAD accumulator in chunks of 8 tree rows (TMEM
    // columns) in a rolled loop: the code stays small and hot in the
    // instruction cache although it runs only once or twice per tile.
    const int q = warp & 3;            // TMEM lane quarter
    const int row = q * 32 + lane;     // row of the 128-row tile
    const int et = threadIdx.x - 64;   // 0..127 epilogue thread id
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
        const int which = (tile == first_tile) ? 0 : 1;
        float* slot = p.ws + (static_cast<size_t>(cta) * 2 + which) * TPAD * 128;
#pragma unroll 1
        for (int c0 = 0; c0 < TPAD; c0 += 8) {
          uint32_t r[8];
          tmem_ld_x8(taddr + c0, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) slot[(c0 + j) * 128 + row] = __uint_as_float(r[j]);
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
        const int mt = tile / p.n_tiles;        // weight tile
        const int tb = (tile % p.n_tiles) * TPAD;  // first token row of the tile
        const int n = mt * 128 + row;
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
                hv[j] = t < p.n_rows ? p.out[static_cast<size_t>(t) * p.ldo + n] : __float2bfloat16_rn(0.0f);
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
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int t = tb + c0 + j;
                const float g = bf16_round(a[j]);
                const float uu = bf16_round(xch[j * 128 + row + 64]);
                const float sg = bf16_round(1.0f / (1.0f + expf(-g)));
                const float sl = bf16_round(g * sg);
                p.out[static_cast<size_t>(t) * p.ldo + jf] = __float2bfloat16_rn(t < p.n_rows ? sl * uu : 0.0f);
              }
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
int gemm_plan_q4(GemmPlan* plan, const void* w_packed, const void* scales, const void* biases, int n_out, int k,
                 const void* x, int t_pad, int x_row_stride_elems, int epi, int grid);
size_t gemm_ws_counter_bytes();  // the counter block at the start of a workspace (zero between launches)
// 4-bit affine weights (MLX layout) -> bf16 [n_out][k]
int dequant_q4_launch(const void* packed, const void* scales, const void* biases, int n_out, int k, void* out,
                      cudaStream_t st);
int gemm_bind_ws(GemmPlan* plan, void* ws, size_t ws_bytes);
int gemm_launch(const GemmPlan& plan, cudaStream_t stream);

}  // namespace dtree
