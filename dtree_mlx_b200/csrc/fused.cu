// Persistent tree-verify forward of a Qwen3 target (bf16 weights, head_dim
// 128, up to 64 tree rows): every layer of qwen3_tree.py:39-83 plus the
// final norm (adapters.py:568-597) in ONE launch with one CTA per SM.
//
// Why: the verify step streams 8 GB of weights for ~28 flop/B, so it is HBM
// bound, but as a chain of nine kernels per layer the weight stream stops at
// every hand-off (launch, ring refill, epilogue tail) and during every glue
// kernel (norm, q/k norm + RoPE, attention, split merge).  Here the weight
// stream never waits for activations: each CTA's producer warp walks the
// CTA's (layer, projection, tile, k-block) units for the whole forward and
// keeps its shared-memory ring full, so the next projection's weights are
// already on chip while the glue phases run; only the activation tile of a
// unit waits for its inputs.
//
// Warp roles (384 threads):
//   warp 0   weight producer: TMA of 128x64 bf16 weight tiles into the ring
//            (never waits on activations; one arrival per stage)
//   warp 1   activation producer: waits for the phase counter of each
//            projection's input, then TMAs the TPAD x 64 activation tile of
//            every unit into the same stage (the second arrival)
//   warp 2   MMA issuer: tcgen05.mma (swap-AB: weights = M 128, tree rows =
//            N TPAD), fp32 accumulators in TMEM, double-buffered
//   warps 4..11  compute: GEMM epilogues (TMEM -> fp32 split partials /
//            SwiGLU) and the glue phases, in layer order
// Per layer the compute warps run:
//   N1  h += sum(down partials); xn = RMSNorm(h)      one CTA per tree row
//   QKV epilogue (split-K partials)
//   FIN q/k RMSNorm + half-split RoPE, q -> buffer, k/v -> cache slots
//   ATT split-KV tree attention (mma.sync), per (kv head, row block, split)
//   CMB log-sum-exp merge of the splits -> attention output
//   O epilogue (split-K partials)
//   N2  h += sum(o partials); xn = RMSNorm(h)
//   GU  epilogue: stream-K gate|up tiles (+ fix-up of tiles split across
//       CTAs), SwiGLU -> act
//   DN  epilogue (split-K partials)
// and after the last layer NF: h += sum(down partials); norm_out = RMSNorm.
// Phases meet through global counters (acquire / release, every wait bounded
// in time: on expiry the kernel sets an abort word that every role polls,
// records an error code and drains).  The counters are zeroed before each
// launch.  The launch is cooperative (all CTAs co-resident).
#include <algorithm>
#include <cmath>
#include <utility>
#include <vector>

#include "fused.cuh"

namespace dtree {

constexpr int kFusedWarpsCompute = 8;
constexpr int kAttChunk = 32;                              // keys per shared-memory chunk
constexpr int kAttLd = 128 + 8;                            // padded row (bf16): conflict-free ldmatrix
constexpr int kAttStage = 2 * kAttChunk * kAttLd * 2;      // K + V chunk
constexpr int kAttBytes = 2 * kAttStage;                   // double buffered
constexpr unsigned long long kFusedTimeoutNs = 2000000000ull;  // 2 s per wait
constexpr int kFusedL2Ahead = 0;  // weight units prefetched into L2 beyond the shared-memory ring

template <int TPAD>
struct FusedCfg {
  static constexpr int kWBytes = 128 * 64 * 2;
  static constexpr int kXBytes = TPAD * 64 * 2;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kFixed = 1024 /*align*/ + kAttBytes + 1024 /*barriers, red, flags*/;
  static constexpr int kBudget = 232448;
  static constexpr int kStages0 = (kBudget - kFixed) / kStageBytes;
  static constexpr int kStages = kStages0 > 12 ? 12 : kStages0;
  static constexpr int kSmem = kFixed + kStages * kStageBytes;
  static constexpr int kTmemCols = 2 * TPAD <= 32 ? 32 : (2 * TPAD <= 64 ? 64 : 128);
  static constexpr uint32_t kIdesc = idesc_bf16_f32(128, TPAD);
  static_assert(kSmem <= kBudget, "fused kernel shared memory");
};

// ------------------------------------------------------------------ sync
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_relaxed(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void abort_set(uint32_t* abort_word, unsigned int code) {
  atomicExch(abort_word, 1u);
  dev_error(code);
}

// wait until *cnt >= target (one thread); false on abort / timeout
__device__ bool wait_count(const uint32_t* cnt, uint32_t target, uint32_t* abort_word, unsigned int where) {
  if (ld_acquire(cnt) >= target) return true;
  const uint64_t t0 = gtimer();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire(cnt) >= target) return true;
    if ((i & 63) == 0) {
      if (ld_relaxed(abort_word)) return false;
      if (gtimer() - t0 > kFusedTimeoutNs) {
        abort_set(abort_word, 0x3000u | where);
        return false;
      }
    }
  }
}

// mbarrier phase wait that gives up on abort / timeout
__device__ bool mbar_wait_ab(uint64_t* bar, uint32_t parity, uint32_t* abort_word, unsigned int where) {
  if (mbar_test_wait(bar, parity)) return true;
  uint64_t t0 = 0;
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 0) {
      if (ld_relaxed(abort_word)) return false;
      const uint64_t t = gtimer();
      if (t0 == 0) {
        t0 = t;
      } else if (t - t0 > kFusedTimeoutNs) {
        abort_set(abort_word, 0x3100u | where);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }  // compute warps
__device__ __forceinline__ void gbar(int g) {  // one 128-thread half of the compute warps
  asm volatile("bar.sync %0, 128;" ::"r"(2 + g) : "memory");
}

// compute-warp barrier that also ANDs / ORs a predicate over its threads
__device__ __forceinline__ bool cbar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred p, 1, 256, p;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ bool cbar_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred p, 1, 256, p;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u)
      : "memory");
  return r != 0;
}
// compute warps: one thread waits, the rest follow; result uniform
__device__ __forceinline__ bool cwait(const uint32_t* cnt, uint32_t target, uint32_t* abort_word, unsigned where,
                                      int ct) {
  bool ok = true;
  if (ct == 0) ok = wait_count(cnt, target, abort_word, where);
  return cbar_and(ok);
}
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// compute warps: every thread's writes are done (the barrier orders them
// before thread 0's release, which is cumulative); one thread publishes
__device__ __forceinline__ void csignal(uint32_t* cnt, int ct) {
  cbar();
  if (ct == 0) red_release_add(cnt, 1u);
}

// ------------------------------------------------------------------ jobs
struct FSeg {
  int tile, kb0, len;
};
struct FJob {
  int n, k;   // output rows (weights), reduction width
  int split;  // > 0: tile-aligned split-K; 0: stream-K over the grid
};
__device__ __forceinline__ FJob fused_job(const FusedParams& p, int j) {
  const int qkv_w = (p.n_heads + 2 * p.n_kv_heads) * 128;
  switch (j) {
    case 0: return {qkv_w, p.hidden, p.qkv_split};
    case 1: return {p.hidden, p.n_heads * 128, p.o_split};
    case 2: return {2 * p.ffn, p.hidden, 0};
    default: return {p.hidden, p.ffn, p.dn_split};
  }
}
// this CTA's segments of job j (at most 3)
__device__ int fused_segs(const FusedParams& p, int j, int c, FSeg* s) {
  const FJob J = fused_job(p, j);
  const int tiles = J.n / 128, kb = J.k / 64;
  if (J.split > 0) {
    if (c >= tiles * J.split) return 0;
    const int t = c / J.split, sp = c % J.split;
    const int k0 = (sp * kb) / J.split, k1 = ((sp + 1) * kb) / J.split;
    s[0] = {t, k0, k1 - k0};
    return k1 > k0 ? 1 : 0;
  }
  const long long U = static_cast<long long>(tiles) * kb;
  long long u = (static_cast<long long>(c) * U) / p.grid;
  const long long u1 = (static_cast<long long>(c + 1) * U) / p.grid;
  int n = 0;
  while (u < u1 && n < 3) {
    const int t = static_cast<int>(u / kb), k0 = static_cast<int>(u % kb);
    const int len = static_cast<int>(min(static_cast<long long>(kb - k0), u1 - u));
    s[n++] = {t, k0, len};
    u += len;
  }
  return n;
}
// walks a CTA's (layer, projection, segment, k-block) units in stream order
struct UnitCursor {
  int l, j, q, k, ns;
  FSeg sg[3];
  __device__ __forceinline__ void skip_empty(const FusedParams& p, int c) {
    while (l < p.layers && q >= ns) {
      if (++j == kFusedJobs) {
        j = 0;
        ++l;
      }
      if (l < p.layers) {
        ns = fused_segs(p, j, c, sg);
        q = 0;
        k = 0;
      }
    }
  }
  __device__ __forceinline__ void init(const FusedParams& p, int c) {
    l = 0;
    j = 0;
    q = 0;
    k = 0;
    ns = fused_segs(p, 0, c, sg);
    skip_empty(p, c);
  }
  __device__ __forceinline__ bool valid(const FusedParams& p) const { return l < p.layers; }
  __device__ __forceinline__ void next(const FusedParams& p, int c) {
    if (++k >= sg[q].len) {
      k = 0;
      ++q;
      skip_empty(p, c);
    }
  }
};

__device__ __forceinline__ void l2_prefetch_tile(const void* tmap, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(tmap), "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ int gu_cta_of(long long u, long long U, int G) {
  return static_cast<int>(((u + 1) * G - 1) / U);
}
__device__ __forceinline__ long long gu_u0(int c, long long U, int G) { return (static_cast<long long>(c) * U) / G; }

// ------------------------------------------------------------------ glue phases
// Row norms are spread over the CTAs: ns slices per row (ns = grid / rows,
// at most 8), one 8-wide vector per thread.
__device__ __forceinline__ int norm_slices(int n_rows, int G) {
  int ns = G / n_rows;
  return ns < 1 ? 1 : (ns > 8 ? 8 : ns);
}

// residual add of a split-K projection + RMSNorm of one slice of one row
// (256 threads).  The slices' sums of squares meet in `ssbuf` (per-row
// arrival counter `rowcnt`, summed in slice order: deterministic).  First
// layer: the row is the token's embedding.  Numerics as
// residual_rmsnorm_kernel: h = bf16(h + bf16(sum of partials)).
template <int TPAD>
__device__ bool fused_norm_slice(const FusedParams& p, int row, int slice, int ns, const float* part, int split,
                                 const __nv_bfloat16* w, __nv_bfloat16* out, __nv_bfloat16* capture, bool embed_row,
                                 int ct, float* red, uint32_t* rowcnt, uint32_t* abort_word) {
  const int H = p.hidden, nv = H / 8;
  const int v0 = (slice * nv) / ns, v1 = ((slice + 1) * nv) / ns;
  const int i = v0 + ct;
  const bool act = i < v1;
  __nv_bfloat16* hrow = p.h + static_cast<size_t>(row) * H;
  uint4 o = make_uint4(0, 0, 0, 0);
  float ss = 0.0f;
  if (act) {
    if (embed_row) {
      int tok = p.tokens[row];
      if (tok < 0 || tok >= p.vocab) {
        dev_error(0x2002u);
        tok = 0;
      }
      o = reinterpret_cast<const uint4*>(p.embed + static_cast<size_t>(tok) * H)[i];
    } else {
      const uint4 h0 = __ldcg(reinterpret_cast<const uint4*>(hrow) + i);
      float y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = 0.0f;
      float4 a[8], b[8];  // every split's loads in flight at once (split <= 8)
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        if (s < split) {
          const float4* pp = reinterpret_cast<const float4*>(part + (static_cast<size_t>(s) * TPAD + row) * H) + 2 * i;
          a[s] = __ldcg(pp);
          b[s] = __ldcg(pp + 1);
        }
      }
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        if (s < split) {
          y[0] += a[s].x; y[1] += a[s].y; y[2] += a[s].z; y[3] += a[s].w;
          y[4] += b[s].x; y[5] += b[s].y; y[6] += b[s].z; y[7] += b[s].w;
        }
      }
      const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&h0);
      __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(hb[q]);
        ob[q] = __floats2bfloat162_rn(f.x + bf16_round(y[2 * q]), f.y + bf16_round(y[2 * q + 1]));
      }
    }
    const __nv_bfloat162* ob = reinterpret_cast<const __nv_bfloat162*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 g = __bfloat1622float2(ob[q]);
      ss += g.x * g.x + g.y * g.y;
    }
    reinterpret_cast<uint4*>(hrow)[i] = o;
    if (capture) reinterpret_cast<uint4*>(capture + static_cast<size_t>(row) * p.ldc)[i] = o;
  }
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((ct & 31) == 0) red[ct >> 5] = ss;
  cbar();
  bool ok = true;
  if (ct == 0) {
    float t = 0.0f;
#pragma unroll
    for (int k = 0; k < kFusedWarpsCompute; ++k) t += red[k];
    p.norm_ss[row * 8 + slice] = t;
    red_release_add(&rowcnt[row], 1u);
    ok = wait_count(&rowcnt[row], static_cast<uint32_t>(ns), abort_word, 0x30);
  }
  if (!cbar_and(ok)) return false;
  float tot = 0.0f;
  for (int k = 0; k < ns; ++k) tot += __ldcg(p.norm_ss + row * 8 + k);
  const float rs = rsqrtf(tot / static_cast<float>(H) + p.eps);
  if (act) {
    const uint4 wv = reinterpret_cast<const uint4*>(w)[i];
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&o);
    const __nv_bfloat162* wb = reinterpret_cast<const __nv_bfloat162*>(&wv);
    uint4 o4;
    __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o4);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __bfloat1622float2(b[q]);
      const float2 g = __bfloat1622float2(wb[q]);
      ob[q] = __floats2bfloat162_rn(f.x * rs * g.x, f.y * rs * g.y);
    }
    reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * H)[i] = o4;
  }
  return true;
}

// q/k RMSNorm + RoPE (q -> buffer, k -> cache) or v -> cache for one (row,
// head): one warp, 4 features per lane.  Numerics as qkv_finish_kernel.
template <int TPAD>
__device__ void fused_fin_item(const FusedParams& p, int l, int t, int gh, int start, int lane) {
  const int Hq = p.n_heads, Hkv = p.n_kv_heads;
  const int W = (Hq + 2 * Hkv) * 128;
  const int d0 = 4 * lane;
  float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  {
    float4 x[8];
#pragma unroll
    for (int s = 0; s < 8; ++s)
      if (s < p.qkv_split)
        x[s] = __ldcg(reinterpret_cast<const float4*>(p.qkv_part + (static_cast<size_t>(s) * TPAD + t) * W +
                                                      gh * 128 + d0));
#pragma unroll
    for (int s = 0; s < 8; ++s)
      if (s < p.qkv_split) {
        a[0] += x[s].x; a[1] += x[s].y; a[2] += x[s].z; a[3] += x[s].w;
      }
  }
  const int slot = start + t;
  const size_t plane = static_cast<size_t>(Hkv) * p.kv_cap * 128;
  __nv_bfloat16* kl = p.kv + static_cast<size_t>(l) * 2 * plane;
  auto store4 = [](__nv_bfloat16* dst, const float (&v)[4]) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]), hi = __floats2bfloat162_rn(v[2], v[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&lo);
    u.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(dst) = u;
  };
  if (gh >= Hq + Hkv) {  // v
    const int kvh = gh - Hq - Hkv;
    if (slot >= 0 && slot < p.kv_cap) store4(kl + plane + (static_cast<size_t>(kvh) * p.kv_cap + slot) * 128 + d0, a);
    else if (lane == 0) dev_error(0x2001u);
    return;
  }
  const bool is_q = gh < Hq;
  const __nv_bfloat16* nwp = (is_q ? p.lp[l].q_norm : p.lp[l].k_norm) + d0;
  float x[4], sq = 0.0f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    x[e] = bf16_round(a[e]);
    sq += x[e] * x[e];
  }
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float rms = rsqrtf(sq / 128.0f + p.eps);
  const float pos = static_cast<float>(p.positions[t]);
  float y[4], out[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) y[e] = bf16_round(x[e] * rms * __bfloat162float(nwp[e]));
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int d = d0 + e;
    const float yp = __shfl_xor_sync(0xffffffffu, y[e], 16);  // feature d +- 64
    const int i_f = d & 63;
    const float inv_freq = exp2f(-(2.0f * static_cast<float>(i_f) / 128.0f) * p.rope_log2_theta);
    float sn, cs;
    sincosf(pos * inv_freq, &sn, &cs);
    out[e] = d < 64 ? (y[e] * cs - yp * sn) : (y[e] * cs + yp * sn);
  }
  if (is_q) {
    store4(p.q + static_cast<size_t>(t) * (Hq * 128) + gh * 128 + d0, out);
  } else {
    const int kvh = gh - Hq;
    if (slot >= 0 && slot < p.kv_cap) store4(kl + (static_cast<size_t>(kvh) * p.kv_cap + slot) * 128 + d0, out);
    else if (lane == 0) dev_error(0x2001u);
  }
}

__device__ __forceinline__ void f_cp_async16(void* smem, const void* gmem, bool pred) {
  const uint32_t s = smem_u32(smem);
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(sz) : "memory");
}
__device__ __forceinline__ void f_ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void f_ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void f_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t f_pack(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ int att_kps(int L, int splits) {
  int kps = (L + splits - 1) / splits;
  if (kps < 2 * kAttChunk) kps = 2 * kAttChunk;
  return ((kps + kAttChunk - 1) / kAttChunk) * kAttChunk;
}

// split-KV tree attention of one (kv head, row block, key split): 128 query
// rows per task (row r -> q head kvh*G + r / T, node r % T); warp cw owns
// rows 16*cw .. +15.  32-key chunks of K / V through shared memory (double
// buffered), bf16 mma.sync with an fp32 online softmax.  Visibility: every
// prefix key, and tree slot j iff bit j of the node's ancestor mask
// (dtree_runtime.py:190-191).  Writes (m, l, unnormalised O).
constexpr int kAttRows = 128;
__device__ void fused_att_task(const FusedParams& p, int l, int kvh, int rbi, int sp, int P, int cw, int lane, int ct,
                               uint8_t* sm) {
  const int T = p.n_rows, G = p.n_heads / p.n_kv_heads;
  const int rows_kv = G * T;
  const int L = P + T;
  const int kps = att_kps(L, p.att_splits);
  const int k_begin = sp * kps;
  if (k_begin >= L) return;  // uniform over the CTA
  const int k_end = min(min(L, k_begin + kps), p.kv_cap);  // (P + T > kv_cap is flagged by the K/V write)
  const int n_chunks = (k_end - k_begin + kAttChunk - 1) / kAttChunk;
  const size_t plane = static_cast<size_t>(p.n_kv_heads) * p.kv_cap * 128;
  const __nv_bfloat16* kpl = p.kv + static_cast<size_t>(l) * 2 * plane + static_cast<size_t>(kvh) * p.kv_cap * 128;
  const __nv_bfloat16* vpl = kpl + plane;
  const int rgrp = cw;

  // this thread's rows: lane/4 and lane/4 + 8 of the warp's 16
  int node[2], qh[2];
  bool rok[2];
  uint64_t a0[2], a1[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int rg = rbi * kAttRows + rgrp * 16 + (lane >> 2) + h * 8;
    rok[h] = rg < rows_kv;
    node[h] = rok[h] ? rg % T : 0;
    qh[h] = kvh * G + (rok[h] ? rg / T : 0);
    a0[h] = rok[h] ? p.anc[2 * node[h]] : 0ull;
    a1[h] = rok[h] ? p.anc[2 * node[h] + 1] : 0ull;
  }
  // Q fragments straight from global (A layout of m16n8k16)
  uint32_t qf[8][4];
  {
    const int c2 = 2 * (lane & 3);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const __nv_bfloat16* qp = p.q + static_cast<size_t>(node[h]) * (p.n_heads * 128) + qh[h] * 128 + kk * 16 + c2;
        // (q is rewritten every layer by other CTAs: read through L2)
        qf[kk][h] = rok[h] ? __ldcg(reinterpret_cast<const unsigned int*>(qp)) : 0u;
        qf[kk][2 + h] = rok[h] ? __ldcg(reinterpret_cast<const unsigned int*>(qp + 8)) : 0u;
      }
    }
  }
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};

  // 32-key chunks of K and V, double buffered: chunk c + 1 loads while c computes
  auto load_chunk = [&](int c, int buf) {
    const int key0 = k_begin + c * kAttChunk;
    __nv_bfloat16* sk = reinterpret_cast<__nv_bfloat16*>(sm + buf * kAttStage);
    __nv_bfloat16* sv = sk + kAttChunk * kAttLd;
    for (int e = ct; e < kAttChunk * 16; e += 256) {
      const int r = e >> 4, v = e & 15;
      const int key = key0 + r;
      const bool ok = key < k_end;
      const size_t off = static_cast<size_t>(ok ? key : 0) * 128 + v * 8;
      f_cp_async16(sk + r * kAttLd + v * 8, kpl + off, ok);
      f_cp_async16(sv + r * kAttLd + v * 8, vpl + off, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  load_chunk(0, 0);
#pragma unroll 1
  for (int c = 0; c < n_chunks; ++c) {
    const int key0 = k_begin + c * kAttChunk;
    if (c + 1 < n_chunks) {
      load_chunk(c + 1, (c + 1) & 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    cbar();
    const __nv_bfloat16* sk = reinterpret_cast<const __nv_bfloat16*>(sm + (c & 1) * kAttStage);
    const __nv_bfloat16* sv = sk + kAttChunk * kAttLd;
    {
      constexpr int kb0 = 0;
      float s[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
        for (int kk = 0; kk < 8; kk += 2) {
          uint32_t b[4];
          const int mi = lane >> 3, i = lane & 7;
          f_ldsm_x4(b, sk + (kb0 + nt * 8 + i) * kAttLd + kk * 16 + 8 * mi);
          f_mma(s[nt], qf[kk], b[0], b[1]);
          f_mma(s[nt], qf[kk + 1], b[2], b[3]);
        }
      }
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = e >> 1;
          const int key = key0 + kb0 + nt * 8 + 2 * (lane & 3) + (e & 1);
          bool vis = rok[h] && key < k_end;
          if (vis && key >= P) {
            const int j = key - P;
            vis = ((j < 64 ? (a0[h] >> j) : (a1[h] >> (j - 64))) & 1ull) != 0ull;
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
      uint32_t pf[2][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const float p0 = exp2f(s[nt][0] - mx[0]), p1 = exp2f(s[nt][1] - mx[0]);
        const float p2 = exp2f(s[nt][2] - mx[1]), p3 = exp2f(s[nt][3] - mx[1]);
        rs[0] += p0 + p1;
        rs[1] += p2 + p3;
        pf[nt >> 1][(nt & 1) * 2 + 0] = f_pack(p0, p1);
        pf[nt >> 1][(nt & 1) * 2 + 1] = f_pack(p2, p3);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
        rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
        l_run[h] = l_run[h] * alpha[h] + rs[h];
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= alpha[0];
        o[j][1] *= alpha[0];
        o[j][2] *= alpha[1];
        o[j][3] *= alpha[1];
      }
#pragma unroll
      for (int kt = 0; kt < 2; ++kt) {
#pragma unroll
        for (int nt = 0; nt < 16; nt += 2) {
          uint32_t b[4];
          const int mi = lane >> 3, i = lane & 7;
          f_ldsm_x4_t(b, sv + (kb0 + kt * 16 + i + 8 * (mi & 1)) * kAttLd + nt * 8 + 8 * (mi >> 1));
          f_mma(o[nt], pf[kt], b[0], b[1]);
          f_mma(o[nt + 1], pf[kt], b[2], b[3]);
        }
      }
    }
    cbar();  // buffer c & 1 is refilled by the next iteration's prefetch
  }
  const int rows_total = p.n_heads * T;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (!rok[h]) continue;
    const int qrow = qh[h] * T + node[h];
    float* po = p.att_o + (static_cast<size_t>(sp) * rows_total + qrow) * 128;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int d = j * 8 + 2 * (lane & 3);
      *reinterpret_cast<float2*>(po + d) = make_float2(o[j][2 * h], o[j][2 * h + 1]);
    }
    if ((lane & 3) == 0) {
      float* pml = p.att_ml + (static_cast<size_t>(sp) * rows_total + qrow) * 2;
      pml[0] = m_run[h];
      pml[1] = l_run[h];
    }
  }
}

// log-sum-exp merge of the key splits for one (row, q head): one warp
__device__ void fused_cmb_item(const FusedParams& p, int t, int head, int P, int lane) {
  const int T = p.n_rows;
  const int rows_total = p.n_heads * T;
  const int qrow = head * T + t;
  const int L = P + T;
  const int kps = att_kps(L, p.att_splits);
  const int active = min(p.att_splits, (L + kps - 1) / kps);
  float m = -INFINITY, lv = 0.0f;
  if (lane < active) {
    const size_t r = static_cast<size_t>(lane) * rows_total + qrow;
    m = __ldcg(p.att_ml + r * 2);
    lv = __ldcg(p.att_ml + r * 2 + 1);
  }
  float M = m;
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  const float m_use = (M == -INFINITY) ? 0.0f : M;
  const float w = lane < active ? exp2f(m - m_use) : 0.0f;
  const float wl = w * lv;
  float Ls = 0.0f;
  for (int s = 0; s < active; ++s) Ls += __shfl_sync(0xffffffffu, wl, s);  // split order: deterministic
  const float inv = Ls > 0.0f ? 1.0f / Ls : 0.0f;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int s0 = 0; s0 < active; s0 += 8) {
    float4 v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (s0 + k < active)
        v[k] = __ldcg(reinterpret_cast<const float4*>(p.att_o + (static_cast<size_t>(s0 + k) * rows_total + qrow) * 128) +
                      lane);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float ws = __shfl_sync(0xffffffffu, w, (s0 + k) & 31);
      if (s0 + k < active) {
        acc[0] += ws * v[k].x;
        acc[1] += ws * v[k].y;
        acc[2] += ws * v[k].z;
        acc[3] += ws * v[k].w;
      }
    }
  }
  __nv_bfloat162 lo = __floats2bfloat162_rn(acc[0] * inv, acc[1] * inv);
  __nv_bfloat162 hi = __floats2bfloat162_rn(acc[2] * inv, acc[3] * inv);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&lo);
  u.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p.attn + static_cast<size_t>(t) * (p.n_heads * 128) + head * 128 + 4 * lane) = u;
}

// ------------------------------------------------------------------ kernel
template <int TPAD>
__global__ void __launch_bounds__(kFusedThreads, 1)
    fused_verify_kernel(const __grid_constant__ CUtensorMap xm_xn, const __grid_constant__ CUtensorMap xm_attn,
                        const __grid_constant__ CUtensorMap xm_act, const __grid_constant__ FusedParams p) {
  using C = FusedCfg<TPAD>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* att_sm = smem + S * C::kStageBytes;  // attention K/V chunk; SwiGLU exchange (disjoint in time)
  uint8_t* misc = att_sm + kAttBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(misc);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* tfull = empty_bar + S;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  float* red = reinterpret_cast<float*>(tmem_slot + 4);  // [8]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const int G = p.grid;
  uint32_t* abort_word = p.cnt + p.layers * kCntPerLayer;
  auto cnt = [&](int l, int k) { return p.cnt + l * kCntPerLayer + k; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 2);  // weight producer + activation producer
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kFusedWarpsCompute);
    }
    fence_barrier_init();
    tma_prefetch_desc(&xm_xn);
    tma_prefetch_desc(&xm_attn);
    tma_prefetch_desc(&xm_act);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int start = p.state->start;

  if (warp == 0) {
    // ---------------------------------------------------------------- weights
    // TMA loads fill the ring as slots free up; L2 prefetches of the units
    // after the ring run kFusedL2Ahead units further ahead, so the stream
    // keeps DRAM busy while the ring is full and the glue phases run.
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      long long i = 0, ipf = 0;
      UnitCursor cur, pf;
      cur.init(p, c);
      pf.init(p, c);
      while (cur.valid(p) && ok) {
        while (pf.valid(p) && ipf < i + S + kFusedL2Ahead) {
          if (ipf >= i + S)
            l2_prefetch_tile(p.wmaps + pf.l * kFusedJobs + pf.j, (pf.sg[pf.q].kb0 + pf.k) * 64, pf.sg[pf.q].tile * 128);
          pf.next(p, c);
          ++ipf;
        }
        if (i >= S) {
          ok = mbar_wait_ab(&empty_bar[s], ph ^ 1u, abort_word, 1);
          if (!ok) break;
        }
        mbar_arrive_expect_tx(&full_bar[s], C::kWBytes);
        tma_load_2d(stages + s * C::kStageBytes, p.wmaps + cur.l * kFusedJobs + cur.j, &full_bar[s],
                    (cur.sg[cur.q].kb0 + cur.k) * 64, cur.sg[cur.q].tile * 128, pol);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
        cur.next(p, c);
        ++i;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- activations
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      long long i = 0;
      for (int l = 0; l < p.layers && ok; ++l) {
        for (int j = 0; j < kFusedJobs && ok; ++j) {
          FSeg sg[3];
          const int ns = fused_segs(p, j, c, sg);
          if (ns == 0) continue;
          // the projection's input is complete
          const uint32_t* wc = j == 0 ? cnt(l, kCntN1) : j == 1 ? cnt(l, kCntCmb) : j == 2 ? cnt(l, kCntN2)
                                                                                          : cnt(l, kCntGu);
          const uint32_t target = (j == 0 || j == 2) ? static_cast<uint32_t>(p.n_rows * norm_slices(p.n_rows, G))
                                                     : static_cast<uint32_t>(G);
          ok = wait_count(wc, target, abort_word, 0x10 + j);
          if (!ok) break;
          fence_proxy_async_global();  // generic-proxy writes of other CTAs -> this thread's TMA reads
          const CUtensorMap* xm = (j == 0 || j == 2) ? &xm_xn : (j == 1 ? &xm_attn : &xm_act);
          for (int q = 0; q < ns && ok; ++q) {
            for (int k = 0; k < sg[q].len; ++k, ++i) {
              if (i >= S) {
                ok = mbar_wait_ab(&empty_bar[s], ph ^ 1u, abort_word, 2);
                if (!ok) break;
              }
              mbar_arrive_expect_tx(&full_bar[s], C::kXBytes);
              tma_load_2d(stages + s * C::kStageBytes + C::kWBytes, xm, &full_bar[s], (sg[q].kb0 + k) * 64, 0, pol);
              if (++s == S) {
                s = 0;
                ph ^= 1u;
              }
            }
          }
        }
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint64_t a_base = sw128_kmajor_desc(smem_u32(stages));
      const uint64_t b_base = sw128_kmajor_desc(smem_u32(stages + C::kWBytes));
      int s = 0, seg = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int l = 0; l < p.layers && ok; ++l) {
        for (int j = 0; j < kFusedJobs && ok; ++j) {
          FSeg sg[3];
          const int ns = fused_segs(p, j, c, sg);
          for (int q = 0; q < ns && ok; ++q, ++seg) {
            const int b = seg & 1, use = seg >> 1;
            if (use >= 1) ok = mbar_wait_ab(&tempty[b], static_cast<uint32_t>(use - 1) & 1u, abort_word, 3);
            if (!ok) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * TPAD);
            for (int k = 0; k < sg[q].len; ++k) {
              ok = mbar_wait_ab(&full_bar[s], ph, abort_word, 4);
              if (!ok) break;
              tc_fence_after();
              const uint64_t off = static_cast<uint64_t>((s * C::kStageBytes) >> 4);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                umma_bf16(d_tmem, a_base + off + kk * 2, b_base + off + kk * 2, C::kIdesc, (k > 0 || kk > 0) ? 1u : 0u);
              umma_commit(&empty_bar[s]);
              if (++s == S) {
                s = 0;
                ph ^= 1u;
              }
            }
            if (ok) umma_commit(&tfull[b]);
          }
        }
      }
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- compute
    const int ct = threadIdx.x - 128;  // 0..255
    const int cw = warp - 4;           // 0..7
    const int qd = warp & 3;           // TMEM lane quarter
    const int g = cw >> 2;             // column half of the accumulator
    const int row = qd * 32 + lane;    // accumulator row (weight row of the tile)
    constexpr int HC = TPAD / 2;       // columns per half
    const int NH = p.n_heads + 2 * p.n_kv_heads;
    const int Hkv = p.n_kv_heads;
    const int tasks_att = Hkv * p.att_rb * p.att_splits;
    int seg = 0;
    bool ok = true;
    float* xch = reinterpret_cast<float*>(att_sm) + g * (128 * 8);  // [8][128] per half

    // split-K epilogue of job j: fp32 partials [split][TPAD][N]
    auto epi_split = [&](int j, float* out) {
      FSeg sg[3];
      const int ns = fused_segs(p, j, c, sg);
      const FJob J = fused_job(p, j);
      for (int q = 0; q < ns && ok; ++q, ++seg) {
        const int b = seg & 1, use = seg >> 1;
        bool w_ok = true;
        if (ct == 0) w_ok = mbar_wait_ab(&tfull[b], static_cast<uint32_t>(use) & 1u, abort_word, 5);
        ok = cbar_and(w_ok);
        if (!ok) break;
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(qd * 32) << 16) + static_cast<uint32_t>(b * TPAD);
        const int n = sg[q].tile * 128 + row;
        float* o = out + static_cast<size_t>(c % J.split) * TPAD * J.n + n;
#pragma unroll
        for (int c0 = g * HC; c0 < (g + 1) * HC; c0 += 8) {
          uint32_t r[8];
          tmem_ld_x8(taddr + c0, r);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (c0 + e < p.n_rows) o[static_cast<size_t>(c0 + e) * J.n] = __uint_as_float(r[e]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
      }
    };

    // Steps 2l (attention half of layer l) and 2l + 1 (MLP half) each start
    // with a residual add + RMSNorm; step 2L is the final norm.  The norm
    // has one call site (inlined once).
    for (int step = 0; step <= 2 * p.layers && ok; ++step) {
      const int l = step >> 1, half = step & 1;
      {
        const uint32_t* wc;
        const float* part;
        int split;
        const __nv_bfloat16* w;
        __nv_bfloat16* out;
        __nv_bfloat16* cap;
        uint32_t* sig;
        if (half == 0) {  // N1 of layer l (NF after the last layer): h += down(l-1)
          wc = l > 0 ? cnt(l - 1, kCntDn) : nullptr;
          part = p.dn_part;
          split = p.dn_split;
          w = l < p.layers ? p.lp[l].input_norm : p.final_norm;
          out = l < p.layers ? p.xn : p.norm_out;
          cap = l > 0 ? p.lp[l - 1].capture : nullptr;  // verifier_hidden of layer l-1
          sig = l < p.layers ? cnt(l, kCntN1) : nullptr;
        } else {  // N2: h += o_proj(l)
          wc = cnt(l, kCntO);
          part = p.o_part;
          split = p.o_split;
          w = p.lp[l].post_norm;
          out = p.xn;
          cap = nullptr;
          sig = cnt(l, kCntN2);
        }
        if (wc) ok = cwait(wc, static_cast<uint32_t>(G), abort_word, 0x20 + half, ct);
        if (!ok) break;
        const int ns = norm_slices(p.n_rows, G);
        if (c < p.n_rows * ns) {
          ok = fused_norm_slice<TPAD>(p, c / ns, c % ns, ns, part, split, w, out, cap, step == 0, ct, red,
                                      p.norm_cnt + step * 64, abort_word);
          if (!ok) break;
          if (sig) csignal(sig, ct);
        }
      }
      if (l == p.layers) break;
      if (half == 0) {
      // ---- q|k|v projection epilogue
      epi_split(0, p.qkv_part);
      if (!ok) break;
      csignal(cnt(l, kCntQkv), ct);
      // prefix keys of this CTA's attention task into L2 while the projections finish
      if (c < tasks_att && ct == 0) {
        const int sp = c % p.att_splits;
        const int kvh = c / (p.att_rb * p.att_splits);
        const int kps = att_kps(start + p.n_rows, p.att_splits);
        const int lo = sp * kps, hi = min(min(start, lo + kps), p.kv_cap);
        if (hi > lo) {
          const size_t plane = static_cast<size_t>(Hkv) * p.kv_cap * 128;
          const __nv_bfloat16* kpl = p.kv + static_cast<size_t>(l) * 2 * plane + static_cast<size_t>(kvh) * p.kv_cap * 128;
          const uint32_t bytes = static_cast<uint32_t>(hi - lo) * 256;
          l2_prefetch_bulk(kpl + static_cast<size_t>(lo) * 128, bytes);
          l2_prefetch_bulk(kpl + plane + static_cast<size_t>(lo) * 128, bytes);
        }
      }
      // ---- FIN: q/k RMSNorm + RoPE, K/V -> cache
      ok = cwait(cnt(l, kCntQkv), static_cast<uint32_t>(G), abort_word, 0x21, ct);
      if (!ok) break;
      for (int it = c * kFusedWarpsCompute + cw; it < p.n_rows * NH; it += G * kFusedWarpsCompute)
        fused_fin_item<TPAD>(p, l, it / NH, it % NH, start, lane);
      csignal(cnt(l, kCntFin), ct);
      // ---- ATT
      ok = cwait(cnt(l, kCntFin), static_cast<uint32_t>(G), abort_word, 0x22, ct);
      if (!ok) break;
      for (int task = c; task < tasks_att; task += G) {
        const int kvh = task / (p.att_rb * p.att_splits);
        const int rem = task % (p.att_rb * p.att_splits);
        fused_att_task(p, l, kvh, rem / p.att_splits, rem % p.att_splits, start, cw, lane, ct, att_sm);
      }
      csignal(cnt(l, kCntAtt), ct);
      // ---- CMB
      ok = cwait(cnt(l, kCntAtt), static_cast<uint32_t>(G), abort_word, 0x23, ct);
      if (!ok) break;
      for (int it = c * kFusedWarpsCompute + cw; it < p.n_rows * p.n_heads; it += G * kFusedWarpsCompute)
        fused_cmb_item(p, it / p.n_heads, it % p.n_heads, start, lane);
      csignal(cnt(l, kCntCmb), ct);
      // ---- o_proj epilogue
      epi_split(1, p.o_part);
      if (!ok) break;
      csignal(cnt(l, kCntO), ct);
      } else {
      // ---- gate|up epilogue (stream-K) + SwiGLU -> act
      {
        FSeg sg[3];
        const int ns = fused_segs(p, 2, c, sg);
        const FJob J = fused_job(p, 2);
        const int kb = J.k / 64;
        const long long U = static_cast<long long>(J.n / 128) * kb;
        const int first_tile = ns > 0 ? sg[0].tile : 0;
        for (int q = 0; q < ns && ok; ++q, ++seg) {
          const int b = seg & 1, use = seg >> 1;
          bool w_ok = true;
          if (ct == 0) w_ok = mbar_wait_ab(&tfull[b], static_cast<uint32_t>(use) & 1u, abort_word, 6);
          ok = cbar_and(w_ok);
          if (!ok) break;
          tc_fence_after();
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(qd * 32) << 16) + static_cast<uint32_t>(b * TPAD);
          const int tile = sg[q].tile;
          const bool full = sg[q].kb0 == 0 && sg[q].len == kb;
          bool have = true;
          int c_first = c, c_last = c;
          if (!full) {
            const int which = tile == first_tile ? 0 : 1;
            float* slot = p.gu_ws + (static_cast<size_t>(c) * 2 + which) * TPAD * 128;
#pragma unroll
            for (int c0 = g * HC; c0 < (g + 1) * HC; c0 += 8) {
              uint32_t r[8];
              tmem_ld_x8(taddr + c0, r);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 8; ++e)
                if (c0 + e < p.n_rows) slot[(c0 + e) * 128 + row] = __uint_as_float(r[e]);
            }
            cbar();  // the partial is written (ordered before thread 0's release below)
            c_first = gu_cta_of(static_cast<long long>(tile) * kb, U, G);
            c_last = gu_cta_of(static_cast<long long>(tile) * kb + kb - 1, U, G);
            bool last = false;
            if (ct == 0) {
              uint32_t prev;
              asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(&p.gu_tile_cnt[tile])
                           : "memory");
              last = prev == static_cast<uint32_t>(c_last - c_first);
              if (last) p.gu_tile_cnt[tile] = 0u;  // every contributor has arrived: reset for the next layer
            }
            have = cbar_or(last);
          }
          if (have) {
#pragma unroll 1
            for (int c0 = g * HC; c0 < (g + 1) * HC; c0 += 8) {
              float a[8];
              if (full) {
                uint32_t r[8];
                tmem_ld_x8(taddr + c0, r);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 8; ++e) a[e] = __uint_as_float(r[e]);
              } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) a[e] = 0.0f;
                for (int cb = c_first; cb <= c_last; cb += 4) {  // four contributors' loads in flight
                  float v[4][8];
#pragma unroll
                  for (int k2 = 0; k2 < 4; ++k2) {
                    const int cc = cb + k2;
                    if (cc <= c_last) {
                      const int w2 = (tile == static_cast<int>(gu_u0(cc, U, G) / kb)) ? 0 : 1;
                      const float* sl = p.gu_ws + (static_cast<size_t>(cc) * 2 + w2) * TPAD * 128 + c0 * 128 + row;
#pragma unroll
                      for (int e = 0; e < 8; ++e) v[k2][e] = __ldcg(sl + e * 128);
                    }
                  }
#pragma unroll
                  for (int k2 = 0; k2 < 4; ++k2)
                    if (cb + k2 <= c_last) {
#pragma unroll
                      for (int e = 0; e < 8; ++e) a[e] += v[k2][e];
                    }
                }
              }
              if (row >= 64) {
#pragma unroll
                for (int e = 0; e < 8; ++e) xch[e * 128 + row] = a[e];
              }
              gbar(g);
              if (row < 64) {
                const int jf = tile * 64 + row;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  const int t = c0 + e;
                  const float gt = bf16_round(a[e]);
                  const float uu = bf16_round(xch[e * 128 + row + 64]);
                  const float sg2 = bf16_round(__fdividef(1.0f, 1.0f + __expf(-gt)));  // as the GEMM epilogue
                  const float sl = bf16_round(gt * sg2);
                  if (t < p.n_rows) p.act[static_cast<size_t>(t) * p.ffn + jf] = __float2bfloat16_rn(sl * uu);
                }
              }
              gbar(g);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[b]);
        }
        if (!ok) break;
        csignal(cnt(l, kCntGu), ct);
      }
      // ---- down_proj epilogue
      epi_split(3, p.dn_part);
      if (!ok) break;
      csignal(cnt(l, kCntDn), ct);
      }
    }
  }
  if (threadIdx.x == 0 && ld_relaxed(abort_word)) {
    // aborted: let every TMA load and MMA already issued land before the
    // CTA's shared and tensor memory are released
    const uint64_t t0 = gtimer();
    while (gtimer() - t0 < 200000ull) __nanosleep(1000);
  }
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ host
static int qkv_width(const dtree_qwen3_desc& d) { return (d.n_heads + 2 * d.n_kv_heads) * d.head_dim; }
static int fused_tpad_max(const dtree_qwen3_desc& d) {
  return d.t_cap <= 16 ? 16 : (d.t_cap <= 32 ? 32 : 64);
}

bool fused_supported(const dtree_qwen3_desc& d) {
  if (d.quant_bits == 4) return false;
  if (d.head_dim != 128) return false;
  if (d.hidden % 128 != 0 || d.ffn % 64 != 0 || (2 * d.ffn) % 128 != 0 || d.hidden > 4096) return false;
  if (d.layers < 1 || d.layers > kFusedMaxLayers) return false;
  if (d.n_heads % d.n_kv_heads != 0) return false;
  // a CTA's stream-K range of gate|up units spans at most three tiles
  const long long gu_units = static_cast<long long>(2 * d.ffn / 128) * (d.hidden / 64);
  if ((gu_units + num_sms() - 1) / num_sms() > d.hidden / 64 + 2) return false;
  return true;
}

// phase counters, the abort word, then per-(norm step, row) arrival counters
static size_t fused_cnt_words(int layers) {
  return static_cast<size_t>(layers) * kCntPerLayer + 8 + static_cast<size_t>(2 * layers + 1) * 64;
}

struct FusedLayout {
  size_t maps, lp, cnt, norm_ss, qkv_part, o_part, dn_part, gu_ws, gu_cnt, att_o, att_ml, total;
  int qkv_split, o_split, dn_split, att_splits, att_rb, grid;
};

static int fused_split(int tiles, int kb, int grid) {
  int s = grid / tiles;
  if (s < 1) s = 1;
  if (s > 8) s = 8;
  if (s > kb) s = kb;
  return s;
}

static FusedLayout fused_layout(const dtree_qwen3_desc& d, int t_pad) {
  FusedLayout L{};
  const int G = num_sms();
  L.grid = G;
  L.qkv_split = fused_split(qkv_width(d) / 128, d.hidden / 64, G);
  L.o_split = fused_split(d.hidden / 128, d.n_heads * 2, G);
  L.dn_split = fused_split(d.hidden / 128, d.ffn / 64, G);
  const int Gq = d.n_heads / d.n_kv_heads;
  L.att_rb = (Gq * t_pad + kAttRows - 1) / kAttRows;
  L.att_splits = std::max(1, std::min(32, G / (d.n_kv_heads * L.att_rb)));
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = (off + bytes + 255) & ~static_cast<size_t>(255);
    return o;
  };
  L.maps = take(static_cast<size_t>(d.layers) * kFusedJobs * sizeof(CUtensorMap));
  L.lp = take(static_cast<size_t>(d.layers) * sizeof(FusedLayerPtrs));
  L.cnt = take(fused_cnt_words(d.layers) * 4);
  L.norm_ss = take(64 * 8 * 4);
  L.qkv_part = take(static_cast<size_t>(L.qkv_split) * t_pad * qkv_width(d) * 4);
  L.o_part = take(static_cast<size_t>(L.o_split) * t_pad * d.hidden * 4);
  L.dn_part = take(static_cast<size_t>(L.dn_split) * t_pad * d.hidden * 4);
  L.gu_ws = take(static_cast<size_t>(G) * 2 * t_pad * 128 * 4);
  L.gu_cnt = take(static_cast<size_t>(2 * d.ffn / 128) * 4);
  // attention partials: room for the largest splits x rows of any t_pad up to this one
  size_t att_rows = 0;
  for (int tp = 16; tp <= t_pad; tp *= 2) {
    const int rb = (Gq * tp + kAttRows - 1) / kAttRows;
    const int sp = std::max(1, std::min(32, G / (d.n_kv_heads * rb)));
    att_rows = std::max(att_rows, static_cast<size_t>(sp) * tp);
  }
  L.att_o = take(att_rows * d.n_heads * 128 * 4);
  L.att_ml = take(att_rows * d.n_heads * 2 * 4);
  L.total = off;
  return L;
}

size_t fused_ws_bytes(const dtree_qwen3_desc& d) {
  if (d.verify_path != 1 || !fused_supported(d)) return 0;
  return fused_layout(d, fused_tpad_max(d)).total;
}

int fused_init(const dtree_qwen3_desc& d, void* ws, const std::pair<int, __nv_bfloat16*>* captures, int n_capture) {
  const FusedLayout L = fused_layout(d, fused_tpad_max(d));
  std::vector<CUtensorMap> maps(static_cast<size_t>(d.layers) * kFusedJobs);
  std::vector<FusedLayerPtrs> lp(d.layers);
  const int qd = d.n_heads * d.head_dim;
  for (int l = 0; l < d.layers; ++l) {
    const dtree_qwen3_layer& W = d.layer[l];
    const void* w[kFusedJobs] = {W.qkv, W.o_proj, W.gate_up, W.down};
    const int n[kFusedJobs] = {qkv_width(d), d.hidden, 2 * d.ffn, d.hidden};
    const int k[kFusedJobs] = {d.hidden, qd, d.hidden, d.ffn};
    for (int j = 0; j < kFusedJobs; ++j) {
      int rc = make_tmap_2d_bf16(&maps[static_cast<size_t>(l) * kFusedJobs + j], w[j], static_cast<uint64_t>(k[j]),
                                 static_cast<uint64_t>(n[j]), static_cast<uint64_t>(k[j]) * 2, 64, 128, true);
      if (rc) return rc;
    }
    lp[l].input_norm = static_cast<const __nv_bfloat16*>(W.input_norm);
    lp[l].q_norm = static_cast<const __nv_bfloat16*>(W.q_norm);
    lp[l].k_norm = static_cast<const __nv_bfloat16*>(W.k_norm);
    lp[l].post_norm = static_cast<const __nv_bfloat16*>(W.post_norm);
    lp[l].capture = nullptr;
    for (int i = 0; i < n_capture; ++i)
      if (captures[i].first == l) lp[l].capture = captures[i].second;
  }
  char* base = static_cast<char*>(ws);
  DTREE_CUDA_RET(cudaMemcpy(base + L.maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice));
  DTREE_CUDA_RET(cudaMemcpy(base + L.lp, lp.data(), lp.size() * sizeof(FusedLayerPtrs), cudaMemcpyHostToDevice));
  DTREE_CUDA_RET(cudaMemset(base + L.gu_cnt, 0, static_cast<size_t>(2 * d.ffn / 128) * 4));
  return kOk;
}

template <int TPAD>
static int fused_smem() {
  return FusedCfg<TPAD>::kSmem;
}

int fused_plan(const dtree_qwen3_desc& d, void* ws, int t_pad, FusedPlan* plan) {
  DTREE_CHECK_ARG(t_pad == 16 || t_pad == 32 || t_pad == 64, "fused verify: t_pad must be 16, 32 or 64");
  DTREE_CHECK_ARG(t_pad <= fused_tpad_max(d), "fused verify: t_pad above the model's t_cap");
  // the workspace is laid out for the largest t_pad; smaller ones use a prefix of each region
  const FusedLayout L = fused_layout(d, fused_tpad_max(d));
  const FusedLayout Lt = fused_layout(d, t_pad);
  char* base = static_cast<char*>(ws);
  int rc;
  if ((rc = make_tmap_2d_bf16(&plan->xmap_xn, d.xn, d.hidden, t_pad, static_cast<uint64_t>(d.hidden) * 2, 64, t_pad,
                              true)))
    return rc;
  if ((rc = make_tmap_2d_bf16(&plan->xmap_attn, d.attn, d.n_heads * 128, t_pad,
                              static_cast<uint64_t>(d.n_heads) * 256, 64, t_pad, true)))
    return rc;
  if ((rc = make_tmap_2d_bf16(&plan->xmap_act, d.act, d.ffn, t_pad, static_cast<uint64_t>(d.ffn) * 2, 64, t_pad,
                              true)))
    return rc;
  FusedParams& p = plan->p;
  p = FusedParams{};
  p.layers = d.layers;
  p.hidden = d.hidden;
  p.n_heads = d.n_heads;
  p.n_kv_heads = d.n_kv_heads;
  p.ffn = d.ffn;
  p.eps = d.rms_eps;
  p.rope_log2_theta = std::log2(d.rope_theta);
  p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(128.0));
  p.kv_cap = d.kv_capacity;
  p.vocab = d.vocab;
  p.ldc = d.hidden * (d.n_capture > 0 ? d.n_capture : 1);
  p.embed = static_cast<const __nv_bfloat16*>(d.embed);
  p.final_norm = static_cast<const __nv_bfloat16*>(d.final_norm);
  p.wmaps = reinterpret_cast<const CUtensorMap*>(base + L.maps);
  p.lp = reinterpret_cast<const FusedLayerPtrs*>(base + L.lp);
  p.kv = static_cast<__nv_bfloat16*>(d.kv_cache);
  p.h = static_cast<__nv_bfloat16*>(d.h);
  p.xn = static_cast<__nv_bfloat16*>(d.xn);
  p.q = static_cast<__nv_bfloat16*>(d.q);
  p.attn = static_cast<__nv_bfloat16*>(d.attn);
  p.act = static_cast<__nv_bfloat16*>(d.act);
  p.norm_out = static_cast<__nv_bfloat16*>(d.norm_out);
  p.qkv_part = reinterpret_cast<float*>(base + L.qkv_part);
  p.o_part = reinterpret_cast<float*>(base + L.o_part);
  p.dn_part = reinterpret_cast<float*>(base + L.dn_part);
  p.gu_ws = reinterpret_cast<float*>(base + L.gu_ws);
  p.gu_tile_cnt = reinterpret_cast<uint32_t*>(base + L.gu_cnt);
  p.att_o = reinterpret_cast<float*>(base + L.att_o);
  p.att_ml = reinterpret_cast<float*>(base + L.att_ml);
  p.cnt = reinterpret_cast<uint32_t*>(base + L.cnt);
  p.norm_cnt = p.cnt + static_cast<size_t>(d.layers) * kCntPerLayer + 8;
  p.norm_ss = reinterpret_cast<float*>(base + L.norm_ss);
  p.qkv_split = L.qkv_split;
  p.o_split = L.o_split;
  p.dn_split = L.dn_split;
  p.att_splits = Lt.att_splits;
  p.att_rb = Lt.att_rb;
  DTREE_CHECK_ARG(static_cast<size_t>(Lt.att_splits) * t_pad * d.n_heads * 128 * 4 <= L.att_ml - L.att_o,
                  "fused verify: attention partials exceed the workspace");
  p.grid = L.grid;
  plan->t_pad = t_pad;
  plan->smem = t_pad == 16 ? fused_smem<16>() : (t_pad == 32 ? fused_smem<32>() : fused_smem<64>());
  return kOk;
}

template <int TPAD>
static int fused_launch_t(FusedPlan& plan, cudaStream_t stream) {
  auto kern = fused_verify_kernel<TPAD>;
  DTREE_CUDA_RET(ensure_smem_attr(kern, plan.smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.p.grid);
  cfg.blockDim = dim3(kFusedThreads);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  DTREE_CUDA_RET(cudaLaunchKernelEx(&cfg, kern, plan.xmap_xn, plan.xmap_attn, plan.xmap_act, plan.p));
  return kOk;
}

int fused_launch(FusedPlan& plan, const int32_t* tokens, const int32_t* positions, const uint64_t* anc, int n_rows,
                 const dtree_step_state* state, cudaStream_t stream) {
  DTREE_CHECK_ARG(n_rows > 0 && n_rows <= plan.t_pad, "fused verify: n_rows out of range");
  plan.p.tokens = tokens;
  plan.p.positions = positions;
  plan.p.anc = anc;
  plan.p.state = state;
  plan.p.n_rows = n_rows;
  DTREE_CUDA_RET(cudaMemsetAsync(plan.p.cnt, 0, fused_cnt_words(plan.p.layers) * 4, stream));
  if (plan.t_pad == 16) return fused_launch_t<16>(plan, stream);
  if (plan.t_pad == 32) return fused_launch_t<32>(plan, stream);
  return fused_launch_t<64>(plan, stream);
}

}  // namespace dtree
