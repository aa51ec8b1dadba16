// Tree construction, acceptance walk, KV compaction and decode-state kernels.
//
// Reference semantics: dtree_mlx/dtree_runtime.py:82-208 (build / compile /
// follow), adapters.py:635-668 (compaction), runtime.py:476-490 (DFlash
// chain block).  All state lives on the device so a decode step needs no
// host round trip.
#include <mutex>
#include <string>

#include "common.cuh"
#include "../../include/dtree_b200.h"

namespace dtree {

constexpr int kTopkThreads = 512;
constexpr int kMaxBudget = DTREE_MAX_TREE - 1;  // 127 nodes + root
constexpr int kMaxRows = 64;
constexpr int kMaxK = 128;                       // k = min(budget, vocab) <= 127

// ============================================================ planted logits
constexpr uint32_t kNoiseTag = 0xD1CEu;
constexpr uint32_t kPlantTag = 0xB1A5u;
constexpr uint32_t kKeyHi = 0x5EED0001u;

__device__ __forceinline__ float u24(uint32_t x) { return __fmul_rn(static_cast<float>(x >> 8), 5.9604644775390625e-08f); }

// grid (ceil(vocab/256), rows), block 256
__global__ void plant_draft_logits_kernel(float* __restrict__ logits, int rows, int vocab, uint32_t seed,
                                          const dtree_step_state* __restrict__ state,
                                          const int32_t* __restrict__ cont, int cont_len, float p_correct) {
  pdl_trigger();
  __shared__ int s_tok;
  const int r = blockIdx.y;
  pdl_wait();
  const int step = state->step;
  const int start = state->start;
  if (threadIdx.x == 0) {
    uint32_t c[4] = {0xFFFFFFFFu, static_cast<uint32_t>(r), static_cast<uint32_t>(step), kPlantTag};
    philox4x32_10(c, seed, kKeyHi);
    const bool take = u24(c[0]) < p_correct;
    int tok = static_cast<int>(c[1] % static_cast<uint32_t>(vocab));
    const int pos = start + r + 1;
    if (take && pos < cont_len && cont[pos] >= 0) tok = cont[pos];
    s_tok = tok;
  }
  __syncthreads();
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= vocab) return;
  float acc = 0.0f;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    uint32_t c[4] = {static_cast<uint32_t>(v), static_cast<uint32_t>(r) | (static_cast<uint32_t>(j) << 16),
                     static_cast<uint32_t>(step), kNoiseTag};
    philox4x32_10(c, seed, kKeyHi);
#pragma unroll
    for (int l = 0; l < 4; ++l) acc = __fadd_rn(acc, u24(c[l]));
  }
  float x = __fsub_rn(acc, 6.0f);
  if (v == s_tok) x = __fadd_rn(x, 8.0f);
  logits[static_cast<size_t>(r) * vocab + v] = x;
}

// ============================================================ top-k + LSE
// Workspace layout (per row r, split s):
//   cand_val [rows][splits][kMaxK] f32, cand_id [rows][splits][kMaxK] i32
//   part_m [rows][splits], part_s [rows][splits]
//   top_id [rows][kMaxK] i32, top_lp [rows][kMaxK] f32
//   counters [rows] u32
struct TreeWs {
  float* cand_val;
  int32_t* cand_id;
  float* part_m;
  float* part_s;
  int32_t* top_id;
  float* top_lp;
  uint32_t* counters;
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

__host__ __device__ inline size_t tree_ws_layout(int rows, int splits, TreeWs* ws, char* base) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t rs = static_cast<size_t>(rows) * splits;
  size_t o_cv = take(rs * kMaxK * 4), o_ci = take(rs * kMaxK * 4), o_pm = take(rs * 4), o_ps = take(rs * 4);
  size_t o_ti = take(static_cast<size_t>(rows) * kMaxK * 4), o_tl = take(static_cast<size_t>(rows) * kMaxK * 4);
  size_t o_ct = take(static_cast<size_t>(rows) * 4);
  if (ws && base) {
    ws->cand_val = reinterpret_cast<float*>(base + o_cv);
    ws->cand_id = reinterpret_cast<int32_t*>(base + o_ci);
    ws->part_m = reinterpret_cast<float*>(base + o_pm);
    ws->part_s = reinterpret_cast<float*>(base + o_ps);
    ws->top_id = reinterpret_cast<int32_t*>(base + o_ti);
    ws->top_lp = reinterpret_cast<float*>(base + o_tl);
    ws->counters = reinterpret_cast<uint32_t*>(base + o_ct);
  }
  return off;
}

__device__ __forceinline__ float block_reduce_max(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = (l < (blockDim.x >> 5)) ? red[l] : -INFINITY;
  for (int o = 16; o > 0; o >>= 1) r = fmaxf(r, __shfl_xor_sync(0xffffffffu, r, o));
  return r;
}
__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = (l < (blockDim.x >> 5)) ? red[l] : 0.0f;
  for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}

// (value desc, id asc) total order
__device__ __forceinline__ bool cand_before(float va, int ia, float vb, int ib) {
  return (va > vb) || (va == vb && ia < ib);
}

// Sorts n (<= kMaxK * splits, held in smem) candidates by rank counting and
// writes the first k into out_val/out_id (smem or global).
__device__ void rank_select(const float* val, const int32_t* id, int n, int k, float* out_val, int32_t* out_id) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float vi = val[i];
    const int ii = id[i];
    int rank = 0;
    for (int j = 0; j < n; ++j) rank += cand_before(val[j], id[j], vi, ii) ? 1 : 0;
    if (rank < k) {
      out_val[rank] = vi;
      out_id[rank] = ii;
    }
  }
}

// 64-bit selection key of (value, index): larger key = earlier in the
// (value desc, index asc) order; unique per element
__device__ __forceinline__ unsigned long long topk_key(float v, int idx) {
  return (static_cast<unsigned long long>(float_order_key(v)) << 32) |
         static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(idx));
}
__device__ __forceinline__ float topk_key_value(unsigned long long key) {
  const uint32_t k = static_cast<uint32_t>(key >> 32);
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}
__device__ __forceinline__ int topk_key_index(unsigned long long key) {
  return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull));
}
__device__ __forceinline__ unsigned long long block_reduce_max_u64(unsigned long long v, unsigned long long* red) {
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  const int wp = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[wp] = v;
  __syncthreads();
  unsigned long long r = (l < (blockDim.x >> 5)) ? red[l] : 0ull;
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, r, o);
    r = w > r ? w : r;
  }
  return r;
}

constexpr int kTopkElems = 48;     // elements per thread (registers)
constexpr int kTopkCandCap = 1024;  // candidates above the threshold kept in shared memory

// Per-row top-k (value desc, index asc; k <= 127) of the draft logits and
// their logsumexp (dtree_runtime.py:92-107).  grid (splits, rows), block
// kTopkThreads; split s covers the chunk [s*chunk, (s+1)*chunk) of its row,
// thread t the elements t + i*blockDim (coalesced), held in registers.
//   theta = the kk-th largest of the per-thread maximum keys: at least kk
//           elements reach theta, so every top-kk element is >= theta;
//   the elements >= theta (few: the strided layout spreads large values over
//           threads) are ranked in shared memory.  If more than
//           kTopkCandCap reach theta, kk rounds of a block-wide maximum
//           below the previous key select them instead (exact, slower).
// The last CTA of a row merges the splits' sorted candidates and subtracts
// the row's logsumexp, as the heap stage reads them.
__global__ void __launch_bounds__(kTopkThreads) topk_lse_kernel(const float* __restrict__ logits, int rows,
                                                                 int vocab, int k, int splits, int chunk,
                                                                 TreeWs ws) {
  pdl_trigger();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* s_cv = reinterpret_cast<float*>(smem_raw);                   // [splits*kMaxK] merge area (last CTA)
  int32_t* s_ci = reinterpret_cast<int32_t*>(s_cv + splits * kMaxK);  // [splits*kMaxK]
  __shared__ unsigned long long s_tmax[kTopkThreads];
  __shared__ unsigned long long s_cand[kTopkCandCap];
  __shared__ unsigned long long s_kred[32];
  __shared__ float s_red[32];
  __shared__ int s_ncand;
  __shared__ bool s_last;

  const int r = blockIdx.y, s = blockIdx.x;
  const int c0 = s * chunk;
  const int c1 = min(vocab, c0 + chunk);
  const int n = max(0, c1 - c0);
  const int kk = min(k, n);
  pdl_wait();
  const float* row = logits + static_cast<size_t>(r) * vocab;
  float x[kTopkElems];
  float lmax = -INFINITY;
#pragma unroll
  for (int i = 0; i < kTopkElems; ++i) {
    const int idx = c0 + threadIdx.x + i * kTopkThreads;
    x[i] = idx < c1 ? __ldcs(row + idx) : -INFINITY;
    lmax = fmaxf(lmax, x[i]);
  }
  const float m = block_reduce_max(lmax, s_red);
  float lsum = 0.0f;
  unsigned long long tmax = 0ull;
#pragma unroll
  for (int i = 0; i < kTopkElems; ++i) {
    const int idx = c0 + threadIdx.x + i * kTopkThreads;
    if (idx < c1) {
      lsum += __expf(x[i] - m);
      const unsigned long long key = topk_key(x[i], idx);
      tmax = key > tmax ? key : tmax;
    }
  }
  const float ssum = block_reduce_sum(lsum, s_red);

  float* cv = ws.cand_val + (static_cast<size_t>(r) * splits + s) * kMaxK;
  int32_t* ci = ws.cand_id + (static_cast<size_t>(r) * splits + s) * kMaxK;
  if (kk > 0) {
    // theta: the smallest of the kk largest per-thread maxima
    s_tmax[threadIdx.x] = tmax;
    if (threadIdx.x == 0) s_ncand = 0;
    __syncthreads();
    int rank = 0;
    for (int j = 0; j < kTopkThreads; ++j) rank += s_tmax[j] > tmax ? 1 : 0;
    const unsigned long long mine = (rank < kk && tmax != 0ull) ? ~tmax : 0ull;  // max of ~key = min key
    const unsigned long long theta = ~block_reduce_max_u64(mine, s_kred);
    const unsigned long long th = (theta == ~0ull) ? 0ull : theta;  // fewer than kk non-empty threads
#pragma unroll
    for (int i = 0; i < kTopkElems; ++i) {
      const int idx = c0 + threadIdx.x + i * kTopkThreads;
      if (idx < c1) {
        const unsigned long long key = topk_key(x[i], idx);
        if (key >= th) {
          const int slot = atomicAdd(&s_ncand, 1);
          if (slot < kTopkCandCap) s_cand[slot] = key;
        }
      }
    }
    __syncthreads();
    const int nc = s_ncand;
    if (nc <= kTopkCandCap) {
      for (int c = threadIdx.x; c < nc; c += blockDim.x) {
        const unsigned long long key = s_cand[c];
        int rk = 0;
        for (int j = 0; j < nc; ++j) rk += s_cand[j] > key ? 1 : 0;
        if (rk < kk) {
          cv[rk] = topk_key_value(key);
          ci[rk] = topk_key_index(key);
        }
      }
    } else {
      unsigned long long prev = ~0ull;
      for (int t = 0; t < kk; ++t) {
        unsigned long long best = 0ull;
#pragma unroll
        for (int i = 0; i < kTopkElems; ++i) {
          const int idx = c0 + threadIdx.x + i * kTopkThreads;
          if (idx < c1) {
            const unsigned long long key = topk_key(x[i], idx);
            if (key < prev && key > best) best = key;
          }
        }
        best = block_reduce_max_u64(best, s_kred);
        if (threadIdx.x == 0) {
          cv[t] = topk_key_value(best);
          ci[t] = topk_key_index(best);
        }
        prev = best;
      }
    }
  }
  for (int i = kk + threadIdx.x; i < k; i += blockDim.x) {  // pad short chunks
    cv[i] = -INFINITY;
    ci[i] = 0x7FFFFFFF;
  }
  if (threadIdx.x == 0) {
    ws.part_m[r * splits + s] = m;
    ws.part_s[r * splits + s] = ssum;
  }
  // last CTA of this row merges the splits
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(&ws.counters[r], 1u);
    s_last = (prev == static_cast<uint32_t>(splits - 1));
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int total = splits * k;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int sp = i / k, j = i % k;
    s_cv[i] = __ldcg(&ws.cand_val[(static_cast<size_t>(r) * splits + sp) * kMaxK + j]);
    s_ci[i] = __ldcg(&ws.cand_id[(static_cast<size_t>(r) * splits + sp) * kMaxK + j]);
  }
  __syncthreads();
  rank_select(s_cv, s_ci, total, k, ws.top_lp + static_cast<size_t>(r) * kMaxK,
              ws.top_id + static_cast<size_t>(r) * kMaxK);
  __syncthreads();
  __threadfence();
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int sp = 0; sp < splits; ++sp) M = fmaxf(M, __ldcg(&ws.part_m[r * splits + sp]));
    float S = 0.0f;
    for (int sp = 0; sp < splits; ++sp)
      S += __ldcg(&ws.part_s[r * splits + sp]) * expf(__ldcg(&ws.part_m[r * splits + sp]) - M);
    s_red[0] = M + logf(S);
    ws.counters[r] = 0;  // ready for the next launch
  }
  __syncthreads();
  const float lse = s_red[0];
  float* lp = ws.top_lp + static_cast<size_t>(r) * kMaxK;
  for (int j = threadIdx.x; j < k; j += blockDim.x) lp[j] = __fsub_rn(__ldcg(&lp[j]), lse);
}

// ============================================================ best-first heap
// One warp.  Entries live in shared memory; each pop is a warp-wide argmin
// under the reference's tuple order (-logw, ranks, parent, depth, rank, logw).
constexpr int kHeapCap = 2 * kMaxBudget + 4;

struct HeapSmem {
  double neg_logw[kHeapCap];
  double logw[kHeapCap];
  int parent[kHeapCap];
  int depth[kHeapCap];
  int rank[kHeapCap];
  int active[kHeapCap];
  uint8_t path[kHeapCap][kMaxRows];  // ranks tuple (length = depth)
  uint8_t node_path[DTREE_MAX_TREE][kMaxRows];
  uint64_t anc[DTREE_MAX_TREE][2];  // emitted nodes' ancestor masks
  int n_entries;
};

__device__ __forceinline__ bool heap_less(const HeapSmem& h, int a, int b) {
  if (h.neg_logw[a] != h.neg_logw[b]) return h.neg_logw[a] < h.neg_logw[b];
  const int da = h.depth[a], db = h.depth[b];
  const int dm = min(da, db);
  for (int i = 0; i < dm; ++i)
    if (h.path[a][i] != h.path[b][i]) return h.path[a][i] < h.path[b][i];
  if (da != db) return da < db;  // shorter tuple sorts first
  if (h.parent[a] != h.parent[b]) return h.parent[a] < h.parent[b];
  if (h.depth[a] != h.depth[b]) return h.depth[a] < h.depth[b];
  if (h.rank[a] != h.rank[b]) return h.rank[a] < h.rank[b];
  return h.logw[a] < h.logw[b];
}

// top_ids/top_lp: [rows][ld] with k valid columns.  block = 32 threads.
__global__ void __launch_bounds__(32) heap_tree_kernel(const int32_t* __restrict__ top_ids,
                                                        const float* __restrict__ top_lp, int ld, int rows, int k,
                                                        int budget, dtree_step_state* state,
                                                        int32_t* __restrict__ tree_tokens,
                                                        int32_t* __restrict__ parents, int32_t* __restrict__ depths,
                                                        int32_t* __restrict__ positions,
                                                        uint64_t* __restrict__ anc_mask) {
  pdl_trigger();
  __shared__ HeapSmem h;
  // the top-k table [rows][k] in shared memory: no global round trip per pop
  extern __shared__ __align__(16) unsigned char heap_dyn[];
  float* s_lp = reinterpret_cast<float*>(heap_dyn);
  int32_t* s_id = reinterpret_cast<int32_t*>(s_lp + rows * k);
  const int lane = threadIdx.x;
  pdl_wait();
  const int start = state->start;
  for (int e = lane; e < rows * k; e += 32) {
    s_lp[e] = top_lp[(e / k) * ld + e % k];
    s_id[e] = top_ids[(e / k) * ld + e % k];
  }
  for (int i = lane; i < kHeapCap; i += 32) h.active[i] = 0;
  __syncwarp();
  if (lane == 0) {
    tree_tokens[0] = state->root_token;
    parents[0] = -1;
    depths[0] = 0;
    positions[0] = start;
    anc_mask[0] = 1ull;
    anc_mask[1] = 0ull;
    h.anc[0][0] = 1ull;
    h.anc[0][1] = 0ull;
    h.n_entries = 0;
    if (budget > 0 && rows > 0 && k > 0) {
      const double lw = static_cast<double>(s_lp[0]);
      h.neg_logw[0] = -lw;
      h.logw[0] = lw;
      h.parent[0] = 0;
      h.depth[0] = 1;
      h.rank[0] = 0;
      h.path[0][0] = 0;
      h.active[0] = 1;
      h.n_entries = 1;
    }
  }
  __syncwarp();
  int n_nodes = 0;
  while (n_nodes < budget) {
    // warp argmin over active entries: compare -logw in registers and fall
    // back to the full tuple order only on exact ties
    int best = -1;
    double bnl = 0.0;
    const int ne = h.n_entries;
    for (int e = lane; e < ne; e += 32) {
      if (!h.active[e]) continue;
      const double nl = h.neg_logw[e];
      if (best < 0 || nl < bnl || (nl == bnl && heap_less(h, e, best))) {
        best = e;
        bnl = nl;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const int other = __shfl_xor_sync(0xffffffffu, best, o);
      const double onl = __shfl_xor_sync(0xffffffffu, bnl, o);
      if (other >= 0 && (best < 0 || onl < bnl || (onl == bnl && heap_less(h, other, best)))) {
        best = other;
        bnl = onl;
      }
    }
    if (best < 0) break;  // heap exhausted
    // every lane reads the popped entry; lane 0 does the scalar updates and the
    // lanes share the byte-wise ranks-tuple copies
    const int depth = h.depth[best], rank = h.rank[best], parent = h.parent[best];
    const double logw = h.logw[best];
    const int cur = n_nodes + 1;
    const bool has_sib = rank + 1 < k;
    const bool has_child = depth < rows;
    // the sibling reuses the popped slot; the child takes a fresh slot when a
    // sibling exists, else the popped one (whose tuple prefix is already right)
    const int child_slot = has_sib ? h.n_entries : best;
    for (int i = lane; i < depth; i += 32) h.node_path[cur][i] = h.path[best][i];
    __syncwarp();
    if (has_child && has_sib)
      for (int i = lane; i < depth; i += 32) h.path[child_slot][i] = h.node_path[cur][i];
    if (lane == 0) {
      tree_tokens[cur] = s_id[(depth - 1) * k + rank];
      parents[cur] = parent;
      depths[cur] = depth;
      positions[cur] = start + depth;
      uint64_t a0 = h.anc[parent][0], a1 = h.anc[parent][1];
      if (cur < 64) a0 |= 1ull << cur; else a1 |= 1ull << (cur - 64);
      h.anc[cur][0] = a0;
      h.anc[cur][1] = a1;
      anc_mask[2 * cur] = a0;
      anc_mask[2 * cur + 1] = a1;
      h.active[best] = 0;
      if (has_sib) {
        const double sib = (logw - static_cast<double>(s_lp[(depth - 1) * k + rank])) +
                           static_cast<double>(s_lp[(depth - 1) * k + rank + 1]);
        h.neg_logw[best] = -sib;
        h.logw[best] = sib;
        h.rank[best] = rank + 1;  // parent and depth unchanged
        h.path[best][depth - 1] = static_cast<uint8_t>(rank + 1);
        h.active[best] = 1;
      }
      if (has_child) {
        if (has_sib) ++h.n_entries;
        const int e = child_slot;
        const double ch = logw + static_cast<double>(s_lp[depth * k + 0]);
        h.neg_logw[e] = -ch;
        h.logw[e] = ch;
        h.parent[e] = cur;
        h.depth[e] = depth + 1;
        h.rank[e] = 0;
        h.path[e][depth] = 0;
        h.active[e] = 1;
      }
    }
    __syncwarp();
    ++n_nodes;
  }
  if (lane == 0) state->n_nodes = n_nodes + 1;
}

// ============================================================ chain (DFlash)
// grid = rows, block 256: per-row argmax (first index on ties); then the last
// block writes the chain tree.
// inv_temp > 0: the drafted token is sampled from softmax(logits * inv_temp)
// (sample_tokens, runtime.py:12-19) by the Gumbel-max rule; 0: argmax
__global__ void chain_argmax_kernel(const float* __restrict__ logits, int rows, int vocab,
                                    dtree_step_state* state, int32_t* __restrict__ tree_tokens,
                                    int32_t* __restrict__ parents, int32_t* __restrict__ depths,
                                    int32_t* __restrict__ positions, uint64_t* __restrict__ anc_mask, float inv_temp,
                                    uint32_t seed) {
  pdl_trigger();
  __shared__ float s_v[32];
  __shared__ int s_i[32];
  const int r = blockIdx.x;
  pdl_wait();
  const uint32_t step = static_cast<uint32_t>(state->step);
  const float* row = logits + static_cast<size_t>(r) * vocab;
  float bv = -INFINITY;
  int bi = 0x7FFFFFFF;
  for (int v = threadIdx.x; v < vocab; v += blockDim.x) {
    float x = row[v];
    if (inv_temp > 0.0f) x = x * inv_temp + gumbel_noise(seed, kSampleTagDraft, step, r, v);
    if (x > bv || (x == bv && v < bi)) {
      bv = x;
      bi = v;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    s_v[w] = bv;
    s_i[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int j = 1; j < (blockDim.x >> 5); ++j)
      if (s_v[j] > bv || (s_v[j] == bv && s_i[j] < bi)) {
        bv = s_v[j];
        bi = s_i[j];
      }
    const int start = state->start;
    const int i = r + 1;
    tree_tokens[i] = bi;
    parents[i] = r;
    depths[i] = i;
    positions[i] = start + i;
    // chain visibility: nodes 0..i
    uint64_t a0 = 0, a1 = 0;
    for (int j = 0; j <= i; ++j) {
      if (j < 64) a0 |= 1ull << j; else a1 |= 1ull << (j - 64);
    }
    anc_mask[2 * i] = a0;
    anc_mask[2 * i + 1] = a1;
    if (r == 0) {
      tree_tokens[0] = state->root_token;
      parents[0] = -1;
      depths[0] = 0;
      positions[0] = start;
      anc_mask[0] = 1ull;
      anc_mask[1] = 0ull;
      state->n_nodes = rows + 1;
    }
  }
}

// ============================================================ accept walk
__global__ void __launch_bounds__(32) accept_walk_kernel(const int32_t* __restrict__ tree_tokens,
                                                          const int32_t* __restrict__ parents,
                                                          const int32_t* __restrict__ posterior,
                                                          dtree_step_state* state, int32_t* __restrict__ accepted,
                                                          int32_t* __restrict__ out_tokens, int out_cap,
                                                          int32_t* __restrict__ history, int hist_cap) {
  pdl_trigger();
  const int lane = threadIdx.x;
  pdl_wait();
  const int n_nodes = min(state->n_nodes, DTREE_MAX_TREE);
  const int start = state->start;
  int cur = 0, n = 1;
  if (lane == 0) accepted[0] = 0;
  int tok = posterior[0];
  for (int it = 0; it < n_nodes; ++it) {
    int found = -1;
    for (int j = 1 + lane; j < n_nodes; j += 32) {
      const bool hit = (parents[j] == cur) && (tree_tokens[j] == tok);
      const unsigned b = __ballot_sync(__activemask(), hit);
      if (b && found < 0) found = j - lane + (__ffs(b) - 1);
    }
    // lanes may disagree only if some lanes did not iterate; take the min found
    for (int o = 16; o > 0; o >>= 1) {
      const int of = __shfl_xor_sync(0xffffffffu, found, o);
      if (of >= 0 && (found < 0 || of < found)) found = of;
    }
    if (found < 0) break;
    cur = found;
    if (lane == 0) accepted[n] = cur;
    ++n;
    tok = posterior[cur];
  }
  if (lane == 0) {
    for (int i = 0; i < n; ++i) {
      const int pos = start + i;
      if (pos < out_cap) out_tokens[pos] = tree_tokens[accepted[i]];
    }
    if (start + n < out_cap) out_tokens[start + n] = tok;
    state->n_accepted = n;
    state->bonus_token = tok;
    state->n_output = start + n + 1;
    const int step = state->step;
    if (history && step < hist_cap) history[step] = n;
  }
}

// ============================================================ compaction
// grid = layers*2*kv_heads planes, block 256; smem holds the accepted rows.
__global__ void kv_compact_kernel(__nv_bfloat16* __restrict__ kv, int capacity, int head_dim,
                                  const int32_t* __restrict__ accepted, const dtree_step_state* state) {
  pdl_trigger();
  extern __shared__ __align__(16) uint4 s_rows[];  // up to DTREE_MAX_TREE rows of head_dim bf16
  pdl_wait();
  const int n = min(state->n_accepted, DTREE_MAX_TREE);
  const int start = state->start;
  bool identity = true;
  for (int i = 0; i < n; ++i) identity &= (accepted[i] == i);
  if (identity || n <= 0) return;
  const int vec_per_row = head_dim * 2 / 16;
  __nv_bfloat16* plane = kv + static_cast<size_t>(blockIdx.x) * capacity * head_dim;
  const uint4* src = reinterpret_cast<const uint4*>(plane);
  uint4* dst = reinterpret_cast<uint4*>(plane);
  for (int e = threadIdx.x; e < n * vec_per_row; e += blockDim.x) {
    const int i = e / vec_per_row, v = e % vec_per_row;
    const int srow = start + accepted[i];
    if (srow < capacity) s_rows[e] = src[static_cast<size_t>(srow) * vec_per_row + v];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < n * vec_per_row; e += blockDim.x) {
    const int i = e / vec_per_row, v = e % vec_per_row;
    const int drow = start + i;
    if (drow < capacity && start + accepted[i] < capacity) dst[static_cast<size_t>(drow) * vec_per_row + v] = s_rows[e];
  }
}

__global__ void gather_rows_kernel(const uint4* __restrict__ src, int vec_per_row, const int32_t* __restrict__ idx,
                                   const dtree_step_state* state, uint4* __restrict__ dst, int max_rows) {
  pdl_trigger();
  pdl_wait();
  const int n = min(state->n_accepted, max_rows);
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n * vec_per_row; e += gridDim.x * blockDim.x) {
    const int i = e / vec_per_row, v = e % vec_per_row;
    dst[static_cast<size_t>(i) * vec_per_row + v] = src[static_cast<size_t>(idx[i]) * vec_per_row + v];
  }
}

__global__ void step_commit_kernel(dtree_step_state* state) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    state->start += state->n_accepted;
    state->root_token = state->bonus_token;
    state->step += 1;
  }
}

// splits per row for the top-k scan: enough that a chunk fits the registers
// of one CTA (kTopkThreads * kTopkElems elements) and at least ~8 CTAs per
// row for large vocabularies.  `cap_bytes` bounds the workspace (the
// no-allocation scratch): splits shrink until it fits, and the caller checks
// that a chunk still fits one CTA.
constexpr int kTopkMaxSplits = 200;  // merge table splits * kMaxK * 8 B of shared memory
static int topk_splits(int rows, int vocab, size_t cap_bytes) {
  const int per_cta = kTopkThreads * kTopkElems;
  int splits = (vocab + per_cta - 1) / per_cta;
  if (splits < 8) splits = vocab >= 8 * 4096 ? 8 : (vocab + 4095) / 4096;
  if (splits < 1) splits = 1;
  if (splits > kTopkMaxSplits) splits = kTopkMaxSplits;
  while (splits > 1 && tree_ws_layout(rows, splits, nullptr, nullptr) > cap_bytes) --splits;
  return splits;
}
constexpr size_t kNoCap = ~static_cast<size_t>(0);

// argument checks shared by the workspace and no-allocation builds
static int tree_build_check(const float* draft_logits, int rows, int vocab, int budget, const dtree_step_state* state,
                            const int32_t* tree_tokens, const int32_t* parents, const int32_t* depths,
                            const int32_t* positions, const uint64_t* anc_mask) {
  DTREE_CHECK_ARG(state && tree_tokens && parents && depths && positions && anc_mask, "null output pointer");
  DTREE_CHECK_ARG(budget >= 0 && budget <= kMaxBudget, "budget must be in [0, 127]");
  DTREE_CHECK_ARG(rows >= 0 && rows <= kMaxRows, "rows must be in [0, 64]");
  DTREE_CHECK_ARG(vocab > 0, "vocab must be positive");
  DTREE_CHECK_ARG(budget == 0 || rows == 0 || draft_logits != nullptr, "null draft_logits");
  return kOk;
}

static int tree_build_impl(const float* draft_logits, int rows, int vocab, int budget, dtree_step_state* state,
                           void* workspace, size_t workspace_bytes, int splits, int32_t* tree_tokens,
                           int32_t* parents, int32_t* depths, int32_t* positions, uint64_t* anc_mask,
                           int32_t* top_ids, float* top_logprobs, cudaStream_t stream) {
  int rc = tree_build_check(draft_logits, rows, vocab, budget, state, tree_tokens, parents, depths, positions,
                            anc_mask);
  if (rc) return rc;
  const int k = budget < vocab ? budget : vocab;
  if (budget == 0 || rows == 0) {
    // root only (dtree_runtime.py:88-90)
    DTREE_CUDA_RET(launch_pdl(heap_tree_kernel, dim3(1), dim3(32), 0, stream, (const int32_t*)nullptr,
                              (const float*)nullptr, 0, 0, 0, 0, state, tree_tokens, parents, depths, positions,
                              anc_mask));
    return kOk;
  }
  const size_t need = tree_ws_layout(rows, splits, nullptr, nullptr);
  DTREE_CHECK_ARG(workspace != nullptr && workspace_bytes >= need, "tree workspace too small");
  const int chunk = (vocab + splits - 1) / splits;
  DTREE_CHECK_ARG(chunk <= kTopkThreads * kTopkElems,
                  "vocab too large for the top-k chunking (at most " +
                      std::to_string(static_cast<long long>(splits) * kTopkThreads * kTopkElems) + " here)");
  TreeWs ws;
  tree_ws_layout(rows, splits, &ws, static_cast<char*>(workspace));
  const size_t smem = static_cast<size_t>(splits) * kMaxK * 8;
  DTREE_CUDA_RET(ensure_smem_attr(topk_lse_kernel, static_cast<int>(smem)));
  DTREE_CUDA_RET(launch_pdl(topk_lse_kernel, dim3(splits, rows), dim3(kTopkThreads), smem, stream, draft_logits,
                            rows, vocab, k, splits, chunk, ws));
  const size_t heap_smem = static_cast<size_t>(rows) * k * 8;
  DTREE_CUDA_RET(ensure_smem_attr(heap_tree_kernel, static_cast<int>(heap_smem)));
  DTREE_CUDA_RET(launch_pdl(heap_tree_kernel, dim3(1), dim3(32), heap_smem, stream, (const int32_t*)ws.top_id,
                            (const float*)ws.top_lp, kMaxK, rows, k, budget, state, tree_tokens, parents, depths,
                            positions, anc_mask));
  if (top_ids) {
    DTREE_CUDA_RET(cudaMemcpy2DAsync(top_ids, sizeof(int32_t) * k, ws.top_id, sizeof(int32_t) * kMaxK,
                                     sizeof(int32_t) * k, rows, cudaMemcpyDeviceToDevice, stream));
  }
  if (top_logprobs) {
    DTREE_CUDA_RET(cudaMemcpy2DAsync(top_logprobs, sizeof(float) * k, ws.top_lp, sizeof(float) * kMaxK,
                                     sizeof(float) * k, rows, cudaMemcpyDeviceToDevice, stream));
  }
  return kOk;
}

}  // namespace dtree

using namespace dtree;

extern "C" size_t dtree_tree_build_workspace_bytes(int rows, int vocab, int budget) {
  (void)budget;
  if (rows <= 0 || vocab <= 0) return 0;
  return tree_ws_layout(rows, topk_splits(rows, vocab, kNoCap), nullptr, nullptr);
}

extern "C" int dtree_tree_build(const float* draft_logits, int rows, int vocab, int budget,
                                dtree_step_state* state, void* workspace, size_t workspace_bytes,
                                int32_t* tree_tokens, int32_t* parents, int32_t* depths, int32_t* positions,
                                uint64_t* anc_mask, int32_t* top_ids, float* top_logprobs, void* stream_) {
  const int splits = (rows > 0 && vocab > 0) ? topk_splits(rows, vocab, kNoCap) : 1;
  return tree_build_impl(draft_logits, rows, vocab, budget, state, workspace, workspace_bytes, splits, tree_tokens,
                         parents, depths, positions, anc_mask, top_ids, top_logprobs,
                         static_cast<cudaStream_t>(stream_));
}

extern "C" int dtree_tree_from_topk(const int32_t* top_ids, const float* top_logprobs, int rows, int topk,
                                    int budget, dtree_step_state* state, int32_t* tree_tokens, int32_t* parents,
                                    int32_t* depths, int32_t* positions, uint64_t* anc_mask, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DTREE_CHECK_ARG(state && tree_tokens && parents && depths && positions && anc_mask, "null output pointer");
  DTREE_CHECK_ARG(budget >= 0 && budget <= kMaxBudget, "budget must be in [0, 127]");
  DTREE_CHECK_ARG(rows >= 0 && rows <= kMaxRows, "rows must be in [0, 64]");
  DTREE_CHECK_ARG(topk >= 0 && topk <= kMaxK, "topk must be in [0, 128]");
  DTREE_CHECK_ARG((rows == 0 || topk == 0) || (top_ids && top_logprobs), "null top-k inputs");
  const size_t heap_smem = (rows == 0 || topk == 0) ? 0 : static_cast<size_t>(rows) * topk * 8;
  DTREE_CUDA_RET(ensure_smem_attr(heap_tree_kernel, static_cast<int>(heap_smem)));
  DTREE_CUDA_RET(launch_pdl(heap_tree_kernel, dim3(1), dim3(32), heap_smem, stream, top_ids, top_logprobs, topk, rows, topk,
                            (rows == 0 || topk == 0) ? 0 : budget, state, tree_tokens, parents, depths, positions,
                            anc_mask));
  return kOk;
}

extern "C" int dtree_chain_build(const float* draft_logits, int rows, int vocab, dtree_step_state* state,
                                 int32_t* tree_tokens, int32_t* parents, int32_t* depths, int32_t* positions,
                                 uint64_t* anc_mask, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DTREE_CHECK_ARG(draft_logits && state && tree_tokens && parents && depths && positions && anc_mask,
                  "null pointer");
  DTREE_CHECK_ARG(rows >= 1 && rows < DTREE_MAX_TREE, "rows must be in [1, 127]");
  DTREE_CHECK_ARG(vocab > 0, "vocab must be positive");
  DTREE_CUDA_RET(launch_pdl(chain_argmax_kernel, dim3(rows), dim3(256), 0, stream, draft_logits, rows, vocab, state,
                            tree_tokens, parents, depths, positions, anc_mask, 0.0f, 0u));
  return kOk;
}

extern "C" int dtree_chain_sample(const float* draft_logits, int rows, int vocab, float temperature, uint32_t seed,
                                  dtree_step_state* state, int32_t* tree_tokens, int32_t* parents, int32_t* depths,
                                  int32_t* positions, uint64_t* anc_mask, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DTREE_CHECK_ARG(draft_logits && state && tree_tokens && parents && depths && positions && anc_mask,
                  "null pointer");
  DTREE_CHECK_ARG(rows >= 1 && rows < DTREE_MAX_TREE, "rows must be in [1, 127]");
  DTREE_CHECK_ARG(vocab > 0, "vocab must be positive");
  DTREE_CHECK_ARG(temperature >= 0.0f, "temperature must be >= 0");
  const float inv_temp = temperature < 1e-5f ? 0.0f : 1.0f / temperature;
  DTREE_CUDA_RET(launch_pdl(chain_argmax_kernel, dim3(rows), dim3(256), 0, stream, draft_logits, rows, vocab, state,
                            tree_tokens, parents, depths, positions, anc_mask, inv_temp, seed));
  return kOk;
}

extern "C" int dtree_plant_draft_logits(float* logits, int rows, int vocab, uint32_t seed,
                                        const dtree_step_state* state, const int32_t* continuation, int cont_len,
                                        float p_correct, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DTREE_CHECK_ARG(logits && state, "null pointer");
  DTREE_CHECK_ARG(rows > 0 && rows <= kMaxRows && vocab > 0, "bad shape");
  DTREE_CHECK_ARG(cont_len == 0 || continuation != nullptr, "null continuation");
  DTREE_CUDA_RET(launch_pdl(plant_draft_logits_kernel, dim3((vocab + 255) / 256, rows), dim3(256), 0, stream, logits,
                            rows, vocab, seed, state, continuation, cont_len, p_correct));
  return kOk;
}

extern "C" int dtree_accept_walk(const int32_t* tree_tokens, const int32_t* parents, const int32_t* posterior,
                                 dtree_step_state* state, int32_t* accepted, int32_t* output_tokens,
                                 int output_capacity, int32_t* accept_history, int history_capacity, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DTREE_CHECK_ARG(tree_tokens && parents && posterior && state && accepted && output_tokens, "null pointer");
  DTREE_CUDA_RET(launch_pdl(accept_walk_kernel, dim3(1), dim3(32), 0, stream, tree_tokens, parents, posterior, state,
                            accepted, output_tokens, output_capacity, accept_history, history_capacity));
  return kOk;
}

// DFlash block input (dtree_runtime.py:366-368): [current token, mask x
// (block-1)] at positions start .. start+block-1.
__global__ void dflash_block_kernel(const dtree_step_state* state, int mask_token_id, int block, int32_t* tokens,
                                    int32_t* positions) {
  pdl_trigger();
  pdl_wait();
  const int i = threadIdx.x;
  if (i < block) {
    tokens[i] = i == 0 ? state->root_token : mask_token_id;
    positions[i] = state->start + i;
  }
}

extern "C" int dtree_dflash_block(const dtree_step_state* state, int mask_token_id, int block, int32_t* tokens,
                                  int32_t* positions, void* stream) {
  DTREE_CHECK_ARG(state && tokens && positions, "null pointer");
  DTREE_CHECK_ARG(block > 0 && block <= DTREE_MAX_TREE, "block must be in [1, 128]");
  DTREE_CUDA_RET(launch_pdl(dflash_block_kernel, dim3(1), dim3(128), 0, static_cast<cudaStream_t>(stream), state,
                            mask_token_id, block, tokens, positions));
  return kOk;
}

extern "C" int dtree_kv_compact(void* kv_cache, int layers, int kv_heads, int capacity, int head_dim,
                                const int32_t* accepted, const dtree_step_state* state, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DTREE_CHECK_ARG(kv_cache && accepted && state, "null pointer");
  DTREE_CHECK_ARG(layers > 0 && kv_heads > 0 && capacity > 0, "bad shape");
  DTREE_CHECK_ARG(head_dim % 8 == 0 && head_dim <= 256, "head_dim must be a multiple of 8 and <= 256");
  const size_t smem = static_cast<size_t>(DTREE_MAX_TREE) * head_dim * 2;
  DTREE_CUDA_RET(ensure_smem_attr(kv_compact_kernel, static_cast<int>(smem)));
  DTREE_CUDA_RET(launch_pdl(kv_compact_kernel, dim3(layers * 2 * kv_heads), dim3(256), smem, stream,
                            static_cast<__nv_bfloat16*>(kv_cache), capacity, head_dim, accepted, state));
  return kOk;
}

extern "C" int dtree_gather_rows(const void* src, size_t row_bytes, const int32_t* accepted,
                                 const dtree_step_state* state, void* dst, int max_rows, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DTREE_CHECK_ARG(src && accepted && state && dst, "null pointer");
  DTREE_CHECK_ARG(row_bytes % 16 == 0 && row_bytes > 0, "row_bytes must be a positive multiple of 16");
  const int vec = static_cast<int>(row_bytes / 16);
  DTREE_CUDA_RET(launch_pdl(gather_rows_kernel, dim3(64), dim3(256), 0, stream, static_cast<const uint4*>(src), vec,
                            accepted, state, static_cast<uint4*>(dst), max_rows));
  return kOk;
}

extern "C" int dtree_step_commit(dtree_step_state* state, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DTREE_CHECK_ARG(state, "null state");
  DTREE_CUDA_RET(launch_pdl(step_commit_kernel, dim3(1), dim3(32), 0, stream, state));
  return kOk;
}

// ============================================================ no-allocation variant
// Tree build for callers that cannot allocate device memory: for example a
// serving loop that must not call cudaMalloc (or any allocating library
// routine) while it runs, or a host runtime that hands this library only the
// buffers it owns.  The top-k scratch lives in this fixed device array instead
// of a caller workspace.  Every GPU that loads the library holds it until the
// process exits.  All calls share it, so calls whose GPU work overlaps (other
// streams, other threads) race on it and must be serialized by the caller.
namespace dtree {
// 1 MiB: draft rows <= 64; the vocabulary limit follows from the split count
// that fits (dtree_tree_build_noalloc_max_vocab)
constexpr size_t kNoAllocScratchBytes = 1u << 20;
static __device__ __align__(256) unsigned char g_tree_scratch[kNoAllocScratchBytes];
constexpr int kMaxDevices = 64;
static void* g_tree_scratch_ptr[kMaxDevices] = {};
static std::mutex g_tree_scratch_mu;

// Device address of g_tree_scratch on the current device.  The host-side
// symbol is only a stand-in, so the address is looked up once per device,
// with that device current, and cached for the life of the process (a
// cudaDeviceReset invalidates it: do not reset a device this library has
// used and then call the no-allocation entry point on it again).
static int tree_scratch_ptr(void** out) {
  int dev = 0;
  DTREE_CUDA_RET(cudaGetDevice(&dev));
  DTREE_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_tree_scratch_mu);
  if (g_tree_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    DTREE_CUDA_RET(cudaGetSymbolAddress(&p, g_tree_scratch));
    g_tree_scratch_ptr[dev] = p;
  }
  *out = g_tree_scratch_ptr[dev];
  return kOk;
}
}  // namespace dtree

extern "C" size_t dtree_tree_build_noalloc_max_bytes(void) { return dtree::kNoAllocScratchBytes; }

extern "C" int dtree_tree_build_noalloc_max_vocab(int rows) {
  if (rows <= 0 || rows > kMaxRows) return 0;
  // the largest split count whose workspace fits the scratch, times a CTA's chunk
  int splits = kTopkMaxSplits;
  while (splits > 1 && tree_ws_layout(rows, splits, nullptr, nullptr) > kNoAllocScratchBytes) --splits;
  return splits * kTopkThreads * kTopkElems;
}

extern "C" int dtree_tree_build_noalloc(const float* draft_logits, int rows, int vocab, int budget,
                                        dtree_step_state* state, int32_t* tree_tokens, int32_t* parents,
                                        int32_t* depths, int32_t* positions, uint64_t* anc_mask, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  // every check comes before the first GPU work, so a rejected call leaves the
  // shared scratch untouched
  int rc = tree_build_check(draft_logits, rows, vocab, budget, state, tree_tokens, parents, depths, positions,
                            anc_mask);
  if (rc) return rc;
  const bool heap_only = budget == 0 || rows == 0;
  const int splits = heap_only ? 1 : topk_splits(rows, vocab, kNoAllocScratchBytes);
  if (!heap_only) {
    const size_t need = tree_ws_layout(rows, splits, nullptr, nullptr);
    const int max_vocab = dtree_tree_build_noalloc_max_vocab(rows);
    if (need > kNoAllocScratchBytes || vocab > max_vocab)
      return fail(kErrCapacity, "dtree_tree_build_noalloc: " + std::to_string(rows) + " draft rows of vocab " +
                                    std::to_string(vocab) + " need more than the fixed " +
                                    std::to_string(kNoAllocScratchBytes) +
                                    "-byte device scratch (at most vocab " + std::to_string(max_vocab) +
                                    " at this row count)");
  }
  void* scratch = nullptr;
  rc = tree_scratch_ptr(&scratch);
  if (rc) return rc;
  if (!heap_only) {
    // the per-row arrival counters must start at zero (a completed call leaves
    // them at zero; an interrupted one may not)
    TreeWs ws;
    tree_ws_layout(rows, splits, &ws, static_cast<char*>(scratch));
    DTREE_CUDA_RET(cudaMemsetAsync(ws.counters, 0, sizeof(uint32_t) * rows, stream));
  }
  return tree_build_impl(draft_logits, rows, vocab, budget, state, scratch, kNoAllocScratchBytes, splits,
                         tree_tokens, parents, depths, positions, anc_mask, nullptr, nullptr, stream);
}
