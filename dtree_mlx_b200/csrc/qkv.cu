// Finish of the fused q|k|v projection (qwen3_tree.py:50-65): sums the
// split-K fp32 partials of the QKV GEMM in split order, then per head
//   q, k: RMSNorm over head_dim (q_norm / k_norm), half-split RoPE at the
//         node's position, q -> q buffer, k -> K cache slot start + t
//   v:    -> V cache slot start + t
// grid = (n_rows, n_q_heads + 2 * n_kv_heads), block = head_dim threads.
//
// Gated variant (Qwen3.5 full attention, qwen35_tree.py:500-527): each q
// head's projection rows are [q (head_dim) | gate (head_dim)]; the gate is
// written (bf16) to gate_out for the attention output gating, and RoPE
// rotates only the first rot_dims features (partial_rotary_factor), pairs
// (i, i + rot_dims/2) with inv_freq_i = theta^(-2i/rot_dims) (mlx RoPE with
// dims = rot_dims, traditional = False); the rest pass through.
#include <algorithm>

#include "qkv.cuh"

namespace dtree {



__global__ void __launch_bounds__(256) qkv_finish_kernel(QkvFinishParams p) {
  pdl_trigger();
  __shared__ float s_red[8];
  __shared__ float s_y[256];
  const int t = blockIdx.x, gh = blockIdx.y, d = threadIdx.x;
  const int hd = p.head_dim;
  pdl_wait();
  const int qcols = p.gated ? 2 * hd : hd;  // projection columns per q head
  const int col = gh < p.n_q_heads ? gh * qcols + d : p.n_q_heads * qcols + (gh - p.n_q_heads) * hd + d;
  const size_t stride = static_cast<size_t>(p.part_rows) * p.width;
  auto sum_splits = [&](int c) {
    // up to 16 splits' loads in flight at once (one round trip), summed in
    // split order
    const float* src = p.partials + static_cast<size_t>(t) * p.width + c;
    float a = 0.0f;
    for (int s0 = 0; s0 < p.split; s0 += 16) {
      float x[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) x[k] = s0 + k < p.split ? __ldcg(src + (s0 + k) * stride) : 0.0f;
#pragma unroll
      for (int k = 0; k < 16; ++k)
        if (s0 + k < p.split) a += x[k];
    }
    return a;
  };
  const float a = sum_splits(col);
  if (p.gated && gh < p.n_q_heads)
    p.gate_out[static_cast<size_t>(t) * (p.n_q_heads * hd) + gh * hd + d] = __float2bfloat16_rn(sum_splits(col + hd));
  const int start = p.state->start;
  int slot = start + t;
  float pos_t = 0.0f;
  if (p.slot_mode != 0) {
    const int cnt = p.slot_mode == 1 ? p.state->n_accepted : p.ctx_count;
    const int base = p.slot_mode == 1 ? start - cnt : p.ctx_base;
    if (t >= cnt) return;  // uniform per block
    slot = base + t;
    pos_t = static_cast<float>(slot);
    if (p.ring_window > 0) {
      const int r = (p.slot_mode == 1 ? p.ring_state->reserved : base) + t;
      slot = ring_slot(r, p.ring_sink, p.ring_window);
    }
  } else {
    pos_t = static_cast<float>(p.positions[t]);
  }
  if (gh >= p.n_q_heads + p.n_kv_heads) {  // v
    const int kvh = gh - p.n_q_heads - p.n_kv_heads;
    if (slot >= 0 && slot < p.kv_cap) p.v_cache[(static_cast<size_t>(kvh) * p.kv_cap + slot) * hd + d] = __float2bfloat16_rn(a);
    else dev_error(0x2001u);
    return;
  }
  const float x = bf16_round(a);  // projection output is bf16
  float sq = x * x;
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((d & 31) == 0) s_red[d >> 5] = sq;
  __syncthreads();
  float ss = 0.0f;
  for (int w = 0; w < hd / 32; ++w) ss += s_red[w];
  const bool is_q = gh < p.n_q_heads;
  const float nw = __bfloat162float((is_q ? p.q_norm : p.k_norm)[d]);
  const float y = bf16_round(x * rsqrtf(ss / static_cast<float>(hd) + p.eps) * nw);
  s_y[d] = y;
  __syncthreads();
  const int rd = p.rot_dims > 0 ? p.rot_dims : hd;
  float outv = y;
  if (d < rd) {
    const int half = rd / 2;
    const int i_f = d % half;
    const float inv_freq = exp2f(-(2.0f * static_cast<float>(i_f) / static_cast<float>(rd)) * p.rope_log2_theta);
    float sn, cs;
    sincosf(pos_t * inv_freq, &sn, &cs);
    const float yp = s_y[d < half ? d + half : d - half];
    outv = (d < half) ? (y * cs - yp * sn) : (y * cs + yp * sn);
  }
  if (is_q) {
    p.q_out[static_cast<size_t>(t) * (p.n_q_heads * hd) + gh * hd + d] = __float2bfloat16_rn(outv);
  } else {
    const int kvh = gh - p.n_q_heads;
    if (slot >= 0 && slot < p.kv_cap) p.k_cache[(static_cast<size_t>(kvh) * p.kv_cap + slot) * hd + d] = __float2bfloat16_rn(outv);
    else dev_error(0x2001u);
  }
}

// Prompt rows (dense bf16 projection [rows][width], slot = start + t): one
// warp per (row, head), EPL = head_dim / 32 consecutive features per lane,
// 16-byte or 8-byte loads; the head's sum of squares and the RoPE partner
// (feature i <-> i + rot/2, lane l <-> l ^ (rot/2 / EPL)) move by shuffles,
// so there is no shared memory and no block barrier.  Same arithmetic and
// rounding points as qkv_finish_kernel.  PART: the tree verify's split-K
// fp32 partials in place of the dense projection (summed in split order and
// rounded to bf16, as qkv_finish_kernel does), for plain heads (no output
// gate, full RoPE) at slots start + t.
template <int EPL, bool PART = false>
__global__ void __launch_bounds__(256) qkv_rows_kernel(QkvFinishParams p) {
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int heads = p.n_q_heads + 2 * p.n_kv_heads;
  const long long tasks = static_cast<long long>(p.n_rows) * heads;
  const int hd = EPL * 32;
  const int qcols = p.gated ? 2 * hd : hd;
  const int rd = p.rot_dims > 0 ? p.rot_dims : hd;
  const int half = rd / 2;
  const int pmask = half / EPL;  // partner lane offset (a power of two)
  pdl_wait();
  const int start = p.state->start;
  for (long long task = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; task < tasks;
       task += (static_cast<long long>(gridDim.x) * blockDim.x) >> 5) {
    const int t = static_cast<int>(task / heads), gh = static_cast<int>(task % heads);
    const int d0 = lane * EPL;
    const int col = gh < p.n_q_heads ? gh * qcols + d0 : p.n_q_heads * qcols + (gh - p.n_q_heads) * hd + d0;
    const __nv_bfloat16* src = PART ? nullptr : p.dense + static_cast<size_t>(t) * p.width + col;
    __nv_bfloat16 xv[EPL];
    if constexpr (PART) {
      // up to 8 splits' loads in flight at once, summed in split order
      static_assert(EPL % 2 == 0, "partials in float2 / float4 pieces");
      const float* fsrc = p.partials + static_cast<size_t>(t) * p.width + col;
      const size_t stride = static_cast<size_t>(p.part_rows) * p.width;
      float a[EPL];
#pragma unroll
      for (int i = 0; i < EPL; ++i) a[i] = 0.0f;
      for (int s0 = 0; s0 < p.split; s0 += 8) {
        float v[8][EPL];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (s0 + k < p.split) {
            const float* q = fsrc + (s0 + k) * stride;
#pragma unroll
            for (int c = 0; c < EPL; c += 2) {
              const float2 w = __ldcg(reinterpret_cast<const float2*>(q + c));
              v[k][c] = w.x, v[k][c + 1] = w.y;
            }
          }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (s0 + k < p.split) {
#pragma unroll
            for (int i = 0; i < EPL; ++i) a[i] += v[k][i];
          }
      }
#pragma unroll
      for (int i = 0; i < EPL; ++i) xv[i] = __float2bfloat16_rn(a[i]);
    } else if constexpr (EPL == 8) {
      *reinterpret_cast<uint4*>(xv) = *reinterpret_cast<const uint4*>(src);
    } else if constexpr (EPL == 4) {
      *reinterpret_cast<uint2*>(xv) = *reinterpret_cast<const uint2*>(src);
    } else {
      *reinterpret_cast<uint32_t*>(xv) = *reinterpret_cast<const uint32_t*>(src);
    }
    const int slot = start + t;
    if (gh >= p.n_q_heads + p.n_kv_heads) {  // v
      const int kvh = gh - p.n_q_heads - p.n_kv_heads;
      if (slot >= 0 && slot < p.kv_cap) {
        __nv_bfloat16* dst = p.v_cache + (static_cast<size_t>(kvh) * p.kv_cap + slot) * hd + d0;
#pragma unroll
        for (int i = 0; i < EPL; ++i) dst[i] = xv[i];
      } else if (lane == 0) {
        dev_error(0x2001u);
      }
      continue;
    }
    if (!PART && p.gated && gh < p.n_q_heads) {
      const __nv_bfloat16* gsrc = src + hd;
      __nv_bfloat16* gdst = p.gate_out + static_cast<size_t>(t) * (p.n_q_heads * hd) + gh * hd + d0;
#pragma unroll
      for (int i = 0; i < EPL; ++i) gdst[i] = gsrc[i];
    }
    float x[EPL];
    float sq = 0.0f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      x[i] = __bfloat162float(xv[i]);
      sq = fmaf(x[i], x[i], sq);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const bool is_q = gh < p.n_q_heads;
    const __nv_bfloat16* nwp = (is_q ? p.q_norm : p.k_norm) + d0;
    const float rs = rsqrtf(sq / static_cast<float>(hd) + p.eps);
    float y[EPL], yp[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) y[i] = bf16_round(x[i] * rs * __bfloat162float(nwp[i]));
#pragma unroll
    for (int i = 0; i < EPL; ++i) yp[i] = __shfl_xor_sync(0xffffffffu, y[i], pmask);
    const float pos_t = static_cast<float>(p.positions[t]);
    __nv_bfloat16 ov[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int d = d0 + i;
      float outv = y[i];
      if (d < rd) {
        const int i_f = d % half;
        const float inv_freq = exp2f(-(2.0f * static_cast<float>(i_f) / static_cast<float>(rd)) * p.rope_log2_theta);
        float sn, cs;
        sincosf(pos_t * inv_freq, &sn, &cs);
        outv = (d < half) ? (y[i] * cs - yp[i] * sn) : (y[i] * cs + yp[i] * sn);
      }
      ov[i] = __float2bfloat16_rn(outv);
    }
    __nv_bfloat16* dst;
    if (is_q) {
      dst = p.q_out + static_cast<size_t>(t) * (p.n_q_heads * hd) + gh * hd + d0;
    } else {
      if (slot < 0 || slot >= p.kv_cap) {
        if (lane == 0) dev_error(0x2001u);
        continue;
      }
      dst = p.k_cache + (static_cast<size_t>(gh - p.n_q_heads) * p.kv_cap + slot) * hd + d0;
    }
    if constexpr (EPL == 8) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(ov);
    } else if constexpr (EPL == 4) {
      *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(ov);
    } else {
      *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(ov);
    }
  }
}

int qkv_rows_launch(const QkvFinishParams& p, int n_rows, cudaStream_t stream) {
  DTREE_CHECK_ARG(p.dense && p.positions && p.state && p.q_out && p.k_cache && p.v_cache, "prompt QKV: null pointer");
  DTREE_CHECK_ARG(p.slot_mode == 0 && p.n_q_heads > 0, "prompt QKV: rows at start + t only");
  DTREE_CHECK_ARG(!p.gated || p.gate_out, "gated projection needs gate_out");
  const int hd = p.head_dim;
  const int rd = p.rot_dims > 0 ? p.rot_dims : hd;
  const int epl = hd / 32;
  DTREE_CHECK_ARG(hd == 64 || hd == 128 || hd == 256, "prompt QKV: head_dim 64, 128 or 256");
  DTREE_CHECK_ARG(rd % 2 == 0 && (rd / 2) % epl == 0 && (((rd / 2) / epl) & ((rd / 2) / epl - 1)) == 0 &&
                      (rd / 2) / epl < 32,
                  "prompt QKV: rot_dims / 2 must be a power-of-two multiple of head_dim / 32");
  DTREE_CHECK_ARG(p.width % 8 == 0, "prompt QKV: width must be a multiple of 8");
  QkvFinishParams q = p;
  q.n_rows = n_rows;
  const long long tasks = static_cast<long long>(n_rows) * (p.n_q_heads + 2 * p.n_kv_heads);
  const int grid = static_cast<int>(std::min<long long>((tasks + 7) / 8, 16ll * num_sms()));
  switch (epl) {
    case 2: DTREE_CUDA_RET(launch_pdl(qkv_rows_kernel<2>, dim3(grid), dim3(256), 0, stream, q)); break;
    case 4: DTREE_CUDA_RET(launch_pdl(qkv_rows_kernel<4>, dim3(grid), dim3(256), 0, stream, q)); break;
    default: DTREE_CUDA_RET(launch_pdl(qkv_rows_kernel<8>, dim3(grid), dim3(256), 0, stream, q)); break;
  }
  return kOk;
}

int qkv_finish_launch(const QkvFinishParams& p, int n_rows, cudaStream_t stream) {
  DTREE_CHECK_ARG(p.head_dim % 32 == 0 && p.head_dim <= 256, "head_dim must be a multiple of 32, <= 256");
  DTREE_CHECK_ARG(p.rot_dims >= 0 && p.rot_dims <= p.head_dim && p.rot_dims % 2 == 0, "bad rot_dims");
  DTREE_CHECK_ARG(!p.gated || p.gate_out, "gated projection needs gate_out");
  DTREE_CHECK_ARG(p.partials && !p.dense, "qkv_finish sums split partials (prompt rows: qkv_rows_launch)");
  // (at most 16 rows the one-block-per-(row, head) kernel below is faster:
  // 2.415 against 2.432 ms per 9-row verify; 25 rows 2.557 against 2.542)
  if (n_rows > 16 && p.slot_mode == 0 && !p.gated && (p.rot_dims == 0 || p.rot_dims == p.head_dim) &&
      p.n_q_heads > 0 &&
      (p.head_dim == 64 || p.head_dim == 128) && p.width % 4 == 0 && p.positions &&
      (reinterpret_cast<uintptr_t>(p.partials) & 15) == 0) {
    // tree rows of plain heads: a warp per (row, head), no block barriers
    QkvFinishParams q = p;
    q.n_rows = n_rows;
    const long long tasks = static_cast<long long>(n_rows) * (p.n_q_heads + 2 * p.n_kv_heads);
    // warps per block: at least two blocks per SM where the tasks allow
    const int wpb = static_cast<int>(std::max(1ll, std::min(8ll, tasks / (2ll * num_sms()))));
    const int grid = static_cast<int>(std::min<long long>((tasks + wpb - 1) / wpb, 16ll * num_sms()));
    if (p.head_dim == 128)
      DTREE_CUDA_RET(launch_pdl(qkv_rows_kernel<4, true>, dim3(grid), dim3(32 * wpb), 0, stream, q));
    else
      DTREE_CUDA_RET(launch_pdl(qkv_rows_kernel<2, true>, dim3(grid), dim3(32 * wpb), 0, stream, q));
    return kOk;
  }
  DTREE_CUDA_RET(launch_pdl(qkv_finish_kernel, dim3(n_rows, p.n_q_heads + 2 * p.n_kv_heads), dim3(p.head_dim), 0,
                            stream, p));
  return kOk;
}

}  // namespace dtree
