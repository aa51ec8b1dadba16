// RMSNorm (mlx nn.RMSNorm / mx.fast.rms_norm: y = x * rsqrt(mean(x^2) + eps) * w)
// with an optional fused embedding gather for the first layer.
#include "common.cuh"

namespace dtree {

// grid = t_pad rows, block 256.  Rows >= n_rows are written as zeros.
// If `tokens` is non-null the input row is embed[tokens[row]] and is also
// copied to h_out (the residual stream).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                      const int32_t* __restrict__ tokens,
                                                      const __nv_bfloat16* __restrict__ embed,
                                                      __nv_bfloat16* __restrict__ h_out,
                                                      const __nv_bfloat16* __restrict__ w,
                                                      __nv_bfloat16* __restrict__ y, int H, int n_rows, float eps) {
  pdl_trigger();
  __shared__ float red[8];
  const int row = blockIdx.x;
  const int nv = H / 8;
  pdl_wait();
  uint4* yrow = reinterpret_cast<uint4*>(y + static_cast<size_t>(row) * H);
  if (row >= n_rows) {
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      yrow[i] = z;
      if (tokens && h_out) reinterpret_cast<uint4*>(h_out + static_cast<size_t>(row) * H)[i] = z;
    }
    return;
  }
  const __nv_bfloat16* src = tokens ? embed + static_cast<size_t>(tokens[row]) * H : x + static_cast<size_t>(row) * ldx;
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  const uint4* w4 = reinterpret_cast<const uint4*>(w);
  // the row stays in registers between the two passes (H <= 4096: two
  // 16-byte vectors per thread); wider rows re-read it
  constexpr int kCache = 2;
  uint4 cache[kCache], wcache[kCache];
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kCache; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < nv) {
      cache[j] = s4[i];
      wcache[j] = w4[i];
    }
  }
#pragma unroll
  for (int j = 0; j < kCache; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < nv) {
      if (tokens && h_out) reinterpret_cast<uint4*>(h_out + static_cast<size_t>(row) * H)[i] = cache[j];
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&cache[j]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(b[q]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
  }
  for (int i = threadIdx.x + kCache * blockDim.x; i < nv; i += blockDim.x) {
    const uint4 v = s4[i];
    if (tokens && h_out) reinterpret_cast<uint4*>(h_out + static_cast<size_t>(row) * H)[i] = v;
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __bfloat1622float2(b[q]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int i = 0; i < (blockDim.x >> 5); ++i) tot += red[i];
  const float rs = rsqrtf(tot / static_cast<float>(H) + eps);
  auto norm_vec = [&](const uint4& v, const uint4& wv) {
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
    const __nv_bfloat162* wb = reinterpret_cast<const __nv_bfloat162*>(&wv);
    uint4 o4;
    __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o4);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __bfloat1622float2(b[q]);
      const float2 g = __bfloat1622float2(wb[q]);
      ob[q] = __floats2bfloat162_rn(f.x * rs * g.x, f.y * rs * g.y);
    }
    return o4;
  };
#pragma unroll
  for (int j = 0; j < kCache; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < nv) yrow[i] = norm_vec(cache[j], wcache[j]);
  }
  for (int i = threadIdx.x + kCache * blockDim.x; i < nv; i += blockDim.x) yrow[i] = norm_vec(s4[i], w4[i]);
}

// Residual add of a split-K projection fused with the next RMSNorm:
//   y      = bf16(sum_s partials[s][row])          (fixed split order)
//   h[row] = bf16(h[row] + y)                      (qwen3_tree.py:78,82 residual adds)
//   capture[row] = h[row]            (optional: verifier_hidden of this layer)
//   xn[row] = RMSNorm(h[row], w)
// A row is spread over a cluster of kNormCluster CTAs (grid (kNormCluster,
// t_pad)), one 8-wide column vector per thread, so every load of the row is
// in flight at once; the CTAs' sums of squares meet through distributed
// shared memory (summed in CTA-rank order: deterministic).  H <= 4096.
constexpr int kNormCluster = 4;
constexpr int kNormThreads = 128;

__global__ void __launch_bounds__(kNormThreads) residual_rmsnorm_kernel(
    __nv_bfloat16* __restrict__ h, const float* __restrict__ partials, int n_split, int part_rows,
    __nv_bfloat16* __restrict__ capture, int ldc, const __nv_bfloat16* __restrict__ w,
    __nv_bfloat16* __restrict__ xn, int H, int n_rows, float eps) {
  pdl_trigger();
  __shared__ float red[kNormThreads / 32];
  __shared__ float s_ss;  // this CTA's share of the row's sum of squares
  const int rank = blockIdx.x, row = blockIdx.y;
  const int nv = H / 8;
  const int per = (nv + kNormCluster - 1) / kNormCluster;
  const int i = rank * per + threadIdx.x;
  const bool act = threadIdx.x < per && i < nv;
  pdl_wait();
  uint4* xrow = reinterpret_cast<uint4*>(xn + static_cast<size_t>(row) * H);
  uint4* hrow = reinterpret_cast<uint4*>(h + static_cast<size_t>(row) * H);
  if (row >= n_rows) {  // uniform over the cluster: no cluster barrier is entered
    if (act) {
      xrow[i] = make_uint4(0, 0, 0, 0);
      hrow[i] = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  float ss = 0.0f;
  uint4 o = make_uint4(0, 0, 0, 0);
  if (act) {
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = 0.0f;
    const uint4 hv = hrow[i];
    // all splits' loads of a batch are in flight together; the sum still
    // runs in split order
    constexpr int kB = 16;  // splits per batch: the projections' split-K (<= 16) in one round trip
    for (int s0 = 0; s0 < n_split; s0 += kB) {
      float4 a[kB], b[kB];
#pragma unroll
      for (int k = 0; k < kB; ++k) {
        if (s0 + k < n_split) {
          const float4* pp =
              reinterpret_cast<const float4*>(partials + (static_cast<size_t>(s0 + k) * part_rows + row) * H) + 2 * i;
          a[k] = __ldcg(pp);
          b[k] = __ldcg(pp + 1);
        }
      }
#pragma unroll
      for (int k = 0; k < kB; ++k) {
        if (s0 + k < n_split) {
          y[0] += a[k].x; y[1] += a[k].y; y[2] += a[k].z; y[3] += a[k].w;
          y[4] += b[k].x; y[5] += b[k].y; y[6] += b[k].z; y[7] += b[k].w;
        }
      }
    }
    const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&hv);
    __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __bfloat1622float2(hb[q]);
      ob[q] = __floats2bfloat162_rn(f.x + bf16_round(y[2 * q]), f.y + bf16_round(y[2 * q + 1]));
      const float2 g = __bfloat1622float2(ob[q]);
      ss += g.x * g.x + g.y * g.y;
    }
    hrow[i] = o;
    if (capture) reinterpret_cast<uint4*>(capture + static_cast<size_t>(row) * ldc)[i] = o;
  }
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int k = 0; k < kNormThreads / 32; ++k) t += red[k];
    s_ss = t;
  }
  cluster_arrive();  // s_ss of every CTA is published
  cluster_wait();
  float tot = 0.0f;
  for (int r = 0; r < kNormCluster; ++r) tot += ld_dsmem_f32(&s_ss, static_cast<uint32_t>(r));
  cluster_arrive();  // done reading the other CTAs' shared memory
  const float rs = rsqrtf(tot / static_cast<float>(H) + eps);
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
    xrow[i] = o4;
  }
  cluster_wait();  // no CTA leaves while another may still read its s_ss
}

int residual_rmsnorm_launch(__nv_bfloat16* h, const float* partials, int n_split, int part_rows,
                            __nv_bfloat16* capture, int ldc, const __nv_bfloat16* w, __nv_bfloat16* xn, int H,
                            int n_rows, int t_pad, float eps, cudaStream_t stream) {
  DTREE_CHECK_ARG(H % 8 == 0 && H / 8 <= kNormCluster * kNormThreads, "hidden size must be a multiple of 8 and <= 4096");
  DTREE_CUDA_RET(launch_pdl_cluster(residual_rmsnorm_kernel, dim3(kNormCluster, t_pad), dim3(kNormThreads), 0, stream,
                                    kNormCluster, h, partials, n_split, part_rows, capture, ldc, w, xn, H, n_rows,
                                    eps));
  return kOk;
}

int rmsnorm_launch(const __nv_bfloat16* x, int ldx, const int32_t* tokens, const __nv_bfloat16* embed,
                   __nv_bfloat16* h_out, const __nv_bfloat16* w, __nv_bfloat16* y, int H, int n_rows, int t_pad,
                   float eps, cudaStream_t stream) {
  DTREE_CHECK_ARG(H % 8 == 0, "hidden size must be a multiple of 8");
  DTREE_CUDA_RET(launch_pdl(rmsnorm_kernel, dim3(t_pad), dim3(256), 0, stream, x, ldx, tokens, embed, h_out, w, y, H,
                            n_rows, eps));
  return kOk;
}

}  // namespace dtree
