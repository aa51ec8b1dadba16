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
  float ss = 0.0f;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const uint4 v = s4[i];
    if (tokens && h_out) reinterpret_cast<uint4*>(h_out + static_cast<size_t>(row) * H)[i] = v;
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(b[j]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int i = 0; i < (blockDim.x >> 5); ++i) tot += red[i];
  const float rs = rsqrtf(tot / static_cast<float>(H) + eps);
  const uint4* w4 = reinterpret_cast<const uint4*>(w);
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const uint4 v = s4[i], wv = w4[i];
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
    const __nv_bfloat162* wb = reinterpret_cast<const __nv_bfloat162*>(&wv);
    uint4 o4;
    __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o4);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(b[j]);
      const float2 g = __bfloat1622float2(wb[j]);
      ob[j] = __floats2bfloat162_rn(f.x * rs * g.x, f.y * rs * g.y);
    }
    yrow[i] = o4;
  }
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
