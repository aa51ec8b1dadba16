// Host side of the stream-K tcgen05 GEMM: plans (tensor maps + params),
// dispatch over tile widths / epilogues, and the dense-linear and LM-head
// argmax entry points.
#include <algorithm>

#include "gemm.cuh"

namespace dtree {

// workspace: [tile counters][argmax keys][done][partials grid*2*t_pad*128 f32]
// The counters sit at fixed offsets so every plan bound to the same workspace
// (any grid, any t_pad) shares them; each fix-up resets its counter to zero.
constexpr int kMaxTileCounters = 8192;
constexpr int kMaxArgmaxRows = 256;
constexpr size_t kCountersBytes = kMaxTileCounters * 4 + kMaxArgmaxRows * 8 + 256;

struct GemmWs {
  float* partials;
  uint32_t* tile_cnt;
  unsigned long long* keys;
  uint32_t* done;
};

static size_t ws_partial_bytes(int t_pad, int grid) {
  return (static_cast<size_t>(grid) * 2 * t_pad * 128 * 4 + 255) & ~static_cast<size_t>(255);
}

size_t gemm_ws_bytes(int t_pad, int grid) { return kCountersBytes + ws_partial_bytes(t_pad, grid); }
size_t gemm_ws_counter_bytes() { return kCountersBytes; }

// MLX affine 4-bit weights -> bf16 [n_out][k] (the prompt path's dense GEMMs
// read bf16): thread = one packed word (8 weights, one 16-byte store), the
// same bf16 fma rounding as the fused q4 verify GEMM (dequant8).
__global__ void __launch_bounds__(256) dequant_q4_kernel(const uint32_t* __restrict__ packed,
                                                         const __nv_bfloat16* __restrict__ scales,
                                                         const __nv_bfloat16* __restrict__ biases, int n_out, int k,
                                                         uint4* __restrict__ out) {
  pdl_trigger();
  const int wpr = k / 8;  // words per row
  const size_t total = static_cast<size_t>(n_out) * wpr;
  pdl_wait();
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = i / wpr;
    const int w = static_cast<int>(i % wpr);
    const size_t g = row * (k / 64) + w / 8;
    const __nv_bfloat16 sc = scales[g], bi = biases[g];
    out[i] = dequant8(__ldg(packed + i), __halves2bfloat162(sc, sc), __halves2bfloat162(bi, bi));
  }
}

int dequant_q4_launch(const void* packed, const void* scales, const void* biases, int n_out, int k, void* out,
                      cudaStream_t st) {
  DTREE_CHECK_ARG(packed && scales && biases && out, "null pointer");
  DTREE_CHECK_ARG(k % 64 == 0 && n_out > 0, "K must be a multiple of 64");
  const size_t total = static_cast<size_t>(n_out) * (k / 8);
  const int grid = static_cast<int>(std::min<size_t>((total + 255) / 256, static_cast<size_t>(num_sms()) * 8));
  DTREE_CUDA_RET(launch_pdl(dequant_q4_kernel, dim3(grid), dim3(256), 0, st, static_cast<const uint32_t*>(packed),
                            static_cast<const __nv_bfloat16*>(scales), static_cast<const __nv_bfloat16*>(biases),
                            n_out, k, static_cast<uint4*>(out)));
  return kOk;
}

static GemmWs ws_split(void* base) {
  GemmWs w;
  char* b = static_cast<char*>(base);
  w.tile_cnt = reinterpret_cast<uint32_t*>(b);
  w.keys = reinterpret_cast<unsigned long long*>(b + kMaxTileCounters * 4);
  w.done = reinterpret_cast<uint32_t*>(b + kMaxTileCounters * 4 + kMaxArgmaxRows * 8);
  w.partials = reinterpret_cast<float*>(b + kCountersBytes);
  return w;
}

static bool valid_tpad(int t) { return t == 16 || t == 32 || t == 64 || t == 80 || t == 128; }

// activation map, split / grid choice and parameters shared by both weight formats
// `wide` kernels (one CTA per SM) would run a second wave above the SM
// count; both weight formats now fit two CTAs per SM.
// `kunit` = K elements per stream-K unit (64 bf16, 128 for 4-bit weights).
static int plan_common(GemmPlan* plan, int n_out, int k, const void* x, int t_pad, int x_row_stride_elems, int epi,
                       int grid, bool wide, int kunit) {
  DTREE_CHECK_ARG(valid_tpad(t_pad), "t_pad must be 16, 32, 64, 80 or 128");
  DTREE_CHECK_ARG(k % 64 == 0 && k > 0, "K must be a positive multiple of 64");
  DTREE_CHECK_ARG(n_out > 0, "N must be positive");
  const int m_tiles = (n_out + 127) / 128;
  DTREE_CHECK_ARG(m_tiles <= kMaxTileCounters, "N too large");
  int rc = make_tmap_2d_bf16(&plan->tmap_x, x, static_cast<uint64_t>(k), static_cast<uint64_t>(t_pad),
                             static_cast<uint64_t>(x_row_stride_elems) * 2, 64, static_cast<uint32_t>(t_pad), true);
  if (rc) return rc;
  GemmParams& p = plan->p;
  p = GemmParams{};
  p.n_out = n_out;
  p.kb = (k + kunit - 1) / kunit;  // (4-bit: the last unit of a row may be partial)
  p.m_tiles = m_tiles;
  p.n_rows = t_pad;
  p.n_tiles = 1;
  const long long units = static_cast<long long>(m_tiles) * p.kb;
  const int sms = num_sms();
  if (epi == kEpiPartial) {
    // tile-aligned split-K: the consumer sums the fp32 partials
    int split = grid > 0 ? grid : sms / m_tiles;
    if (split < 1) split = 1;
    if (split > p.kb) split = p.kb;
    p.split = split;
    p.grid = m_tiles * split;
  } else if (grid > 0) {
    p.grid = static_cast<int>(units < grid ? units : grid);
  } else if (m_tiles >= (sms * 9) / 10 && m_tiles <= (wide ? sms : 2 * sms)) {
    // one whole tile per CTA, up to two CTAs per SM (both fit), all in one
    // wave: no partial tiles at all (the Qwen3.5-9B gate|up, 192 tiles, ran
    // 0.16 ms faster per verify than stream-K over 148 CTAs)
    p.grid = m_tiles;
  } else if (m_tiles < (sms * 9) / 10 && 2 * m_tiles >= (sms * 9) / 10 && units >= 2ll * m_tiles) {
    // two CTAs per tile (the K halves), both CTA slots of an SM busy, one
    // fix-up per tile (the Qwen3.5-9B in_proj, 97 tiles: 0.11 ms per verify
    // faster than stream-K over 148 CTAs)
    p.grid = 2 * m_tiles;
  } else {
    p.grid = static_cast<int>(units < sms ? units : sms);
  }
  DTREE_CHECK_ARG(units * p.grid < (1ll << 31), "stream-K index range exceeds 32 bits");
  plan->t_pad = t_pad;
  plan->epi = epi;
  plan->q4 = false;
  return kOk;
}

int gemm_plan(GemmPlan* plan, const void* w, int n_out, int k, const void* x, int t_pad, int x_row_stride_elems,
              int epi, int grid) {
  int rc = plan_common(plan, n_out, k, x, t_pad, x_row_stride_elems, epi, grid, false, 64);
  if (rc) return rc;
  return make_tmap_2d_bf16(&plan->tmap_w, w, static_cast<uint64_t>(k), static_cast<uint64_t>(n_out),
                           static_cast<uint64_t>(k) * 2, 64, 128, true);
}

int gemm_plan_q4(GemmPlan* plan, const void* w_packed, const void* sb, int n_out, int k, const void* x, int t_pad,
                 int x_row_stride_elems, int epi, int grid) {
  DTREE_CHECK_ARG(w_packed && sb, "null q4 weight pointer");
  DTREE_CHECK_ARG(reinterpret_cast<uintptr_t>(sb) % 16 == 0, "q4 scale / bias blocks must be 16-byte aligned");
  DTREE_CHECK_ARG(epi == kEpiStore || epi == kEpiPartial || epi == kEpiSwiglu || epi == kEpiArgmax,
                  "q4 GEMM supports the store, split-K partial, SwiGLU and argmax epilogues");
  int rc = plan_common(plan, n_out, k, x, t_pad, x_row_stride_elems, epi, grid, false, 64 * kQ4Kb);
  if (rc) return rc;
  // packed weight map: box 8 * kQ4Kb words (one stream-K unit of K, 64 B)
  // x 128 rows, 64-byte swizzled
  rc = make_tmap_2d_u32(&plan->tmap_w, w_packed, static_cast<uint64_t>(k / 8), static_cast<uint64_t>(n_out),
                        static_cast<uint64_t>(k / 2), 8 * kQ4Kb, 128, 32 * kQ4Kb);
  if (rc) return rc;
  plan->p.q_sb = static_cast<const uint8_t*>(sb);
  plan->q4 = true;
  return kOk;
}

size_t q4_sb_bytes(int n_out, int k) {
  const size_t m_tiles = (static_cast<size_t>(n_out) + 127) / 128;
  const size_t units = (static_cast<size_t>(k) + 64 * kQ4Kb - 1) / (64 * kQ4Kb);
  return m_tiles * units * kQ4SbBlock;
}

// One thread per (m tile, unit, row): the row's (s0, s1, b0, b1) for the
// unit's groups 2u, 2u + 1 (MLX bf16 [n][k/64] scales and biases), zeros
// past the last row or group.
__global__ void q4_sb_repack_kernel(const __nv_bfloat16* __restrict__ scales, const __nv_bfloat16* __restrict__ biases,
                                    int n_out, int groups, int units, long long total, uint2* __restrict__ out) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int r = static_cast<int>(i % 128);
  const long long tu = i / 128;
  const int u = static_cast<int>(tu % units);
  const long long n = (tu / units) * 128 + r;
  __nv_bfloat16 v[4];
  const __nv_bfloat16 z = __float2bfloat16_rn(0.0f);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int g = u * kQ4Kb + j;
    const bool in = n < n_out && g < groups;
    v[j] = in ? scales[n * groups + g] : z;
    v[2 + j] = in ? biases[n * groups + g] : z;
  }
  uint2 o;
  o.x = static_cast<uint32_t>(__bfloat16_as_ushort(v[0])) | (static_cast<uint32_t>(__bfloat16_as_ushort(v[1])) << 16);
  o.y = static_cast<uint32_t>(__bfloat16_as_ushort(v[2])) | (static_cast<uint32_t>(__bfloat16_as_ushort(v[3])) << 16);
  out[i] = o;
}

int q4_sb_repack_launch(const void* scales, const void* biases, int n_out, int k, void* sb, cudaStream_t stream) {
  DTREE_CHECK_ARG(scales && biases && sb, "null pointer");
  DTREE_CHECK_ARG(k % 64 == 0 && k > 0 && n_out > 0, "q4 repack: K must be a positive multiple of 64");
  static_assert(kQ4Kb == 2, "a scale / bias block holds two groups per row");
  const int groups = k / 64;
  const int units = (k + 64 * kQ4Kb - 1) / (64 * kQ4Kb);
  const long long total = static_cast<long long>((n_out + 127) / 128) * units * 128;
  const int threads = 256;
  q4_sb_repack_kernel<<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(scales), static_cast<const __nv_bfloat16*>(biases), n_out, groups, units,
      total, static_cast<uint2*>(sb));
  DTREE_CUDA_RET(cudaGetLastError());
  return kOk;
}

int gemm_plan_dense(GemmPlan* plan, const void* w, int n_out, int k, const void* x, int n_rows, int x_rows,
                    int x_row_stride_elems, int epi) {
  DTREE_CHECK_ARG(w && x, "null pointer");
  DTREE_CHECK_ARG(epi == kEpiStore || epi == kEpiResidual || epi == kEpiSwiglu,
                  "dense GEMM supports the store, residual and SwiGLU epilogues");
  DTREE_CHECK_ARG(k % 64 == 0 && k > 0, "K must be a positive multiple of 64");
  DTREE_CHECK_ARG(n_out > 0 && n_rows > 0, "N and rows must be positive");
  const int n_tiles = (n_rows + kDenseRows - 1) / kDenseRows;
  DTREE_CHECK_ARG(x_rows >= n_tiles * kDenseRows, "activation buffer must hold the rows padded to 256");
  const int m_tiles = (n_out + 127) / 128;
  DTREE_CHECK_ARG(static_cast<long long>(m_tiles) * n_tiles <= kMaxTileCounters, "N x rows too large");
  int rc = make_tmap_2d_bf16(&plan->tmap_x, x, static_cast<uint64_t>(k), static_cast<uint64_t>(x_rows),
                             static_cast<uint64_t>(x_row_stride_elems) * 2, 64, kDenseRows, true);
  if (rc) return rc;
  if ((rc = make_tmap_2d_bf16(&plan->tmap_w, w, static_cast<uint64_t>(k), static_cast<uint64_t>(n_out),
                              static_cast<uint64_t>(k) * 2, 64, 128, true)))
    return rc;
  GemmParams& p = plan->p;
  p = GemmParams{};
  p.n_out = n_out;
  p.kb = k / 64;
  p.m_tiles = m_tiles;
  p.n_tiles = n_tiles;
  p.n_rows = n_rows;
  const long long units = static_cast<long long>(m_tiles) * n_tiles * p.kb;
  const int sms = num_sms();
  p.grid = static_cast<int>(units < sms ? units : sms);
  DTREE_CHECK_ARG(units * p.grid < (1ll << 31), "stream-K index range exceeds 32 bits");
  plan->t_pad = kDenseRows;
  plan->epi = epi;
  plan->q4 = false;
  return kOk;
}

int gemm_bind_ws(GemmPlan* plan, void* ws, size_t ws_bytes) {
  // split-K partial plans write every tile straight to out_f32: only the
  // counter block of the workspace is touched
  const size_t need = plan->epi == kEpiPartial ? kCountersBytes : gemm_ws_bytes(plan->t_pad, plan->p.grid);
  DTREE_CHECK_ARG(ws != nullptr && ws_bytes >= need, "GEMM workspace too small");
  GemmWs w = ws_split(ws);
  plan->p.ws = w.partials;
  plan->p.tile_cnt = w.tile_cnt;
  plan->p.argmax_keys = w.keys;
  plan->p.done_cnt = w.done;
  return kOk;
}

template <int TPAD, int EPI, bool Q4 = false>
static int launch_t(const GemmPlan& pl, cudaStream_t st) {
  using C = GemmCfg<TPAD, EPI, Q4>;
  auto kern = gemm_streamk_kernel<TPAD, EPI, Q4>;
  DTREE_CUDA_RET(ensure_smem_attr(kern, C::kSmem));
  DTREE_CUDA_RET(launch_pdl(kern, dim3(pl.p.grid), dim3(Q4 ? kGemmThreadsQ4 : kGemmThreads),
                            static_cast<size_t>(C::kSmem), st, pl.tmap_w, pl.tmap_x, pl.p));
  return kOk;
}

template <int TPAD>
static int launch_epi(const GemmPlan& pl, cudaStream_t st) {
  if (pl.q4) {
    switch (pl.epi) {
      case kEpiStore: return launch_t<TPAD, kEpiStore, true>(pl, st);
      case kEpiSwiglu: return launch_t<TPAD, kEpiSwiglu, true>(pl, st);
      case kEpiPartial: return launch_t<TPAD, kEpiPartial, true>(pl, st);
      case kEpiArgmax: return launch_t<TPAD, kEpiArgmax, true>(pl, st);
    }
    return fail(kErrInvalidArg, "epilogue not available for q4 weights");
  }
  switch (pl.epi) {
    case kEpiStore: return launch_t<TPAD, kEpiStore>(pl, st);
    case kEpiResidual: return launch_t<TPAD, kEpiResidual>(pl, st);
    case kEpiSwiglu: return launch_t<TPAD, kEpiSwiglu>(pl, st);
    case kEpiQkv: return launch_t<TPAD, kEpiQkv>(pl, st);
    case kEpiArgmax: return launch_t<TPAD, kEpiArgmax>(pl, st);
    case kEpiPartial: return launch_t<TPAD, kEpiPartial>(pl, st);
  }
  return fail(kErrInvalidArg, "unknown epilogue");
}

int gemm_launch(const GemmPlan& pl, cudaStream_t st) {
  switch (pl.t_pad) {
    case 16: return launch_epi<16>(pl, st);
    case 32: return launch_epi<32>(pl, st);
    case 64: return launch_epi<64>(pl, st);
    case 80: return launch_epi<80>(pl, st);
    case 128: return launch_epi<128>(pl, st);
    case kDenseRows:
      switch (pl.epi) {  // dense (prefill) tiles: bf16 weights, no split-K / argmax / q|k|v epilogues
        case kEpiStore: return launch_t<kDenseRows, kEpiStore>(pl, st);
        case kEpiResidual: return launch_t<kDenseRows, kEpiResidual>(pl, st);
        case kEpiSwiglu: return launch_t<kDenseRows, kEpiSwiglu>(pl, st);
      }
      return fail(kErrInvalidArg, "epilogue not available for dense tiles");
  }
  return fail(kErrInvalidArg, "bad t_pad");
}

}  // namespace dtree

using namespace dtree;

extern "C" size_t dtree_linear_workspace_bytes(int t_pad, int n) {
  (void)n;
  return gemm_ws_bytes(t_pad, 2 * num_sms());
}

extern "C" int dtree_linear_bf16(const void* x, int t_pad, int k, const void* w, int n, void* y, void* workspace,
                                 size_t workspace_bytes, int split_k, void* stream) {
  DTREE_CHECK_ARG(x && w && y, "null pointer");
  GemmPlan plan;
  int rc = gemm_plan(&plan, w, n, k, x, t_pad, k, kEpiStore, split_k > 0 ? split_k : 0);
  if (rc) return rc;
  rc = gemm_bind_ws(&plan, workspace, workspace_bytes);
  if (rc) return rc;
  plan.p.out = static_cast<__nv_bfloat16*>(y);
  plan.p.ldo = n;
  return gemm_launch(plan, static_cast<cudaStream_t>(stream));
}

extern "C" size_t dtree_linear_q4_workspace_bytes(int t_pad, int n, int k) {
  return ((gemm_ws_bytes(t_pad, 2 * num_sms()) + 255) & ~static_cast<size_t>(255)) + q4_sb_bytes(n, k);
}

extern "C" int dtree_linear_q4(const void* x, int t_pad, int k, const void* w_packed, const void* scales,
                               const void* biases, int n, void* y, void* workspace, size_t workspace_bytes,
                               int split_k, void* stream) {
  DTREE_CHECK_ARG(x && y && workspace, "null pointer");
  DTREE_CHECK_ARG(n > 0 && k > 0 && k % 64 == 0, "N must be positive and K a positive multiple of 64");
  DTREE_CHECK_ARG(workspace_bytes >= dtree_linear_q4_workspace_bytes(t_pad, n, k),
                  "workspace smaller than dtree_linear_q4_workspace_bytes");
  const size_t ws_gemm = (gemm_ws_bytes(t_pad, 2 * num_sms()) + 255) & ~static_cast<size_t>(255);
  void* sb = static_cast<char*>(workspace) + ws_gemm;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the scale / bias blocks of this call's weight, then the GEMM
  int rc = q4_sb_repack_launch(scales, biases, n, k, sb, st);
  if (rc) return rc;
  GemmPlan plan;
  rc = gemm_plan_q4(&plan, w_packed, sb, n, k, x, t_pad, k, kEpiStore, split_k > 0 ? split_k : 0);
  if (rc) return rc;
  rc = gemm_bind_ws(&plan, workspace, ws_gemm);
  if (rc) return rc;
  plan.p.out = static_cast<__nv_bfloat16*>(y);
  plan.p.ldo = n;
  return gemm_launch(plan, static_cast<cudaStream_t>(stream));
}

extern "C" size_t dtree_lm_head_workspace_bytes(int t_pad) { return gemm_ws_bytes(t_pad, 2 * num_sms()); }

extern "C" int dtree_lm_head_sample(const void* h, int t_pad, int n_rows, int hidden, const void* embed, int vocab,
                                    float temperature, uint32_t seed, const dtree_step_state* state, int32_t* out,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  DTREE_CHECK_ARG(h && embed && out, "null pointer");
  DTREE_CHECK_ARG(n_rows > 0 && n_rows <= t_pad, "n_rows must be in [1, t_pad]");
  DTREE_CHECK_ARG(temperature >= 0.0f, "temperature must be >= 0");
  GemmPlan plan;
  int rc = gemm_plan(&plan, embed, vocab, hidden, h, t_pad, hidden, kEpiArgmax, 0);
  if (rc) return rc;
  rc = gemm_bind_ws(&plan, workspace, workspace_bytes);
  if (rc) return rc;
  plan.p.n_rows = n_rows;
  plan.p.vocab = vocab;
  plan.p.argmax_out = out;
  plan.p.inv_temp = temperature < 1e-5f ? 0.0f : 1.0f / temperature;
  plan.p.sample_seed = seed;
  plan.p.sample_state = state;
  return gemm_launch(plan, static_cast<cudaStream_t>(stream));
}

extern "C" int dtree_lm_head_argmax(const void* h, int t_pad, int n_rows, int hidden, const void* embed, int vocab,
                                    int32_t* out, void* workspace, size_t workspace_bytes, void* stream) {
  DTREE_CHECK_ARG(h && embed && out, "null pointer");
  DTREE_CHECK_ARG(n_rows > 0 && n_rows <= t_pad, "n_rows must be in [1, t_pad]");
  GemmPlan plan;
  int rc = gemm_plan(&plan, embed, vocab, hidden, h, t_pad, hidden, kEpiArgmax, 0);
  if (rc) return rc;
  rc = gemm_bind_ws(&plan, workspace, workspace_bytes);
  if (rc) return rc;
  plan.p.n_rows = n_rows;
  plan.p.vocab = vocab;
  plan.p.argmax_out = out;
  return gemm_launch(plan, static_cast<cudaStream_t>(stream));
}
