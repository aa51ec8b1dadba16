// Library-wide state: last-error string, device error word, tensor maps.
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "../../include/dtree_b200.h"

namespace dtree {

__device__ unsigned int g_dtree_dev_error = 0;

static thread_local std::string t_last_error = "no error";

void set_last_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                      uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(kErrCuda, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return fail(kErrInvalidArg, "TMA base not 16-byte aligned");
  if (row_stride_bytes % 16 != 0) return fail(kErrInvalidArg, "TMA row stride not a multiple of 16 bytes");
  if ((box_inner * 2) % 16 != 0) return fail(kErrInvalidArg, "TMA box inner extent not a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(kErrCuda, "cuTensorMapEncodeTiled failed: " + std::to_string(static_cast<int>(r)));
  return kOk;
}

int make_tmap_2d_u32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                     uint32_t box_inner, uint32_t box_outer, int swizzle_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(kErrCuda, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return fail(kErrInvalidArg, "TMA base not 16-byte aligned");
  if (row_stride_bytes % 16 != 0) return fail(kErrInvalidArg, "TMA row stride not a multiple of 16 bytes");
  if ((box_inner * 4) % 16 != 0) return fail(kErrInvalidArg, "TMA box inner extent not a multiple of 16 bytes");
  if (swizzle_bytes != 0 && swizzle_bytes != 64 && swizzle_bytes != 128) return fail(kErrInvalidArg, "bad TMA swizzle");
  if (swizzle_bytes && box_inner * 4 != static_cast<uint32_t>(swizzle_bytes))
    return fail(kErrInvalidArg, "a swizzled u32 box row must span the swizzle width");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                       : (swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE),
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(kErrCuda, "cuTensorMapEncodeTiled failed: " + std::to_string(static_cast<int>(r)));
  return kOk;
}

cudaError_t ensure_smem_attr_fn(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> done;
  std::lock_guard<std::mutex> lock(mu);
  auto it = done.find(kernel);
  if (it != done.end() && it->second >= bytes) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done[kernel] = bytes;
  return e;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

}  // namespace dtree

extern "C" const char* dtree_last_error(void) { return dtree::t_last_error.c_str(); }

extern "C" int dtree_version(void) { return 100; }

extern "C" int dtree_device_error(uint32_t* code_out, int clear) {
  DTREE_CUDA_RET(cudaDeviceSynchronize());
  unsigned int v = 0;
  DTREE_CUDA_RET(cudaMemcpyFromSymbol(&v, dtree::g_dtree_dev_error, sizeof(v)));
  if (code_out) *code_out = v;
  if (clear) {
    unsigned int z = 0;
    DTREE_CUDA_RET(cudaMemcpyToSymbol(dtree::g_dtree_dev_error, &z, sizeof(z)));
  }
  return dtree::kOk;
}

// ------------------------------------------------------------ test hook
namespace dtree {
// One thread: let the next kernel on the stream start (programmatic dependent
// launch), wait `delay_ns` on the global timer (bounded: at most 2^22 polls),
// then store `value` -- a device write that lands while a dependent kernel
// that read the old value early is already running.
__global__ void delayed_store_kernel(int32_t* dst, int32_t value, unsigned long long delay_ns) {
  pdl_trigger();
  unsigned long long t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 >= delay_ns) break;
  }
  *dst = value;
}
}  // namespace dtree

extern "C" int dtree_test_delayed_store(int32_t* dst, int32_t value, int delay_ns, void* stream) {
  DTREE_CHECK_ARG(dst, "null pointer");
  DTREE_CHECK_ARG(delay_ns >= 0 && delay_ns <= 10000000, "delay_ns must be in [0, 1e7]");
  DTREE_CUDA_RET(dtree::launch_pdl(dtree::delayed_store_kernel, dim3(1), dim3(1), 0,
                                   static_cast<cudaStream_t>(stream), dst, value,
                                   static_cast<unsigned long long>(delay_ns)));
  return dtree::kOk;
}
