// extern "C" entry points of libglacier_cuda.so (declared in include/glacier_cuda.h).
#include <stdarg.h>

#include <mutex>
#include <vector>

#include "common.cuh"

namespace glacier {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    cache[dev] = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0 ? n : 148;
  }
  return cache[dev];
}

int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                   uint64_t outer, uint64_t outer_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                   CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo) {
  using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  if (!fn) return set_error(GLACIER_CUDA_ECUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {outer_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(GLACIER_CUDA_ECUDA, "cuTensorMapEncodeTiled failed (%d): inner=%llu outer=%llu stride=%llu",
                     (int)r, (unsigned long long)inner, (unsigned long long)outer,
                     (unsigned long long)outer_stride_bytes);
  return GLACIER_CUDA_OK;
}

int allow_dynamic_smem(const void* kernel, int bytes) {
  GLC_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  return GLACIER_CUDA_OK;
}

template <typename ScaleT>
int gemv_int4(const float* x, size_t ldx, size_t batch, const uint8_t* packed, const ScaleT* scales,
              size_t scale_stride, const float* bias, float* y, size_t ldy, size_t M, size_t K,
              size_t group, cudaStream_t stream);

int gemv_device_error(int clear);

}  // namespace glacier

using namespace glacier;

extern "C" {

const char* glacier_cuda_last_error(void) { return g_last_error; }

int glacier_cuda_version(void) { return (0 << 16) | 1; }

int glacier_cuda_device_status(int clear) {
  GLC_CHECK_CUDA(cudaDeviceSynchronize());
  const int v = gemv_device_error(clear);
  if (v < 0) return set_error(GLACIER_CUDA_ECUDA, "device status read failed");
  return v;
}

int glacier_cuda_int4_matvec_f32(const float* x, const uint8_t* packed, const float* scales,
                                 const float* bias, float* y, size_t out_features, size_t in_features,
                                 size_t group_size, void* stream) {
  GLC_REQUIRE(x && packed && scales && y, "int4_matvec_f32: null pointer");
  return gemv_int4<float>(x, in_features, 1, packed, scales, 0, bias, y, out_features, out_features,
                          in_features, group_size, (cudaStream_t)stream);
}

int glacier_cuda_int4_matvec_f16scale(const float* x, const uint8_t* packed, const uint16_t* scales,
                                      const float* bias, float* y, size_t out_features,
                                      size_t in_features, size_t group_size, void* stream) {
  GLC_REQUIRE(x && packed && scales && y, "int4_matvec_f16scale: null pointer");
  return gemv_int4<__half>(x, in_features, 1, packed, reinterpret_cast<const __half*>(scales), 0, bias,
                           y, out_features, out_features, in_features, group_size, (cudaStream_t)stream);
}

int glacier_cuda_int4_linear(const float* x, size_t batch, const uint8_t* packed, const void* scales,
                             int scale_is_f16, const float* bias, float* y, size_t out_features,
                             size_t in_features, size_t group_size, void* stream) {
  GLC_REQUIRE(x && packed && scales && y, "int4_linear: null pointer");
  if (scale_is_f16)
    return gemv_int4<__half>(x, in_features, batch, packed, static_cast<const __half*>(scales), 0, bias, y,
                             out_features, out_features, in_features, group_size, (cudaStream_t)stream);
  return gemv_int4<float>(x, in_features, batch, packed, static_cast<const float*>(scales), 0, bias, y,
                          out_features, out_features, in_features, group_size, (cudaStream_t)stream);
}

}  // extern "C"
