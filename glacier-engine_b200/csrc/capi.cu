// extern "C" entry points of libglacier_cuda.so (declared in include/glacier_cuda.h).
#include <stdarg.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace glacier {

static thread_local char g_last_error[512] = "";
static std::atomic<unsigned long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

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

void* device_symbol_address_raw(const void* symbol) {
  constexpr int kMaxDevices = 64, kMaxSymbols = 16;
  struct Slot {
    const void* symbol;
    void* address;
  };
  static Slot table[kMaxDevices][kMaxSymbols] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  for (auto& e : table[dev]) {
    if (e.symbol == symbol) return e.address;
    if (!e.symbol) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, symbol) != cudaSuccess) return nullptr;
      e.symbol = symbol;
      e.address = p;
      return p;
    }
  }
  void* p = nullptr;
  return cudaGetSymbolAddress(&p, symbol) == cudaSuccess ? p : nullptr;
}

// The attribute belongs to the kernel on one device, so the largest size set so
// far is remembered per (kernel, current device) under a mutex: a process that
// drives several GPUs sets it once on each, and concurrent host threads neither
// race on the record nor skip the call.
int allow_dynamic_smem(const void* kernel, int bytes) {
  struct Entry {
    const void* kernel;
    int device;
    int bytes;
  };
  static std::mutex mu;
  static std::vector<Entry> done;
  int dev = 0;
  GLC_CHECK_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  Entry* e = nullptr;
  for (auto& d : done)
    if (d.kernel == kernel && d.device == dev) e = &d;
  if (e && e->bytes >= bytes) return GLACIER_CUDA_OK;
  GLC_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  if (e)
    e->bytes = bytes;
  else
    done.push_back({kernel, dev, bytes});
  return GLACIER_CUDA_OK;
}

template <typename ScaleT>
int gemv_int4(const float* x, size_t ldx, size_t batch, const uint8_t* packed, const ScaleT* scales,
              size_t scale_stride, const float* bias, float* y, size_t ldy, size_t M, size_t K,
              size_t group, cudaStream_t stream);

int gemv_device_error(int clear);
int q8_device_error(int clear);
int ops_device_error(int clear);
int add_rmsnorm(const float* a, size_t lda, const float* b, size_t ldb, size_t b_split_stride, int nb,
                float* residual, size_t ldr, const float* w, float eps, float* out, size_t ldo, size_t batch,
                size_t dim, cudaStream_t stream, SplitOut so = SplitOut());
int silu_mul(const float* gate, const float* up, size_t ld_in, float* out, size_t ld_out, size_t batch, size_t n,
             cudaStream_t stream, SplitOut so = SplitOut());
int embed_gather(const __half* table, size_t vocab, size_t dim, const int32_t* tokens, size_t batch, float* out,
                 size_t ldo, cudaStream_t stream);
int qkv_rope_append(const float* qkv, size_t ld, size_t split_stride, int nsplit, const float* bias,
                    const float* cos_t, const float* sin_t, size_t positions, const int32_t* pos, size_t batch,
                    size_t num_heads, size_t num_kv_heads, size_t head_dim, float* q_out, size_t ldq, float* pool,
                    size_t page_floats, const int32_t* block_tables, size_t max_pages, size_t layer,
                    cudaStream_t stream);
size_t attention_workspace_floats(size_t lanes, size_t num_heads, size_t head_dim, size_t nsplit);
int attention_segments(size_t lanes, size_t num_heads, size_t head_dim, size_t max_ctx);
int paged_attention(const float* q, size_t ldq, const float* pool, size_t page_floats, const int32_t* block_tables,
                    size_t max_pages, const int32_t* ctx_lens, size_t max_ctx, size_t lanes, size_t layer,
                    size_t num_heads, size_t num_kv_heads, size_t head_dim, float* out, size_t ldo, float* workspace,
                    size_t workspace_floats, int chunk, cudaStream_t stream, SplitOut so = SplitOut(),
                    StepProfiler* prof = nullptr, int combine_kind = -1);
size_t argmax_workspace_bytes(size_t batch, size_t n);
int argmax_rows(const float* logits, size_t ld, size_t batch, size_t n, const uint64_t* words, size_t word_count,
                glacier_argmax_result* out, int32_t* tokens, int32_t* status, void* workspace, size_t ws_bytes,
                cudaStream_t stream);

size_t gemm_split_bytes(size_t np, size_t K);
bool gemm_tc_supported(const Int4Weight& w);
int split_activation(const float* x, size_t ldx, size_t n, size_t K, size_t np, __half* xs, float* xscale,
                     cudaStream_t stream);
int encode_split_map(CUtensorMap* map, const __half* xs, size_t np, size_t K);
int gemm_device_error(int clear);
int attn_device_error(int clear);
int persist_device_error(int clear);
int gemm_splits(size_t M, size_t K);
int reduce_splits(const float* part, size_t split_stride, int nsplit, float* y, size_t n, cudaStream_t stream);

}  // namespace glacier

using namespace glacier;

namespace glacier {

// Workspace of the batched matmul: the split activations (padded to 16 rows)
// and, when K is split, the per-split partial outputs.
size_t matmul_workspace_bytes(size_t batch, size_t in_features, size_t out_features) {
  const size_t np = ceil_div(batch < 16 ? 16 : batch, 16) * 16;
  const int ns = gemm_splits(out_features, in_features);
  const size_t part = ns > 1 ? (size_t)ns * batch * out_features * sizeof(float) : 0;
  return ceil_div(gemm_split_bytes(np, in_features), 256) * 256 + part;
}

// y[batch, M] = x[batch, K] * dequant(W)^T + bias: the tcgen05 GEMM for up to
// 128 rows when the weight qualifies, else the GEMV kernels.
int int4_matmul(const Int4Weight& w, const float* x, size_t batch, const float* bias, float* y, void* workspace,
                size_t workspace_bytes, cudaStream_t st) {
  const size_t in_features = w.K, out_features = w.M;
  if (!gemm_tc_supported(w) || batch > 128) return int4_linear(w, x, in_features, batch, bias, y, out_features, st);
  const size_t np = ceil_div(batch < 16 ? 16 : batch, 16) * 16;
  const size_t need = matmul_workspace_bytes(batch, in_features, out_features);
  GLC_REQUIRE(workspace && workspace_bytes >= need, "int4_matmul: workspace of %zu bytes needed", need);
  __half* xs = static_cast<__half*>(workspace);
  float* xscale = reinterpret_cast<float*>(xs + 2 * np * in_features);
  GLC_CHECK_CUDA(cudaMemsetAsync(xs, 0, 2 * np * in_features * sizeof(__half), st));
  int rc = split_activation(x, in_features, batch, in_features, np, xs, xscale, st);
  if (rc) return rc;
  CUtensorMap map;
  if ((rc = encode_split_map(&map, xs, np, in_features))) return rc;
  const int ns = gemm_splits(out_features, in_features);
  if (ns == 1) return gemm_int4_tc(w, map, xscale, batch, np, y, out_features, 1, 0, bias, st);
  float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                         ceil_div(gemm_split_bytes(np, in_features), 256) * 256);
  const size_t stride = batch * out_features;
  if ((rc = gemm_int4_tc(w, map, xscale, batch, np, part, out_features, ns, stride, bias, st))) return rc;
  return reduce_splits(part, stride, ns, y, stride, st);
}

}  // namespace glacier

extern "C" {

const char* glacier_cuda_last_error(void) { return g_last_error; }

int glacier_cuda_version(void) { return (0 << 16) | 1; }

unsigned long long glacier_cuda_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int glacier_cuda_device_status(int clear) {
  GLC_CHECK_CUDA(cudaDeviceSynchronize());
  const int v = gemv_device_error(clear), w = ops_device_error(clear), g = gemm_device_error(clear),
            a = attn_device_error(clear), q = q8_device_error(clear), p = persist_device_error(clear);
  if (v < 0 || w < 0 || g < 0 || a < 0 || q < 0 || p < 0)
    return set_error(GLACIER_CUDA_ECUDA, "device status read failed");
  return (v || g || a || q || p == 1) ? 1 : ((w || p) ? 2 : 0);
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

int glacier_cuda_int4_linear_q8(const float* x, size_t batch, const uint8_t* packed, const void* scales,
                                int scale_is_f16, const float* bias, float* y, size_t out_features,
                                size_t in_features, size_t group_size, void* stream) {
  GLC_REQUIRE(x && packed && scales && y, "int4_linear_q8: null pointer");
  Int4Weight w;
  w.packed = packed;
  w.scales = scales;
  w.f16 = scale_is_f16 != 0;
  w.M = out_features;
  w.K = in_features;
  w.group = group_size;
  const int rc = int4_weight_prepare(w);
  if (rc) return rc;
  return int4_linear_q8(w, x, in_features, batch, bias, y, out_features, (cudaStream_t)stream);
}

size_t glacier_cuda_int4_matmul_workspace(size_t batch, size_t in_features, size_t out_features) {
  return matmul_workspace_bytes(batch, in_features, out_features);
}

int glacier_cuda_int4_matmul_f16scale(const float* x, size_t batch, const uint8_t* packed, const uint16_t* scales,
                                      const float* bias, float* y, size_t out_features, size_t in_features,
                                      size_t group_size, void* workspace, size_t workspace_bytes, void* stream) {
  GLC_REQUIRE(x && packed && scales && y && batch > 0, "int4_matmul: null or empty argument");
  Int4Weight w;
  w.packed = packed;
  w.scales = scales;
  w.f16 = true;
  w.M = out_features;
  w.K = in_features;
  w.group = group_size;
  const int rc = int4_weight_prepare(w);
  if (rc) return rc;
  return int4_matmul(w, x, batch, bias, y, workspace, workspace_bytes, (cudaStream_t)stream);
}

int glacier_cuda_rmsnorm_f32(const float* x, const float* weight, float eps, float* out, size_t batch, size_t dim,
                             void* stream) {
  return add_rmsnorm(x, dim, nullptr, dim, 0, 0, nullptr, dim, weight, eps, out, dim, batch, dim,
                     (cudaStream_t)stream);
}

int glacier_cuda_add_rmsnorm_f32(const float* a, const float* b, float* residual, const float* weight, float eps,
                                 float* out, size_t batch, size_t dim, void* stream) {
  GLC_REQUIRE(b && residual, "add_rmsnorm: null argument");
  return add_rmsnorm(a, dim, b, dim, 0, 1, residual, dim, weight, eps, out, dim, batch, dim, (cudaStream_t)stream);
}

int glacier_cuda_silu_mul_f32(const float* gate, const float* up, size_t ld_in, float* out, size_t ld_out,
                              size_t batch, size_t n, void* stream) {
  return silu_mul(gate, up, ld_in, out, ld_out, batch, n, (cudaStream_t)stream);
}

int glacier_cuda_embedding_f16(const uint16_t* table, size_t vocab, size_t dim, const int32_t* tokens, size_t batch,
                               float* out, void* stream) {
  return embed_gather(reinterpret_cast<const __half*>(table), vocab, dim, tokens, batch, out, dim,
                      (cudaStream_t)stream);
}

int glacier_cuda_qkv_rope_append_f32(const float* qkv, size_t ld, const float* bias, const float* cos_table,
                                     const float* sin_table, size_t positions, const int32_t* pos, size_t batch,
                                     size_t num_heads, size_t num_kv_heads, size_t head_dim, float* q_out, size_t ldq,
                                     float* kv_pages, size_t page_floats, const int32_t* block_tables,
                                     size_t max_pages, size_t layer, void* stream) {
  return qkv_rope_append(qkv, ld, 0, 1, bias, cos_table, sin_table, positions, pos, batch, num_heads, num_kv_heads,
                         head_dim, q_out, ldq, kv_pages, page_floats, block_tables, max_pages, layer,
                         (cudaStream_t)stream);
}

size_t glacier_cuda_paged_attention_workspace(size_t lanes, size_t num_heads, size_t num_kv_heads, size_t head_dim,
                                              size_t max_ctx) {
  if (!lanes || !num_kv_heads || !max_ctx) return 0;
  return attention_workspace_floats(lanes, num_heads, head_dim,
                                    attention_segments(lanes, num_heads, head_dim, max_ctx));
}

int glacier_cuda_paged_attention_f32(const float* q, const float* kv_pages, size_t page_floats,
                                     const int32_t* block_tables, size_t max_pages, const int32_t* ctx_lens,
                                     size_t max_ctx, size_t lanes, size_t layer, size_t num_heads, size_t num_kv_heads,
                                     size_t head_dim, float* out, float* workspace, size_t workspace_floats,
                                     void* stream) {
  GLC_REQUIRE(lanes > 0 && num_kv_heads > 0, "paged_attention: empty batch");
  const size_t need = glacier_cuda_paged_attention_workspace(lanes, num_heads, num_kv_heads, head_dim, max_ctx);
  GLC_REQUIRE(workspace && workspace_floats >= need, "paged_attention: workspace of %zu floats needed", need);
  return paged_attention(q, num_heads * head_dim, kv_pages, page_floats, block_tables, max_pages, ctx_lens, max_ctx,
                         lanes, layer, num_heads, num_kv_heads, head_dim, out, num_heads * head_dim, workspace,
                         workspace_floats, attention_segments(lanes, num_heads, head_dim, max_ctx), (cudaStream_t)stream);
}

size_t glacier_cuda_argmax_workspace(size_t batch, size_t n) { return argmax_workspace_bytes(batch, n); }

int glacier_cuda_argmax_eligible_f32(const float* logits, size_t batch, size_t n, const uint64_t* words,
                                     size_t word_count, int32_t* tokens, int32_t* status,
                                     glacier_argmax_result* results, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  return argmax_rows(logits, n, batch, n, words, word_count, results, tokens, status, workspace, workspace_bytes,
                     (cudaStream_t)stream);
}

}  // extern "C"
