// Kernels (c): the norm / rotary / activation steps around the INT4 GEMVs of a
// decode step, each fused with its neighbouring element-wise work.
//
//  * embedding gather         generate.zig:3653-3663 loadEmbeddingRow (fp16 table)
//  * residual add + RMSNorm   kernels.zig:141-220 rmsNormF32, :322-401 addRmsNormF32
//  * q/k RoPE + KV append     generate.zig:816-831 RopeTable.apply,
//                             paged_kv_cache.zig:1074-1103 appendRowTxn
//  * SwiGLU                   kernels.zig:465-507 siluMulF32
//
// All activations stay fp32 (the reference's --fp32-activations mode); the only
// numeric difference from the reference is the reduction order of the RMSNorm
// sum of squares (block tree instead of 16 lanes + ordered sum).
#include "common.cuh"

namespace glacier {

namespace {

constexpr int kNormThreads = 512;

__device__ __forceinline__ float block_sum(float v, float* sh) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float t = (threadIdx.x < nw) ? sh[threadIdx.x] : 0.f;
  if (w == 0) t = warp_sum(t);
  if (threadIdx.x == 0) sh[0] = t;
  __syncthreads();
  return sh[0];
}

// One CTA per row.  x = a (+ sum of nb partial rows of b, in order) ; the sum
// is written to `residual` when given; out = x * (1/sqrt(mean(x^2)+eps)) * w.
// The rows are held in shared memory between the two passes.
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(
    const float* __restrict__ a, size_t lda, const float* __restrict__ b, size_t ldb, size_t b_split_stride,
    int nb, float* __restrict__ residual, size_t ldr, const float* __restrict__ w, float eps, float* __restrict__ out,
    size_t ldo, int dim) {
  extern __shared__ float row[];
  __shared__ float sh[32];
  const int r = blockIdx.x;
  const float* ar = a + r * lda;
  float ss = 0.f;
  for (int k = threadIdx.x; k < dim; k += blockDim.x) {
    float v = ar[k];
    // addInto (generate.zig:3642): dst = a + b; split-K partial rows of b are
    // summed first, in split order.
    if (nb > 0) {
      float bv = b[r * ldb + k];
      for (int s = 1; s < nb; ++s) bv += b[s * b_split_stride + r * ldb + k];
      v = v + bv;
    }
    row[k] = v;
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, sh);
  const float rms = sqrtf(ss / (float)dim + eps);
  const float inv = 1.0f / rms;
  for (int k = threadIdx.x; k < dim; k += blockDim.x) {
    const float v = row[k];
    if (residual) residual[r * ldr + k] = v;
    out[r * ldo + k] = v * inv * w[k];
  }
}

// out[b, i] = silu(gate[b, i]) * up[b, i]; silu(g) = g * (1 / (1 + exp(-g))).
__global__ void silu_mul_kernel(const float* __restrict__ gate, const float* __restrict__ up, size_t ld_in,
                                float* __restrict__ out, size_t ld_out, int n, int batch) {
  const size_t total = (size_t)n * batch;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / n), k = (int)(i % n);
    const float g = gate[b * ld_in + k];
    const float sig = 1.0f / (1.0f + expf(-g));
    out[b * ld_out + k] = g * sig * up[b * ld_in + k];
  }
}

// x[b, :] = float(table[token[b], :])
__global__ void embed_kernel(const __half* __restrict__ table, const int32_t* __restrict__ tokens, int vocab, int dim,
                             float* __restrict__ out, size_t ldo, int* __restrict__ bad) {
  const int b = blockIdx.y;
  const int tok = tokens[b];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(bad, 1);
    return;
  }
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < dim; k += gridDim.x * blockDim.x)
    out[b * ldo + k] = __half2float(table[(size_t)tok * dim + k]);
}

// One CTA per lane: adds the q/k/v biases to the fused projection row (summing
// nsplit split-K partials first), rotates q and k (NeoX half-split pairs with
// the host-built cos/sin table), writes q to q_out and the k/v rows into the
// lane's current page slot: page = block_table[pos / 16], row = pos % 16,
// payload offset ((layer*2 + kind)*16 + row) * kv_dim.
__global__ void qkv_rope_append_kernel(const float* __restrict__ qkv, size_t ld, size_t split_stride, int nsplit,
                                       const float* __restrict__ bias, const float* __restrict__ cos_t,
                                       const float* __restrict__ sin_t, int positions, const int32_t* __restrict__ pos,
                                       int num_heads, int num_kv_heads, int head_dim, float* __restrict__ q_out,
                                       size_t ldq, float* __restrict__ pool, size_t page_floats,
                                       const int32_t* __restrict__ block_tables, int max_pages, int layer,
                                       int* __restrict__ bad) {
  const int b = blockIdx.x;
  const int p = pos[b];
  const int half = head_dim >> 1;
  const int q_dim = num_heads * head_dim, kv_dim = num_kv_heads * head_dim;
  const int page_idx = p >> 4;
  if (p < 0 || p >= positions || page_idx >= max_pages) {
    if (threadIdx.x == 0) atomicExch(bad, 1);
    return;
  }
  const int32_t page = block_tables[b * max_pages + page_idx];
  float* kdst = pool + (size_t)page * page_floats + ((size_t)(layer * 2 + 0) * 16 + (p & 15)) * kv_dim;
  float* vdst = pool + (size_t)page * page_floats + ((size_t)(layer * 2 + 1) * 16 + (p & 15)) * kv_dim;
  const float* row = qkv + b * ld;
  auto val = [&](int i) {
    float v = row[i];
    for (int s = 1; s < nsplit; ++s) v += row[s * split_stride + i];
    return bias ? v + bias[i] : v;
  };
  const float* ct = cos_t + (size_t)p * half;
  const float* st = sin_t + (size_t)p * half;
  // Rotated pairs: (head, j) and (head, j + half) for q and k heads.
  const int pairs = (num_heads + num_kv_heads) * half;
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int hh = i / half, j = i % half;
    const float c = ct[j], s = st[j];
    if (hh < num_heads) {
      const int i0 = hh * head_dim + j;
      const float x0 = val(i0), x1 = val(i0 + half);
      q_out[b * ldq + i0] = x0 * c - x1 * s;
      q_out[b * ldq + i0 + half] = x0 * s + x1 * c;
    } else {
      const int kh = hh - num_heads;
      const int i0 = kh * head_dim + j;
      const float x0 = val(q_dim + i0), x1 = val(q_dim + i0 + half);
      kdst[i0] = x0 * c - x1 * s;
      kdst[i0 + half] = x0 * s + x1 * c;
    }
  }
  for (int i = threadIdx.x; i < kv_dim; i += blockDim.x) vdst[i] = val(q_dim + kv_dim + i);
}

}  // namespace

__device__ int g_ops_error;

int ops_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_ops_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_ops_error, &z, sizeof(int));
  }
  return v;
}

static int* ops_err_ptr() {
  int* p = nullptr;
  cudaGetSymbolAddress((void**)&p, g_ops_error);
  return p;
}

int add_rmsnorm(const float* a, size_t lda, const float* b, size_t ldb, size_t b_split_stride, int nb,
                float* residual, size_t ldr, const float* w, float eps, float* out, size_t ldo, size_t batch,
                size_t dim, cudaStream_t stream) {
  GLC_REQUIRE(a && w && out && batch > 0 && dim > 0, "rmsnorm: empty or null argument");
  GLC_REQUIRE(dim * sizeof(float) <= 160 * 1024, "rmsnorm: dim %zu too large", dim);
  const size_t smem = dim * sizeof(float);
  static size_t attr = 0;
  if (smem > 48 * 1024 && attr < smem) {
    const int rc = allow_dynamic_smem((const void*)add_rmsnorm_kernel, (int)smem);
    if (rc) return rc;
    attr = smem;
  }
  add_rmsnorm_kernel<<<(unsigned)batch, kNormThreads, smem, stream>>>(a, lda, b, ldb, b_split_stride, nb, residual,
                                                                      ldr, w, eps, out, ldo, (int)dim);
  GLC_CHECK_LAUNCH();
  return GLACIER_CUDA_OK;
}

int silu_mul(const float* gate, const float* up, size_t ld_in, float* out, size_t ld_out, size_t batch, size_t n,
             cudaStream_t stream) {
  GLC_REQUIRE(gate && up && out && batch > 0 && n > 0, "silu_mul: empty or null argument");
  const size_t total = batch * n;
  const unsigned grid = (unsigned)std::min<size_t>(ceil_div(total, 256), (size_t)sm_count() * 8);
  silu_mul_kernel<<<grid, 256, 0, stream>>>(gate, up, ld_in, out, ld_out, (int)n, (int)batch);
  GLC_CHECK_LAUNCH();
  return GLACIER_CUDA_OK;
}

int embed_gather(const __half* table, size_t vocab, size_t dim, const int32_t* tokens, size_t batch, float* out,
                 size_t ldo, cudaStream_t stream) {
  GLC_REQUIRE(table && tokens && out && batch > 0 && dim > 0, "embedding: empty or null argument");
  dim3 grid((unsigned)std::min<size_t>(ceil_div(dim, 256), 16), (unsigned)batch);
  embed_kernel<<<grid, 256, 0, stream>>>(table, tokens, (int)vocab, (int)dim, out, ldo, ops_err_ptr());
  GLC_CHECK_LAUNCH();
  return GLACIER_CUDA_OK;
}

int qkv_rope_append(const float* qkv, size_t ld, size_t split_stride, int nsplit, const float* bias,
                    const float* cos_t, const float* sin_t, size_t positions, const int32_t* pos, size_t batch,
                    size_t num_heads, size_t num_kv_heads, size_t head_dim, float* q_out, size_t ldq, float* pool,
                    size_t page_floats, const int32_t* block_tables, size_t max_pages, size_t layer,
                    cudaStream_t stream) {
  GLC_REQUIRE(qkv && cos_t && sin_t && pos && q_out && pool && block_tables && batch > 0,
              "qkv_rope_append: null argument");
  GLC_REQUIRE(head_dim % 2 == 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0,
              "qkv_rope_append: bad head geometry");
  qkv_rope_append_kernel<<<(unsigned)batch, 256, 0, stream>>>(
      qkv, ld, split_stride, nsplit, bias, cos_t, sin_t, (int)positions, pos, (int)num_heads, (int)num_kv_heads,
      (int)head_dim, q_out, ldq, pool, page_floats, block_tables, (int)max_pages, (int)layer, ops_err_ptr());
  GLC_CHECK_LAUNCH();
  return GLACIER_CUDA_OK;
}

}  // namespace glacier
