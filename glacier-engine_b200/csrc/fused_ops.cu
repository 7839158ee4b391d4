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

// Reduces one float per CTA across the cluster (in rank order) through
// distributed shared memory.  `slot` is this CTA's shared word.
__device__ __forceinline__ float cluster_sum(float* slot, float v) {
  if (threadIdx.x == 0) *slot = v;
  cluster_sync_all();
  const uint32_t n = cluster_nctarank();
  const uint32_t a = smem_u32(slot);
  float t = 0.f;
  for (uint32_t q = 0; q < n; ++q) t += ld_dsmem_f32(mapa_shared(a, q));
  return t;
}
__device__ __forceinline__ float cluster_max(float* slot, float v) {
  if (threadIdx.x == 0) *slot = v;
  cluster_sync_all();
  const uint32_t n = cluster_nctarank();
  const uint32_t a = smem_u32(slot);
  float t = 0.f;
  for (uint32_t q = 0; q < n; ++q) t = fmaxf(t, ld_dsmem_f32(mapa_shared(a, q)));
  return t;
}

__device__ __forceinline__ float block_max(float v, float* sh) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float t = (threadIdx.x < nw) ? sh[threadIdx.x] : 0.f;
  if (w == 0) t = warp_max(t);
  if (threadIdx.x == 0) sh[0] = t;
  __syncthreads();
  return sh[0];
}

// Few rows (GEMV decode): one CTA per row, each thread holding up to two float4
// of it in registers, so one block reduction and no cluster exchange are
// needed.  Same arithmetic as add_rmsnorm_kernel with fp32 output.
__global__ void __launch_bounds__(1024) add_rmsnorm_row_kernel(
    const float* __restrict__ a, size_t lda, const float* __restrict__ b, size_t ldb, size_t b_split_stride,
    int nb, float* __restrict__ residual, size_t ldr, const float* __restrict__ w, float eps, float* __restrict__ out,
    size_t ldo, int dim) {
  griddep_launch();
  griddep_wait();
  __shared__ float sh[32];
  const int r = blockIdx.x, n4 = dim / 4;
  float4 v[2];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < n4) {
      float4 x = reinterpret_cast<const float4*>(a + r * lda)[i];
      if (nb > 0) {
        // addInto (generate.zig:3642): dst = a + b, split-K partials summed first.
        float4 bv = reinterpret_cast<const float4*>(b + r * ldb)[i];
        for (int sp = 1; sp < nb; ++sp) {
          const float4 t = reinterpret_cast<const float4*>(b + sp * b_split_stride + r * ldb)[i];
          bv.x += t.x;
          bv.y += t.y;
          bv.z += t.z;
          bv.w += t.w;
        }
        x.x = x.x + bv.x;
        x.y = x.y + bv.y;
        x.z = x.z + bv.z;
        x.w = x.w + bv.w;
      }
      v[j] = x;
      ss = fmaf(x.x, x.x, ss);
      ss = fmaf(x.y, x.y, ss);
      ss = fmaf(x.z, x.z, ss);
      ss = fmaf(x.w, x.w, ss);
    }
  }
  ss = block_sum(ss, sh);
  const float inv = 1.0f / sqrtf(ss / (float)dim + eps);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < n4) {
      if (residual) reinterpret_cast<float4*>(residual + r * ldr)[i] = v[j];
      const float4 wv = reinterpret_cast<const float4*>(w)[i];
      reinterpret_cast<float4*>(out + r * ldo)[i] =
          make_float4(v[j].x * inv * wv.x, v[j].y * inv * wv.y, v[j].z * inv * wv.z, v[j].w * inv * wv.w);
    }
  }
}

// A cluster of CTAs per row (blockIdx.y = row, cluster rank = slice of the row):
// x = a (+ the nb split-K partial rows of b, summed in split order); the sum
// goes to `residual` when given; out = x * (1/sqrt(mean(x^2)+eps)) * w, written
// as fp32 or in split form.  The sum of squares (and for split outputs the row
// max) is combined across the cluster through distributed shared memory.
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(
    const float* __restrict__ a, size_t lda, const float* __restrict__ b, size_t ldb, size_t b_split_stride,
    int nb, float* __restrict__ residual, size_t ldr, const float* __restrict__ w, float eps, float* __restrict__ out,
    size_t ldo, SplitOut so, int dim) {
  griddep_launch();
  griddep_wait();
  extern __shared__ float row[];
  __shared__ float sh[32];
  __shared__ float xch[2];
  const int r = blockIdx.y;
  const int cr = (int)cluster_ctarank(), cn = (int)cluster_nctarank();
  const int slice = ((dim + cn - 1) / cn + 7) & ~7;
  const int k0 = min(dim, cr * slice), k1 = min(dim, k0 + slice);
  const float* ar = a + r * lda;
  float ss = 0.f;
  for (int k = k0 + threadIdx.x; k < k1; k += blockDim.x) {
    float v = ar[k];
    // addInto (generate.zig:3642): dst = a + b, split-K partials summed first.
    if (nb > 0) {
      float bv = b[r * ldb + k];
      for (int s = 1; s < nb; ++s) bv += b[s * b_split_stride + r * ldb + k];
      v = v + bv;
    }
    row[k - k0] = v;
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, sh);
  const float total = cluster_sum(&xch[0], ss);
  const float rms = sqrtf(total / (float)dim + eps);
  const float inv = 1.0f / rms;
  float m = 0.f;
  for (int k = k0 + threadIdx.x; k < k1; k += blockDim.x) {
    const float v = row[k - k0];
    if (residual) residual[r * ldr + k] = v;
    const float o = v * inv * w[k];
    if (so.xs) {
      row[k - k0] = o;
      m = fmaxf(m, fabsf(o));
    } else {
      out[r * ldo + k] = o;
    }
  }
  if (so.xs) {
    m = block_max(m, sh);
    const float scale = split_scale(cluster_max(&xch[1], m));
    const float iscale = 1.0f / scale;
    for (int k8 = k0 / 8 + threadIdx.x; k8 < k1 / 8; k8 += blockDim.x) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = row[k8 * 8 - k0 + i];
      store_split8(so, r, dim, (size_t)k8 * 8, v, iscale);
    }
    if (cr == 0 && threadIdx.x == 0) so.xscale[r] = scale;
  }
  cluster_sync_all();  // peers may still read this CTA's exchange words
}

// Vectorised RoPE + append: one CTA per lane; a thread owns 4 consecutive rotary
// pairs of one q or k head (or 4 consecutive v values), loads every split-K
// partial of them at once, and writes the rotated q, k and the v row.
__global__ void __launch_bounds__(1024) qkv_rope_append4_kernel(
    const float* __restrict__ qkv, size_t ld, size_t split_stride, int nsplit, const float* __restrict__ bias,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, int positions, const int32_t* __restrict__ pos,
    int num_heads, int num_kv_heads, int head_dim, float* __restrict__ q_out, size_t ldq, float* __restrict__ pool,
    size_t page_floats, const int32_t* __restrict__ block_tables, int max_pages, int layer, int* __restrict__ bad) {
  griddep_launch();
  griddep_wait();
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
  auto val4 = [&](int i) {  // split-K partials summed in split order, then the bias
    float4 v = *reinterpret_cast<const float4*>(row + i);
#pragma unroll 4
    for (int s = 1; s < nsplit; ++s) {
      const float4 u = *reinterpret_cast<const float4*>(row + (size_t)s * split_stride + i);
      v.x += u.x; v.y += u.y; v.z += u.z; v.w += u.w;
    }
    if (bias) {
      const float4 c = *reinterpret_cast<const float4*>(bias + i);
      v.x += c.x; v.y += c.y; v.z += c.z; v.w += c.w;
    }
    return v;
  };
  const int pair_quads = (num_heads + num_kv_heads) * half / 4;
  const int t = threadIdx.x;
  if (t < pair_quads) {
    const int i = 4 * t;
    const int hh = i / half, j = i - hh * half;
    const int src = hh < num_heads ? hh * head_dim + j : q_dim + (hh - num_heads) * head_dim + j;
    const float4 x0 = val4(src), x1 = val4(src + half);
    const float4 c = *reinterpret_cast<const float4*>(cos_t + (size_t)p * half + j);
    const float4 sn = *reinterpret_cast<const float4*>(sin_t + (size_t)p * half + j);
    const float4 y0 = make_float4(x0.x * c.x - x1.x * sn.x, x0.y * c.y - x1.y * sn.y, x0.z * c.z - x1.z * sn.z,
                                  x0.w * c.w - x1.w * sn.w);
    const float4 y1 = make_float4(x0.x * sn.x + x1.x * c.x, x0.y * sn.y + x1.y * c.y, x0.z * sn.z + x1.z * c.z,
                                  x0.w * sn.w + x1.w * c.w);
    float* dst = hh < num_heads ? q_out + b * ldq + hh * head_dim + j : kdst + (hh - num_heads) * head_dim + j;
    *reinterpret_cast<float4*>(dst) = y0;
    *reinterpret_cast<float4*>(dst + half) = y1;
  } else if (t < pair_quads + kv_dim / 4) {
    const int i = 4 * (t - pair_quads);
    *reinterpret_cast<float4*>(vdst + i) = val4(q_dim + kv_dim + i);
  }
}

// ---- Split-output forms: each thread owns 8 consecutive values in registers ----
// A row is cut into `cn` CTAs (a cluster when cn > 1); thread t of CTA c owns
// values [8g, 8g + 8) with g = c * per + t.  One block (and cluster) reduction
// gives the row's statistics, then every thread writes its 8 values straight
// to the GEMM's split form.

// residual = a + sum of b's split-K partials (in split order); split(rmsnorm(residual) * w).
__global__ void __launch_bounds__(1024) add_rmsnorm_split8_kernel(
    const float* __restrict__ a, size_t lda, const float* __restrict__ b, size_t ldb, size_t b_split_stride, int nb,
    float* __restrict__ residual, size_t ldr, const float* __restrict__ w, float eps, SplitOut so, int dim) {
  griddep_launch();
  griddep_wait();
  __shared__ float2 sh[32];
  __shared__ __align__(8) float2 xch;
  const int r = blockIdx.y;
  const int per = blockDim.x;
  const int g = (int)cluster_ctarank() * per + threadIdx.x;
  const bool active = 8 * g < dim;
  const int k = 8 * g;
  float v[8], wv[8];
  float ss = 0.f, mx = 0.f;
  if (active) {
    load8(a + (size_t)r * lda + k, v);
    if (nb > 0) {
      float t[8];
      load8(b + (size_t)r * ldb + k, t);
#pragma unroll 4
      for (int s = 1; s < nb; ++s) {
        float u[8];
        load8(b + (size_t)s * b_split_stride + (size_t)r * ldb + k, u);
#pragma unroll
        for (int i = 0; i < 8; ++i) t[i] += u[i];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = v[i] + t[i];  // addInto (generate.zig:3642)
    }
    load8(w + k, wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ss = fmaf(v[i], v[i], ss);
      mx = fmaxf(mx, fabsf(v[i] * wv[i]));
    }
  }
  const float2 tot = row_sum_max(ss, mx, sh, &xch);
  const float inv = 1.0f / sqrtf(tot.x / (float)dim + eps);
  const float scale = split_scale(tot.y * inv);
  if (active) {
    if (residual) {
      float4* rp = reinterpret_cast<float4*>(residual + (size_t)r * ldr + k);
      rp[0] = make_float4(v[0], v[1], v[2], v[3]);
      rp[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = v[i] * inv * wv[i];
    store_split8(so, r, (size_t)dim, (size_t)k, o, 1.0f / scale);
  }
  if (g == 0) so.xscale[r] = scale;
  if (cluster_nctarank() > 1) cluster_sync_all();  // peers may still read this CTA's exchange slot
}

// split(silu(gate) * up) per row (kernels.zig:465-507).
__global__ void __launch_bounds__(1024) silu_mul_split8_kernel(const float* __restrict__ gate,
                                                               const float* __restrict__ up, size_t ld_in,
                                                               SplitOut so, int n) {
  griddep_launch();
  griddep_wait();
  __shared__ float2 sh[32];
  __shared__ __align__(8) float2 xch;
  const int r = blockIdx.y;
  const int g = (int)cluster_ctarank() * blockDim.x + threadIdx.x;
  const bool active = 8 * g < n;
  const int k = 8 * g;
  float h[8];
  float mx = 0.f;
  if (active) {
    float gv[8], uv[8];
    load8(gate + (size_t)r * ld_in + k, gv);
    load8(up + (size_t)r * ld_in + k, uv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float sig = 1.0f / (1.0f + expf(-gv[i]));
      h[i] = gv[i] * sig * uv[i];
      mx = fmaxf(mx, fabsf(h[i]));
    }
  }
  const float2 tot = row_sum_max(0.f, mx, sh, &xch);
  const float scale = split_scale(tot.y);
  if (active) store_split8(so, r, (size_t)n, (size_t)k, h, 1.0f / scale);
  if (g == 0) so.xscale[r] = scale;
  if (cluster_nctarank() > 1) cluster_sync_all();
}

// Threads per CTA and cluster size for a split8 row of `dim` values.
static void split8_shape(size_t dim, int* threads, int* cl) {
  const size_t groups = dim / 8;
  int c = 1;
  while (c < 8 && ceil_div(groups, (size_t)c) > 1024) c *= 2;
  *cl = c;
  *threads = (int)(ceil_div(ceil_div(groups, (size_t)c), 32) * 32);
}

// One cluster per row: out = silu(gate) * up (kernels.zig:465-507), as fp32
// or in split form with the row max combined across the cluster.
__global__ void __launch_bounds__(kNormThreads) silu_mul_split_kernel(const float* __restrict__ gate,
                                                                        const float* __restrict__ up, size_t ld_in,
                                                                        float* __restrict__ out, size_t ld_out,
                                                                        SplitOut so, int n) {
  griddep_launch();
  griddep_wait();
  extern __shared__ float row[];
  __shared__ float sh[32];
  __shared__ float xch;
  const int r = blockIdx.y;
  const int cr = (int)cluster_ctarank(), cn = (int)cluster_nctarank();
  const int slice = ((n + cn - 1) / cn + 7) & ~7;
  const int k0 = min(n, cr * slice), k1 = min(n, k0 + slice);
  float m = 0.f;
  for (int k = k0 + threadIdx.x; k < k1; k += blockDim.x) {
    const float g = gate[r * ld_in + k];
    const float sig = 1.0f / (1.0f + expf(-g));
    const float h = g * sig * up[r * ld_in + k];
    if (so.xs) {
      row[k - k0] = h;
      m = fmaxf(m, fabsf(h));
    } else {
      out[r * ld_out + k] = h;
    }
  }
  if (so.xs) {
    m = block_max(m, sh);
    const float scale = split_scale(cluster_max(&xch, m));
    const float iscale = 1.0f / scale;
    for (int k8 = k0 / 8 + threadIdx.x; k8 < k1 / 8; k8 += blockDim.x) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = row[k8 * 8 - k0 + i];
      store_split8(so, r, n, (size_t)k8 * 8, v, iscale);
    }
    if (cr == 0 && threadIdx.x == 0) so.xscale[r] = scale;
    cluster_sync_all();
  }
}

// out[b, i] = silu(gate[b, i]) * up[b, i]; silu(g) = g * (1 / (1 + exp(-g))).
__global__ void silu_mul_kernel(const float* __restrict__ gate, const float* __restrict__ up, size_t ld_in,
                                float* __restrict__ out, size_t ld_out, int n, int batch) {
  griddep_launch();
  griddep_wait();
  const size_t total = (size_t)n * batch;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / n), k = (int)(i % n);
    const float g = gate[b * ld_in + k];
    const float sig = 1.0f / (1.0f + expf(-g));
    out[b * ld_out + k] = g * sig * up[b * ld_in + k];
  }
}

// x[b, :] = float(table[token[b], :])
__device__ __forceinline__ float embed_value(__half v) { return __half2float(v); }
__device__ __forceinline__ float embed_value(float v) { return v; }

template <typename T>
__global__ void embed_kernel(const T* __restrict__ table, const int32_t* __restrict__ tokens, int vocab, int dim,
                             float* __restrict__ out, size_t ldo, int* __restrict__ bad) {
  griddep_launch();
  griddep_wait();
  const int b = blockIdx.y;
  const int tok = tokens[b];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(bad, 1);
    return;
  }
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < dim; k += gridDim.x * blockDim.x)
    out[b * ldo + k] = embed_value(table[(size_t)tok * dim + k]);
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
  griddep_launch();
  griddep_wait();
  const int b = blockIdx.x;
  const int p = pos[b];
  const int half = head_dim >> 1;
  // blockIdx.y / gridDim.y: this CTA's share of the lane's pairs and v values.
  const int part = blockIdx.y, nparts = gridDim.y;
  const int tid = part * blockDim.x + threadIdx.x, nthreads = nparts * blockDim.x;
  const int q_dim = num_heads * head_dim, kv_dim = num_kv_heads * head_dim;
  const int page_idx = p >> 4;
  if (p < 0 || p >= positions || page_idx >= max_pages) {
    if (threadIdx.x == 0 && part == 0) atomicExch(bad, 1);
    return;
  }
  const int32_t page = block_tables[b * max_pages + page_idx];
  float* kdst = pool + (size_t)page * page_floats + ((size_t)(layer * 2 + 0) * 16 + (p & 15)) * kv_dim;
  float* vdst = pool + (size_t)page * page_floats + ((size_t)(layer * 2 + 1) * 16 + (p & 15)) * kv_dim;
  const float* row = qkv + b * ld;
  auto val = [&](int i) {
    float v = row[i];
#pragma unroll 4
    for (int s = 1; s < nsplit; ++s) v += row[s * split_stride + i];
    return bias ? v + bias[i] : v;
  };
  const float* ct = cos_t + (size_t)p * half;
  const float* st = sin_t + (size_t)p * half;
  // Rotated pairs: (head, j) and (head, j + half) for q and k heads.
  const int pairs = (num_heads + num_kv_heads) * half;
  for (int i = tid; i < pairs; i += nthreads) {
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
  for (int i = tid; i < kv_dim; i += nthreads) vdst[i] = val(q_dim + kv_dim + i);
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

static int* ops_err_ptr() { return device_symbol_address(g_ops_error); }
int* ops_error_word() { return ops_err_ptr(); }

// Cluster size for a row of `dim` values: about 1024 values per CTA, at most 8.
static int row_cluster(size_t dim) {
  int c = 1;
  while (c < 8 && dim / (size_t)(2 * c) >= 1024) c *= 2;
  return c;
}

static int launch_row_cluster(const void* kern, void** args, size_t rows, int cl, size_t smem, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)cl, (unsigned)rows);
  cfg.blockDim = dim3(kNormThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see launch_pdl
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  GLC_CHECK_CUDA(cudaLaunchKernelExC(&cfg, kern, args));
  note_launch();
  return GLACIER_CUDA_OK;
}

int add_rmsnorm(const float* a, size_t lda, const float* b, size_t ldb, size_t b_split_stride, int nb,
                float* residual, size_t ldr, const float* w, float eps, float* out, size_t ldo, size_t batch,
                size_t dim, cudaStream_t stream, SplitOut so) {
  GLC_REQUIRE(a && w && (out || so.xs) && batch > 0 && dim > 0, "rmsnorm: empty or null argument");
  GLC_REQUIRE(!so.xs || dim % 8 == 0, "rmsnorm: split output needs dim %% 8 == 0");
  if (so.xs && lda % 4 == 0 && ldb % 4 == 0 && b_split_stride % 4 == 0 && ldr % 4 == 0) {
    int threads, cl;
    split8_shape(dim, &threads, &cl);
    return launch_pdl(add_rmsnorm_split8_kernel, dim3((unsigned)cl, (unsigned)batch), dim3(threads), 0, stream, cl,
                      a, lda, b, ldb, b_split_stride, nb, residual, ldr, w, eps, so, (int)dim);
  }
  const bool vec = dim % 4 == 0 && lda % 4 == 0 && (!b || (ldb % 4 == 0 && b_split_stride % 4 == 0)) &&
                   (!residual || ldr % 4 == 0) && ldo % 4 == 0 && ((uintptr_t)a | (uintptr_t)b | (uintptr_t)w |
                                                                 (uintptr_t)out | (uintptr_t)residual) % 16 == 0;
  if (!so.xs && vec && batch <= 8 && dim <= 8 * 1024) {
    const unsigned threads = (unsigned)std::min<size_t>(1024, ceil_div(ceil_div(dim / 4, (size_t)2), (size_t)32) * 32);
    return launch_pdl(add_rmsnorm_row_kernel, dim3((unsigned)batch), dim3(threads), 0, stream, 1, a, lda, b, ldb,
                      b_split_stride, nb, residual, ldr, w, eps, out, ldo, (int)dim);
  }
  const int cl = row_cluster(dim);
  const size_t slice = ((ceil_div(dim, (size_t)cl)) + 7) & ~(size_t)7;
  const size_t smem = slice * sizeof(float);
  GLC_REQUIRE(smem <= 160 * 1024, "rmsnorm: dim %zu too large", dim);
  if (smem > 48 * 1024) {
    const int rc = allow_dynamic_smem((const void*)add_rmsnorm_kernel, (int)smem);
    if (rc) return rc;
  }
  int d = (int)dim;
  void* args[] = {(void*)&a, &lda, (void*)&b, &ldb, &b_split_stride, &nb, &residual, &ldr, (void*)&w, &eps, &out,
                  &ldo, &so, &d};
  return launch_row_cluster((const void*)add_rmsnorm_kernel, args, batch, cl, smem, stream);
}

int silu_mul(const float* gate, const float* up, size_t ld_in, float* out, size_t ld_out, size_t batch, size_t n,
             cudaStream_t stream, SplitOut so) {
  GLC_REQUIRE(gate && up && (out || so.xs) && batch > 0 && n > 0, "silu_mul: empty or null argument");
  GLC_REQUIRE(!so.xs || n % 8 == 0, "silu_mul: split output needs n %% 8 == 0");
  if (!so.xs) {
    const size_t total = batch * n;
    const unsigned grid = (unsigned)std::min<size_t>(ceil_div(total, 256), (size_t)sm_count() * 8);
    return launch_pdl(silu_mul_kernel, dim3(grid), dim3(256), 0, stream, 1, gate, up, ld_in, out, ld_out, (int)n,
                      (int)batch);
  }
  if (ld_in % 4 == 0) {
    int threads, cl;
    split8_shape(n, &threads, &cl);
    return launch_pdl(silu_mul_split8_kernel, dim3((unsigned)cl, (unsigned)batch), dim3(threads), 0, stream, cl, gate,
                      up, ld_in, so, (int)n);
  }
  const int cl = row_cluster(n);
  const size_t slice = ((ceil_div(n, (size_t)cl)) + 7) & ~(size_t)7;
  const size_t smem = slice * sizeof(float);
  GLC_REQUIRE(smem <= 160 * 1024, "silu_mul: row %zu too long", n);
  if (smem > 48 * 1024) {
    const int rc = allow_dynamic_smem((const void*)silu_mul_split_kernel, (int)smem);
    if (rc) return rc;
  }
  int nn = (int)n;
  void* args[] = {(void*)&gate, (void*)&up, &ld_in, &out, &ld_out, &so, &nn};
  return launch_row_cluster((const void*)silu_mul_split_kernel, args, batch, cl, smem, stream);
}

template <typename T>
int embed_gather_t(const T* table, size_t vocab, size_t dim, const int32_t* tokens, size_t batch, float* out,
                   size_t ldo, cudaStream_t stream) {
  GLC_REQUIRE(table && tokens && out && batch > 0 && dim > 0, "embedding: empty or null argument");
  dim3 grid((unsigned)std::min<size_t>(ceil_div(dim, 256), 16), (unsigned)batch);
  return launch_pdl(embed_kernel<T>, grid, dim3(256), 0, stream, 1, table, tokens, (int)vocab, (int)dim, out, ldo,
                    ops_err_ptr());
}

int embed_gather(const __half* table, size_t vocab, size_t dim, const int32_t* tokens, size_t batch, float* out,
                 size_t ldo, cudaStream_t stream) {
  return embed_gather_t(table, vocab, dim, tokens, batch, out, ldo, stream);
}

int embed_gather(const float* table, size_t vocab, size_t dim, const int32_t* tokens, size_t batch, float* out,
                 size_t ldo, cudaStream_t stream) {
  return embed_gather_t(table, vocab, dim, tokens, batch, out, ldo, stream);
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
  const int quads = (int)((num_heads + num_kv_heads) * (head_dim / 2) / 4 + num_kv_heads * head_dim / 4);
  if (head_dim % 8 == 0 && ld % 4 == 0 && split_stride % 4 == 0 && ldq % 4 == 0 && page_floats % 4 == 0 &&
      quads <= 1024)
    return launch_pdl(qkv_rope_append4_kernel, dim3((unsigned)batch), dim3((unsigned)ceil_div(quads, 32) * 32), 0,
                      stream, 1, qkv, ld, split_stride, nsplit, bias, cos_t, sin_t, (int)positions, pos,
                      (int)num_heads, (int)num_kv_heads, (int)head_dim, q_out, ldq, pool, page_floats, block_tables,
                      (int)max_pages, (int)layer, ops_err_ptr());
  return launch_pdl(qkv_rope_append_kernel, dim3((unsigned)batch, 4), dim3(256), 0, stream, 1, qkv, ld, split_stride,
                    nsplit, bias, cos_t, sin_t, (int)positions, pos, (int)num_heads, (int)num_kv_heads,
                    (int)head_dim, q_out, ldq, pool, page_floats, block_tables, (int)max_pages, (int)layer,
                    ops_err_ptr());
}

}  // namespace glacier
