// Kernel (d): paged-KV decode attention over the reference's FP32 page layout.
//
// Same operator as attentionMultiHead (src/paged_attention.zig:108-216) for one
// query row per lane: causal GQA (kv head = h / (H / Hkv)), scale 1/sqrt(hd),
// softmax over positions 0..ctx-1.  Pages hold 16 positions of every layer:
// payload offset ((layer*2 + kind)*16 + row) * kv_dim floats
// (src/paged_kv_cache.zig:1421-1442); block_tables[lane][logical page] gives
// the physical page.
//
// B200 design (flash-decoding): the context is split into chunks; one CTA owns
// (lane, kv head, chunk) and serves all G = H/Hkv query heads of the GQA
// group from a single read of each K and V row (the reference's shared-KV
// tile, forward.zig:544-620).  Pass 1: one thread per position computes the G
// scores from its K row.  Pass 2: per-head chunk max and exp-sum.  Pass 3:
// one thread per head dimension accumulates p * V with coalesced row reads.
// A combine kernel merges the chunks with the usual max/sum rescaling, in
// chunk order (deterministic).
#include "common.cuh"

namespace glacier {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kMaxGroup = 8;      // query heads per kv head
constexpr int kMaxHeadDim = 128;

struct AttnParams {
  const float* q;  // [lanes, H*hd]
  size_t ldq;
  const float* pool;
  size_t page_floats;
  const int32_t* block_tables;  // [lanes, max_pages]
  int max_pages;
  const int32_t* ctx_lens;      // [lanes]
  int layer, num_heads, num_kv_heads, head_dim, group;
  int chunk;                    // positions per split (multiple of 16)
  int nsplit;                   // splits per (lane, kv head)
  float scale;
  float* part_o;                // [lanes, H, nsplit, hd]
  float* part_ml;               // [lanes, H, nsplit, 2]  (max, sum)
};

__global__ void __launch_bounds__(kAttnThreads) attn_chunk_kernel(const AttnParams p) {
  extern __shared__ float sm[];
  float* qs = sm;                          // [G][hd]
  float* sc = qs + kMaxGroup * kMaxHeadDim;  // [G][chunk]
  __shared__ float red[kMaxGroup][kAttnThreads / 32];
  __shared__ float mx[kMaxGroup], sumv[kMaxGroup];

  const int lane_id = blockIdx.z;
  const int kvh = blockIdx.y;
  const int split = blockIdx.x;
  const int G = p.group, hd = p.head_dim;
  const int ctx = p.ctx_lens[lane_id];
  const int j0 = split * p.chunk;
  const int j1 = min(ctx, j0 + p.chunk);
  const int n = j1 - j0;
  const int kv_dim = p.num_kv_heads * hd;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t part_base = ((size_t)lane_id * p.num_heads + (size_t)kvh * G) * p.nsplit + split;

  if (n <= 0) {  // empty chunk: neutral partial (max -inf, sum 0)
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
      p.part_ml[(part_base + (size_t)g * p.nsplit) * 2 + 0] = -INFINITY;
      p.part_ml[(part_base + (size_t)g * p.nsplit) * 2 + 1] = 0.f;
    }
    return;
  }
  for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
    const int g = i / hd, d = i % hd;
    qs[g * kMaxHeadDim + d] = p.q[lane_id * p.ldq + (size_t)(kvh * G + g) * hd + d];
  }
  __syncthreads();

  const int32_t* bt = p.block_tables + (size_t)lane_id * p.max_pages;
  const size_t k_off = (size_t)(p.layer * 2 + 0) * 16 * kv_dim + (size_t)kvh * hd;
  const size_t v_off = (size_t)(p.layer * 2 + 1) * 16 * kv_dim + (size_t)kvh * hd;

  // Pass 1: scores.
  for (int jj = threadIdx.x; jj < n; jj += blockDim.x) {
    const int j = j0 + jj;
    const float* krow = p.pool + (size_t)bt[j >> 4] * p.page_floats + k_off + (size_t)(j & 15) * kv_dim;
    float dot[kMaxGroup];
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) dot[g] = 0.f;
    for (int d = 0; d < hd; d += 4) {
      const float4 kv = __ldg(reinterpret_cast<const float4*>(krow + d));
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        if (g < G) {
          const float4 qv = *reinterpret_cast<const float4*>(qs + g * kMaxHeadDim + d);
          dot[g] = fmaf(qv.x, kv.x, dot[g]);
          dot[g] = fmaf(qv.y, kv.y, dot[g]);
          dot[g] = fmaf(qv.z, kv.z, dot[g]);
          dot[g] = fmaf(qv.w, kv.w, dot[g]);
        }
      }
    }
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g)
      if (g < G) sc[g * p.chunk + jj] = dot[g] * p.scale;
  }
  __syncthreads();

  // Pass 2: per-head max and exp-sum over the chunk.
  for (int g = 0; g < G; ++g) {
    float m = -INFINITY;
    for (int jj = threadIdx.x; jj < n; jj += blockDim.x) m = fmaxf(m, sc[g * p.chunk + jj]);
    m = warp_max(m);
    if (lane == 0) red[g][warp] = m;
  }
  __syncthreads();
  if (threadIdx.x < G) {
    float m = red[threadIdx.x][0];
    for (int w = 1; w < kAttnThreads / 32; ++w) m = fmaxf(m, red[threadIdx.x][w]);
    mx[threadIdx.x] = m;
  }
  __syncthreads();
  for (int g = 0; g < G; ++g) {
    float s = 0.f;
    for (int jj = threadIdx.x; jj < n; jj += blockDim.x) {
      const float e = expf(sc[g * p.chunk + jj] - mx[g]);
      sc[g * p.chunk + jj] = e;
      s += e;
    }
    s = warp_sum(s);
    if (lane == 0) red[g][warp] = s;
  }
  __syncthreads();
  if (threadIdx.x < G) {
    float s = 0.f;
    for (int w = 0; w < kAttnThreads / 32; ++w) s += red[threadIdx.x][w];
    sumv[threadIdx.x] = s;
    p.part_ml[(part_base + (size_t)threadIdx.x * p.nsplit) * 2 + 0] = mx[threadIdx.x];
    p.part_ml[(part_base + (size_t)threadIdx.x * p.nsplit) * 2 + 1] = s;
  }

  // Pass 3: o[g][d] = sum_j p[g][j] * v_j[d]  (threads over d, rows coalesced).
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc[kMaxGroup];
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) acc[g] = 0.f;
    for (int jj = 0; jj < n; ++jj) {
      const int j = j0 + jj;
      const float v = __ldg(p.pool + (size_t)bt[j >> 4] * p.page_floats + v_off + (size_t)(j & 15) * kv_dim + d);
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g)
        if (g < G) acc[g] = fmaf(sc[g * p.chunk + jj], v, acc[g]);
    }
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g)
      if (g < G) p.part_o[(part_base + (size_t)g * p.nsplit) * hd + d] = acc[g];
  }
}

// out[lane, h, :] = sum_s o_s * e^(m_s - M) / sum_s l_s * e^(m_s - M), in split order.
__global__ void attn_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int nsplit,
                                    int head_dim, int num_heads, float* __restrict__ out, size_t ldo) {
  const int h = blockIdx.x, lane_id = blockIdx.y;
  const size_t base = ((size_t)lane_id * num_heads + h) * nsplit;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, part_ml[(base + s) * 2]);
  float L = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float m = part_ml[(base + s) * 2];
    if (m != -INFINITY) L += part_ml[(base + s) * 2 + 1] * expf(m - M);
  }
  const float inv = 1.0f / L;
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float m = part_ml[(base + s) * 2];
      if (m != -INFINITY) acc = fmaf(part_o[(base + s) * head_dim + d], expf(m - M), acc);
    }
    out[lane_id * ldo + (size_t)h * head_dim + d] = acc * inv;
  }
}

}  // namespace

// Workspace floats needed by paged_attention for the given split count.
size_t attention_workspace_floats(size_t lanes, size_t num_heads, size_t head_dim, size_t nsplit) {
  return lanes * num_heads * nsplit * (head_dim + 2);
}

// Positions per chunk: splits so that lanes * kv_heads * splits covers the
// SMs about twice, chunks of 64..1024 positions in whole pages.
int attention_chunk(size_t lanes, size_t num_kv_heads, size_t max_ctx) {
  const size_t units = lanes * num_kv_heads;
  size_t want = ceil_div(2 * (size_t)sm_count(), units);
  size_t chunk = ceil_div(max_ctx, want);
  chunk = ceil_div(chunk, 16) * 16;
  if (chunk < 64) chunk = 64;
  if (chunk > 1024) chunk = 1024;
  return (int)chunk;
}

int paged_attention(const float* q, size_t ldq, const float* pool, size_t page_floats, const int32_t* block_tables,
                    size_t max_pages, const int32_t* ctx_lens, size_t max_ctx, size_t lanes, size_t layer,
                    size_t num_heads, size_t num_kv_heads, size_t head_dim, float* out, size_t ldo, float* workspace,
                    size_t workspace_floats, int chunk, cudaStream_t stream) {
  GLC_REQUIRE(q && pool && block_tables && ctx_lens && out && workspace, "paged_attention: null argument");
  GLC_REQUIRE(num_kv_heads > 0 && num_heads % num_kv_heads == 0, "paged_attention: heads %zu / kv heads %zu",
              num_heads, num_kv_heads);
  const size_t group = num_heads / num_kv_heads;
  GLC_REQUIRE(group <= kMaxGroup && head_dim <= kMaxHeadDim && head_dim % 4 == 0,
              "paged_attention: group %zu / head_dim %zu outside the kernel contract", group, head_dim);
  GLC_REQUIRE(max_ctx > 0 && max_ctx <= max_pages * 16, "paged_attention: context %zu exceeds the block table",
              max_ctx);
  if (chunk <= 0) chunk = attention_chunk(lanes, num_kv_heads, max_ctx);
  GLC_REQUIRE(chunk % 16 == 0, "paged_attention: chunk must be whole pages");
  const int nsplit = (int)ceil_div(max_ctx, (size_t)chunk);
  GLC_REQUIRE(workspace_floats >= attention_workspace_floats(lanes, num_heads, head_dim, nsplit),
              "paged_attention: workspace too small");
  AttnParams prm;
  prm.q = q;
  prm.ldq = ldq;
  prm.pool = pool;
  prm.page_floats = page_floats;
  prm.block_tables = block_tables;
  prm.max_pages = (int)max_pages;
  prm.ctx_lens = ctx_lens;
  prm.layer = (int)layer;
  prm.num_heads = (int)num_heads;
  prm.num_kv_heads = (int)num_kv_heads;
  prm.head_dim = (int)head_dim;
  prm.group = (int)group;
  prm.chunk = chunk;
  prm.nsplit = nsplit;
  prm.scale = 1.0f / sqrtf((float)head_dim);
  prm.part_o = workspace;
  prm.part_ml = workspace + lanes * num_heads * nsplit * head_dim;
  const size_t smem = (kMaxGroup * kMaxHeadDim + group * chunk) * sizeof(float);
  static size_t attr = 0;
  if (smem > 48 * 1024 && attr < smem) {
    const int rc = allow_dynamic_smem((const void*)attn_chunk_kernel, (int)smem);
    if (rc) return rc;
    attr = smem;
  }
  attn_chunk_kernel<<<dim3(nsplit, (unsigned)num_kv_heads, (unsigned)lanes), kAttnThreads, smem, stream>>>(prm);
  GLC_CHECK_LAUNCH();
  attn_combine_kernel<<<dim3((unsigned)num_heads, (unsigned)lanes), 128, 0, stream>>>(
      prm.part_o, prm.part_ml, nsplit, (int)head_dim, (int)num_heads, out, ldo);
  GLC_CHECK_LAUNCH();
  return GLACIER_CUDA_OK;
}

}  // namespace glacier
