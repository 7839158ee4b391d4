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
// tile, forward.zig:544-620).  Pass 1: each warp takes 8 positions at a time,
// four lanes per position (a quarter of the head dims each, contiguous K loads,
// q from bank-padded shared memory, packed fp32x2 FMAs, a two-step shuffle
// reduction).  Pass 2: per-head chunk max and exp-sum.  Pass 3: lanes over head
// dims accumulate p * V from coalesced V rows with packed FMAs.
// A combine kernel merges the chunks with the usual max/sum rescaling, in
// chunk order (deterministic).
#include <type_traits>

#include "common.cuh"

namespace glacier {

namespace {

constexpr int kAttnThreads = 128;  // 4 warps
constexpr int kMaxGroup = 8;       // query heads per kv head
constexpr int kBlock = 8;          // positions per warp iteration

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

// Pass 1 maps a warp onto 8 positions x 4 head-dim slices (HD/4 dims per lane,
// contiguous 16-byte loads of each K row), pass 3 onto head dims (HD/32 per
// lane, one coalesced row load per position).
template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attn_chunk_kernel(const AttnParams p) {
  constexpr int SL = HD / 4;      // dims per lane in pass 1
  constexpr int SL4 = SL / 4;     // float4 per lane in pass 1
  constexpr int QPITCH = SL + 4;  // padded q slice pitch (floats): slices land in different banks
  constexpr int DPL = HD / 32;    // dims per lane in pass 3
  extern __shared__ float sm[];
  float* qs = sm;                                  // [G][4 slices][QPITCH]
  float* sc = qs + kMaxGroup * 4 * QPITCH;         // [chunk][8]  scores, then probabilities
  float* red = sc + (size_t)p.chunk * kMaxGroup;   // [4 warps][G][HD] pass-3 partials
  __shared__ float mx[kMaxGroup], wred[kAttnThreads / 32][kMaxGroup];

  const int lane_id = blockIdx.z;
  const int kvh = blockIdx.y;
  const int split = blockIdx.x;
  const int G = p.group;
  const int ctx = p.ctx_lens[lane_id];
  const int j0 = split * p.chunk;
  const int j1 = min(ctx, j0 + p.chunk);
  const int n = j1 - j0;
  const int kv_dim = p.num_kv_heads * HD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t part_base = ((size_t)lane_id * p.num_heads + (size_t)kvh * G) * p.nsplit + split;

  if (n <= 0) {  // empty chunk: neutral partial (max -inf, sum 0)
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
      p.part_ml[(part_base + (size_t)g * p.nsplit) * 2 + 0] = -INFINITY;
      p.part_ml[(part_base + (size_t)g * p.nsplit) * 2 + 1] = 0.f;
    }
    return;
  }
  for (int i = threadIdx.x; i < kMaxGroup * HD; i += blockDim.x) {
    const int g = i / HD, d = i % HD;
    const float v = g < G ? p.q[lane_id * p.ldq + (size_t)(kvh * G + g) * HD + d] * p.scale : 0.f;
    qs[(g * 4 + d / SL) * QPITCH + d % SL] = v;
  }
  __syncthreads();

  const int32_t* bt = p.block_tables + (size_t)lane_id * p.max_pages;
  const size_t k_off = (size_t)(p.layer * 2 + 0) * 16 * kv_dim + (size_t)kvh * HD;
  const size_t v_off = (size_t)(p.layer * 2 + 1) * 16 * kv_dim + (size_t)kvh * HD;
  const int nblocks = (n + kBlock - 1) / kBlock;

  // ---- pass 1: scores = (q * scale) . k for the G heads -------------------------
  // The K loads of the warp's next block are issued before the current block is
  // consumed (register double buffering), so every lane keeps 2 x HD/4 floats in flight.
  {
    const int pp = lane >> 2, sl = lane & 3;
    auto krow_of = [&](int bk) {
      const int j = j0 + min(bk * kBlock + pp, n - 1);  // clamp the tail to a valid row
      return reinterpret_cast<const float4*>(p.pool + (size_t)bt[j >> 4] * p.page_floats + k_off +
                                             (size_t)(j & 15) * kv_dim + sl * SL);
    };
    float4 kv[SL4], kn[SL4];
    int bk = warp;
    if (bk < nblocks) {
      const float4* kr = krow_of(bk);
#pragma unroll
      for (int i = 0; i < SL4; ++i) kv[i] = __ldg(kr + i);
    }
    for (; bk < nblocks; bk += kAttnThreads / 32) {
      const int bn = bk + kAttnThreads / 32;
      if (bn < nblocks) {
        const float4* kr = krow_of(bn);
#pragma unroll
        for (int i = 0; i < SL4; ++i) kn[i] = __ldg(kr + i);
      }
      const int jj = bk * kBlock + pp;
      float2 acc[kMaxGroup];
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) acc[g] = make_float2(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < SL4; ++i) {
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) {
          if (g < G) {
            const float4 qv = *reinterpret_cast<const float4*>(qs + (g * 4 + sl) * QPITCH + 4 * i);
            acc[g] = __ffma2_rn(make_float2(qv.x, qv.y), make_float2(kv[i].x, kv[i].y), acc[g]);
            acc[g] = __ffma2_rn(make_float2(qv.z, qv.w), make_float2(kv[i].z, kv[i].w), acc[g]);
          }
        }
      }
      float sv[kMaxGroup];
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        float v = acc[g].x + acc[g].y;
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        sv[g] = v;
      }
      if (sl == 0 && jj < n) {
        float4* dst = reinterpret_cast<float4*>(sc + (size_t)jj * kMaxGroup);
        dst[0] = make_float4(sv[0], sv[1], sv[2], sv[3]);
        dst[1] = make_float4(sv[4], sv[5], sv[6], sv[7]);
      }
#pragma unroll
      for (int i = 0; i < SL4; ++i) kv[i] = kn[i];
    }
  }
  __syncthreads();

  // ---- pass 2: per-head chunk max, exp, sum ---------------------------------------
  {
    // thread t covers head g = t & 7 over positions (t >> 3), (t >> 3) + 16, ...
    const int g = threadIdx.x & 7, r = threadIdx.x >> 3;  // r in 0..15
    float m = -INFINITY;
    for (int jj = r; jj < n; jj += 16) m = fmaxf(m, sc[jj * kMaxGroup + g]);
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
    if (lane < 8) wred[warp][g] = m;
    __syncthreads();
    if (threadIdx.x < kMaxGroup) {
      float v = wred[0][threadIdx.x];
      for (int w = 1; w < kAttnThreads / 32; ++w) v = fmaxf(v, wred[w][threadIdx.x]);
      mx[threadIdx.x] = v;
    }
    __syncthreads();
    const float mg = mx[g];
    float sum = 0.f;
    for (int jj = r; jj < n; jj += 16) {
      const float e = g < G ? expf(sc[jj * kMaxGroup + g] - mg) : 0.f;
      sc[jj * kMaxGroup + g] = e;
      sum += e;
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 8);
    sum += __shfl_xor_sync(0xffffffffu, sum, 16);
    __syncthreads();
    if (lane < 8) wred[warp][g] = sum;
    __syncthreads();
    if (threadIdx.x < G) {
      float v = 0.f;
      for (int w = 0; w < kAttnThreads / 32; ++w) v += wred[w][threadIdx.x];
      p.part_ml[(part_base + (size_t)threadIdx.x * p.nsplit) * 2 + 0] = mx[threadIdx.x];
      p.part_ml[(part_base + (size_t)threadIdx.x * p.nsplit) * 2 + 1] = v;
    }
  }
  __syncthreads();

  // ---- pass 3: o[g][d] = sum_j p[g][j] * v_j[d], lanes over head dims ------------
  {
    float2 acc[kMaxGroup][DPL / 2];
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g)
#pragma unroll
      for (int i = 0; i < DPL / 2; ++i) acc[g][i] = make_float2(0.f, 0.f);
    // All 8 V rows of a block are loaded before use, and the next block's rows
    // are in flight while the current block is accumulated.
    using VecT = typename std::conditional<DPL == 4, float4, float2>::type;
    auto vrow_of = [&](int bk, int pp) {
      const int j = j0 + min(bk * kBlock + pp, n - 1);
      return reinterpret_cast<const VecT*>(p.pool + (size_t)bt[j >> 4] * p.page_floats + v_off +
                                           (size_t)(j & 15) * kv_dim) + lane;
    };
    VecT vc[kBlock], vn[kBlock];
    int bk = warp;
    if (bk < nblocks) {
#pragma unroll
      for (int pp = 0; pp < kBlock; ++pp) vc[pp] = __ldg(vrow_of(bk, pp));
    }
    for (; bk < nblocks; bk += kAttnThreads / 32) {
      const int bn = bk + kAttnThreads / 32;
      if (bn < nblocks) {
#pragma unroll
        for (int pp = 0; pp < kBlock; ++pp) vn[pp] = __ldg(vrow_of(bn, pp));
      }
#pragma unroll
      for (int pp = 0; pp < kBlock; ++pp) {
        const int jj = bk * kBlock + pp;
        if (jj < n) {  // positions past the chunk end carry no probability
          float vv[DPL];
          if constexpr (DPL == 4) {
            vv[0] = vc[pp].x; vv[1] = vc[pp].y; vv[2] = vc[pp].z; vv[3] = vc[pp].w;
          } else {
            vv[0] = vc[pp].x; vv[1] = vc[pp].y;
          }
          const float4 p0 = *reinterpret_cast<const float4*>(sc + (size_t)jj * kMaxGroup);
          const float4 p1 = *reinterpret_cast<const float4*>(sc + (size_t)jj * kMaxGroup + 4);
          const float pg[kMaxGroup] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
          for (int g = 0; g < kMaxGroup; ++g) {
            if (g < G) {
#pragma unroll
              for (int i = 0; i < DPL / 2; ++i)
                acc[g][i] = __ffma2_rn(make_float2(pg[g], pg[g]), make_float2(vv[2 * i], vv[2 * i + 1]), acc[g][i]);
            }
          }
        }
      }
#pragma unroll
      for (int pp = 0; pp < kBlock; ++pp) vc[pp] = vn[pp];
    }
    // reduce the 4 warps' partials through shared memory (scores are no longer needed)
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      if (g < G) {
#pragma unroll
        for (int i = 0; i < DPL / 2; ++i) {
          red[((size_t)warp * kMaxGroup + g) * HD + lane * DPL + 2 * i] = acc[g][i].x;
          red[((size_t)warp * kMaxGroup + g) * HD + lane * DPL + 2 * i + 1] = acc[g][i].y;
        }
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
      const int g = i / HD, d = i % HD;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kAttnThreads / 32; ++w) v += red[((size_t)w * kMaxGroup + g) * HD + d];
      p.part_o[(part_base + (size_t)g * p.nsplit) * HD + d] = v;
    }
  }
}

// out[lane, h, :] = sum_s o_s * e^(m_s - M) / sum_s l_s * e^(m_s - M), in split
// order.  A cluster of CTAs covers one lane (blockIdx.y), each a range of
// heads; split outputs (the o-projection's GEMM input) share the lane's row
// max through distributed shared memory.
__global__ void __launch_bounds__(256) attn_combine_kernel(const float* __restrict__ part_o,
                                                           const float* __restrict__ part_ml, int nsplit, int head_dim,
                                                           int num_heads, float* __restrict__ out, size_t ldo,
                                                           SplitOut so) {
  extern __shared__ float row[];  // this CTA's heads x head_dim (split outputs)
  __shared__ float hm[kMaxGroup * 4], hinv[kMaxGroup * 4];
  __shared__ float sh[32], xch;
  const int lane_id = blockIdx.y;
  const int cr = (int)cluster_ctarank(), cn = (int)cluster_nctarank();
  const int hpc = (num_heads + cn - 1) / cn;
  const int h0 = min(num_heads, cr * hpc), h1 = min(num_heads, h0 + hpc);
  for (int t = threadIdx.x; t < h1 - h0; t += blockDim.x) {
    const size_t base = ((size_t)lane_id * num_heads + h0 + t) * nsplit;
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, part_ml[(base + s) * 2]);
    float L = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float m = part_ml[(base + s) * 2];
      if (m != -INFINITY) L += part_ml[(base + s) * 2 + 1] * expf(m - M);
    }
    hm[t] = M;
    hinv[t] = 1.0f / L;
  }
  __syncthreads();
  float mx = 0.f;
  for (int i = threadIdx.x; i < (h1 - h0) * head_dim; i += blockDim.x) {
    const int t = i / head_dim, d = i % head_dim;
    const size_t base = ((size_t)lane_id * num_heads + h0 + t) * nsplit;
    float acc = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float m = part_ml[(base + s) * 2];
      if (m != -INFINITY) acc = fmaf(part_o[(base + s) * head_dim + d], expf(m - hm[t]), acc);
    }
    const float v = acc * hinv[t];
    if (so.xs) {
      row[i] = v;
      mx = fmaxf(mx, fabsf(v));
    } else {
      out[lane_id * ldo + (size_t)(h0 + t) * head_dim + d] = v;
    }
  }
  if (so.xs) {
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t = fmaxf(t, sh[w]);
      xch = t;
    }
    cluster_sync_all();
    float rm = 0.f;
    const uint32_t a = smem_u32(&xch);
    for (int q = 0; q < cn; ++q) rm = fmaxf(rm, ld_dsmem_f32(mapa_shared(a, (uint32_t)q)));
    const float scale = split_scale(rm);
    const float iscale = 1.0f / scale;
    const int K = num_heads * head_dim;
    for (int k8 = threadIdx.x; k8 < (h1 - h0) * head_dim / 8; k8 += blockDim.x) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = row[k8 * 8 + i];
      store_split8(so, lane_id, K, (size_t)h0 * head_dim + (size_t)k8 * 8, v, iscale);
    }
    if (cr == 0 && threadIdx.x == 0) so.xscale[lane_id] = scale;
    cluster_sync_all();
  }
}

}  // namespace

// Workspace floats needed by paged_attention for the given split count.
size_t attention_workspace_floats(size_t lanes, size_t num_heads, size_t head_dim, size_t nsplit) {
  return lanes * num_heads * nsplit * (head_dim + 2);
}

// Positions per chunk: splits so that lanes * kv_heads * splits covers the
// SMs about four times, chunks of 64..512 positions in whole pages.
int attention_chunk(size_t lanes, size_t num_kv_heads, size_t max_ctx) {
  const size_t units = lanes * num_kv_heads;
  size_t want = ceil_div(4 * (size_t)sm_count(), units);
  size_t chunk = ceil_div(max_ctx, want);
  chunk = ceil_div(chunk, 32) * 32;
  if (chunk < 64) chunk = 64;
  if (chunk > 512) chunk = 512;
  return (int)chunk;
}

int paged_attention(const float* q, size_t ldq, const float* pool, size_t page_floats, const int32_t* block_tables,
                    size_t max_pages, const int32_t* ctx_lens, size_t max_ctx, size_t lanes, size_t layer,
                    size_t num_heads, size_t num_kv_heads, size_t head_dim, float* out, size_t ldo, float* workspace,
                    size_t workspace_floats, int chunk, cudaStream_t stream, SplitOut so, StepProfiler* prof,
                    int combine_kind) {
  GLC_REQUIRE(q && pool && block_tables && ctx_lens && (out || so.xs) && workspace, "paged_attention: null argument");
  GLC_REQUIRE(num_kv_heads > 0 && num_heads % num_kv_heads == 0, "paged_attention: heads %zu / kv heads %zu",
              num_heads, num_kv_heads);
  const size_t group = num_heads / num_kv_heads;
  GLC_REQUIRE(group <= kMaxGroup && (head_dim == 64 || head_dim == 128),
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
  const size_t smem =
      ((size_t)kMaxGroup * 4 * (head_dim / 4 + 4) + (size_t)chunk * kMaxGroup + 4 * kMaxGroup * head_dim) * sizeof(float);
  auto kern = head_dim == 128 ? attn_chunk_kernel<128> : attn_chunk_kernel<64>;
  static size_t attr[2] = {0, 0};
  size_t& done = attr[head_dim == 128 ? 1 : 0];
  if (smem > 48 * 1024 && done < smem) {
    const int rc = allow_dynamic_smem((const void*)kern, (int)smem);
    if (rc) return rc;
    done = smem;
  }
  kern<<<dim3(nsplit, (unsigned)num_kv_heads, (unsigned)lanes), kAttnThreads, smem, stream>>>(prm);
  GLC_CHECK_LAUNCH();
  if (prof) prof->mark(combine_kind, stream);
  {
    // Cluster of CTAs per lane over its heads (about 7 heads per CTA).
    int cl = 1;
    while (cl < 8 && (size_t)cl * 7 < num_heads) cl *= 2;
    const int hpc = (int)ceil_div(num_heads, (size_t)cl);
    GLC_REQUIRE(hpc <= 4 * kMaxGroup, "paged_attention: too many heads per combine CTA");
    const size_t csmem = so.xs ? (size_t)hpc * head_dim * sizeof(float) : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)cl, (unsigned)lanes);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = csmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    GLC_CHECK_CUDA(cudaLaunchKernelEx(&cfg, attn_combine_kernel, (const float*)prm.part_o, (const float*)prm.part_ml,
                                      nsplit, (int)head_dim, (int)num_heads, out, ldo, so));
    note_launch();
  }
  return GLACIER_CUDA_OK;
}

}  // namespace glacier
