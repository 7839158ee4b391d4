// Kernel (d): paged-KV decode attention over the reference's FP32 page layout.
//
// Same operator as attentionMultiHead (src/paged_attention.zig:108-216) for one
// query row per lane: causal GQA (kv head = h / (H / Hkv)), scale 1/sqrt(hd),
// softmax over positions 0..ctx-1.  Pages hold 16 positions of every layer:
// payload offset ((layer*2 + kind)*16 + row) * kv_dim floats
// (src/paged_kv_cache.zig:1421-1442); block_tables[lane][logical page] gives
// the physical page.
//
// B200 design (flash-decoding over TMA-fed warps): the K/V stages of every
// (lane, kv head) pair are split evenly over all warps of the grid (static
// stream-K: each warp streams the same number of bytes); a warp serves all
// G = H/Hkv query heads of the GQA group from a single read of each K and V
// row (the reference's shared-KV tile, forward.zig:544-620).  A combine kernel
// merges a pair's segments with the usual max/sum rescaling, in segment order
// (deterministic).
#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace glacier {

__device__ int g_attn_error;

namespace {

constexpr int kMaxGroup = 8;  // query heads per kv head

struct AttnParams {
  const float* q;  // [lanes, H*hd]
  size_t ldq;
  const float* pool;
  size_t page_floats;
  const int32_t* block_tables;  // [lanes, max_pages]
  int max_pages;
  const int32_t* ctx_lens;      // [lanes]
  int layer, num_heads, num_kv_heads, head_dim, group;
  int warps;                    // warps of the attention grid (W)
  int nsplit;                   // segment slots per (lane, kv head)
  float scale;
  float* part_o;                // [lanes, H, nsplit, hd]
  float* part_ml;               // [lanes, H, nsplit, 2]  (max, sum)
};

constexpr int kStagePositions = 8;  // positions per pipeline stage

// A lane's context as the kernels use it: clamped to [0, cap] (cap = the block
// table's positions), so a context past the table never reads past it.
__device__ __forceinline__ int lane_ctx(const int32_t* __restrict__ ctx_lens, int l, int cap) {
  return min(max(ctx_lens[l], 0), cap);
}
constexpr int kMaxPlanLanes = 128;  // lanes one stage plan covers (4 per thread of a warp)

// Static work split shared by the attention and combine kernels (stream-K):
// the stages (8 positions of one kv head) of every (lane, kv head) pair are
// laid end to end, lane-major, and warp w of the grid takes stages
// [w * Q, (w + 1) * Q).  A pair cut by warp boundaries leaves one partial per
// warp (segment), numbered from the pair's first warp.  Q is the even share,
// raised when needed so no pair has more than seg_cap segments.  Run by one
// warp; C[l] = first stage of lane l (C[lanes] = total); plan = {total, Q}.
__device__ __forceinline__ void attn_stage_plan(const int32_t* __restrict__ ctx_lens, int lanes, int hkv, int warps,
                                                int seg_cap, int* C, int* plan, int ctx_cap) {
  const int lane = threadIdx.x & 31;
  int v[4], sum = 0, mx = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = 4 * lane + i;
    const int ns = idx < lanes ? (lane_ctx(ctx_lens, idx, ctx_cap) + kStagePositions - 1) / kStagePositions : 0;
    v[i] = hkv * ns;
    sum += v[i];
    mx = max(mx, ns);
  }
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  int excl = incl - sum;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = 4 * lane + i;
    if (idx <= lanes) C[idx] = excl;
    excl += v[i];
  }
  const int total = __shfl_sync(0xffffffffu, incl, 31);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const int q = max(1, max((total + warps - 1) / warps, (mx + seg_cap - 2) / max(1, seg_cap - 1)));
  if (lane == 0) {
    plan[0] = total;
    plan[1] = q;
  }
}

// Segments of pair (lane l, kv head h): its stages [P, P + ns) over warps of Q stages.
__device__ __forceinline__ int attn_pair_segments(const int* C, const int32_t* ctx_lens, int l, int h, int q,
                                                  int ctx_cap) {
  const int ns = (lane_ctx(ctx_lens, l, ctx_cap) + kStagePositions - 1) / kStagePositions;
  if (ns == 0) return 0;
  const int P = C[l] + h * ns;
  return (P + ns - 1) / q - P / q + 1;
}

// ---------------------------------------------------------------------------
// TMA-fed persistent form.  Each warp takes its contiguous share of the stage
// sequence (attn_stage_plan), i.e. one segment of one or more consecutive
// (lane, kv head) pairs; it owns a private ring of half-page stages (8
// positions of K and V of one kv head), so no warp ever waits for another and
// every warp streams the same number of K/V bytes:
//   * lane 0 streams each stage's K and V tiles (8 rows x HD floats, two 2D TMA
//     boxes over the pool viewed as [rows, kv_dim]) into the next free slot,
//     running kAttnStages stages ahead across item boundaries;
//   * scores: 16 lanes per position, 2 positions per step, q of all G heads in
//     registers (HD/16 dims per lane, interleaved so a step's shared-memory
//     reads are conflict-free), packed fp32x2 FMAs and a butterfly that leaves
//     lanes (16p + 2h, 16p + 2h + 1) with the score of position p, head h;
//   * online softmax per stage (running max and sum per head, acc rescaled);
//   * P.V: lanes over head dims, V rows and probabilities from shared memory.
// Each segment writes one (max, sum, unnormalised o) partial for the combine.
// Warps per CTA (one CTA per SM) and half-page stages per warp.  Many lanes:
// twelve warps of two stages keep the same 192 KB of K/V in flight per SM as
// eight warps of three, with half again as many warps to hide each warp's
// dependency latency (the kernel fits 168 registers a thread): 97.6 against
// 105.6 us a 64-lane 7B layer (0.89 against 0.82 of the measured HBM copy
// rate).  Four lanes or fewer keep eight warps of three stages: a single
// context spread over the grid gives each warp a stage or two, and the larger
// CTA only lengthens the prologue (11.8 against 10.6 us a layer at batch 1).
constexpr int kAttnWarpsWide = 12, kAttnStagesWide = 2;
constexpr int kAttnWarpsFew = 8, kAttnStagesFew = 3;
constexpr int kStageRows = kStagePositions;

__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 2^x on the special-function unit (relative error about 2^-22; results below
// the normal range flush to zero, far below what a softmax weight can matter).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One half-page stage of one warp: base-2 scores of its 8 positions for the NG
// heads, the online-softmax update of (m, l, acc) and P.V.  Kt / Vt: the stage's
// K and V rows in shared memory; nvalid: positions inside the context; scr / prb:
// the warp's score and probability scratch.  Shared by the stream-K kernel and
// the cluster kernel for few lanes.
template <int HD, int NG>
__device__ __forceinline__ void attn_stage_math(const float* __restrict__ Kt, const float* __restrict__ Vt,
                                                int nvalid, const float2 (&q2)[NG][HD / 32], float (&m)[NG],
                                                float (&l)[NG], float2 (&acc)[NG][HD / 64], float* scr, float2* prb,
                                                int lane) {
  constexpr int DL4 = HD / 64;  // score phase: float4 loads per lane (16 lanes per position)
  constexpr int VD = HD / 32;   // P.V phase: dims per lane
  constexpr int G = NG;
  const int l16 = lane & 15, ph = lane >> 4;
  // -- scores (base-2 logits) for 8 positions, 2 per step --
#pragma unroll
  for (int step = 0; step < kStageRows / 2; ++step) {
    const int pos = 2 * step + ph;
    float4 kv[DL4];
#pragma unroll
    for (int i = 0; i < DL4; ++i) kv[i] = *reinterpret_cast<const float4*>(Kt + pos * HD + 4 * l16 + 64 * i);
    float v[kMaxGroup];
#pragma unroll
    for (int g = NG; g < kMaxGroup; ++g) v[g] = 0.f;
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      float2 a = __fmul2_rn(q2[g][0], make_float2(kv[0].x, kv[0].y));
      a = __ffma2_rn(q2[g][1], make_float2(kv[0].z, kv[0].w), a);
#pragma unroll
      for (int i = 1; i < DL4; ++i) {
        a = __ffma2_rn(q2[g][2 * i], make_float2(kv[i].x, kv[i].y), a);
        a = __ffma2_rn(q2[g][2 * i + 1], make_float2(kv[i].z, kv[i].w), a);
      }
      v[g] = a.x + a.y;
    }
    // Butterfly over the 16 lanes of this position: lanes 2h, 2h+1 end with head h.
    const bool b8 = (l16 & 8) != 0, b4 = (l16 & 4) != 0, b2 = (l16 & 2) != 0;
    float w4[4], w2[2];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float send = b8 ? v[k] : v[k + 4];
      const float keep = b8 ? v[k + 4] : v[k];
      w4[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float send = b4 ? w4[k] : w4[k + 2];
      const float keep = b4 ? w4[k + 2] : w4[k];
      w2[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    const float send = b2 ? w2[0] : w2[1];
    const float keep = b2 ? w2[1] : w2[0];
    float sc = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    sc += __shfl_xor_sync(0xffffffffu, sc, 1);
    const int h = l16 >> 1;
    if (h >= G || (nvalid < kStageRows && pos >= nvalid)) sc = -INFINITY;
    if ((l16 & 1) == 0) scr[pos * kMaxGroup + h] = sc;
  }
  __syncwarp();
  // -- online softmax over this stage: lane = (head lane & 7, positions (lane >> 3) + 4k) --
  const int hh = lane & 7, r0 = lane >> 3;
  const float s0 = scr[r0 * kMaxGroup + hh], s1 = scr[(r0 + 4) * kMaxGroup + hh];
  float mp = fmaxf(s0, s1);
  mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 8));
  mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 16));
  float alpha[NG], mh = 0.f;
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const float mn = fmaxf(m[g], __shfl_sync(0xffffffffu, mp, g));
    alpha[g] = (m[g] == -INFINITY) ? 0.f : ex2_approx(m[g] - mn);
    m[g] = mn;
    if (g == hh) mh = mn;
  }
  // Masked scores are -inf and give ex2(-inf) = 0; padding heads (hh >= G) are zeroed.
  const float e0 = hh < G ? ex2_approx(s0 - mh) : 0.f;
  const float e1 = hh < G ? ex2_approx(s1 - mh) : 0.f;
  prb[r0 * kMaxGroup + hh] = make_float2(e0, e0);
  prb[(r0 + 4) * kMaxGroup + hh] = make_float2(e1, e1);
  float ps = e0 + e1;
  ps += __shfl_xor_sync(0xffffffffu, ps, 8);
  ps += __shfl_xor_sync(0xffffffffu, ps, 16);
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    l[g] = l[g] * alpha[g] + __shfl_sync(0xffffffffu, ps, g);
    const float2 a2 = make_float2(alpha[g], alpha[g]);
#pragma unroll
    for (int i = 0; i < VD / 2; ++i) acc[g][i] = __fmul2_rn(acc[g][i], a2);
  }
  __syncwarp();
  // -- P.V over the stage (positions past the context carry probability 0
  //    and are skipped, so stale rows never enter the sum) --
  auto pv_row = [&](int pos) {
    float vv[VD];
    if constexpr (VD == 4) {
      const float4 t = *reinterpret_cast<const float4*>(Vt + pos * HD + 4 * lane);
      vv[0] = t.x; vv[1] = t.y; vv[2] = t.z; vv[3] = t.w;
    } else {
      const float2 t = *reinterpret_cast<const float2*>(Vt + pos * HD + 2 * lane);
      vv[0] = t.x; vv[1] = t.y;
    }
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      const float2 pp = prb[pos * kMaxGroup + g];
#pragma unroll
      for (int i = 0; i < VD / 2; ++i)
        acc[g][i] = __ffma2_rn(pp, make_float2(vv[2 * i], vv[2 * i + 1]), acc[g][i]);
    }
  };
  if (nvalid == kStageRows) {
#pragma unroll
    for (int pos = 0; pos < kStageRows; ++pos) pv_row(pos);
  } else {
    for (int pos = 0; pos < nvalid; ++pos) pv_row(pos);
  }
}

// NG = query heads per kv head (compile time); HD = head dim; kAttnWarps and
// kAttnStages as above.
template <int HD, int NG, int kAttnWarps, int kAttnStages>
__global__ void __launch_bounds__(kAttnWarps * 32, 1)
    attn_tma_kernel(const __grid_constant__ CUtensorMap kvmap, const AttnParams p, int lanes, int rows_per_page,
                    int* err) {
  constexpr int TILE = kStageRows * HD;  // floats per K (or V) stage tile of one kv head
  constexpr int DL = HD / 16;            // score phase: dims per lane (16 lanes per position)
  constexpr int DL4 = DL / 4;
  constexpr int VD = HD / 32;            // P.V phase: dims per lane
  constexpr float kLog2e = 1.4426950408889634f;
  extern __shared__ __align__(128) float sm[];
  __shared__ uint64_t bars[kAttnWarps][kAttnStages];
  __shared__ __align__(16) float scr_all[kAttnWarps][kStageRows * kMaxGroup];
  __shared__ __align__(16) float2 prb_all[kAttnWarps][kStageRows * kMaxGroup];  // {p, p} per (position, head)
  __shared__ int queue[kAttnWarps][8];  // pairs queued by lane 0, in issue order (-1 ends the list)
  __shared__ int Cs[kMaxPlanLanes + 1];
  __shared__ int plan[2];

  griddep_launch();
  griddep_wait();  // q, the KV pages and the context lengths come from earlier kernels
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int l16 = lane & 15;
  float* ring = sm + (size_t)warp * kAttnStages * 2 * TILE;
  float* scr = scr_all[warp];
  float2* prb = prb_all[warp];
  constexpr int G = NG;
  const int Hkv = p.num_kv_heads;
  const int ctx_cap = p.max_pages * 16;
  if (warp == 0) attn_stage_plan(p.ctx_lens, lanes, Hkv, p.warps, p.nsplit, Cs, plan, ctx_cap);
  if (lane == 0) {
    for (int i = 0; i < kAttnStages; ++i) mbar_init(&bars[warp][i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int total = plan[0], Q = plan[1];
  const int gw = blockIdx.x * kAttnWarps + warp;
  const int g0 = min(total, gw * Q), g1 = min(total, g0 + Q);  // this warp's stages
  // Pair geometry: stages ns of lane l, first stage P of (l, h), this warp's part [sb, se).
  auto pair_span = [&](int pair, int& lid, int& kvh, int& P, int& sb, int& se) {
    lid = pair / Hkv;
    kvh = pair - lid * Hkv;
    const int ns = (lane_ctx(p.ctx_lens, lid, ctx_cap) + kStageRows - 1) / kStageRows;
    P = Cs[lid] + kvh * ns;
    sb = max(0, g0 - P);
    se = min(ns, g1 - P);
  };
  // First pair of the warp: the lane whose stages hold g0 (largest l with C[l] <= g0).
  int first_pair = lanes * Hkv;
  if (g0 < g1) {
    int lo = 0, hi = lanes - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (Cs[mid] <= g0) lo = mid; else hi = mid - 1;
    }
    const int ns = (lane_ctx(p.ctx_lens, lo, ctx_cap) + kStageRows - 1) / kStageRows;
    first_pair = lo * Hkv + min(Hkv - 1, (g0 - Cs[lo]) / max(ns, 1));
  }

  // ---- issue cursor (lane 0): the next stage of this warp's sequence ----
  int c_pair = first_pair - 1, c_st = 0, c_se = 0, c_lid = 0, c_kvh = 0;
  uint32_t claimed = 0;
  bool drained = false;  // no pair left (the -1 marker is queued)
  auto claim = [&]() {  // lane 0: next pair with stages in [g0, g1) into the queue, or the end marker
    while (true) {
      ++c_pair;
      int P, sb, se;
      if (c_pair < lanes * Hkv) pair_span(c_pair, c_lid, c_kvh, P, sb, se);
      if (c_pair >= lanes * Hkv || P >= g1) {
        queue[warp][claimed++ & 7] = -1;
        drained = true;
        return;
      }
      if (sb < se) {
        c_st = sb;
        c_se = se;
        queue[warp][claimed++ & 7] = c_pair;
        return;
      }
    }
  };
  if (lane == 0) claim();
  uint64_t pol = 0;
  if (lane == 0) {
    prefetch_tmap(&kvmap);
    pol = l2_evict_first_policy();
  }
  uint32_t issued = 0;
  auto issue_next = [&]() {  // lane 0 only
    if (drained) return;
    if (c_st >= c_se) {
      claim();
      if (drained) return;
    }
    const int s = issued % kAttnStages;
    const int j = c_st * kStageRows;  // first position of the stage
    const int phys = p.block_tables[(size_t)c_lid * p.max_pages + (j >> 4)];
    const int yk = phys * rows_per_page + p.layer * 32 + (j & 15);
    float* dst = ring + (size_t)s * 2 * TILE;
    mbar_arrive_expect_tx(&bars[warp][s], 2 * TILE * (uint32_t)sizeof(float));
    tma_load_2d(dst, &kvmap, c_kvh * HD, yk, &bars[warp][s], pol);
    tma_load_2d(dst + TILE, &kvmap, c_kvh * HD, yk + 16, &bars[warp][s], pol);
    ++issued;
    ++c_st;
  };
  if (lane == 0)
    for (int i = 0; i < kAttnStages; ++i) issue_next();

  uint32_t consumed = 0, taken = 0;
  bool ok = true;
  while (ok) {
    __syncwarp();
    const int item = queue[warp][taken++ & 7];
    if (item < 0) break;
    int lid, kvh, P, sb, se;
    pair_span(item, lid, kvh, P, sb, se);
    const int nst = se - sb, ctx = lane_ctx(p.ctx_lens, lid, ctx_cap);
    const size_t part_base = ((size_t)lid * p.num_heads + (size_t)kvh * G) * p.nsplit + (gw - P / Q);
    // q of the G heads, scaled by 1/sqrt(hd) * log2(e) (softmax in base 2), this
    // lane's dims 4*l16 + 64*i + c.
    const float qs = p.scale * kLog2e;
    float2 q2[NG][DL / 2];
    const float* qrow = p.q + (size_t)lid * p.ldq + (size_t)kvh * G * HD;
#pragma unroll
    for (int g = 0; g < NG; ++g) {
#pragma unroll
      for (int i = 0; i < DL4; ++i) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(qrow + (size_t)g * HD + 4 * l16 + 64 * i));
        q2[g][2 * i] = make_float2(v.x * qs, v.y * qs);
        q2[g][2 * i + 1] = make_float2(v.z * qs, v.w * qs);
      }
    }
    float m[NG], l[NG];
    float2 acc[NG][VD / 2];
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      m[g] = -INFINITY;
      l[g] = 0.f;
#pragma unroll
      for (int i = 0; i < VD / 2; ++i) acc[g][i] = make_float2(0.f, 0.f);
    }
    for (int st = 0; st < nst; ++st, ++consumed) {
      const int s = consumed % kAttnStages;
      if (!__all_sync(0xffffffffu, mbar_wait(&bars[warp][s], (consumed / kAttnStages) & 1, err))) {
        ok = false;
        break;
      }
      const float* Kt = ring + (size_t)s * 2 * TILE;
      const float* Vt = Kt + TILE;
      const int nvalid = min(kStageRows, ctx - kStageRows * (sb + st));
      attn_stage_math<HD, NG>(Kt, Vt, nvalid, q2, m, l, acc, scr, prb, lane);
      __syncwarp();
      if (lane == 0) {
        fence_async_shared();  // this slot's generic reads precede the next async write into it
        issue_next();
      }
    }
    if (!ok) break;
    // -- partial of this item: unnormalised o, running max (natural log base) and sum --
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      {
        float* dst = p.part_o + (part_base + (size_t)g * p.nsplit) * HD + VD * lane;
        if constexpr (VD == 4) {
          *reinterpret_cast<float4*>(dst) = make_float4(acc[g][0].x, acc[g][0].y, acc[g][1].x, acc[g][1].y);
        } else {
          *reinterpret_cast<float2*>(dst) = acc[g][0];
        }
      }
    }
    if (lane < G) {
      float mm = m[0], ll = l[0];
#pragma unroll
      for (int g = 1; g < NG; ++g)
        if (g == lane) {
          mm = m[g];
          ll = l[g];
        }
      p.part_ml[(part_base + (size_t)lane * p.nsplit) * 2 + 0] = mm / kLog2e;
      p.part_ml[(part_base + (size_t)lane * p.nsplit) * 2 + 1] = ll;
    }
  }
  // Leave no copy in flight (a wait that gave up leaves some outstanding).
  if (lane == 0)
    for (uint32_t i = consumed; i < issued; ++i) mbar_wait(&bars[warp][i % kAttnStages], (i / kAttnStages) & 1, err);
  __syncwarp();
}

// ---------------------------------------------------------------------------
// Few lanes (4 or fewer, fp32 output): one cluster of kClusterCtas CTAs per
// (lane, kv head) and no combine launch.  CTA c of the cluster takes stages
// [c*ns/C, (c+1)*ns/C) of the pair's ns stages and its warps split those evenly;
// each warp streams its stages through a private TMA ring (attn_stage_math).  The
// warps' (max, sum, o) states merge in shared memory (warp g merges head g in
// warp order), then CTA rank 0 merges the CTAs' states over distributed shared
// memory in rank order and writes the normalised rows: the reduction order is
// fixed, so the result is deterministic.  A pair of context 0 writes zeros.
constexpr int kClusterCtas = 8;
constexpr int kCWarps = 8, kCStages = 3;

template <int HD, int NG>
__global__ void __launch_bounds__(kCWarps * 32, 1)
    attn_cluster_kernel(const __grid_constant__ CUtensorMap kvmap, const AttnParams p, int rows_per_page, int* err,
                        float* __restrict__ out, size_t ldo) {
  constexpr int TILE = kStageRows * HD;
  constexpr int DL = HD / 16, DL4 = DL / 4, VD = HD / 32;
  constexpr int SLOT = HD + 4;  // acc, then max (base 2) and sum; a multiple of 4 floats keeps float4 stores aligned
  constexpr float kLog2e = 1.4426950408889634f;
  extern __shared__ __align__(128) float sm[];
  __shared__ uint64_t bars[kCWarps][kCStages];
  __shared__ __align__(16) float scr_all[kCWarps][kStageRows * kMaxGroup];
  __shared__ __align__(16) float2 prb_all[kCWarps][kStageRows * kMaxGroup];

  griddep_launch();
  griddep_wait();  // q, the KV pages and the context lengths come from earlier kernels
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, l16 = lane & 15;
  const uint32_t cr = cluster_ctarank();
  const int pair = blockIdx.x / kClusterCtas;
  const int lid = pair / p.num_kv_heads, kvh = pair - lid * p.num_kv_heads;
  const int ctx = lane_ctx(p.ctx_lens, lid, p.max_pages * 16);
  const int ns = (ctx + kStageRows - 1) / kStageRows;
  const int cb = (int)((long long)ns * cr / kClusterCtas), ce = (int)((long long)ns * (cr + 1) / kClusterCtas);
  const int wb = cb + (ce - cb) * warp / kCWarps, we = cb + (ce - cb) * (warp + 1) / kCWarps;
  float* ring = sm + (size_t)warp * kCStages * 2 * TILE;
  if (lane == 0) {
    for (int i = 0; i < kCStages; ++i) mbar_init(&bars[warp][i], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // q of the G heads, scaled by 1/sqrt(hd) * log2(e), this lane's dims 4*l16 + 64*i + c.
  const float qs = p.scale * kLog2e;
  float2 q2[NG][DL / 2];
  const float* qrow = p.q + (size_t)lid * p.ldq + (size_t)kvh * NG * HD;
#pragma unroll
  for (int g = 0; g < NG; ++g) {
#pragma unroll
    for (int i = 0; i < DL4; ++i) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(qrow + (size_t)g * HD + 4 * l16 + 64 * i));
      q2[g][2 * i] = make_float2(v.x * qs, v.y * qs);
      q2[g][2 * i + 1] = make_float2(v.z * qs, v.w * qs);
    }
  }
  float m[NG], l[NG];
  float2 acc[NG][VD / 2];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < VD / 2; ++i) acc[g][i] = make_float2(0.f, 0.f);
  }

  uint64_t pol = 0;
  if (lane == 0) {
    prefetch_tmap(&kvmap);
    pol = l2_evict_first_policy();
  }
  int issued = wb;  // lane 0: next stage to load
  auto issue = [&](int st) {
    const int s = (st - wb) % kCStages;
    const int j = st * kStageRows;  // first position of the stage
    const int phys = p.block_tables[(size_t)lid * p.max_pages + (j >> 4)];
    const int yk = phys * rows_per_page + p.layer * 32 + (j & 15);
    float* dst = ring + (size_t)s * 2 * TILE;
    mbar_arrive_expect_tx(&bars[warp][s], 2 * TILE * (uint32_t)sizeof(float));
    tma_load_2d(dst, &kvmap, kvh * HD, yk, &bars[warp][s], pol);
    tma_load_2d(dst + TILE, &kvmap, kvh * HD, yk + 16, &bars[warp][s], pol);
  };
  if (lane == 0)
    for (; issued < min(we, wb + kCStages); ++issued) issue(issued);
  int consumed = 0;
  for (int st = wb; st < we; ++st, ++consumed) {
    const int s = consumed % kCStages;
    if (!__all_sync(0xffffffffu, mbar_wait(&bars[warp][s], (consumed / kCStages) & 1, err))) break;
    const float* Kt = ring + (size_t)s * 2 * TILE;
    const int nvalid = min(kStageRows, ctx - kStageRows * st);
    attn_stage_math<HD, NG>(Kt, Kt + TILE, nvalid, q2, m, l, acc, scr_all[warp], prb_all[warp], lane);
    __syncwarp();
    if (lane == 0) {
      fence_async_shared();  // this slot's generic reads precede the next async write into it
      if (issued < we) issue(issued++);
    }
  }
  // Leave no copy in flight (a wait that gave up leaves some outstanding).
  if (lane == 0)
    for (int i = consumed; i < issued - wb; ++i) mbar_wait(&bars[warp][i % kCStages], (i / kCStages) & 1, err);
  __syncthreads();  // every ring is idle: the states go where the stages were

  float* slots = sm;                         // [kCWarps][NG][SLOT]
  float* cpart = sm + kCWarps * NG * SLOT;   // [NG][SLOT], read by rank 0 over DSMEM
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    float* d = slots + (warp * NG + g) * SLOT;
    if constexpr (VD == 4) {
      *reinterpret_cast<float4*>(d + 4 * lane) = make_float4(acc[g][0].x, acc[g][0].y, acc[g][1].x, acc[g][1].y);
    } else {
      *reinterpret_cast<float2*>(d + 2 * lane) = acc[g][0];
    }
    if (lane == 0) {
      d[HD] = m[g];
      d[HD + 1] = l[g];
    }
  }
  __syncthreads();
  if (warp < NG) {  // this CTA's state of head `warp`, over its warps in order
    const int g = warp;
    float M = -INFINITY;
    for (int w = 0; w < kCWarps; ++w) M = fmaxf(M, slots[(w * NG + g) * SLOT + HD]);
    float L = 0.f, a[VD];
#pragma unroll
    for (int i = 0; i < VD; ++i) a[i] = 0.f;
    for (int w = 0; w < kCWarps; ++w) {
      const float* d = slots + (w * NG + g) * SLOT;
      const float e = d[HD] == -INFINITY ? 0.f : ex2_approx(d[HD] - M);
      L = fmaf(d[HD + 1], e, L);
#pragma unroll
      for (int i = 0; i < VD; ++i) a[i] = fmaf(d[VD * lane + i], e, a[i]);
    }
    float* c = cpart + g * SLOT;
#pragma unroll
    for (int i = 0; i < VD; ++i) c[VD * lane + i] = a[i];
    if (lane == 0) {
      c[HD] = M;
      c[HD + 1] = L;
    }
  }
  cluster_sync_all();  // every CTA's state is visible to the cluster
  if (cr == 0 && warp < NG) {
    const int g = warp;
    const uint32_t local = smem_u32(cpart + g * SLOT);
    float M = -INFINITY;
    for (uint32_t q = 0; q < kClusterCtas; ++q) M = fmaxf(M, ld_dsmem_f32(mapa_shared(local + 4 * HD, q)));
    float L = 0.f, a[VD];
#pragma unroll
    for (int i = 0; i < VD; ++i) a[i] = 0.f;
    for (uint32_t q = 0; q < kClusterCtas; ++q) {
      const uint32_t base = mapa_shared(local, q);
      const float mq = ld_dsmem_f32(base + 4 * HD);
      const float e = mq == -INFINITY ? 0.f : ex2_approx(mq - M);
      L = fmaf(ld_dsmem_f32(base + 4 * (HD + 1)), e, L);
#pragma unroll
      for (int i = 0; i < VD; ++i) a[i] = fmaf(ld_dsmem_f32(base + 4 * (VD * lane + i)), e, a[i]);
    }
    const float inv = L > 0.f ? 1.0f / L : 0.f;
    float* o = out + (size_t)lid * ldo + (size_t)(kvh * NG + g) * HD + VD * lane;
#pragma unroll
    for (int i = 0; i < VD; ++i) o[i] = a[i] * inv;
  }
  cluster_sync_all();  // keep every CTA's shared memory until rank 0 has read it
}

// out[lane, h, :] = sum_s o_s * e^(m_s - M) / sum_s l_s * e^(m_s - M), in segment
// order.  One CTA per (lane, block of heads): a warp per head computes the segment
// weights once, then each thread combines 8 consecutive values of one head from
// registers and writes them as fp32 or, for the o-projection GEMM, in split form
// with the lane's row max from one block reduction (one block of all heads).
__global__ void __launch_bounds__(1024) attn_combine_kernel(const float* __restrict__ part_o,
                                                            const float* __restrict__ part_ml, int nsplit,
                                                            int head_dim, int num_heads, float* __restrict__ out,
                                                            size_t ldo, SplitOut so,
                                                            const int32_t* __restrict__ ctx_lens, int lanes,
                                                            int num_kv_heads, int warps_total, int heads_per_block,
                                                            int ctx_cap) {
  griddep_launch();
  griddep_wait();
  extern __shared__ float wts[];  // [num_heads][nsplit] segment weights
  __shared__ float2 sh[32];
  __shared__ __align__(8) float2 xch;
  __shared__ int Cs[kMaxPlanLanes + 1], plan[2], segs[kMaxPlanLanes];
  const int lane_id = blockIdx.y;
  const int head0 = blockIdx.x * heads_per_block;  // the head blocks of a lane form one cluster
  const int nh = min(heads_per_block, num_heads - head0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  // The segments each head of this lane was cut into (the attention kernel's plan).
  if (warp == 0) attn_stage_plan(ctx_lens, lanes, num_kv_heads, warps_total, nsplit, Cs, plan, ctx_cap);
  __syncthreads();
  const int group = num_heads / num_kv_heads;
  for (int t = threadIdx.x; t < nh; t += blockDim.x)
    segs[t] = attn_pair_segments(Cs, ctx_lens, lane_id, (head0 + t) / group, plan[1], ctx_cap);
  __syncthreads();
  for (int t = warp; t < nh; t += nwarps) {
    const int nsplit_lane = segs[t];
    const size_t base = ((size_t)lane_id * num_heads + head0 + t) * nsplit;
    if (nsplit_lane <= 32) {  // one chunk per lane of the warp: one load of (max, sum)
      const float2 ml = lane < nsplit_lane ? *reinterpret_cast<const float2*>(part_ml + (base + lane) * 2)
                                           : make_float2(-INFINITY, 0.f);
      const float M = warp_max(ml.x);
      const float e = ml.x == -INFINITY ? 0.f : expf(ml.x - M);
      const float L = warp_sum(ml.y * e);
      if (lane < nsplit_lane) wts[t * nsplit + lane] = e * (1.0f / L);
      continue;
    }
    float M = -INFINITY;
    for (int s = lane; s < nsplit_lane; s += 32) M = fmaxf(M, part_ml[(base + s) * 2]);
    M = warp_max(M);
    float L = 0.f;
    for (int s = lane; s < nsplit_lane; s += 32) {
      const float m = part_ml[(base + s) * 2];
      const float e = m == -INFINITY ? 0.f : expf(m - M);
      wts[t * nsplit + s] = e;
      L += part_ml[(base + s) * 2 + 1] * e;
    }
    L = warp_sum(L);
    const float inv = 1.0f / L;
    for (int s = lane; s < nsplit_lane; s += 32) wts[t * nsplit + s] *= inv;
  }
  __syncthreads();
  const int e0 = 8 * threadIdx.x;
  const bool active = e0 < nh * head_dim;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float mx = 0.f;
  if (active) {
    const int t = e0 / head_dim, d = e0 - t * head_dim;
    const float* po = part_o + ((size_t)lane_id * num_heads + head0 + t) * nsplit * head_dim + d;
    const float* wt = wts + t * nsplit;
    const int nsplit_lane = segs[t];
#pragma unroll 4
    for (int s = 0; s < nsplit_lane; ++s) {
      float v[8];
      load8(po + (size_t)s * head_dim, v);
      const float w = wt[s];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(v[i], w, acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(acc[i]));
  }
  if (so.xs) {
    const float2 tot = row_sum_max(0.f, mx, sh, &xch);
    const float scale = split_scale(tot.y);
    if (active)
      store_split8(so, lane_id, (size_t)num_heads * head_dim, (size_t)head0 * head_dim + e0, acc, 1.0f / scale);
    if (threadIdx.x == 0) so.xscale[lane_id] = scale;
    if (cluster_nctarank() > 1) cluster_sync_all();  // no CTA leaves while another reads its row max
  } else if (active) {
    float4* dst = reinterpret_cast<float4*>(out + lane_id * ldo + (size_t)head0 * head_dim + e0);
    dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

// fp32 output of one (lane, head) per CTA, for few lanes: warp 0 computes the
// chunk weights, then the W warps take chunks s = warp, warp + W, ... (each lane
// 4 consecutive dims) and warp 0 adds the W partial sums in warp order.  Many
// chunks (one lane's context cut into one-page items) take W = 32, so each
// warp has at most a few dependent partial loads in flight.
template <int W>
__global__ void __launch_bounds__(W * 32) attn_combine_head_kernel(const float* __restrict__ part_o,
                                                                   const float* __restrict__ part_ml, int nsplit,
                                                                   int head_dim, int num_heads,
                                                                   float* __restrict__ out, size_t ldo,
                                                                   const int32_t* __restrict__ ctx_lens, int lanes,
                                                                   int num_kv_heads, int warps_total, int ctx_cap) {
  griddep_launch();
  griddep_wait();
  extern __shared__ float wts[];  // [nsplit]
  __shared__ float4 part[W][32];
  __shared__ int Cs[kMaxPlanLanes + 1], plan[2];
  const int lane_id = blockIdx.x, head = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) attn_stage_plan(ctx_lens, lanes, num_kv_heads, warps_total, nsplit, Cs, plan, ctx_cap);
  __syncthreads();
  const int nsplit_lane =
      attn_pair_segments(Cs, ctx_lens, lane_id, head / (num_heads / num_kv_heads), plan[1], ctx_cap);
  const size_t base = ((size_t)lane_id * num_heads + head) * nsplit;
  if (warp == 0) {
    float M = -INFINITY;
    for (int s = lane; s < nsplit_lane; s += 32) M = fmaxf(M, part_ml[(base + s) * 2]);
    M = warp_max(M);
    float L = 0.f;
    for (int s = lane; s < nsplit_lane; s += 32) {
      const float m = part_ml[(base + s) * 2];
      const float e = m == -INFINITY ? 0.f : expf(m - M);
      wts[s] = e;
      L += part_ml[(base + s) * 2 + 1] * e;
    }
    L = warp_sum(L);
    const float inv = 1.0f / L;
    for (int s = lane; s < nsplit_lane; s += 32) wts[s] *= inv;
  }
  __syncthreads();
  const bool active = 4 * lane < head_dim;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (active) {
    const float* po = part_o + base * head_dim + 4 * lane;
    for (int s = warp; s < nsplit_lane; s += W) {
      const float4 v = *reinterpret_cast<const float4*>(po + (size_t)s * head_dim);
      const float w = wts[s];
      acc.x = fmaf(v.x, w, acc.x);
      acc.y = fmaf(v.y, w, acc.y);
      acc.z = fmaf(v.z, w, acc.z);
      acc.w = fmaf(v.w, w, acc.w);
    }
  }
  part[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && active) {
    float4 t = part[0][lane];
#pragma unroll
    for (int w = 1; w < W; ++w) {
      const float4 q = part[w][lane];
      t.x += q.x;
      t.y += q.y;
      t.z += q.z;
      t.w += q.w;
    }
    *reinterpret_cast<float4*>(out + lane_id * ldo + (size_t)head * head_dim + 4 * lane) = t;
  }
}

}  // namespace

// Workspace floats needed by paged_attention for the given split count.
size_t attention_workspace_floats(size_t lanes, size_t num_heads, size_t head_dim, size_t nsplit) {
  return 4 + lanes * num_heads * nsplit * (head_dim + 2);  // 4 reserved + segment partials
}

// Segment slots per (lane, kv head): as many as the combine's weight table (one
// float per head and segment in 44 KB of shared memory) and a 64 MiB partial
// buffer allow, and no more than a context of max_ctx can use.  Few lanes get
// many slots (one context spread over every warp); 64 lanes get ~70, while the
// even share of such a batch cuts a pair into about a dozen segments.
int attention_segments(size_t lanes, size_t num_heads, size_t head_dim, size_t max_ctx) {
  // 44 KB: the combine kernels' static shared memory shares the 48 KB a launch gets by default.
  const size_t by_smem = (44 * 1024) / (sizeof(float) * num_heads);
  const size_t by_mem = ((size_t)64 << 20) / (lanes * num_heads * (head_dim + 2) * sizeof(float));
  const size_t by_ctx = ceil_div(max_ctx, (size_t)kStagePositions) + 1;
  return (int)std::max<size_t>(2, std::min({by_smem, std::max<size_t>(16, by_mem), by_ctx}));
}

int attn_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_attn_error, &z, sizeof(int));
  }
  return v;
}

// TMA view of a KV pool: [rows, kv_dim] floats, boxes of 16 rows x head_dim;
// encoded once per (pool, geometry) and cached per host thread.
static int attn_kv_map(const float* pool, size_t kv_dim, size_t head_dim, const CUtensorMap** out) {
  struct Entry {
    const float* pool;
    size_t kv_dim, head_dim;
    CUtensorMap map;
  };
  thread_local Entry cache[4];
  thread_local int next = 0;
  for (auto& e : cache)
    if (e.pool == pool && e.kv_dim == kv_dim && e.head_dim == head_dim) {
      *out = &e.map;
      return GLACIER_CUDA_OK;
    }
  Entry& e = cache[next];
  next = (next + 1) % 4;
  // Rows cover any pool that fits in device memory; block tables select within it.
  const uint64_t rows = ((uint64_t)192 << 30) / (kv_dim * sizeof(float));
  e.pool = nullptr;
  const int rc = encode_tmap_2d(&e.map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, pool, kv_dim, rows, kv_dim * sizeof(float),
                                (uint32_t)head_dim, kStageRows, CU_TENSOR_MAP_SWIZZLE_NONE,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  e.pool = pool;
  e.kv_dim = kv_dim;
  e.head_dim = head_dim;
  *out = &e.map;
  return GLACIER_CUDA_OK;
}

int paged_attention(const float* q, size_t ldq, const float* pool, size_t page_floats, const int32_t* block_tables,
                    size_t max_pages, const int32_t* ctx_lens, size_t max_ctx, size_t lanes, size_t layer,
                    size_t num_heads, size_t num_kv_heads, size_t head_dim, float* out, size_t ldo, float* workspace,
                    size_t workspace_floats, int seg_cap, cudaStream_t stream, SplitOut so, StepProfiler* prof,
                    int combine_kind) {
  GLC_REQUIRE(q && pool && block_tables && ctx_lens && (out || so.xs) && workspace, "paged_attention: null argument");
  GLC_REQUIRE(num_kv_heads > 0 && num_heads % num_kv_heads == 0, "paged_attention: heads %zu / kv heads %zu",
              num_heads, num_kv_heads);
  const size_t group = num_heads / num_kv_heads;
  GLC_REQUIRE(group <= kMaxGroup && (head_dim == 64 || head_dim == 128),
              "paged_attention: group %zu / head_dim %zu outside the kernel contract", group, head_dim);
  GLC_REQUIRE(max_ctx > 0 && max_ctx <= max_pages * 16, "paged_attention: context %zu exceeds the block table",
              max_ctx);
  if (seg_cap <= 1) seg_cap = attention_segments(lanes, num_heads, head_dim, max_ctx);
  GLC_REQUIRE(lanes <= (size_t)kMaxPlanLanes, "paged_attention: at most %d lanes per launch", kMaxPlanLanes);
  const int nsplit = seg_cap;
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
  const int grid = sm_count();
  const bool wide = lanes > 4;
  const int warps_per_cta = wide ? kAttnWarpsWide : kAttnWarpsFew;
  const int stages = wide ? kAttnStagesWide : kAttnStagesFew;
  prm.warps = grid * warps_per_cta;
  prm.nsplit = nsplit;
  prm.scale = 1.0f / sqrtf((float)head_dim);
  // Workspace: two work counters (4 floats reserved), then the chunk partials.
  prm.part_o = workspace + 4;
  prm.part_ml = prm.part_o + lanes * num_heads * nsplit * head_dim;
  const size_t kv_dim = num_kv_heads * head_dim;
  GLC_REQUIRE(page_floats % kv_dim == 0 && page_floats / kv_dim >= (layer + 1) * 32,
              "paged_attention: page of %zu floats does not hold layer %zu", page_floats, layer);
  const CUtensorMap* kvmap = nullptr;
  int rc = attn_kv_map(pool, kv_dim, head_dim, &kvmap);
  if (rc) return rc;
  if (lanes <= 4 && !so.xs) {
    // Few lanes: one cluster per (lane, kv head) merges its own partials (no combine launch).
    using CKern = void (*)(const CUtensorMap, const AttnParams, int, int*, float*, size_t);
    CKern ck = nullptr;
#define GLC_ATTN_CLUSTER_CASE(hd, ng) \
  if (head_dim == hd && group == ng) ck = attn_cluster_kernel<hd, ng>;
    GLC_ATTN_CLUSTER_CASE(128, 1) GLC_ATTN_CLUSTER_CASE(128, 2) GLC_ATTN_CLUSTER_CASE(128, 3)
    GLC_ATTN_CLUSTER_CASE(128, 4) GLC_ATTN_CLUSTER_CASE(128, 5) GLC_ATTN_CLUSTER_CASE(128, 6)
    GLC_ATTN_CLUSTER_CASE(128, 7) GLC_ATTN_CLUSTER_CASE(128, 8) GLC_ATTN_CLUSTER_CASE(64, 1)
    GLC_ATTN_CLUSTER_CASE(64, 2) GLC_ATTN_CLUSTER_CASE(64, 3) GLC_ATTN_CLUSTER_CASE(64, 4)
    GLC_ATTN_CLUSTER_CASE(64, 5) GLC_ATTN_CLUSTER_CASE(64, 6) GLC_ATTN_CLUSTER_CASE(64, 7)
    GLC_ATTN_CLUSTER_CASE(64, 8)
#undef GLC_ATTN_CLUSTER_CASE
    GLC_REQUIRE(ck != nullptr, "paged_attention: no kernel for head_dim %zu / group %zu", head_dim, group);
    GLC_REQUIRE(ldo % 4 == 0 && (uintptr_t)out % 16 == 0, "paged_attention: output rows must be 16-byte aligned");
    const size_t csmem = (size_t)kCWarps * kCStages * 2 * kStageRows * head_dim * sizeof(float);
    if ((rc = allow_dynamic_smem((const void*)ck, (int)csmem))) return rc;
    int* cerr = device_symbol_address(g_attn_error);
    GLC_REQUIRE(cerr != nullptr, "paged_attention: device status word unavailable");
    return launch_pdl(ck, dim3((unsigned)(lanes * num_kv_heads * kClusterCtas)), dim3(kCWarps * 32), csmem, stream,
                      kClusterCtas, *kvmap, prm, (int)(page_floats / kv_dim), cerr, out, ldo);
  }
  const size_t smem = (size_t)warps_per_cta * stages * 2 * kStageRows * head_dim * sizeof(float);
  using Kern = void (*)(const CUtensorMap, const AttnParams, int, int, int*);
  Kern kern = nullptr;
#define GLC_ATTN_CASE(hd, ng)                                                                    \
  if (head_dim == hd && group == ng)                                                             \
    kern = wide ? attn_tma_kernel<hd, ng, kAttnWarpsWide, kAttnStagesWide>                       \
                : attn_tma_kernel<hd, ng, kAttnWarpsFew, kAttnStagesFew>;
  GLC_ATTN_CASE(128, 1) GLC_ATTN_CASE(128, 2) GLC_ATTN_CASE(128, 3) GLC_ATTN_CASE(128, 4)
  GLC_ATTN_CASE(128, 5) GLC_ATTN_CASE(128, 6) GLC_ATTN_CASE(128, 7) GLC_ATTN_CASE(128, 8)
  GLC_ATTN_CASE(64, 1) GLC_ATTN_CASE(64, 2) GLC_ATTN_CASE(64, 3) GLC_ATTN_CASE(64, 4)
  GLC_ATTN_CASE(64, 5) GLC_ATTN_CASE(64, 6) GLC_ATTN_CASE(64, 7) GLC_ATTN_CASE(64, 8)
#undef GLC_ATTN_CASE
  GLC_REQUIRE(kern != nullptr, "paged_attention: no kernel for head_dim %zu / group %zu", head_dim, group);
  if ((rc = allow_dynamic_smem((const void*)kern, (int)smem))) return rc;
  int* err = device_symbol_address(g_attn_error);
  GLC_REQUIRE(err != nullptr, "paged_attention: device status word unavailable");
  // One CTA per SM; every warp streams the same number of K/V stages.
  if ((rc = launch_pdl(kern, dim3(grid), dim3(warps_per_cta * 32), smem, stream, 1, *kvmap, prm, (int)lanes,
                       (int)(page_floats / kv_dim), err)))
    return rc;
  if (prof) prof->mark(combine_kind, stream);
  {
    GLC_REQUIRE(head_dim % 8 == 0 && ldo % 4 == 0 && (num_heads * head_dim) / 8 <= 1024,
                "paged_attention: combine geometry %zu x %zu unsupported", num_heads, head_dim);
    const size_t csmem = num_heads * (size_t)nsplit * sizeof(float);
    GLC_REQUIRE(csmem <= 44 * 1024, "paged_attention: %d segments per lane exceed the combine's shared memory",
                nsplit);
    // The split output needs the lane's row max over all heads (one block per
    // lane); fp32 output with few lanes takes a block per (lane, head).
    if (!so.xs && lanes * num_heads < (size_t)sm_count()) {
      GLC_REQUIRE(head_dim <= 128 && head_dim % 4 == 0 && ldo % 4 == 0, "paged_attention: head_dim %zu", head_dim);
      const dim3 hgrid((unsigned)lanes, (unsigned)num_heads);
      if (nsplit > 64)
        return launch_pdl(attn_combine_head_kernel<32>, hgrid, dim3(1024), (size_t)nsplit * sizeof(float), stream, 1,
                          (const float*)prm.part_o, (const float*)prm.part_ml, nsplit, (int)head_dim,
                          (int)num_heads, out, ldo, ctx_lens, (int)lanes, (int)num_kv_heads, prm.warps,
                          (int)max_pages * 16);
      return launch_pdl(attn_combine_head_kernel<8>, hgrid, dim3(256), (size_t)nsplit * sizeof(float), stream, 1,
                        (const float*)prm.part_o, (const float*)prm.part_ml, nsplit, (int)head_dim, (int)num_heads,
                        out, ldo, ctx_lens, (int)lanes, (int)num_kv_heads, prm.warps, (int)max_pages * 16);
    }
    // Two head blocks per lane (a cluster of 2, whose row max is combined over
    // distributed shared memory) while that stays within one CTA per SM.
    const size_t nblk = 2 * lanes <= (size_t)sm_count() && num_heads >= 2 ? 2 : 1;
    const size_t hpb = ceil_div(num_heads, nblk);
    // One warp per head for the weights (up to 32 warps), enough threads for 8 values each.
    const size_t vals = ceil_div(hpb * head_dim / 8, (size_t)32) * 32;
    const unsigned threads = (unsigned)std::min<size_t>(1024, std::max(vals, hpb * (size_t)32));
    const dim3 cgrid((unsigned)ceil_div(num_heads, hpb), (unsigned)lanes);
    if ((rc = launch_pdl(attn_combine_kernel, cgrid, dim3(threads), hpb * (size_t)nsplit * sizeof(float), stream,
                         (int)cgrid.x,
                         (const float*)prm.part_o, (const float*)prm.part_ml, nsplit, (int)head_dim, (int)num_heads,
                         out, ldo, so, ctx_lens, (int)lanes, (int)num_kv_heads, prm.warps, (int)hpb,
                         (int)max_pages * 16)))
      return rc;
  }
  return GLACIER_CUDA_OK;
}

}  // namespace glacier
