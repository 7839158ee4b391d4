// Kernel (a), tensor-core form: TMA-fed INT4 dequant GEMV for group size 32
// (the BASELINE shapes); other groups use the FFMA2 kernel in int4_gemv.cu.
//
// y[b, m] = bias[m] + sum_g s[m, g] * sum_{k in g} (u[m, k] - 7) * x[b, k]
// over the reference's exact packing (src/core/quant.zig:164-177); same
// operator as linearInt4OnTheFly (src/backends/cpu/int4_matmul.zig:215-305).
//
// B200 design:
//  * A CTA owns 128 rows (8 consumer warps x one 16-row MMA tile) and a
//    K-slice.  A producer warp streams 128-row x 256-code tiles (16 KB, 2D TMA,
//    SWIZZLE_128B) plus the matching 128 x 8 scale tile into a 4-stage
//    shared-memory ring guarded by mbarriers, so memory traffic never waits on
//    arithmetic.  Only the B-fragment lanes of live batch rows are stored.
//  * Consumers unpack each 32-bit word of 8 codes into four half2 registers
//    holding the exact integers (u - 7) with 1 shift + 4 LOP3 + 4 HFMA2, which
//    are mma.sync A fragments as they are; the activation is split into fp16
//    hi + lo parts (x = hi + lo to ~22 bits) in the B fragment columns, so the
//    tensor core does the multiply-adds exactly up to fp32 accumulation.
//  * Each 32-code group accumulates in the MMA accumulator and is scaled by its
//    fp32 group scale once per group (one FFMA per row per group).
//  * A K-split across the CTAs of a thread-block cluster is reduced through
//    distributed shared memory in rank order (deterministic, no workspace).
//  * The LM head's instantiation ends with the eligible argmax of each row:
//    each warp reduces the 32 results it writes to one winner record, which a
//    one-CTA-per-row kernel reduces (logits are written only on request).
//  * Every mbarrier wait is bounded; on timeout the kernel raises a device
//    error word, drains its own TMA copies and leaves through the cluster
//    barriers so no CTA is left waiting.
#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace glacier {

__device__ int g_gemv_error;

namespace {

constexpr int kWarps = 8;                      // consumer warps, one 16-row MMA tile each
constexpr int kTilesPerWarp = 1;
constexpr int kThreads = (kWarps + 1) * 32;    // + producer warp
constexpr int kRows = 16 * kTilesPerWarp * kWarps;  // 128 rows per CTA tile
constexpr int kNibBytes = kRows * 128;         // 128 rows x 256 codes
constexpr int kStages = 4;
constexpr int kBlocksPerStage = 8;             // 32-code groups per stage
constexpr int kMaxStagesPerCta = 16;

struct GemvParams {
  const float* x;
  size_t ldx;
  const float* bias;
  float* y;
  size_t ldy;
  int M, K, batch;
  int stages_total;    // ceil(K / 256)
  int stages_per_cta;  // K-slice length in stages
  int* err;
  const float* xu;     // SwiGLU input: x = silu(x) * xu elementwise (same leading dimension), or null
};

struct NoEpi {};  // the plain instantiation's (empty) epilogue argument


__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Same with a zero accumulator input (first k-step of a group).
__device__ __forceinline__ void mma_16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Eight codes of one word -> four half2 of exact (u - 7):
//   q0 = {u0, u4}, q1 = {u1, u5}, q2 = {u2, u6}, q3 = {u3, u7}  (nibble i = bits 4i..4i+3)
__device__ __forceinline__ void unpack8(uint32_t w, uint32_t (&q)[4]) {
  const uint32_t kOne = 0x3C003C00u;        // {1, 1}
  const uint32_t kM1031 = 0xE407E407u;      // {-1031, -1031}
  const uint32_t kSixteenth = 0x2C002C00u;  // {1/16, 1/16}
  const uint32_t kM71 = 0xD470D470u;        // {-71, -71}
  const uint32_t w8 = w >> 8;
  // 0x6400 = 1024.0: low nibble of each half -> 1024 + u, bits 4..7 -> 1024 + 16u.
  const uint32_t t0 = lop3_and_or(w, 0x000F000Fu, 0x64006400u);
  const uint32_t t1 = lop3_and_or(w, 0x00F000F0u, 0x64006400u);
  const uint32_t t2 = lop3_and_or(w8, 0x000F000Fu, 0x64006400u);
  const uint32_t t3 = lop3_and_or(w8, 0x00F000F0u, 0x64006400u);
  q[0] = hfma2_u32(t0, kOne, kM1031);      // (1024 + u) - 1031
  q[1] = hfma2_u32(t1, kSixteenth, kM71);  // (1024 + 16u)/16 - 71
  q[2] = hfma2_u32(t2, kOne, kM1031);
  q[3] = hfma2_u32(t3, kSixteenth, kM71);
}

__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// Eight consecutive group scales of one row (one stage), converted on use.
template <typename ScaleT>
struct RowScales;
template <>
struct RowScales<__half> {
  uint4 v;
  __device__ void load(const uint8_t* p) { v = *reinterpret_cast<const uint4*>(p); }
  __device__ float get(int g) const {
    const uint32_t w = g < 2 ? v.x : g < 4 ? v.y : g < 6 ? v.z : v.w;
    return half_to_float_bits((g & 1) ? (w >> 16) : (w & 0xFFFFu));
  }
};
// fp16 scales of a weight that holds a non-finite one: the conversion
// instruction keeps infinities and NaNs (rare; the fast form assumes finite).
struct HalfExact {
  uint16_t bits;
};
template <>
struct RowScales<HalfExact> {
  uint4 v;
  __device__ void load(const uint8_t* p) { v = *reinterpret_cast<const uint4*>(p); }
  __device__ float get(int g) const {
    const uint32_t w = g < 2 ? v.x : g < 4 ? v.y : g < 6 ? v.z : v.w;
    return __half2float(__ushort_as_half((unsigned short)((g & 1) ? (w >> 16) : (w & 0xFFFFu))));
  }
};
template <>
struct RowScales<float> {
  float4 a, b;
  __device__ void load(const uint8_t* p) {
    a = reinterpret_cast<const float4*>(p)[0];
    b = reinterpret_cast<const float4*>(p)[1];
  }
  __device__ float get(int g) const {
    const float4& q = g < 4 ? a : b;
    const int j = g & 3;
    return j == 0 ? q.x : j == 1 ? q.y : j == 2 ? q.z : q.w;
  }
};

// Epi: NoEpi (y = W x + bias) or ArgmaxEpi (the LM head: y optional, then the
// eligible argmax of each row).
template <typename ScaleT, typename Epi>
__global__ void __launch_bounds__(kThreads, 2) gemv_tc_kernel(const __grid_constant__ CUtensorMap tmap_w,
                                                              const __grid_constant__ CUtensorMap tmap_s,
                                                              const GemvParams p, const Epi epi) {
  constexpr bool kArgmax = std::is_same<Epi, ArgmaxEpi>::value;
  // Weights do not depend on the previous kernel: the producer streams them at
  // once; the consumers wait for its writes (griddep_wait) before reading x, and
  // every thread waits before the stores of y.
  griddep_launch();
  constexpr int kScaleBytes = kRows * 8 * (int)sizeof(ScaleT);  // 8 groups per row per stage
  constexpr int kStageBytes = kNibBytes + kScaleBytes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled TMA destination.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint4* xfrag = reinterpret_cast<uint4*>(smem + kStages * kStageBytes);
  const int max_blocks = p.stages_per_cta * kBlocksPerStage;
  const int flanes = 8 * p.batch;  // lanes whose B columns (n = lane / 4 < 2 * batch) are live
  float* red = reinterpret_cast<float*>(xfrag + (size_t)max_blocks * flanes);  // [4][kRows]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 4 * kRows);
  uint64_t* empty = full + kStages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  uint32_t nrank;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(nrank));
  const int tile = blockIdx.x / nrank;
  const int row0 = tile * kRows;
  const int st0 = (int)crank * p.stages_per_cta;
  const int st1 = min(p.stages_total, st0 + p.stages_per_cta);
  const int nst = max(0, st1 - st0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kWarps) {
    // ---------------- producer: nibble tile + scale tile per stage ----------------
    if (lane == 0) {
      prefetch_tmap(&tmap_w);
      prefetch_tmap(&tmap_s);
      const uint64_t pol = l2_evict_first_policy();
      int issued = 0;
      for (int i = 0; i < nst; ++i) {
        const int slot = i % kStages, round = i / kStages;
        if (!mbar_wait(&empty[slot], (round & 1) ^ 1, p.err)) break;
        uint8_t* dst = ring + slot * kStageBytes;
        mbar_arrive_expect_tx(&full[slot], kStageBytes);
        tma_load_2d(dst, &tmap_w, (st0 + i) * 128, row0, &full[slot], pol);
        tma_load_2d(dst + kNibBytes, &tmap_s, (st0 + i) * 8, row0, &full[slot], pol);
        ++issued;
      }
      // Drain: never leave with copies into this CTA's shared memory in flight.
      for (int i = max(0, issued - kStages); i < issued; ++i)
        mbar_wait(&full[i % kStages], (i / kStages) & 1, p.err);
    }
  } else {
    // ---------------- consumers ----------------
    griddep_wait();
    // 1) B fragments (activation hi/lo columns) for this CTA's K-slice.
    const int nblk = nst * kBlocksPerStage;
    for (int idx = threadIdx.x; idx < nblk * flanes; idx += kWarps * 32) {
      const int blk = idx / flanes, l = idx % flanes;
      const int n = l >> 2, c = l & 3;
      const int b = n >> 1;
      const int k0 = (st0 * kBlocksPerStage + blk) * 32 + 8 * c;
      float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (k0 < p.K) {
        const float4* xp = reinterpret_cast<const float4*>(p.x + b * p.ldx + k0);
        const float4 a = __ldg(xp), bq = __ldg(xp + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = bq.x; v[5] = bq.y; v[6] = bq.z; v[7] = bq.w;
        if (p.xu) {
          // SwiGLU (kernels.zig:465): silu(gate) * up, the same expression as silu_mul_kernel.
          const float4* up = reinterpret_cast<const float4*>(p.xu + b * p.ldx + k0);
          const float4 ua = __ldg(up), ub = __ldg(up + 1);
          const float u[8] = {ua.x, ua.y, ua.z, ua.w, ub.x, ub.y, ub.z, ub.w};
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = v[j] * (1.0f / (1.0f + expf(-v[j]))) * u[j];
        }
      }
      __half h[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const __half hi = __float2half_rn(v[j]);
        h[j] = (n & 1) ? __float2half_rn(v[j] - __half2float(hi)) : hi;
      }
      // k-step 0: {k 8c, 8c+4}, {8c+1, 8c+5}; k-step 1: {8c+2, 8c+6}, {8c+3, 8c+7}
      xfrag[idx] = make_uint4(pack_half2(h[0], h[4]), pack_half2(h[1], h[5]), pack_half2(h[2], h[6]),
                              pack_half2(h[3], h[7]));
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kWarps * 32) : "memory");

    const int r = lane >> 2, c = lane & 3;
    const bool bcol = lane < flanes;  // lanes whose B columns belong to a live batch row
    // Rows of tile t: rho_t = 64*warp + 16*t + r and rho_t + 8 (all share rho & 7 == r & 7).
    const uint32_t swz = (uint32_t)(r & 7);
    float acc[kTilesPerWarp][2];
#pragma unroll
    for (int t = 0; t < kTilesPerWarp; ++t) acc[t][0] = acc[t][1] = 0.f;
    for (int i = 0; i < nst; ++i) {
      const int slot = i % kStages, round = i / kStages;
      if (!mbar_wait(&full[slot], round & 1, p.err)) break;
      const uint8_t* stg = ring + slot * kStageBytes;
      const uint8_t* sstg = stg + kNibBytes;
      RowScales<ScaleT> sc[kTilesPerWarp][2];
#pragma unroll
      for (int t = 0; t < kTilesPerWarp; ++t) {
        const int rho = 16 * kTilesPerWarp * warp + 16 * t + r;
        sc[t][0].load(sstg + rho * 8 * sizeof(ScaleT));
        sc[t][1].load(sstg + (rho + 8) * 8 * sizeof(ScaleT));
      }
      const uint8_t* rowbase = stg + (16 * kTilesPerWarp * warp + r) * 128 + 4 * c;
#pragma unroll
      for (int bl = 0; bl < kBlocksPerStage; ++bl) {
        const uint32_t off = ((uint32_t)bl ^ swz) << 4;
        uint4 bf = make_uint4(0, 0, 0, 0);
        if (bcol) bf = xfrag[(i * kBlocksPerStage + bl) * flanes + lane];
#pragma unroll
        for (int t = 0; t < kTilesPerWarp; ++t) {
          const uint32_t w0 = *reinterpret_cast<const uint32_t*>(rowbase + t * 16 * 128 + off);
          const uint32_t w1 = *reinterpret_cast<const uint32_t*>(rowbase + (t * 16 + 8) * 128 + off);
          uint32_t q0[4], q1[4];
          unpack8(w0, q0);
          unpack8(w1, q1);
          float ca[4];
          mma_16816_z(ca, q0[0], q1[0], q0[1], q1[1], bf.x, bf.y);
          mma_16816(ca, q0[2], q1[2], q0[3], q1[3], bf.z, bf.w);
          acc[t][0] = fmaf(sc[t][0].get(bl), ca[0] + ca[1], acc[t][0]);
          acc[t][1] = fmaf(sc[t][1].get(bl), ca[2] + ca[3], acc[t][1]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
#pragma unroll
    for (int t = 0; t < kTilesPerWarp; ++t) {
      const int rho = 16 * kTilesPerWarp * warp + 16 * t + r;
      red[c * kRows + rho] = acc[t][0];  // lane c's batch column
      red[c * kRows + rho + 8] = acc[t][1];
    }
  }

  // Cross-CTA K reduction through distributed shared memory, in rank order.
  griddep_wait();
  cluster_sync_all();
  if (crank == 0) {
    for (int idx = threadIdx.x; idx < p.batch * kRows; idx += kThreads) {
      const int b = idx / kRows, rr = idx % kRows;
      const int row = row0 + rr;
      float v = 0.f;
      if (row < p.M) {
        const uint32_t local = smem_u32(&red[b * kRows + rr]);
        for (uint32_t q = 0; q < nrank; ++q) v += ld_dsmem_f32(mapa_shared(local, q));
        v += p.bias ? p.bias[row] : 0.f;
        if (!kArgmax || p.y) p.y[b * p.ldy + row] = v;
      }
      if constexpr (kArgmax) {
        // The warp's 32 consecutive rows (one batch row b: kRows is a multiple of
        // 32) reduce to one winner record; argmax_tiles_kernel reduces the records.
        bool ok = row < p.M;
        if (ok && epi.words) ok = (epi.words[(size_t)b * epi.word_count + (row >> 6)] >> (row & 63)) & 1ull;
        int nan = ok && v != v, elig = ok;
        float bv = v;
        int bi = ok && !nan ? row : -1;
        arg_warp_reduce(bv, bi, nan, elig);
        if (lane == 0)
          epi.partials[(size_t)b * (gridDim.x / nrank) * (kRows / 32) + (size_t)tile * (kRows / 32) + rr / 32] =
              make_int4(__float_as_int(bv), bi, nan, elig);
      }
    }
  }
  cluster_sync_all();
}

// The LM head's argmax, second part: row b's winner records (one per 32 rows)
// reduced by one CTA.
// The order (value, then lowest index) is total, so this gives the result of
// argmax_rows whatever the tiling; the statuses follow argmax_final_kernel.
__global__ void __launch_bounds__(1024) argmax_tiles_kernel(const ArgmaxEpi a, int tiles, int n) {
  griddep_launch();
  griddep_wait();
  __shared__ float sv[32];
  __shared__ int si[32], sn[32], se[32];
  const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float bv = 0.f;
  int bi = -1, nan = 0, elig = 0;
  const int4* rec = a.partials + (size_t)b * tiles;
  // Four independent loads in flight per thread before any is compared.
  for (int t0 = threadIdx.x; t0 < tiles; t0 += 4 * blockDim.x) {
    int4 r[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = t0 + u * blockDim.x;
      r[u] = t < tiles ? rec[t] : make_int4(0, -1, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (arg_better(__int_as_float(r[u].x), r[u].y, bv, bi)) {
        bv = __int_as_float(r[u].x);
        bi = r[u].y;
      }
      nan |= r[u].z;
      elig += r[u].w;
    }
  }
  arg_warp_reduce(bv, bi, nan, elig);
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
    sn[warp] = nan;
    se[warp] = elig;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
    if (arg_better(sv[w], si[w], bv, bi)) {
      bv = sv[w];
      bi = si[w];
    }
    nan |= sn[w];
    elig += se[w];
  }
  int tail = 0;
  if (a.words && (n & 63)) {
    const uint64_t valid = (1ull << (n & 63)) - 1;
    tail = (a.words[(size_t)b * a.word_count + a.word_count - 1] & ~valid) != 0;
  }
  int st = GLACIER_CUDA_OK;
  if (a.words && (tail || elig == 0)) st = GLACIER_CUDA_EMASK;
  else if (nan) st = GLACIER_CUDA_ENAN;
  else if (bi < 0) st = GLACIER_CUDA_EMASK;
  if (a.tokens) a.tokens[b] = st == GLACIER_CUDA_OK ? bi : -1;
  if (a.status) a.status[b] = st;
  if (a.results) {
    glacier_argmax_result& r = a.results[b];
    r.value = bi >= 0 ? bv : -INFINITY;
    r.index = bi >= 0 ? (size_t)bi : 0;
    r.valid = st == GLACIER_CUDA_OK;
    r.saw_nan = nan;
  }
}

template <typename ScaleT, typename Epi>
int launch_gemv_tc(const Int4Weight& w, const float* x, const float* xu, size_t ldx, size_t batch, const float* bias,
                   float* y, size_t ldy, cudaStream_t stream, const Epi& epi) {
  const size_t M = w.M, K = w.K;
  int rc = 0;
  const int tiles = (int)ceil_div(M, kRows);
  const int stages = (int)ceil_div(K, 256);
  // Cluster size (the K split): as many CTAs per row tile as keep the grid within
  // one wave of two CTAs per SM (at most 8 per cluster: 10-CTA non-portable
  // clusters measured slower), then as few as give every CTA the same number of
  // stages; K-slices short enough that the B fragments leave room for two CTAs
  // per SM.
  auto frag_bytes = [&](int c) { return (size_t)ceil_div(stages, c) * kBlocksPerStage * 8 * batch * 16; };
  int cs = std::max(1, std::min({8, stages, 2 * sm_count() / tiles}));
  while (cs < std::min(8, stages) &&
         ((int)ceil_div(stages, cs) > kMaxStagesPerCta || frag_bytes(cs) > 24 * 1024))
    ++cs;
  const int spc = (int)ceil_div(stages, cs);
  cs = (int)ceil_div(stages, spc);
  const size_t stage_bytes = kNibBytes + (size_t)kRows * 8 * sizeof(ScaleT);
  const size_t smem = 1024 + (size_t)kStages * stage_bytes + (size_t)spc * kBlocksPerStage * 8 * batch * 16 +
                      4 * kRows * sizeof(float) + 2 * kStages * sizeof(uint64_t);
  GLC_REQUIRE(smem <= 200 * 1024, "int4 gemv: K slice too long for shared memory (K=%zu)", K);
  auto kern = gemv_tc_kernel<ScaleT, Epi>;
  rc = allow_dynamic_smem((const void*)kern, (int)smem);
  if (rc) return rc;
  int* err = device_symbol_address(g_gemv_error);
  GLC_REQUIRE(err != nullptr, "int4 gemv: device status word unavailable");
  GemvParams prm{x, ldx, bias, y, ldy, (int)M, (int)K, (int)batch, stages, spc, err, xu};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * cs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see launch_pdl
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  GLC_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, w.tmap_w, w.tmap_s, prm, epi));
  note_launch();
  return GLACIER_CUDA_OK;
}

}  // namespace

// The tensor-core GEMV handles group 32, whole 32-code chunks, 16-byte aligned
// operands and scale rows whose byte stride is a multiple of 16 (TMA).
int int4_weight_prepare(Int4Weight& w) {
  GLC_REQUIRE(w.packed && w.scales && w.M > 0 && w.K > 0 && w.group > 0, "int4 weight: empty or null");
  GLC_REQUIRE(w.M < (1u << 31) && w.K < (1u << 31), "int4 weight: dimension too large");
  const size_t esz = w.f16 ? 2 : 4;
  const size_t stride = w.scale_stride ? w.scale_stride : (w.K % w.group == 0 ? w.K / w.group : 0);
  // Maps for 128-row x 256-code tiles and their 256/group scales: the GEMV takes
  // group 32, the tcgen05 GEMM groups 8, 16 and 32 (one scale row of 16, 32 or 64
  // bytes per tile row and super-stage).
  w.tcg = (w.group == 8 || w.group == 16 || w.group == 32) && w.K % 32 == 0 && stride != 0 &&
          (stride * esz) % 16 == 0 && (uintptr_t)w.packed % 16 == 0 && (uintptr_t)w.scales % 16 == 0;
  w.tc = w.tcg && w.group == 32;
  if (!w.tcg) return GLACIER_CUDA_OK;
  w.scale_stride = stride;
  int rc = encode_tmap_2d(&w.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.packed, w.K / 2, w.M, w.K / 2, 128, kRows,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  rc = encode_tmap_2d(&w.tmap_s, w.f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.scales,
                      w.K / w.group, w.M, stride * esz, (uint32_t)(256 / w.group), kRows, CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_NONE);
  return rc;
}

int gemv_int4_tc(const Int4Weight& w, const float* x, size_t ldx, size_t batch, const float* bias, float* y,
                 size_t ldy, cudaStream_t stream, const float* xu) {
  if (!w.f16) return launch_gemv_tc<float>(w, x, xu, ldx, batch, bias, y, ldy, stream, NoEpi());
  return w.nonfinite ? launch_gemv_tc<HalfExact>(w, x, xu, ldx, batch, bias, y, ldy, stream, NoEpi())
                     : launch_gemv_tc<__half>(w, x, xu, ldx, batch, bias, y, ldy, stream, NoEpi());
}

size_t argmax_records_bytes(size_t rows, size_t M) {
  return rows * ceil_div(M, (size_t)kRows) * (kRows / 32) * sizeof(int4);  // one record per 32 rows of a 128-row tile
}

int argmax_records_reduce(const ArgmaxEpi& a, size_t rows, size_t records, size_t n, cudaStream_t stream) {
  return launch_pdl(argmax_tiles_kernel, dim3((unsigned)rows), dim3(1024), 0, stream, 1, a, (int)records, (int)n);
}

int int4_linear_argmax(const Int4Weight& w, const float* x, size_t ldx, size_t batch, float* y, size_t ldy,
                       const ArgmaxEpi& a, cudaStream_t stream) {
  GLC_REQUIRE(x && batch > 0 && a.partials, "int4 linear argmax: null argument");
  const bool aligned = (uintptr_t)x % 16 == 0 && ldx % 4 == 0;
  if (!w.tc || !aligned || batch > 4) return GLACIER_CUDA_EUNSUPPORTED;
  GLC_REQUIRE(!a.words || (size_t)a.word_count == ceil_div(w.M, (size_t)64),
              "int4 linear argmax: eligible mask needs %zu words per row", ceil_div(w.M, (size_t)64));
  const int rc = !w.f16 ? launch_gemv_tc<float>(w, x, nullptr, ldx, batch, nullptr, y, ldy, stream, a)
                 : w.nonfinite ? launch_gemv_tc<HalfExact>(w, x, nullptr, ldx, batch, nullptr, y, ldy, stream, a)
                               : launch_gemv_tc<__half>(w, x, nullptr, ldx, batch, nullptr, y, ldy, stream, a);
  if (rc) return rc;
  return argmax_records_reduce(a, batch, ceil_div(w.M, (size_t)kRows) * (kRows / 32), w.M, stream);
}

int gemv_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemv_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_gemv_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace glacier
