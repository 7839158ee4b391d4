// INT4 GEMV with Q8 activations: the reference's default decode numerics,
// linearInt4Q8OnTheFly (src/backends/cpu/int4_matmul.zig:335-418) as dispatched
// by linearInt4WeightQ8 (:422-532) on a non-AArch64 host.
//
//   per batch row and activation block of 32 (g8) or g codes:
//     scale = max|x| / 127,  q = clamp(round(x * (1/scale)), -127, 127)
//   per output row: acc = bias; for each weight group in order
//     acc += (float)(sum (u - 7) * q) * w_scale * a_scale
//
// The integer dot products are exact, so the result is bit-identical to the
// reference's portable path when the float steps keep its order: every term is
// formed as ((float)dot * w_scale) * a_scale and added to acc group by group,
// with no fused multiply-add (__fmul_rn / __fadd_rn) and no K split.
//
// B200 form (group 32): a CTA owns 16*W weight rows and the whole K.  A TMA
// producer streams 256-code nibble tiles (SWIZZLE_128B) plus scale tiles into a
// 4-stage mbarrier ring; the consumer warps first quantize x into int8
// mma.sync B fragments in shared memory (one warp per 32-code block), then turn
// each 8-code word into two int8 A registers with 3 instructions (mask, shift,
// mask: the codes u as unsigned bytes, even codes in one register, odd in the
// other) and run one m16n8k32 integer MMA per 32-code group; -7 * sum q
// restores the zero point exactly.  Other groups and layouts take a warp-per-row
// CUDA-core kernel with the same arithmetic.
#include "common.cuh"

namespace glacier {

__device__ int g_gemv_q8_error;

namespace {

constexpr int kQ8MaxK = 16384;  // the reference quantizes inputs up to this length (int4_matmul.zig:369)

struct Q8Params {
  const float* x;
  size_t ldx;
  const float* bias;
  float* y;
  size_t ldy;
  int M, K, batch;
  int stages;  // ceil(K / 256)
  int* err;
};

__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// Q8 code of one activation (int4_matmul.zig:388-392): round half away from zero, clamp.
__device__ __forceinline__ int q8_code(float v, float inv) {
  int q = (int)roundf(__fmul_rn(v, inv));
  return max(-127, min(127, q));
}

// The eight group scales of one row in one stage, loaded once and read by
// compile-time index.
template <typename ScaleT>
struct StageScales;
template <>
struct StageScales<__half> {
  uint4 v;
  __device__ void load(const uint8_t* p) { v = *reinterpret_cast<const uint4*>(p); }
  __device__ float get(int g) const {
    const uint32_t w = g < 2 ? v.x : g < 4 ? v.y : g < 6 ? v.z : v.w;
    return half_to_float_bits((g & 1) ? (w >> 16) : (w & 0xFFFFu));
  }
};
template <>
struct StageScales<float> {
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

// Ring depth: 4 stages for 128-row tiles, more for shorter tiles so that about
// the same bytes stay in flight per SM.
template <int T>
constexpr int q8_stages() { return T >= 8 ? 4 : T >= 4 ? 8 : 12; }

// T row tiles of 16 per CTA and KP K-parts: W = T * KP consumer warps; warp w
// takes tile w % T and the stages i with i % KP == w / T.  With KP > 1 every
// group's term goes to shared memory and one pass per (row, batch row) adds the
// bias and the terms in group order, so the float sum keeps the reference's order.
template <typename ScaleT, int T, int KP>
__global__ void __launch_bounds__((T * KP + 1) * 32) gemv_q8_kernel(const __grid_constant__ CUtensorMap tmap_w,
                                                                    const __grid_constant__ CUtensorMap tmap_s,
                                                                    const Q8Params p) {
  constexpr int W = T * KP;
  constexpr int kRows = 16 * T;
  constexpr int kNib = kRows * 128;  // rows x 256 codes
  constexpr int kScl = kRows * 8 * (int)sizeof(ScaleT);
  // Stages start on 1024-byte boundaries: the 128-byte swizzle pattern of the
  // nibble tiles follows the shared-memory address bits.
  constexpr int kStage = (kNib + kScl + 1023) & ~1023;
  constexpr int kQ8Stages = q8_stages<T>();
  // Weights do not depend on the previous kernel: the producer streams them at
  // once, the consumers wait (griddep_wait) before reading x or writing y.
  griddep_launch();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nblk = p.K / 32;
  uint8_t* ring = smem;
  uint2* xq = reinterpret_cast<uint2*>(ring + kQ8Stages * kStage);  // [nblk][4 batch cols][4 k-quads]
  int2* stat = reinterpret_cast<int2*>(xq + (size_t)nblk * 16);     // [nblk][4]: {a_scale bits, sum q}
  // KP > 1: per-group terms [batch][kRows][tstride], an odd row stride so that the
  // final per-row passes read distinct banks.
  const int tstride = nblk | 1;
  float* terms = reinterpret_cast<float*>(stat + (size_t)nblk * 4);
  uint64_t* full =
      reinterpret_cast<uint64_t*>(terms + (KP > 1 ? (((size_t)p.batch * kRows * tstride + 1) & ~(size_t)1) : 0));
  uint64_t* empty = full + kQ8Stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kRows;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kQ8Stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], T);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == W) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tmap_w);
      prefetch_tmap(&tmap_s);
      const uint64_t pol = l2_evict_first_policy();
      int issued = 0;
      for (int i = 0; i < p.stages; ++i) {
        const int slot = i % kQ8Stages, round = i / kQ8Stages;
        if (!mbar_wait(&empty[slot], (round & 1) ^ 1, p.err)) break;
        uint8_t* dst = ring + slot * kStage;
        mbar_arrive_expect_tx(&full[slot], kNib + kScl);  // bytes copied (kStage includes padding)
        tma_load_2d(dst, &tmap_w, i * 128, row0, &full[slot], pol);
        tma_load_2d(dst + kNib, &tmap_s, i * 8, row0, &full[slot], pol);
        ++issued;
      }
      for (int i = max(0, issued - kQ8Stages); i < issued; ++i)
        mbar_wait(&full[i % kQ8Stages], (i / kQ8Stages) & 1, p.err);
    }
    return;
  }

  // ---------------- consumers ----------------
  griddep_wait();
  // 1) Q8 activations (int4_matmul.zig:379-394): per warp iteration four 32-code
  //    blocks of one batch row, eight lanes per block and four codes per lane.
  //    Code e of block g lands in the B fragment of k-quad c = e / 8: even codes in
  //    the first register, odd codes in the second (the order the A unpack gives).
  {
    const int sub = lane >> 3, e0 = (lane & 7) * 4;
    const int nquad = (nblk + 3) / 4;
    for (int it = warp; it < nquad * p.batch; it += W) {
      const int qd = it / p.batch, b = it - qd * p.batch;
      const int g = qd * 4 + sub;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (g < nblk) v = *reinterpret_cast<const float4*>(p.x + (size_t)b * p.ldx + (size_t)g * 32 + e0);
      float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float scale = m / 127.0f;
      int q[4] = {0, 0, 0, 0};
      if (scale != 0.f) {
        const float inv = 1.0f / scale;
        q[0] = q8_code(v.x, inv);
        q[1] = q8_code(v.y, inv);
        q[2] = q8_code(v.z, inv);
        q[3] = q8_code(v.w, inv);
      }
      int sum = (q[0] + q[1]) + (q[2] + q[3]);
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (g < nblk) {
        uint8_t* base = reinterpret_cast<uint8_t*>(&xq[((size_t)g * 4 + b) * 4]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int e = e0 + i, c = e >> 3, j = e & 7;
          base[c * 8 + ((j & 1) ? 4 : 0) + (j >> 1)] = (uint8_t)(int8_t)q[i];
        }
        if ((lane & 7) == 0) stat[g * 4 + b] = make_int2(__float_as_int(scale), sum);
      }
    }
  }
  asm volatile("bar.sync 1, %0;" ::"n"(W * 32) : "memory");

  // 2) Integer MMAs, one per 32-code group, and the group-ordered float combine.
  const int r = lane >> 2, c = lane & 3;
  const int n = lane >> 2;  // this lane's B column (batch row) in the fragment load
  const bool bload = n < p.batch;
  const uint32_t swz = (uint32_t)(r & 7);
  const int tile = warp % T, part = warp / T;
  const int rho = 16 * tile + r;  // rows rho and rho + 8 of the tile
  float acc[2][2];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int row = row0 + rho + 8 * rr;
    const float bias = (p.bias && row < p.M) ? p.bias[row] : 0.f;
    acc[rr][0] = acc[rr][1] = bias;
  }
  const int bc0 = 2 * c, bc1 = 2 * c + 1;  // accumulator columns of this lane
  for (int i = part; i < p.stages; i += KP) {
    const int slot = i % kQ8Stages, round = i / kQ8Stages;
    if (!mbar_wait(&full[slot], round & 1, p.err)) break;
    const uint8_t* stg = ring + slot * kStage;
    StageScales<ScaleT> sc0, sc1;
    sc0.load(stg + kNib + (size_t)rho * 8 * sizeof(ScaleT));
    sc1.load(stg + kNib + (size_t)(rho + 8) * 8 * sizeof(ScaleT));
    const uint8_t* rowbase = stg + rho * 128 + 4 * c;
#pragma unroll
    for (int bl = 0; bl < 8; ++bl) {
      const int g = i * 8 + bl;
      if (g < nblk) {
        const uint32_t off = ((uint32_t)bl ^ swz) << 4;
        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(rowbase + off);
        const uint32_t w1 = *reinterpret_cast<const uint32_t*>(rowbase + 8 * 128 + off);
        const uint2 bf = bload ? xq[((size_t)g * 4 + n) * 4 + c] : make_uint2(0, 0);
        int d[4];
        mma_s8_16832(d, w0 & 0x0F0F0F0Fu, w1 & 0x0F0F0F0Fu, (w0 >> 4) & 0x0F0F0F0Fu, (w1 >> 4) & 0x0F0F0F0Fu, bf.x,
                     bf.y);
        const float ws0 = sc0.get(bl), ws1 = sc1.get(bl);
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int bcol = jj ? bc1 : bc0;
          if (bcol < p.batch) {
            const int2 st = stat[g * 4 + bcol];
            const int corr = 7 * st.y;
            const float as = __int_as_float(st.x);
            const float t0 = __fmul_rn(__fmul_rn((float)(d[jj] - corr), ws0), as);
            const float t1 = __fmul_rn(__fmul_rn((float)(d[2 + jj] - corr), ws1), as);
            if constexpr (KP == 1) {
              acc[0][jj] = __fadd_rn(acc[0][jj], t0);
              acc[1][jj] = __fadd_rn(acc[1][jj], t1);
            } else {
              terms[((size_t)bcol * kRows + rho) * tstride + g] = t0;
              terms[((size_t)bcol * kRows + rho + 8) * tstride + g] = t1;
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  if constexpr (KP == 1) {
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int row = row0 + rho + 8 * rr;
      if (row >= p.M) continue;
      if (bc0 < p.batch) p.y[(size_t)bc0 * p.ldy + row] = acc[rr][0];
      if (bc1 < p.batch) p.y[(size_t)bc1 * p.ldy + row] = acc[rr][1];
    }
  } else {
    asm volatile("bar.sync 1, %0;" ::"n"(W * 32) : "memory");
    for (int idx = threadIdx.x; idx < kRows * p.batch; idx += W * 32) {
      const int rr = idx % kRows, b = idx / kRows, row = row0 + rr;
      if (row >= p.M) continue;
      const float* tr = terms + ((size_t)b * kRows + rr) * tstride;
      float a = p.bias ? p.bias[row] : 0.f;
      for (int g = 0; g < nblk; ++g) a = __fadd_rn(a, tr[g]);
      p.y[(size_t)b * p.ldy + row] = a;
    }
  }
}

// Any group size (flat-index scales): one warp per (output row, batch row).  For
// each weight group in order the warp rebuilds the Q8 codes of its activation
// block (the scale from the block's max), forms the exact integer dot with a warp
// reduction and lane 0 adds the term.
template <typename ScaleT>
__global__ void gemv_q8_generic_kernel(const float* __restrict__ x, size_t ldx, const uint8_t* __restrict__ packed,
                                       const ScaleT* __restrict__ scales, const float* __restrict__ bias,
                                       float* __restrict__ y, size_t ldy, int M, int K, int group, int batch) {
  griddep_launch();
  griddep_wait();
  const int gw = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (gw >= M * batch) return;
  const int row = gw % M, b = gw / M;
  const int ag = group == 8 ? 32 : group;
  const float* xr = x + (size_t)b * ldx;
  float acc = bias ? bias[row] : 0.f;
  const size_t row_start = (size_t)row * K;
  for (int og = 0; og < K / group; ++og) {
    const int start = og * group, blk0 = (start / ag) * ag;
    float m = 0.f;
    for (int k = blk0 + lane; k < min(K, blk0 + ag); k += 32) m = fmaxf(m, fabsf(xr[k]));
    m = warp_max(m);
    const float scale = m / 127.0f;
    const float inv = scale == 0.f ? 0.f : 1.0f / scale;
    int dot = 0;
    for (int k = start + lane; k < start + group; k += 32) {
      const size_t idx = row_start + k;
      const uint8_t byte = packed[idx / 2];
      const int nib = (idx & 1) == 0 ? (byte & 0x0F) : (byte >> 4);
      const int q = scale == 0.f ? 0 : q8_code(xr[k], inv);
      dot += (nib - 7) * q;
    }
    dot = __reduce_add_sync(0xffffffffu, dot);
    const float ws = (float)scales[(row_start + start) / group];
    acc = __fadd_rn(acc, __fmul_rn(__fmul_rn((float)dot, ws), scale));
  }
  if (lane == 0) y[(size_t)b * ldy + row] = acc;
}

template <typename ScaleT, int T, int KP>
int launch_q8(const uint8_t* packed, const ScaleT* scales, const float* x, size_t ldx, size_t batch, const float* bias,
              float* y, size_t ldy, size_t M, size_t K, cudaStream_t stream) {
  constexpr int kRows = 16 * T, W = T * KP;
  CUtensorMap tw, ts;
  int rc = encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, packed, K / 2, M, K / 2, 128, kRows,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  rc = encode_tmap_2d(&ts, sizeof(ScaleT) == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                      scales, K / 32, M, (K / 32) * sizeof(ScaleT), 8, kRows, CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_NONE);
  if (rc) return rc;
  const size_t nblk = K / 32;
  const size_t stage = ((size_t)kRows * 128 + (size_t)kRows * 8 * sizeof(ScaleT) + 1023) & ~(size_t)1023;
  constexpr int kQ8Stages = q8_stages<T>();
  const size_t smem = 1024 + kQ8Stages * stage + nblk * 16 * sizeof(uint2) + nblk * 4 * sizeof(int2) +
                      (KP > 1 ? (batch * kRows * (nblk | 1) + 1) * sizeof(float) : 0) + 8 +
                      2 * kQ8Stages * sizeof(uint64_t);
  GLC_REQUIRE(smem <= 227 * 1024, "int4 q8 gemv: %zu bytes of shared memory", smem);
  auto kern = gemv_q8_kernel<ScaleT, T, KP>;
  if ((rc = allow_dynamic_smem((const void*)kern, (int)smem))) return rc;
  int* err = device_symbol_address(g_gemv_q8_error);
  GLC_REQUIRE(err != nullptr, "int4 q8 gemv: device status word unavailable");
  Q8Params prm{x, ldx, bias, y, ldy, (int)M, (int)K, (int)batch, (int)ceil_div(K, 256), err};
  return launch_pdl(kern, dim3((unsigned)ceil_div(M, kRows)), dim3((W + 1) * 32), smem, stream, 1, tw, ts, prm);
}

}  // namespace

int q8_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemv_q8_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_gemv_q8_error, &z, sizeof(int));
  }
  return v;
}

// linearInt4WeightQ8 on a non-AArch64 host (int4_matmul.zig:422-532): outputs
// longer than 65536 (the vocabulary head, :460) and inputs longer than 16384 or
// with more than 2048 activation blocks (:369) take the FP32-activation GEMV;
// everything else the Q8 path above.
int int4_linear_q8(const Int4Weight& w, const float* x, size_t ldx, size_t batch, const float* bias, float* y,
                   size_t ldy, cudaStream_t stream) {
  GLC_REQUIRE(x && y && batch > 0 && w.packed && w.scales && w.group > 0, "int4 linear q8: empty or null argument");
  GLC_REQUIRE(w.K % w.group == 0, "int4 linear q8: in_features %zu not a multiple of group %zu", w.K, w.group);
  const size_t M = w.M, K = w.K, ag = w.group == 8 ? 32 : w.group;
  if (M > 65536 || K > (size_t)kQ8MaxK || ceil_div(K, ag) > 2048) return int4_linear(w, x, ldx, batch, bias, y, ldy, stream);
  const size_t stride = w.scale_stride ? w.scale_stride : K / w.group;
  // (Weights with a non-finite fp16 scale take the generic kernel, which converts scales exactly.)
  const bool tc = !w.nonfinite && w.group == 32 && K % 256 == 0 && stride == K / 32 &&
                  (uintptr_t)w.packed % 16 == 0 && (uintptr_t)w.scales % 16 == 0 && (uintptr_t)x % 16 == 0 &&
                  ldx % 4 == 0;
  if (tc) {
    for (size_t b = 0; b < batch; b += 4) {
      const size_t nb = batch - b < 4 ? batch - b : 4;
      const float* xb = x + b * ldx;
      float* yb = y + b * ldy;
      // 128-row tiles when they fill the GPU; else 64-row tiles; else 32-row tiles
      // whose K is split over four warp pairs (per-group terms in shared memory,
      // up to 96 KB of them, else one warp pair per tile).
      const size_t sms = (size_t)sm_count();
      const bool split = (size_t)32 * (K / 32) * nb * sizeof(float) <= 96 * 1024;
      int rc;
      if (w.f16) {
        const __half* s = static_cast<const __half*>(w.scales);
        rc = ceil_div(M, 128) >= sms ? launch_q8<__half, 8, 1>(w.packed, s, xb, ldx, nb, bias, yb, ldy, M, K, stream)
             : ceil_div(M, 64) >= sms ? launch_q8<__half, 4, 1>(w.packed, s, xb, ldx, nb, bias, yb, ldy, M, K, stream)
             : split ? launch_q8<__half, 2, 4>(w.packed, s, xb, ldx, nb, bias, yb, ldy, M, K, stream)
                     : launch_q8<__half, 2, 1>(w.packed, s, xb, ldx, nb, bias, yb, ldy, M, K, stream);
      } else {
        const float* s = static_cast<const float*>(w.scales);
        rc = ceil_div(M, 128) >= sms ? launch_q8<float, 8, 1>(w.packed, s, xb, ldx, nb, bias, yb, ldy, M, K, stream)
             : ceil_div(M, 64) >= sms ? launch_q8<float, 4, 1>(w.packed, s, xb, ldx, nb, bias, yb, ldy, M, K, stream)
             : split ? launch_q8<float, 2, 4>(w.packed, s, xb, ldx, nb, bias, yb, ldy, M, K, stream)
                     : launch_q8<float, 2, 1>(w.packed, s, xb, ldx, nb, bias, yb, ldy, M, K, stream);
      }
      if (rc) return rc;
    }
    return GLACIER_CUDA_OK;
  }
  GLC_REQUIRE(stride == 0 || stride * w.group == K, "int4 linear q8: flat group layout required");
  const size_t warps = M * batch;
  if (w.f16)
    return launch_pdl(gemv_q8_generic_kernel<__half>, dim3((unsigned)ceil_div(warps, 8)), dim3(256), 0, stream, 1, x,
                      ldx, w.packed, static_cast<const __half*>(w.scales), bias, y, ldy, (int)M, (int)K, (int)w.group,
                      (int)batch);
  return launch_pdl(gemv_q8_generic_kernel<float>, dim3((unsigned)ceil_div(warps, 8)), dim3(256), 0, stream, 1, x, ldx,
                    w.packed, static_cast<const float*>(w.scales), bias, y, ldy, (int)M, (int)K, (int)w.group,
                    (int)batch);
}

}  // namespace glacier
