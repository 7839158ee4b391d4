// Kernel (a): memory-bound INT4 group-dequant GEMV with FP32 activations.
//
// Computes y[b, m] = bias[m] + sum_k x[b, k] * (u[m, k] - 7) * s[m, k / g]
// over the reference's exact packing (src/core/quant.zig:164-177: row-major,
// two codes per byte, low nibble first, zero point 7) -- the same result as
// linearInt4OnTheFly (src/backends/cpu/int4_matmul.zig:215-305) up to fp32
// summation order.
//
// Design (B200, sm_100a):
//  * A CTA's 8 warps form row groups of R rows; KS warps of a group split the
//    row's 16-byte chunks (32 codes), lanes stride over chunks, so every weight
//    load is a coalesced 128-bit streaming load (L1 no-allocate, L2
//    evict-first) and each byte is read exactly once.  The next chunk of every
//    row is prefetched into registers before the current one is consumed, so
//    each lane keeps 2R loads in flight.
//  * Codes become floats without integer conversion: a byte-permute places
//    0x80 | (u << 3) into bits 16..23 under exponent 0x3F, giving exactly
//    f = 1 + u/16.  Packed fp32x2 FMAs (FFMA2) accumulate T = sum f*x, and the
//    exact identity  sum (u-7) x = 16 T - 23 X  (X = sum x over the chunk)
//    recovers the dot product.  One 64-bit FMA therefore does two
//    multiply-adds, so the SM issue budget stays below the HBM time.
//  * Per-row partial sums are reduced across the warp with shuffles and across
//    the KS K-slices through shared memory.
#include "common.cuh"

namespace glacier {

namespace {

constexpr uint32_t kExp = 0x3F000000u;  // byte 3 = 0x3F, bytes 0..2 = 0 when used as PRMT source b

// f = 1 + u/16 for the code in byte `i` of a prepared word (0x80 | u<<3 per byte).
__device__ __forceinline__ float code_to_float(uint32_t prepared, int i) {
  // result bytes: [0] <- b.byte0 (0), [1] <- b.byte0 (0), [2] <- a.byte i, [3] <- b.byte3 (0x3F)
  return __uint_as_float(prmt(prepared, kExp, 0x7044u | ((uint32_t)i << 8)));
}

template <int B, int R, int KS, typename ScaleT, int GPC>
__global__ void __launch_bounds__(256) gemv_int4_kernel(
    const float* __restrict__ x, size_t ldx, const uint8_t* __restrict__ packed,
    const ScaleT* __restrict__ scales, size_t scale_stride, const float* __restrict__ bias,
    float* __restrict__ y, size_t ldy, int M, int K, int group_shift) {
  griddep_launch();
  griddep_wait();
  // 8 warps = (8 / KS) row groups x KS K-slices; a row group owns R rows.
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int rg = warp / KS, ks = warp % KS;
  const int row0 = (blockIdx.x * (8 / KS) + rg) * R;
  const int nchunks = K >> 5;  // 32 codes (16 bytes) per chunk
  const size_t row_bytes = (size_t)K >> 1;
  constexpr int SUB = 32 / GPC;  // codes per scale sub-group within a chunk
  constexpr int STRIDE = 32 * KS;
  const uint64_t policy = l2_evict_first_policy();
  __shared__ float red[8][R * B];

  int rows[R];
#pragma unroll
  for (int r = 0; r < R; ++r) rows[r] = row0 + r < M ? row0 + r : M - 1;

  float acc[R][B];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) acc[r][b] = 0.f;

  int c = ks * 32 + lane;
  uint4 cur[R];
  if (row0 < M && c < nchunks) {
#pragma unroll
    for (int r = 0; r < R; ++r) cur[r] = ld_stream_u4(packed + (size_t)rows[r] * row_bytes + (size_t)c * 16, policy);
  }
  for (; row0 < M && c < nchunks; c += STRIDE) {
    // Prefetch the next chunk of every row before consuming this one.
    uint4 nxt[R];
    const bool more = c + STRIDE < nchunks;
    if (more) {
#pragma unroll
      for (int r = 0; r < R; ++r)
        nxt[r] = ld_stream_u4(packed + (size_t)rows[r] * row_bytes + (size_t)(c + STRIDE) * 16, policy);
    }
    // Activations for this chunk (shared by the R rows).
    float2 xv[B][16];
    float xc[B][GPC];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const float4* xp = reinterpret_cast<const float4*>(x + b * ldx + (size_t)c * 32);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 t = __ldg(xp + q);
        xv[b][2 * q] = make_float2(t.x, t.y);
        xv[b][2 * q + 1] = make_float2(t.z, t.w);
      }
#pragma unroll
      for (int s = 0; s < GPC; ++s) {
        float2 sum = make_float2(0.f, 0.f);
#pragma unroll
        for (int p = 0; p < SUB / 2; ++p) sum = __fadd2_rn(sum, xv[b][s * (SUB / 2) + p]);
        xc[b][s] = (sum.x + sum.y) * 1.4375f;  // 23/16 (exact power-of-two-free scaling of the sum)
      }
    }
    // Group index of each scale sub-group of this chunk (power-of-two groups).
    int gidx[GPC];
#pragma unroll
    for (int s = 0; s < GPC; ++s) gidx[s] = (c * 32 + s * SUB) >> group_shift;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float sc[GPC];
      const ScaleT* srow = scales + (size_t)rows[r] * scale_stride;
#pragma unroll
      for (int s = 0; s < GPC; ++s) sc[s] = 16.f * load_scale(srow, gidx[s]);
      const uint32_t words[4] = {cur[r].x, cur[r].y, cur[r].z, cur[r].w};
      float2 t[B][GPC];
#pragma unroll
      for (int b = 0; b < B; ++b)
#pragma unroll
        for (int s = 0; s < GPC; ++s) t[b][s] = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t lo = lop3_and_or(words[j] << 3, 0x78787878u, 0x80808080u);
        const uint32_t hi = lop3_and_or(words[j] >> 1, 0x78787878u, 0x80808080u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = make_float2(code_to_float(lo, i), code_to_float(hi, i));
          const int s = (8 * j + 2 * i) / SUB;
#pragma unroll
          for (int b = 0; b < B; ++b) t[b][s] = __ffma2_rn(f, xv[b][4 * j + i], t[b][s]);
        }
      }
#pragma unroll
      for (int b = 0; b < B; ++b)
#pragma unroll
        for (int s = 0; s < GPC; ++s) acc[r][b] = fmaf(sc[s], (t[b][s].x + t[b][s].y) - xc[b][s], acc[r][b]);
    }
    if (more) {
#pragma unroll
      for (int r = 0; r < R; ++r) cur[r] = nxt[r];
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) acc[r][b] = warp_sum(acc[r][b]);
  if (KS > 1) {
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int b = 0; b < B; ++b) red[warp][r * B + b] = acc[r][b];
    }
    __syncthreads();
    if (ks != 0) return;
    if (lane < R * B) {
      float v = 0.f;
#pragma unroll
      for (int k2 = 0; k2 < KS; ++k2) v += red[rg * KS + k2][lane];
      const int row = row0 + lane / B;
      if (row < M) y[(lane % B) * ldy + row] = v + (bias ? bias[row] : 0.f);
    }
    return;
  }
  if (lane < R * B) {
    // lane -> (r, b); select without dynamic register indexing.
    float out = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int b = 0; b < B; ++b)
        if (lane == r * B + b) out = acc[r][b];
    const int row = row0 + lane / B;
    if (row < M) y[(lane % B) * ldy + row] = out + (bias ? bias[row] : 0.f);
  }
}

// Any shape (groups may cross rows, K not a multiple of 32): one warp per
// (row, batch) pair, flat element indexing exactly like dequantElement
// (int4_matmul.zig:3198-3207).  Used only for layouts the fast kernel rejects.
template <typename ScaleT>
__global__ void __launch_bounds__(256) gemv_int4_generic_kernel(
    const float* __restrict__ x, size_t ldx, const uint8_t* __restrict__ packed,
    const ScaleT* __restrict__ scales, size_t scale_stride, const float* __restrict__ bias,
    float* __restrict__ y, size_t ldy, int M, int K, int group, int batch) {
  griddep_launch();
  griddep_wait();
  const int lane = threadIdx.x & 31;
  const size_t wid = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (wid >= (size_t)M * batch) return;
  const int row = (int)(wid % M);
  const int b = (int)(wid / M);
  float acc = 0.f;
  for (int k = lane; k < K; k += 32) {
    const size_t idx = (size_t)row * K + k;
    const uint8_t byte = packed[idx >> 1];
    const int u = (idx & 1) ? (byte >> 4) : (byte & 0xF);
    // scale_stride 0: the reference's flat group array (groups may cross rows).
    const size_t sidx = scale_stride ? (size_t)row * scale_stride + k / group : idx / group;
    acc = fmaf(x[b * ldx + k], (float)(u - 7) * load_scale(scales, sidx), acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) y[b * ldy + row] = acc + (bias ? bias[row] : 0.f);
}

template <int B, int R, int KS, typename ScaleT>
cudaError_t launch_fast(const float* x, size_t ldx, const uint8_t* packed, const ScaleT* scales,
                        size_t scale_stride, const float* bias, float* y, size_t ldy, int M, int K,
                        int group, cudaStream_t stream) {
  const int rows_per_cta = (8 / KS) * R;
  dim3 grid((M + rows_per_cta - 1) / rows_per_cta);
  const int gs = __builtin_ctz((unsigned)group);
  if (group >= 32)
    gemv_int4_kernel<B, R, KS, ScaleT, 1><<<grid, 256, 0, stream>>>(x, ldx, packed, scales, scale_stride,
                                                                     bias, y, ldy, M, K, gs);
  else if (group == 16)
    gemv_int4_kernel<B, R, KS, ScaleT, 2><<<grid, 256, 0, stream>>>(x, ldx, packed, scales, scale_stride,
                                                                     bias, y, ldy, M, K, gs);
  else
    gemv_int4_kernel<B, R, KS, ScaleT, 4><<<grid, 256, 0, stream>>>(x, ldx, packed, scales, scale_stride,
                                                                     bias, y, ldy, M, K, gs);
  note_launch();
  return cudaGetLastError();
}

template <int B, int KS, typename ScaleT>
cudaError_t launch_rows(const float* x, size_t ldx, const uint8_t* packed, const ScaleT* scales,
                        size_t scale_stride, const float* bias, float* y, size_t ldy, int M, int K,
                        int group, cudaStream_t stream) {
  // Largest rows-per-warp that still gives >= 3 CTAs per SM.
  const int target = 3 * sm_count();
  const int groups = 8 / KS;
  if (M / (groups * 8) >= target)
    return launch_fast<B, 8, KS>(x, ldx, packed, scales, scale_stride, bias, y, ldy, M, K, group, stream);
  if (M / (groups * 4) >= target)
    return launch_fast<B, 4, KS>(x, ldx, packed, scales, scale_stride, bias, y, ldy, M, K, group, stream);
  if (M / (groups * 2) >= target)
    return launch_fast<B, 2, KS>(x, ldx, packed, scales, scale_stride, bias, y, ldy, M, K, group, stream);
  return launch_fast<B, 1, KS>(x, ldx, packed, scales, scale_stride, bias, y, ldy, M, K, group, stream);
}

template <int B, typename ScaleT>
cudaError_t launch_split(const float* x, size_t ldx, const uint8_t* packed, const ScaleT* scales,
                         size_t scale_stride, const float* bias, float* y, size_t ldy, int M, int K,
                         int group, cudaStream_t stream) {
  // K-slices per row group: about 48 chunks (1.5 lane iterations) per warp.
  const int nchunks = K / 32;
  if (nchunks >= 8 * 48)
    return launch_rows<B, 8>(x, ldx, packed, scales, scale_stride, bias, y, ldy, M, K, group, stream);
  if (nchunks >= 4 * 48)
    return launch_rows<B, 4>(x, ldx, packed, scales, scale_stride, bias, y, ldy, M, K, group, stream);
  if (nchunks >= 2 * 48)
    return launch_rows<B, 2>(x, ldx, packed, scales, scale_stride, bias, y, ldy, M, K, group, stream);
  return launch_rows<B, 1>(x, ldx, packed, scales, scale_stride, bias, y, ldy, M, K, group, stream);
}

}  // namespace

// True when the fast kernel handles this layout: whole 32-code chunks per row
// and power-of-two groups >= 8 that divide the row.
bool gemv_fast_layout(size_t K, size_t group) {
  if (K == 0 || K % 32 != 0 || group < 8 || K % group != 0) return false;
  return (group & (group - 1)) == 0;
}

int gemv_int4_tc(const Int4Weight& w, const float* x, size_t ldx, size_t batch, const float* bias, float* y,
                 size_t ldy, cudaStream_t stream, const float* xu = nullptr);

// y = W (silu(gate) * up) on the tensor-core GEMV, the SwiGLU folded into the
// activation loads; GLACIER_CUDA_EUNSUPPORTED when the weight or operands do not
// fit that kernel (the caller then runs silu_mul and int4_linear).
int int4_linear_swiglu(const Int4Weight& w, const float* gate, const float* up, size_t ld, size_t batch,
                       const float* bias, float* y, size_t ldy, cudaStream_t stream) {
  GLC_REQUIRE(gate && up && y && batch > 0, "int4 linear swiglu: empty or null argument");
  const bool aligned = ((uintptr_t)gate % 16 == 0) && ((uintptr_t)up % 16 == 0) && (ld % 4 == 0);
  if (!w.tc || !aligned) return GLACIER_CUDA_EUNSUPPORTED;
  for (size_t b = 0; b < batch; b += 4) {
    const size_t nb = batch - b < 4 ? batch - b : 4;
    const int rc = gemv_int4_tc(w, gate + b * ld, ld, nb, bias, y + b * ldy, ldy, stream, up + b * ld);
    if (rc) return rc;
  }
  return GLACIER_CUDA_OK;
}

int int4_linear(const Int4Weight& w, const float* x, size_t ldx, size_t batch, const float* bias, float* y,
                size_t ldy, cudaStream_t stream) {
  GLC_REQUIRE(x && y && batch > 0, "int4 linear: empty or null argument");
  const size_t M = w.M, K = w.K, group = w.group;
  const bool xaligned = ((uintptr_t)x % 16 == 0) && (ldx % 4 == 0);
  if (w.tc && xaligned) {
    // Tensor-core GEMV: up to four activation rows per launch.
    for (size_t b = 0; b < batch; b += 4) {
      const size_t nb = batch - b < 4 ? batch - b : 4;
      const int rc = gemv_int4_tc(w, x + b * ldx, ldx, nb, bias, y + b * ldy, ldy, stream);
      if (rc) return rc;
    }
    return GLACIER_CUDA_OK;
  }
  const size_t scale_stride = w.scale_stride;
  if (gemv_fast_layout(K, group) && xaligned && (uintptr_t)w.packed % 16 == 0) {
    const size_t ss = scale_stride ? scale_stride : K / group;
    for (size_t b = 0; b < batch; b += 2) {
      const bool two = b + 2 <= batch;
      cudaError_t e;
      if (w.f16)
        e = two ? launch_split<2, __half>(x + b * ldx, ldx, w.packed, (const __half*)w.scales, ss, bias, y + b * ldy,
                                          ldy, (int)M, (int)K, (int)group, stream)
                : launch_split<1, __half>(x + b * ldx, ldx, w.packed, (const __half*)w.scales, ss, bias, y + b * ldy,
                                          ldy, (int)M, (int)K, (int)group, stream);
      else
        e = two ? launch_split<2, float>(x + b * ldx, ldx, w.packed, (const float*)w.scales, ss, bias, y + b * ldy,
                                         ldy, (int)M, (int)K, (int)group, stream)
                : launch_split<1, float>(x + b * ldx, ldx, w.packed, (const float*)w.scales, ss, bias, y + b * ldy,
                                         ldy, (int)M, (int)K, (int)group, stream);
      GLC_CHECK_CUDA(e);
    }
    return GLACIER_CUDA_OK;
  }
  // Generic layout: flat element index (scale_stride 0 = flat group array).
  GLC_REQUIRE(scale_stride == 0 || K % group == 0, "int4 gemv: per-row scale stride needs group-aligned rows");
  const size_t warps = M * batch;
  if (w.f16)
    gemv_int4_generic_kernel<__half><<<(unsigned)ceil_div(warps, 8), 256, 0, stream>>>(
        x, ldx, w.packed, (const __half*)w.scales, scale_stride, bias, y, ldy, (int)M, (int)K, (int)group, (int)batch);
  else
    gemv_int4_generic_kernel<float><<<(unsigned)ceil_div(warps, 8), 256, 0, stream>>>(
        x, ldx, w.packed, (const float*)w.scales, scale_stride, bias, y, ldy, (int)M, (int)K, (int)group, (int)batch);
  GLC_CHECK_LAUNCH();
  return GLACIER_CUDA_OK;
}

template <typename ScaleT>
int gemv_int4(const float* x, size_t ldx, size_t batch, const uint8_t* packed, const ScaleT* scales,
              size_t scale_stride, const float* bias, float* y, size_t ldy, size_t M, size_t K,
              size_t group, cudaStream_t stream) {
  Int4Weight w;
  w.packed = packed;
  w.scales = scales;
  w.f16 = sizeof(ScaleT) == 2;
  w.scale_stride = scale_stride;
  w.M = M;
  w.K = K;
  w.group = group;
  const int rc = int4_weight_prepare(w);
  if (rc) return rc;
  return int4_linear(w, x, ldx, batch, bias, y, ldy, stream);
}

template int gemv_int4<__half>(const float*, size_t, size_t, const uint8_t*, const __half*, size_t,
                               const float*, float*, size_t, size_t, size_t, size_t, cudaStream_t);
template int gemv_int4<float>(const float*, size_t, size_t, const uint8_t*, const float*, size_t,
                              const float*, float*, size_t, size_t, size_t, size_t, cudaStream_t);

}  // namespace glacier
