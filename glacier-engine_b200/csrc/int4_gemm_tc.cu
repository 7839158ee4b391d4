// Kernel (b): batched INT4 dequant GEMM on the 5th-generation tensor cores
// (tcgen05 + TMEM), for decode lanes and prefill tokens.
//
// Y[n, m] = sum_k X[n, k] * (u[m, k] - 7) * s[m, k / 32]   (+ split-K partials)
// on the reference's exact packing (src/core/quant.zig:164-177), the batched
// form of linearInt4OnTheFly (src/backends/cpu/int4_matmul.zig:215-305) and of
// the reference's M4 weight-stationary GEMM (int4_neon.c:1439-1621).
//
// Numerics: there is no INT4 x FP32 tensor-core MMA, and a single fp16/bf16
// rounding of either operand would miss the 1e-3 tolerance, so both operands
// are split exactly:
//   W = q*s = Whi + Wlo   (fp16 pair; q*s has <= 15 significant bits, so the
//                          split is exact up to fp16 underflow)
//   X = xs*(Xhi + Xlo)    (fp16 pair with a per-row power-of-two scale xs,
//                          ~22 significant bits)
//   Y = xs*(Whi*Xhi + Whi*Xlo + Wlo*Xhi)      (dropped term ~2^-22)
// One MMA per 16-K step runs Whi against the stacked [Xhi | Xlo] columns
// (N = 2*Np) and a second runs Wlo against Xhi into the same TMEM columns, all
// accumulated in fp32.
//
// Pipeline (one CTA = 128 weight rows x Np activation rows x a K range):
//   warp 0  TMA producer: 128 x 256-code nibble tiles (SWIZZLE_128B) + the
//           128 x 8 scale tiles into a 3-slot ring
//   warp 1  TMA producer: 64-K activation tiles [Xhi | Xlo] (SWIZZLE_128B)
//   warp 2  allocates TMEM and issues tcgen05.mma from one thread
//   warps 3-10 (256 threads, two per weight row) convert nibbles + scales to
//           the -Whi / Wlo tiles in the canonical K-major SWIZZLE_128B layout
//           (the MMA descriptor negates A back), then run the epilogue
//           (tcgen05.ld, xs scaling, coalesced stores).
// Code order inside each 8-code word is permuted to (0,4,1,5,2,6,3,7) by the
// unpack; the activation split kernel stores X in the same order, so the
// contraction is unchanged.  Every wait is bounded; no multicast is used.
#include "common.cuh"

namespace glacier {

__device__ int g_gemm_error;

namespace {

constexpr int kRowsTile = 128;
constexpr int kChunkK = 64;                     // K per MMA stage (one 128-byte swizzle row of fp16)
constexpr int kSuperK = 256;                    // K per nibble/scale TMA stage
constexpr int kMaxSlots = 8;                    // ring slots (runtime counts below this)
constexpr int kConvWarps = 8;                   // two converter threads per weight row
constexpr int kNibBytes = kRowsTile * 128;      // 128 rows x 256 codes
constexpr int kSclBytes = kRowsTile * 16;       // 128 rows x 8 fp16 scales
constexpr int kATileBytes = kRowsTile * 128;    // 128 rows x 64 fp16
constexpr int kThreads = (3 + kConvWarps) * 32;

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t neg_half2(uint32_t a) { return a ^ 0x80008000u; }

// Eight codes -> four half2 of exact (u - 7) in the order {u0,u4},{u1,u5},{u2,u6},{u3,u7}.
__device__ __forceinline__ void unpack8(uint32_t w, uint32_t (&q)[4]) {
  const uint32_t w8 = w >> 8;
  const uint32_t t0 = lop3_and_or(w, 0x000F000Fu, 0x64006400u);   // 1024 + u
  const uint32_t t1 = lop3_and_or(w, 0x00F000F0u, 0x64006400u);   // 1024 + 16u
  const uint32_t t2 = lop3_and_or(w8, 0x000F000Fu, 0x64006400u);
  const uint32_t t3 = lop3_and_or(w8, 0x00F000F0u, 0x64006400u);
  q[0] = hfma2_u32(t0, 0x3C003C00u, 0xE407E407u);  // *1 - 1031
  q[1] = hfma2_u32(t1, 0x2C002C00u, 0xD470D470u);  // /16 - 71
  q[2] = hfma2_u32(t2, 0x3C003C00u, 0xE407E407u);
  q[3] = hfma2_u32(t3, 0x2C002C00u, 0xD470D470u);
}

// UMMA shared-memory descriptor: K-major, SWIZZLE_128B, 8-row core groups 1024 B apart.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
  d |= (uint64_t)1 << 46;             // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, A = B = f16, D = f32, both K-major, M = 128;
// negate_a flips the sign of A (bit 13).
__host__ __device__ constexpr uint32_t idesc_f16(int n, bool negate_a = false) {
  return (1u << 4) | ((negate_a ? 1u : 0u) << 13) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

struct GemmParams {
  const float* xscale;  // [Np] per activation row
  const float* bias;    // [M] or null, added by split 0
  float* y;             // [n, ldy] (+ split * split_stride)
  size_t ldy, split_stride;
  int M, K, n, np;      // weight rows, K, live activation rows, padded rows (multiple of 16)
  int chunks_total;     // ceil(K / 64)
  int chunks_per_split; // multiple of 4
  int nib_slots, a_slots, b_slots;
  int* err;
};

__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_w,
                                                              const __grid_constant__ CUtensorMap tmap_s,
                                                              const __grid_constant__ CUtensorMap tmap_x,
                                                              const GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bbytes = 2 * p.np * 128;  // [Xhi | Xlo] tile: 2*Np rows x 64 fp16
  const int kNibSlots = p.nib_slots, kASlots = p.a_slots, kBSlots = p.b_slots;
  uint8_t* nib = smem;                                        // kNibSlots x (nibbles + scales)
  uint8_t* atile = nib + kNibSlots * (kNibBytes + kSclBytes); // kASlots x (-Whi, Wlo)
  uint8_t* btile = atile + kASlots * 2 * kATileBytes;         // kBSlots x bbytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(btile + kBSlots * bbytes);
  uint64_t* nib_full = bars;
  uint64_t* nib_empty = nib_full + kMaxSlots;
  uint64_t* a_full = nib_empty + kMaxSlots;
  uint64_t* a_empty = a_full + kMaxSlots;
  uint64_t* b_full = a_empty + kMaxSlots;
  uint64_t* b_empty = b_full + kMaxSlots;
  uint64_t* acc_full = b_empty + kMaxSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int row0 = tile * kRowsTile;
  const int c0 = split * p.chunks_per_split;
  const int c1 = min(p.chunks_total, c0 + p.chunks_per_split);
  const int nch = max(0, c1 - c0);
  const uint32_t ncols = (2 * p.np <= 32) ? 32 : (2 * p.np <= 64 ? 64 : (2 * p.np <= 128 ? 128 : 256));

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < kNibSlots; ++i) {
      mbar_init(&nib_full[i], 1);
      mbar_init(&nib_empty[i], kConvWarps);
    }
    for (int i = 0; i < kASlots; ++i) {
      mbar_init(&a_full[i], kConvWarps);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < kBSlots; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- nibble + scale producer (one 256-K super-stage per 4 chunks) ----
    if (lane == 0 && nch > 0) {
      prefetch_tmap(&tmap_w);
      prefetch_tmap(&tmap_s);
      const uint64_t pol = l2_evict_first_policy();
      const int nsup = (nch + 3) / 4;
      int issued = 0;
      for (int i = 0; i < nsup; ++i) {
        const int slot = i % kNibSlots, round = i / kNibSlots;
        if (!mbar_wait(&nib_empty[slot], (round & 1) ^ 1, p.err)) { s_abort = 1; break; }
        uint8_t* dst = nib + slot * (kNibBytes + kSclBytes);
        mbar_arrive_expect_tx(&nib_full[slot], kNibBytes + kSclBytes);
        const int ks = (c0 / 4 + i);  // super-stage index along K
        tma_load_2d(dst, &tmap_w, ks * 128, row0, &nib_full[slot], pol);
        tma_load_2d(dst + kNibBytes, &tmap_s, ks * 8, row0, &nib_full[slot], pol);
        ++issued;
      }
      for (int i = max(0, issued - kNibSlots); i < issued; ++i)
        mbar_wait(&nib_full[i % kNibSlots], (i / kNibSlots) & 1, p.err);
    }
  } else if (warp == 1) {
    // ---- activation producer: one [Xhi | Xlo] tile per 64-K chunk ----
    if (lane == 0 && nch > 0) {
      prefetch_tmap(&tmap_x);
      uint64_t keep;
      asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(keep));
      int issued = 0;
      for (int i = 0; i < nch; ++i) {
        const int slot = i % kBSlots, round = i / kBSlots;
        if (!mbar_wait(&b_empty[slot], (round & 1) ^ 1, p.err)) { s_abort = 1; break; }
        mbar_arrive_expect_tx(&b_full[slot], (uint32_t)bbytes);
        tma_load_2d(btile + slot * bbytes, &tmap_x, (c0 + i) * kChunkK, 0, &b_full[slot], keep);
        ++issued;
      }
      for (int i = max(0, issued - kBSlots); i < issued; ++i)
        mbar_wait(&b_full[i % kBSlots], (i / kBSlots) & 1, p.err);
    }
  } else if (warp == 2) {
    // ---- MMA issuer ----
    if (lane == 0 && nch > 0) {
      // A holds -Whi (negated back by the descriptor) and Wlo.
      const uint32_t id_hl = idesc_f16(2 * p.np, true), id_h = idesc_f16(p.np);
      int done = 0;
      for (int i = 0; i < nch; ++i) {
        const int as = i % kASlots, bs = i % kBSlots;
        if (!mbar_wait(&a_full[as], (i / kASlots) & 1, p.err)) { s_abort = 1; break; }
        if (!mbar_wait(&b_full[bs], (i / kBSlots) & 1, p.err)) { s_abort = 1; break; }
        tc_fence_after();
        const uint32_t ahi = smem_u32(atile + as * 2 * kATileBytes);
        const uint32_t alo = ahi + kATileBytes;
        const uint32_t bx = smem_u32(btile + bs * bbytes);
#pragma unroll
        for (int kk = 0; kk < kChunkK / 16; ++kk) {
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          umma_f16(tmem, sdesc(ahi + kk * 32), sdesc(bx + kk * 32), id_hl, acc);  // Whi x [Xhi | Xlo]
          umma_f16(tmem, sdesc(alo + kk * 32), sdesc(bx + kk * 32), id_h, 1u);     // Wlo x Xhi
        }
        umma_commit(&a_empty[as]);
        umma_commit(&b_empty[bs]);
        ++done;
      }
      umma_commit(acc_full);  // fires when every MMA issued above has completed
      (void)done;
    }
  } else {
    // ---- converters (256 threads: two per weight row, 32 codes each), then the epilogue ----
    const int t = threadIdx.x - 3 * 32;   // 0..255
    const int rrow = t & (kRowsTile - 1);  // row within the tile
    const int hf = t >> 7;                 // which 32-code half of the 64-code chunk
    const uint32_t swz = (uint32_t)(rrow & 7);
    for (int i = 0; i < nch && !s_abort; ++i) {
      const int sup = i / 4, sub = i % 4;
      const int ns = sup % kNibSlots;
      if (sub == 0 && !mbar_wait(&nib_full[ns], (sup / kNibSlots) & 1, p.err)) { s_abort = 1; break; }
      const int as = i % kASlots;
      if (!mbar_wait(&a_empty[as], ((i / kASlots) & 1) ^ 1, p.err)) { s_abort = 1; break; }
      const uint8_t* nrow = nib + ns * (kNibBytes + kSclBytes) + rrow * 128;
      const uint8_t* srow = nib + ns * (kNibBytes + kSclBytes) + kNibBytes + rrow * 16;
      const int grp = 2 * sub + hf;  // 32-code group within the 256-code super stage
      const uint4 g = *reinterpret_cast<const uint4*>(nrow + (((uint32_t)grp ^ swz) << 4));
      const uint32_t sh = *reinterpret_cast<const uint16_t*>(srow + 2 * grp);
      const uint32_t s2 = sh * 0x10001u;           // {s, s}
      const uint32_t ns2 = s2 ^ 0x80008000u;       // {-s, -s}
      uint8_t* ahi = atile + as * 2 * kATileBytes + rrow * 128;
      uint8_t* alo = ahi + kATileBytes;
      const uint32_t words[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t q[4], h[4], l[4];
        unpack8(words[j], q);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          h[e] = hmul2_u32(q[e], ns2);        // -RN(q*s)
          l[e] = hfma2_u32(q[e], s2, h[e]);   // q*s - RN(q*s), exact
        }
        const uint32_t off = ((uint32_t)(4 * hf + j) ^ swz) << 4;
        *reinterpret_cast<uint4*>(ahi + off) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(alo + off) = make_uint4(l[0], l[1], l[2], l[3]);
      }
      fence_proxy_async();  // make the generic-proxy stores visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[as]);
        if (sub == 3 || i == nch - 1) mbar_arrive(&nib_empty[ns]);
      }
    }
    // Epilogue: TMEM lane = row (this warp's quarter), columns b (hi) and Np + b (lo);
    // the two converter warps of a quarter split the column blocks.
    const int quarter = warp & 3;
    const int row = row0 + quarter * 32 + lane;
    float* ybase = p.y + (size_t)split * p.split_stride;
    if (nch > 0 && !s_abort && mbar_wait(acc_full, 0, p.err)) {
      tc_fence_after();
      const uint32_t tq = tmem + ((uint32_t)(quarter * 32) << 16);
      const int nblk16 = p.np / 16;
      for (int bi = hf; bi < nblk16; bi += 2) {
        const int b0 = bi * 16;
        float vh[16], vl[16];
        tmem_ld16(tq + (uint32_t)b0, vh);
        tmem_ld16(tq + (uint32_t)(p.np + b0), vl);
        if (row < p.M) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int b = b0 + j;
            if (b < p.n)
              ybase[(size_t)b * p.ldy + row] =
                  (vh[j] + vl[j]) * p.xscale[b] + ((p.bias && split == 0) ? p.bias[row] : 0.f);
          }
        }
      }
    } else if (nch == 0 && hf == 0) {
      // Empty K-range: this split contributes zeros (plus the bias on split 0).
      if (row < p.M)
        for (int b = 0; b < p.n; ++b) ybase[(size_t)b * p.ldy + row] = (p.bias && split == 0) ? p.bias[row] : 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    // Never release TMEM while an MMA may still write it (aborted runs included).
    if (lane == 0 && nch > 0) mbar_wait(acc_full, 0, p.err);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  }
}

// x [n, K] fp32 -> [Xhi ; Xlo] fp16 rows (Np each) in the code order
// (0,4,1,5,2,6,3,7) per 8 and xscale[row] = 2^e with max|x|/2^e in [2^14, 2^15).
__global__ void split_activation_kernel(const float* __restrict__ x, size_t ldx, int K, int np,
                                        __half* __restrict__ xs, float* __restrict__ xscale) {
  const int r = blockIdx.x;
  const float* xr = x + (size_t)r * ldx;
  float m = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) m = fmaxf(m, fabsf(xr[k]));
  __shared__ float sh[32];
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) sh[0] = v;
  }
  __syncthreads();
  m = sh[0];
  float scale = 1.f;
  if (m > 0.f && isfinite(m)) {
    int e;
    frexpf(m, &e);             // m = f * 2^e, f in [0.5, 1)
    scale = ldexpf(1.f, e - 15);  // m / scale in [2^14, 2^15)
  }
  const float inv = 1.f / scale;  // exact (power of two)
  __half* hi = xs + (size_t)r * K;
  __half* lo = xs + ((size_t)np + r) * K;
  for (int k8 = threadIdx.x; k8 < K / 8; k8 += blockDim.x) {
    const int base = k8 * 8;
    __half h[8], l[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int src = base + ((i & 1) ? 4 + (i >> 1) : (i >> 1));  // (0,4,1,5,2,6,3,7)
      const float v = xr[src] * inv;
      h[i] = __float2half_rn(v);
      l[i] = __float2half_rn(v - __half2float(h[i]));
    }
    *reinterpret_cast<uint4*>(hi + base) = *reinterpret_cast<uint4*>(h);
    *reinterpret_cast<uint4*>(lo + base) = *reinterpret_cast<uint4*>(l);
  }
  if (threadIdx.x == 0) xscale[r] = scale;
}

}  // namespace

size_t gemm_split_bytes(size_t np, size_t K) { return 2 * np * K * sizeof(__half) + np * sizeof(float) + 256; }

bool gemm_tc_supported(const Int4Weight& w) { return w.tc && w.f16 && w.K % kChunkK == 0; }

// Activations in split form for the GEMM: xs [2*np, K] fp16 + xscale [np].
int split_activation(const float* x, size_t ldx, size_t n, size_t K, size_t np, __half* xs, float* xscale,
                     cudaStream_t stream) {
  GLC_REQUIRE(K % 8 == 0 && n <= np, "split_activation: K %% 8 and n <= np required");
  split_activation_kernel<<<(unsigned)n, 256, 0, stream>>>(x, ldx, (int)K, (int)np, xs, xscale);
  GLC_CHECK_LAUNCH();
  return GLACIER_CUDA_OK;
}

int encode_split_map(CUtensorMap* map, const __half* xs, size_t np, size_t K) {
  return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xs, K, 2 * np, K * sizeof(__half), kChunkK,
                        (uint32_t)(2 * np), CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}

// Ring depths for a padded activation width.  The activation ring is the
// deepest: its tiles come from L2 with ~1 us of TMA latency and each covers only
// 64 K, so six of them keep the MMA fed; then three nibble stages (768 K of
// HBM reads in flight) and two converted weight tiles; all within 227 KB.
static void gemm_slots(size_t np, int* nib, int* a, int* b) {
  *nib = 3;
  *a = 4;
  *b = 6;
  auto bytes = [&]() {
    return 1024 + (size_t)*nib * (kNibBytes + kSclBytes) + (size_t)*a * 2 * kATileBytes + (size_t)*b * 2 * np * 128 +
           (6 * kMaxSlots + 1) * 8 + 16;
  };
  while (bytes() > 227 * 1024 && *b > 3) --*b;
  if (bytes() > 227 * 1024) *nib = 2;
  while (bytes() > 227 * 1024 && *a > 2) --*a;
  while (bytes() > 227 * 1024 && *b > 2) --*b;
}

size_t gemm_smem_bytes(size_t np) {
  int nib, a, b;
  gemm_slots(np, &nib, &a, &b);
  return 1024 + (size_t)nib * (kNibBytes + kSclBytes) + (size_t)a * 2 * kATileBytes + (size_t)b * 2 * np * 128 +
         (6 * kMaxSlots + 1) * 8 + 16;
}

// The tensor core's fp32 accumulation does not round every addition, so an
// accumulation chain of n k-steps drifts by up to ~n * 2^-24 of the running
// sum.  Chains are therefore capped at kMaxChainK, and longer reductions are
// finished on the CUDA cores in rounded fp32 (split-K partials summed in order).
constexpr size_t kMaxChainK = 4096;

// Number of K splits for a GEMM: enough CTAs to cover the SMs, whole 256-K
// super-stages, and no accumulation chain longer than kMaxChainK.
int gemm_splits(size_t M, size_t K) {
  const int tiles = (int)ceil_div(M, kRowsTile);
  const int sup = (int)ceil_div(K, kSuperK);
  int s = 1;
  while (s < 16 && s * 2 <= sup && (tiles * s < sm_count() || ceil_div(K, (size_t)s) > kMaxChainK)) s *= 2;
  return s;
}

namespace {
__global__ void reduce_splits_kernel(const float* __restrict__ part, size_t split_stride, int nsplit,
                                     float* __restrict__ y, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float v = part[i];
    for (int s = 1; s < nsplit; ++s) v += part[s * split_stride + i];
    y[i] = v;
  }
}
}  // namespace

// y[i] = sum over nsplit partial arrays (in split order), i < n.
int reduce_splits(const float* part, size_t split_stride, int nsplit, float* y, size_t n, cudaStream_t stream) {
  const unsigned grid = (unsigned)std::min<size_t>(ceil_div(n, 256), (size_t)sm_count() * 8);
  reduce_splits_kernel<<<grid, 256, 0, stream>>>(part, split_stride, nsplit, y, n);
  GLC_CHECK_LAUNCH();
  return GLACIER_CUDA_OK;
}

// y (+ split * split_stride) = X W^T for the np-padded activation block whose
// TMA map is `xmap`; nsplit K-partials are written when nsplit > 1.
int gemm_int4_tc(const Int4Weight& w, const CUtensorMap& xmap, const float* xscale, size_t n, size_t np, float* y,
                 size_t ldy, int nsplit, size_t split_stride, const float* bias, cudaStream_t stream) {
  GLC_REQUIRE(gemm_tc_supported(w), "int4 gemm: weight layout not supported by the tensor-core GEMM");
  GLC_REQUIRE(np % 16 == 0 && np >= 16 && np <= 128 && n <= np, "int4 gemm: padded rows %zu (n=%zu)", np, n);
  const int chunks = (int)(w.K / kChunkK);
  const int sup = (int)ceil_div(w.K, kSuperK);
  const int per = (int)ceil_div(sup, nsplit) * 4;
  const size_t smem = gemm_smem_bytes(np);
  GLC_REQUIRE(smem <= 227 * 1024, "int4 gemm: %zu bytes of shared memory", smem);
  static size_t attr = 0;
  if (attr < smem) {
    const int rc = allow_dynamic_smem((const void*)gemm_tc_kernel, (int)smem);
    if (rc) return rc;
    attr = smem;
  }
  int* err = nullptr;
  GLC_CHECK_CUDA(cudaGetSymbolAddress((void**)&err, g_gemm_error));
  int nib_slots, a_slots, b_slots;
  gemm_slots(np, &nib_slots, &a_slots, &b_slots);
  GemmParams prm{xscale, bias, y, ldy, split_stride, (int)w.M, (int)w.K, (int)n, (int)np, chunks, per,
                 nib_slots, a_slots, b_slots, err};
  dim3 grid((unsigned)ceil_div(w.M, kRowsTile), (unsigned)nsplit);
  gemm_tc_kernel<<<grid, kThreads, smem, stream>>>(w.tmap_w, w.tmap_s, xmap, prm);
  GLC_CHECK_LAUNCH();
  return GLACIER_CUDA_OK;
}

int gemm_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_gemm_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace glacier
