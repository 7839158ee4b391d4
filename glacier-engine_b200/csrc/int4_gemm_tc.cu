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
// Persistent pipeline: one CTA per SM walks a static list of work units
// (128 weight rows x one K split), with TMEM allocated and barriers set up once:
//   warp 0      TMA producer: 128 x 256-code nibble tiles (SWIZZLE_128B) plus the
//               matching 128 x 8 fp16 scale tiles, into a ring of super-stages
//   warp 1      TMA producer: 64-K activation tiles [Xhi | Xlo] (SWIZZLE_128B)
//   warp 2      allocates TMEM; runs the MMA loop converged, one elected lane
//               issues every tcgen05.mma and commit
//   warps 3-10  converters (two per 32-row TMEM lane quarter, alternate chunks): nibbles + scales
//               -> -Whi / Wlo fp16 pairs written straight into TMEM with
//               tcgen05.st; the MMA reads A from TMEM (the descriptor's negate
//               bit restores the sign of Whi), so shared memory carries only
//               the nibble and activation tiles
//   warps 11-14 epilogue: tcgen05.ld of a finished accumulator, per-row
//               activation scale, bias, coalesced stores
// Accumulators are double-buffered in TMEM when they fit, so a unit's
// epilogue overlaps the next unit's MMAs.
// Code order inside each 8-code word is permuted to (0,4,1,5,2,6,3,7) by the
// unpack; the activation split kernel stores X in the same order, so the
// contraction is unchanged.  Every wait is bounded; no multicast is used.
#include "common.cuh"

namespace glacier {

__device__ int g_gemm_error;

namespace {

constexpr int kRowsTile = 128;
constexpr int kChunkK = 64;                     // K per MMA group (one 128-byte swizzle row of fp16)
constexpr int kSub = 2;                         // MMA groups per pipeline chunk
constexpr int kPipeK = kChunkK * kSub;          // K per pipeline chunk: one A slot, one B stage, one commit
constexpr int kSuperK = 256;                    // K per nibble/scale TMA stage
constexpr int kChunksPerSuper = kSuperK / kPipeK;
constexpr int kMaxSlots = 8;                    // shared-memory ring slots (runtime counts below this)
constexpr int kConvWarps = 8;                   // two converter warps per TMEM lane quarter
constexpr int kEpiWarps = 4;                    // one epilogue warp per TMEM lane quarter
constexpr int kASlots = 2;                      // A chunks (-Whi | Wlo) resident in TMEM
constexpr int kDoneRing = 8;                    // chunk-completion barriers (>= kASlots and >= B slots)
constexpr uint32_t kAColsPerSlot = 128;         // 64 columns of -Whi + 64 of Wlo (2 fp16 per column)
constexpr uint32_t kTmemCols = 512;             // the whole TMEM of the SM (one CTA per SM)
constexpr int kNibBytes = kRowsTile * 128;      // 128 rows x 256 codes
// Scale tile of a super-stage: 128 rows x 256/group fp16 scales (16, 32 or 64 bytes a row).
__host__ __device__ constexpr int scl_bytes(int per32) { return kRowsTile * 16 * per32; }
constexpr int kThreads = (3 + kConvWarps + kEpiWarps) * 32;
constexpr int kMinSmem = 120 * 1024;            // keeps a second CTA (and its TMEM request) off the SM

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

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

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

// tcgen05.mma with A read from TMEM (kind::f16, cta_group::1).
__device__ __forceinline__ void umma_f16_ts(uint32_t dtmem, uint32_t atmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(dtmem),
      "r"(atmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Each thread writes 16 consecutive 32-bit columns of its own TMEM lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

struct GemmParams {
  const float* xscale;  // [Np] per activation row
  const float* bias;    // [M] or null, added by split 0
  float* y;             // [n, ldy] (+ split * split_stride)
  size_t ldy, split_stride;
  int M, K, n, np;      // weight rows, K, live activation rows, padded rows (multiple of 16)
  int chunks_total;     // K / kPipeK
  int chunks_per_split; // multiple of kChunksPerSuper
  int nsplit, tiles, units;
  int nib_slots, b_slots;
  int acc_cols, acc_bufs;  // TMEM columns per accumulator buffer, number of buffers
  int sc_x;                // scale-tile x coordinate per super-stage (256 / group)
  int* err;
};

struct Unit {
  int row0, split, c0, nch;
};

__device__ __forceinline__ Unit unit_of(const GemmParams& p, int u) {
  Unit w;
  const int tile = u / p.nsplit;
  w.split = u - tile * p.nsplit;
  w.row0 = tile * kRowsTile;
  w.c0 = w.split * p.chunks_per_split;
  w.nch = max(0, min(p.chunks_total, w.c0 + p.chunks_per_split) - w.c0);
  return w;
}

// S = scale groups per 32 codes: 1 (group 32), 2 (group 16) or 4 (group 8).
template <int S>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_w,
                                                              const __grid_constant__ CUtensorMap tmap_s,
                                                              const __grid_constant__ CUtensorMap tmap_x,
                                                              const GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bbytes = 2 * p.np * 128;  // [Xhi | Xlo] box: 2*Np rows x 64 fp16; a B stage holds kSub boxes
  const int NS = p.nib_slots, BS = p.b_slots;
  uint8_t* nib = smem;                                 // NS x (nibbles + scales)
  constexpr int kSclBytes = scl_bytes(S);
  uint8_t* btile = nib + NS * (kNibBytes + kSclBytes);  // BS x kSub x bbytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(btile + BS * kSub * bbytes);
  uint64_t* nib_full = bars;
  uint64_t* nib_empty = nib_full + kMaxSlots;
  uint64_t* b_full = nib_empty + kMaxSlots;
  uint64_t* done = b_full + kMaxSlots;             // chunk c's MMAs completed: done[c % kDoneRing]
  uint64_t* a_full = done + kDoneRing;
  uint64_t* acc_full = a_full + kASlots;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Weights do not depend on the previous kernel: the nibble producer and the
  // converters start at once; the activation producer and the epilogue wait for
  // the previous kernel's writes (griddep_wait) before touching its outputs.
  griddep_launch();

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < NS; ++i) {
      mbar_init(&nib_full[i], 1);
      mbar_init(&nib_empty[i], kConvWarps);
    }
    for (int i = 0; i < BS; ++i) mbar_init(&b_full[i], 1);
    for (int i = 0; i < kDoneRing; ++i) mbar_init(&done[i], 1);
    for (int i = 0; i < kASlots; ++i) mbar_init(&a_full[i], kConvWarps / 2);  // one warp per lane quarter
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiWarps);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t a_base = (uint32_t)(p.acc_bufs * p.acc_cols);  // A ring follows the accumulators

  if (warp == 0) {
    // ---- nibble + scale producer: one 256-K super-stage per kChunksPerSuper chunks ----
    if (lane == 0) {
      prefetch_tmap(&tmap_w);
      prefetch_tmap(&tmap_s);
      const uint64_t pol = l2_evict_first_policy();
      uint32_t it = 0, slot = 0, ph = 0;
      for (int u = blockIdx.x; u < p.units && !s_abort; u += gridDim.x) {
        const Unit w = unit_of(p, u);
        const int nsup = (w.nch + kChunksPerSuper - 1) / kChunksPerSuper;
        for (int i = 0; i < nsup; ++i, ++it) {
          if (!mbar_wait(&nib_empty[slot], ph ^ 1, p.err)) { s_abort = 1; break; }
          uint8_t* dst = nib + slot * (kNibBytes + kSclBytes);
          mbar_arrive_expect_tx(&nib_full[slot], kNibBytes + kSclBytes);
          const int ks = w.c0 / kChunksPerSuper + i;  // super-stage index along K
          tma_load_2d(dst, &tmap_w, ks * 128, w.row0, &nib_full[slot], pol);
          tma_load_2d(dst + kNibBytes, &tmap_s, ks * p.sc_x, w.row0, &nib_full[slot], pol);
          if (++slot == (uint32_t)NS) { slot = 0; ph ^= 1; }
        }
      }
      // Leave no copy in flight (matters only when a wait gave up).
      for (uint32_t i = it > (uint32_t)NS ? it - NS : 0; i < it; ++i)
        mbar_wait(&nib_full[i % NS], (i / NS) & 1, p.err);
    }
  } else if (warp == 1) {
    // ---- activation producer: kSub [Xhi | Xlo] boxes per 128-K chunk ----
    griddep_wait();
    if (lane == 0) {
      prefetch_tmap(&tmap_x);
      uint64_t keep;
      asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(keep));
      uint32_t it = 0, slot = 0, prev = 0;  // chunk counter, its B slot, chunk that last held the slot
      for (int u = blockIdx.x; u < p.units && !s_abort; u += gridDim.x) {
        const Unit w = unit_of(p, u);
        for (int i = 0; i < w.nch; ++i, ++it) {
          // The slot last held chunk it - BS; wait until its MMAs completed.
          if (it >= (uint32_t)BS) {
            if (!mbar_wait(&done[prev % kDoneRing], (prev / kDoneRing) & 1, p.err)) { s_abort = 1; break; }
            ++prev;
          }
          mbar_arrive_expect_tx(&b_full[slot], (uint32_t)(kSub * bbytes));
#pragma unroll
          for (int j = 0; j < kSub; ++j)
            tma_load_2d(btile + (slot * kSub + j) * bbytes, &tmap_x, (w.c0 + i) * kPipeK + j * kChunkK, 0,
                        &b_full[slot], keep);
          if (++slot == (uint32_t)BS) slot = 0;
        }
      }
      for (uint32_t i = it > (uint32_t)BS ? it - BS : 0; i < it; ++i)
        mbar_wait(&b_full[i % BS], (i / BS) & 1, p.err);
    }
  } else if (warp == 2) {
    // ---- MMA issuer ----
    // The whole warp runs this loop so that descriptors and TMEM addresses stay
    // warp-uniform; one lane, elected once, issues every MMA and every commit (a
    // commit tracks the MMAs of the thread that issues it).  Issuing from a
    // diverged single lane instead costs about 47 cycles per tcgen05.mma, which
    // is longer than an M128 x N64 x K16 MMA takes on the tensor pipe.
    const bool leader = elect_one();
    // A holds -Whi (negated back by the descriptor) and Wlo.
    const uint32_t id_hl = idesc_f16(2 * p.np, true), id_h = idesc_f16(p.np);
    const uint64_t bdesc0 = sdesc(smem_u32(btile));
    const uint64_t bbox = (uint64_t)(bbytes >> 4);  // descriptor address units per B box
    uint32_t ch = 0, acc_i = 0;
    uint32_t as = 0, a_ph = 0, bs = 0, b_ph = 0;  // ring positions and phases, advanced per chunk
    for (int u = blockIdx.x; u < p.units && !s_abort; u += gridDim.x) {
      const Unit w = unit_of(p, u);
      if (w.nch == 0) continue;
      const int ab = acc_i % p.acc_bufs;
      const uint32_t use = acc_i / p.acc_bufs;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_empty[ab], (use & 1) ^ 1, p.err))) { s_abort = 1; break; }
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(ab * p.acc_cols);
      bool ok = true;
      for (int i = 0; i < w.nch; ++i, ++ch) {
        if (!__all_sync(0xffffffffu,
                        mbar_wait_poll(&b_full[bs], b_ph, p.err) && mbar_wait_poll(&a_full[as], a_ph, p.err))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ahi = tmem + a_base + (uint32_t)as * kAColsPerSlot;
        const uint32_t alo = ahi + kAColsPerSlot / 2;
        const uint64_t bd = bdesc0 + (uint64_t)bs * kSub * bbox;  // +2 per 16-K step (32 bytes)
        if (leader) {
          umma_f16_ts(d, ahi, bd, id_hl, i > 0 ? 1u : 0u);  // Whi x [Xhi | Xlo]
          umma_f16_ts(d, alo, bd, id_h, 1u);                // Wlo x Xhi
#pragma unroll
          for (int kk = 1; kk < kPipeK / 16; ++kk) {
            const uint32_t ac = (uint32_t)(kk * 8);                           // 8 columns per 16 K
            const uint64_t bk = (uint64_t)((kk >> 2) * bbox + 2 * (kk & 3));  // box, then 32 B steps
            umma_f16_ts(d, ahi + ac, bd + bk, id_hl, 1u);
            umma_f16_ts(d, alo + ac, bd + bk, id_h, 1u);
          }
          umma_commit(&done[ch % kDoneRing]);  // frees A slot ch % kASlots and B slot ch % BS
        }
        __syncwarp();
        if (++as == (uint32_t)kASlots) { as = 0; a_ph ^= 1; }
        if (++bs == (uint32_t)BS) { bs = 0; b_ph ^= 1; }
      }
      if (!ok) { s_abort = 1; break; }
      if (leader) umma_commit(&acc_full[ab]);  // fires when every MMA of this unit has completed
      __syncwarp();
      ++acc_i;
    }
    if (leader) umma_commit(mma_done);  // fires once every MMA issued above has completed
    __syncwarp();
    mbar_wait(mma_done, 0, p.err);
  } else if (warp < 3 + kConvWarps) {
    // ---- converters: thread = weight row (its TMEM lane).  The two warps of a TMEM
    //      lane quarter take alternate chunks of each unit (cw = 0 the even ones,
    //      cw = 1 the odd ones), so one converts while the other waits on a
    //      barrier; each converts all four 32-code scale groups of its chunk and
    //      hands every group to TMEM (asynchronous tcgen05.st) as soon as it is done ----
    const int quarter = warp & 3;
    const int cw = (warp - 3) >> 2;
    const int rrow = quarter * 32 + lane;
    const uint32_t swz = (uint32_t)(rrow & 7);
    const uint32_t tlane = tmem + ((uint32_t)(quarter * 32) << 16) + a_base;
    uint32_t ch = 0, ns = 0, ns_ph = 0;  // chunk counter; nibble slot and phase
    for (int u = blockIdx.x; u < p.units && !s_abort; u += gridDim.x) {
      const Unit w = unit_of(p, u);
      bool ok = true;
      for (int i = 0; i < w.nch; ++i, ++ch) {
        const int sub = i % kChunksPerSuper;
        const bool stage_end = sub == kChunksPerSuper - 1 || i == w.nch - 1;
        if (sub == cw) {
          if (!__all_sync(0xffffffffu, mbar_wait_poll(&nib_full[ns], ns_ph, p.err))) {
            ok = false;
            break;
          }
          const int as = ch % kASlots;
          const uint8_t* nrow = nib + ns * (kNibBytes + kSclBytes) + rrow * 128;
          const uint8_t* srow = nib + ns * (kNibBytes + kSclBytes) + kNibBytes + rrow * 16 * S;
          const uint32_t ta = tlane + (uint32_t)as * kAColsPerSlot;
#pragma unroll
          for (int gi = 0; gi < 2 * kSub; ++gi) {
            const int grp = sub * 2 * kSub + gi;  // 32-code group within the 256-code super stage
            const uint4 g = *reinterpret_cast<const uint4*>(nrow + (((uint32_t)grp ^ swz) << 4));
            // Word j (codes 8j..8j+7) uses scale grp*S + j*S/4 of the super-stage.
            uint32_t s2w[S];
#pragma unroll
            for (int k = 0; k < S; ++k)
              s2w[k] = (uint32_t)reinterpret_cast<const uint16_t*>(srow)[grp * S + k] * 0x10001u;  // {s, s}
            const uint32_t words[4] = {g.x, g.y, g.z, g.w};
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t s2 = s2w[j * S / 4];
              const uint32_t ns2 = s2 ^ 0x80008000u;  // {-s, -s}
              uint32_t q[4];
              unpack8(words[j], q);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                hi[4 * j + e] = hmul2_u32(q[e], ns2);                // -RN(q*s)
                lo[4 * j + e] = hfma2_u32(q[e], s2, hi[4 * j + e]);  // q*s - RN(q*s), exact
              }
            }
            if (gi == 0) {
              // The A slot last held chunk ch - kASlots; wait until its MMAs completed.
              if (ch >= (uint32_t)kASlots) {
                const uint32_t prev = ch - kASlots;
                if (!__all_sync(0xffffffffu,
                                mbar_wait_poll(&done[prev % kDoneRing], (prev / kDoneRing) & 1, p.err))) {
                  ok = false;
                  break;
                }
              }
              tc_fence_after();
            }
            // Group (gsub, half) of the chunk: 16 columns at 32 * gsub + 16 * half.
            const uint32_t col = (uint32_t)(32 * (gi >> 1) + 16 * (gi & 1));
            tmem_st16(ta + col, hi);
            tmem_st16(ta + kAColsPerSlot / 2 + col, lo);
          }
          if (!ok) break;
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&a_full[as]);
            mbar_arrive(&nib_empty[ns]);
          }
        } else if (stage_end && sub < cw) {
          // The stage ended before this warp's chunk (odd chunk count): release its share.
          __syncwarp();
          if (lane == 0) mbar_arrive(&nib_empty[ns]);
        }
        if (stage_end) {
          if (++ns == (uint32_t)NS) { ns = 0; ns_ph ^= 1; }
        }
      }
      if (!ok) { s_abort = 1; break; }
    }
  } else {
    // ---- epilogue: TMEM lane = weight row; columns b (Whi-side hi) and Np + b (lo) ----
    griddep_wait();
    const int quarter = warp & 3;
    uint32_t acc_i = 0;
    for (int u = blockIdx.x; u < p.units && !s_abort; u += gridDim.x) {
      const Unit w = unit_of(p, u);
      const int row = w.row0 + quarter * 32 + lane;
      float* ybase = p.y + (size_t)w.split * p.split_stride;
      const float bias = (p.bias && w.split == 0 && row < p.M) ? p.bias[row] : 0.f;
      if (w.nch == 0) {
        // Empty K-range: this split contributes zeros (plus the bias on split 0).
        if (row < p.M)
          for (int b = 0; b < p.n; ++b) ybase[(size_t)b * p.ldy + row] = bias;
        continue;
      }
      const int ab = acc_i % p.acc_bufs;
      const uint32_t use = acc_i / p.acc_bufs;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[ab], use & 1, p.err))) { s_abort = 1; break; }
      tc_fence_after();
      const uint32_t tq = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(ab * p.acc_cols);
      for (int b0 = 0; b0 < p.np; b0 += 16) {
        float vh[16], vl[16];
        tmem_ld16(tq + (uint32_t)b0, vh);
        tmem_ld16(tq + (uint32_t)(p.np + b0), vl);
        if (row < p.M) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int b = b0 + j;
            if (b < p.n) ybase[(size_t)b * p.ldy + row] = (vh[j] + vl[j]) * p.xscale[b] + bias;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
      ++acc_i;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    // Every MMA has completed (the issuer waited on mma_done) before TMEM is released.
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// x [n, K] fp32 -> [Xhi ; Xlo] fp16 rows (Np each) in the code order
// (0,4,1,5,2,6,3,7) per 8 and xscale[row] = 2^e with max|x|/2^e in [2^14, 2^15).
__global__ void split_activation_kernel(const float* __restrict__ x, size_t ldx, int K, int np,
                                        __half* __restrict__ xs, float* __restrict__ xscale) {
  griddep_launch();
  griddep_wait();
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

// Groups 8, 16 and 32 (the maps int4_weight_prepare encodes), fp16 scales, K a
// multiple of the 128-K pipeline chunk.
bool gemm_tc_supported(const Int4Weight& w) { return w.tcg && w.f16 && w.K % kPipeK == 0; }

// Activations in split form for the GEMM: xs [2*np, K] fp16 + xscale [np].
int split_activation(const float* x, size_t ldx, size_t n, size_t K, size_t np, __half* xs, float* xscale,
                     cudaStream_t stream) {
  GLC_REQUIRE(K % 8 == 0 && n <= np, "split_activation: K %% 8 and n <= np required");
  return launch_pdl(split_activation_kernel, dim3((unsigned)n), dim3(256), 0, stream, 1, x, ldx, (int)K, (int)np, xs,
                    xscale);
}

int encode_split_map(CUtensorMap* map, const __half* xs, size_t np, size_t K) {
  return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xs, K, 2 * np, K * sizeof(__half), kChunkK,
                        (uint32_t)(2 * np), CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}

// Shared-memory rings for a padded activation width: four nibble super-stages
// (1024 K of HBM reads in flight) and as many 64-K activation tiles as fit,
// at most eight; the footprint never drops below kMinSmem so that exactly one
// CTA (which takes the whole TMEM) runs per SM.
static void gemm_slots(size_t np, int per32, int* nib, int* b) {
  *nib = 4;
  *b = kMaxSlots;
  const size_t fixed = 1024 + (size_t)(3 * kMaxSlots + kDoneRing + kASlots + 5) * 8 + 16;
  const size_t stage = (size_t)(kNibBytes + scl_bytes(per32));
  auto bytes = [&]() { return fixed + (size_t)*nib * stage + (size_t)*b * kSub * 2 * np * 128; };
  while (bytes() > 227 * 1024 && *b > 3) --*b;
  while (bytes() > 227 * 1024 && *nib > 2) --*nib;
  while (bytes() > 227 * 1024 && *b > 2) --*b;
}

size_t gemm_smem_bytes(size_t np, int per32) {
  int nib, b;
  gemm_slots(np, per32, &nib, &b);
  const size_t bytes = 1024 + (size_t)(3 * kMaxSlots + kDoneRing + kASlots + 5) * 8 + 16 +
                       (size_t)nib * (kNibBytes + scl_bytes(per32)) + (size_t)b * kSub * 2 * np * 128;
  return bytes < (size_t)kMinSmem ? (size_t)kMinSmem : bytes;
}

// The tensor core's fp32 accumulation does not round every addition, so an
// accumulation chain of n k-steps drifts by up to ~n * 2^-24 of the running
// sum.  Chains are therefore capped at kMaxChainK, and longer reductions are
// finished on the CUDA cores in rounded fp32 (split-K partials summed in order).
constexpr size_t kMaxChainK = 4096;

// Number of K splits: the persistent grid (one CTA per SM) runs units of
// (128 rows, K split) round-robin, so pick the split count that minimises the
// busiest CTA's chunk count (ties go to fewer splits: fewer partials to sum),
// with whole 256-K super-stages, no empty split and no chain above kMaxChainK.
int gemm_splits(size_t M, size_t K) {
  const long tiles = (long)ceil_div(M, kRowsTile);
  const long sup = (long)ceil_div(K, kSuperK);
  const long sms = sm_count();
  int best = 1;
  long best_cost = -1;
  for (long s = 1; s <= 16 && s <= sup; ++s) {
    const long per = (sup + s - 1) / s;       // super-stages per split
    if ((s - 1) * per >= sup) continue;       // would leave an empty split
    if ((size_t)per * kSuperK > kMaxChainK && per > 1) continue;
    const long cost = ((tiles * s + sms - 1) / sms) * per;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = (int)s;
    }
  }
  return best;
}

namespace {
__global__ void reduce_splits_kernel(const float* __restrict__ part, size_t split_stride, int nsplit,
                                     float* __restrict__ y, size_t n) {
  griddep_launch();
  griddep_wait();
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
  return launch_pdl(reduce_splits_kernel, dim3(grid), dim3(256), 0, stream, 1, part, split_stride, nsplit, y, n);
}

// y (+ split * split_stride) = X W^T for the np-padded activation block whose
// TMA map is `xmap`; nsplit K-partials are written when nsplit > 1.
int gemm_int4_tc(const Int4Weight& w, const CUtensorMap& xmap, const float* xscale, size_t n, size_t np, float* y,
                 size_t ldy, int nsplit, size_t split_stride, const float* bias, cudaStream_t stream) {
  GLC_REQUIRE(gemm_tc_supported(w), "int4 gemm: weight layout not supported by the tensor-core GEMM");
  GLC_REQUIRE(np % 16 == 0 && np >= 16 && np <= 128 && n <= np, "int4 gemm: padded rows %zu (n=%zu)", np, n);
  GLC_REQUIRE(nsplit >= 1, "int4 gemm: %d splits", nsplit);
  const int chunks = (int)(w.K / kPipeK);
  const int sup = (int)ceil_div(w.K, kSuperK);
  const int per = (int)ceil_div(sup, nsplit) * kChunksPerSuper;
  const int tiles = (int)ceil_div(w.M, kRowsTile);
  const int per32 = (int)(32 / w.group);  // scale groups per 32 codes
  const size_t smem = gemm_smem_bytes(np, per32);
  GLC_REQUIRE(smem <= 227 * 1024, "int4 gemm: %zu bytes of shared memory", smem);
  const void* kern = per32 == 1 ? (const void*)gemm_tc_kernel<1>
                     : per32 == 2 ? (const void*)gemm_tc_kernel<2> : (const void*)gemm_tc_kernel<4>;
  {
    const int rc = allow_dynamic_smem(kern, (int)smem);
    if (rc) return rc;
  }
  int* err = device_symbol_address(g_gemm_error);
  GLC_REQUIRE(err != nullptr, "int4 gemm: device status word unavailable");
  int nib_slots, b_slots;
  gemm_slots(np, per32, &nib_slots, &b_slots);
  // Accumulator columns: 2*np (hi | lo products), a power of two >= 32; two
  // buffers when they fit beside the A ring in the 512 TMEM columns.
  int acc_cols = 32;
  while (acc_cols < (int)(2 * np)) acc_cols *= 2;
  const int acc_bufs = (2 * acc_cols + kASlots * (int)kAColsPerSlot <= (int)kTmemCols) ? 2 : 1;
  GLC_REQUIRE(acc_bufs * acc_cols + kASlots * (int)kAColsPerSlot <= (int)kTmemCols, "int4 gemm: TMEM budget");
  GemmParams prm{};
  prm.xscale = xscale;
  prm.bias = bias;
  prm.y = y;
  prm.ldy = ldy;
  prm.split_stride = split_stride;
  prm.M = (int)w.M;
  prm.K = (int)w.K;
  prm.n = (int)n;
  prm.np = (int)np;
  prm.chunks_total = chunks;
  prm.chunks_per_split = per;
  prm.nsplit = nsplit;
  prm.tiles = tiles;
  prm.units = tiles * nsplit;
  prm.nib_slots = nib_slots;
  prm.b_slots = b_slots;
  prm.acc_cols = acc_cols;
  prm.acc_bufs = acc_bufs;
  prm.sc_x = 8 * per32;
  prm.err = err;
  const int grid = std::min(prm.units, sm_count());
  if (per32 == 2)
    return launch_pdl(gemm_tc_kernel<2>, dim3(grid), dim3(kThreads), smem, stream, 1, w.tmap_w, w.tmap_s, xmap, prm);
  if (per32 == 4)
    return launch_pdl(gemm_tc_kernel<4>, dim3(grid), dim3(kThreads), smem, stream, 1, w.tmap_w, w.tmap_s, xmap, prm);
  return launch_pdl(gemm_tc_kernel<1>, dim3(grid), dim3(kThreads), smem, stream, 1, w.tmap_w, w.tmap_s, xmap, prm);
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
