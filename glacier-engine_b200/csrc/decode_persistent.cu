// Persistent decode step for few lanes: the whole step (every layer, then the
// LM head) as ONE cooperative kernel with one CTA per SM.
//
// Same operator sequence as the multi-kernel step in decode.cu (the reference's
// forwardLayerCached, src/generate.zig:1511-1967, and its decode loop at
// :5366-5450), with the same arithmetic per element:
//   x = embed(token)
//   per layer:  h = rmsnorm(x (+ down_prev)) -> qkv = W_qkv h -> rope, KV append,
//               paged attention -> x += W_o a -> h2 = rmsnorm(x) -> gu = W_gu h2
//               -> down = W_d (silu(gate) * up)
//   logits = W_lm rmsnorm(x + down)
//
// Why one kernel: at one lane a 7B layer streams 131 MB of INT4 weights in
// about 20 us at HBM speed, but the multi-kernel step spends ~70 us per layer
// in a chain of ~10 dependent launches.  Here:
//  * every CTA walks a static list of every weight tile it consumes in the
//    whole step; the tiles stream with TMA into a shared-memory ring, and the
//    warp that releases a ring slot last refills it with the stage `ring`
//    places further on, so the ring keeps filling across phase boundaries and
//    grid barriers (weights never depend on activations);
//  * sixteen warps run the phases, separated by grid barriers (a global
//    arrival counter, cleared by the host before each launch; every wait is
//    bounded and a timeout raises the device error word and unwinds);
//  * each GEMV splits its (128-row tile, 256-code stage) sequence evenly over
//    the CTAs (stream-K); a tile's K-segments go to per-segment partial rows
//    that the consumers sum in segment order (deterministic, no atomics);
//  * the unpack/MMA arithmetic per stage is the tensor-core GEMV's (exact
//    (u - 7) fp16 A fragments, x as fp16 hi + lo B columns, fp32 group scales);
//  * attention items are (lane, kv head, chunk of positions); the CTA that
//    finishes a (lane, kv head) last merges its chunks (atomic arrival count);
//  * every CTA normalises the full residual row itself, so no CTA waits for
//    another to publish normalised activations.
// Reads of data other CTAs wrote during the launch bypass L1 (ld.global.cg).
#include <algorithm>
#include <memory>
#include <vector>

#include "persistent.cuh"

namespace glacier {

__device__ int g_persist_error;

namespace {

constexpr int kCW = 16;                  // consumer warps (two per 16-row tile slice of a stage)
constexpr int kCThreads = kCW * 32;      // consumer threads
constexpr int kThreadsP = kCThreads;    // every warp consumes; the last to release a stage refills it
constexpr int kTileRows = 128;
constexpr int kNib = kTileRows * 128;    // 128 rows x 256 codes
constexpr int kScl = kTileRows * 8 * 2;  // 128 rows x 8 fp16 group scales
constexpr int kStage = kNib + kScl;
constexpr int kMaxB = 4;
constexpr int kMaxG = 8;
constexpr int kNumMats = 5;              // qkv, o, gate_up, down, lm_head
constexpr int kSegSlots = 32;            // per-CTA segment counters (a warp runs at most a ring ahead)
enum { kQKV = 0, kO = 1, kGU = 2, kDN = 3, kLM = 4 };
// Device error words: 1 = a wait gave up, 2 = a token or position out of range.
constexpr int kErrBadInput = 2;

struct MatPlan {
  int M, K, S, T;  // rows, columns, 256-code stages per tile, 128-row tiles
  int per;         // stages per CTA
};

struct LayerPtrs {
  const float* bqkv;
  const float* in_norm;
  const float* post_norm;
};

struct PParams {
  const CUtensorMap* maps;  // (w, s) per matrix: layer l's qkv, o, gu, d at 2*(4l + m), LM head last
  const LayerPtrs* layers;
  const float* final_norm;
  const void* embedding;
  int emb_f32;
  const float* rope_cos;
  const float* rope_sin;
  int positions;
  float* pool;
  long long page_floats;
  const int32_t* block_tables;
  int max_pages;
  const int32_t* tokens;
  const int32_t* pos;
  int B, L, D, F, H, Hkv, hd, V;
  float eps, qscale;
  MatPlan mp[kNumMats];
  float* part[kNumMats];  // [2 * segment + K-half][B][M] partial rows
  float* out[kNumMats];   // [B][M] final rows (the LM head's only when logits are asked for)
  unsigned* tilecnt;      // per (matrix, tile): CTAs that finished their segment of it
  int tile_off[kNumMats];
  float* tw_v;            // LM head: best eligible value per (lane, tile),
  int* tw_i;              //   its index,
  int* tw_f;              //   flags (bit 0 NaN among eligible) and eligible count
  float* x0;
  float* x1;              // residual rows [B][D], alternating
  float* part_o;          // attention chunk partials [B][H][max_items][hd]
  float* part_ml;         // [B][H][max_items][2]
  int max_items;
  float* attn_out;        // [B][H * hd]
  float* logits;          // [B][V], or null: no logits written (greedy ids only)
  const uint64_t* words;  // eligibility bitsets [B][word_count], or null
  int word_count;
  int32_t* tokens_out;    // [B] greedy ids
  int32_t* status_out;    // [B] selection status
  unsigned* sync;         // [0] grid arrivals; [1 + b * Hkv + kvh] attention chunk arrivals; [1 + B * Hkv] argmax
  int* err;
  unsigned long long* phase_ns;  // optional [8] accumulated phase times (CTA 0)
  unsigned long long* phase_n;   // optional [8] phase counts
  int ring;               // ring slots
  int slots;              // B-fragment slots per matrix (max over matrices)
};

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
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
// Eight codes of one word -> four half2 of the exact integers (u - 7), pairs
// {u0,u4}, {u1,u5}, {u2,u6}, {u3,u7}: 1024 + u (or 1024 + 16u) built in the
// fp16 mantissa, then one fp16x2 FMA removes the offset.
__device__ __forceinline__ void unpack8(uint32_t w, uint32_t (&q)[4]) {
  const uint32_t w8 = w >> 8;
  const uint32_t t0 = lop3_and_or(w, 0x000F000Fu, 0x64006400u);
  const uint32_t t1 = lop3_and_or(w, 0x00F000F0u, 0x64006400u);
  const uint32_t t2 = lop3_and_or(w8, 0x000F000Fu, 0x64006400u);
  const uint32_t t3 = lop3_and_or(w8, 0x00F000F0u, 0x64006400u);
  q[0] = hfma2_u32(t0, 0x3C003C00u, 0xE407E407u);  // (1024 + u) * 1 - 1031
  q[1] = hfma2_u32(t1, 0x2C002C00u, 0xD470D470u);  // (1024 + 16u) / 16 - 71
  q[2] = hfma2_u32(t2, 0x3C003C00u, 0xE407E407u);
  q[3] = hfma2_u32(t3, 0x2C002C00u, 0xD470D470u);
}
__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}
// Scale g of four consecutive fp16 group scales, widened to fp32 with integer and
// FMA-pipe operations only (half_to_float_bits).
__device__ __forceinline__ float scale_of4(const uint2& v, int g) {
  const uint32_t w = g < 2 ? v.x : v.y;
  return half_to_float_bits((g & 1) ? (w >> 16) : (w & 0xFFFFu));
}
// Greedy candidate: a beats b with a larger value, or an equal value and a lower
// index (sampling.zig:92); i < 0 is no candidate.
struct Cand {
  float v;
  int i;
};
__device__ __forceinline__ bool better(const Cand& a, const Cand& b) {
  if (a.i < 0) return false;
  if (b.i < 0) return true;
  return a.v > b.v || (a.v == b.v && a.i < b.i);
}
__device__ __forceinline__ Cand warp_best(Cand c) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Cand t;
    t.v = __shfl_xor_sync(0xffffffffu, c.v, o);
    t.i = __shfl_xor_sync(0xffffffffu, c.i, o);
    if (better(t, c)) c = t;
  }
  return c;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Stage range of CTA `c` in a matrix's (tile, stage) sequence.
__device__ __forceinline__ void stage_range(const MatPlan& mp, int c, int& s0, int& n) {
  s0 = c * mp.per;
  n = max(0, min(s0 + mp.per, mp.T * mp.S) - s0);
}
// First CTA holding a stage of tile t, and how many CTAs do (segments of t).
__device__ __forceinline__ int seg_first(const MatPlan& mp, int t) { return (t * mp.S) / mp.per; }
__device__ __forceinline__ int seg_count(const MatPlan& mp, int t) {
  return ((t + 1) * mp.S - 1) / mp.per - (t * mp.S) / mp.per + 1;
}

struct Smem {
  uint8_t* ring;
  uint64_t* full;
  unsigned* relcnt;  // [ring] warps that released the slot's current stage
  int* nstage;       // [5] stages of each matrix per layer (this CTA), [5] = all stages
  unsigned* issued;  // [1] highest stage sequence number issued + 1
  unsigned* segcnt;  // [kSegSlots] warps that ended the CTA's segment of that sequence number
  uint4* xfrag;   // [slots][8 blocks][8 * B lanes]
  float* xs;      // [B][D] normalised rows / scratch
  float* qs;      // [G][hd] rotated, scaled q of the current attention item
  float* wpo;     // [8][G][hd] warp partials
  float* wpm;     // [8][G][2] warp (max, sum)
  float* red;     // [64]
  int* flag;      // [4]
};

struct Ctx {
  const PParams& p;
  Smem& s;
  int cta, nct, tid, warp, lane;
  unsigned target;      // grid barrier arrivals expected so far (thread 0)
  unsigned ring_pos;    // consumer position in the stage sequence
  unsigned seg_seq;     // segments this warp has ended
  int ring_slot;        // ring_pos mod ring
  uint32_t ring_par;    // (ring_pos / ring) & 1
  bool ok;
  unsigned long long t_phase;
};

// Sum over the 256 consumer threads (same order in every CTA).
__device__ float csum(Ctx& c, float v) {
  v = warp_sum(v);
  if (c.lane == 0) c.s.red[c.warp] = v;
  cbar();
  float t = c.lane < kCW ? c.s.red[c.lane] : 0.f;
  t = warp_sum(t);
  cbar();
  return t;
}

// Grid barrier over the consumer warps of every CTA; false when the launch is
// being abandoned (a wait gave up here or elsewhere).
__device__ bool grid_sync(Ctx& c, int phase_kind) {
  cbar();
  if (c.tid == 0) {
    bool ok = true;
    c.target += c.nct;
    __threadfence();
    atomicAdd(c.p.sync, 1u);
    const long long t0 = clock64();
    int it = 0;
    while (ld_acquire_u32(c.p.sync) < c.target) {
      if ((++it & 255) == 0 && (clock64() - t0 > kSpinLimitCycles || *(volatile int*)c.p.err != 0)) {
        atomicExch(c.p.err, kErrTimeout);
        ok = false;
        break;
      }
    }
    __threadfence();
    c.s.flag[0] = ok ? 0 : 1;
    if (c.cta == 0 && c.p.phase_ns && phase_kind >= 0) {
      const unsigned long long t = globaltimer_ns();
      c.p.phase_ns[phase_kind] += t - c.t_phase;
      c.p.phase_n[phase_kind] += 1;
      c.t_phase = t;
    }
  }
  cbar();
  c.ok = c.s.flag[0] == 0;
  return c.ok;
}

// x = src (+ the final rows `add` of a projection), written to dst for this
// CTA's own rows; xs = x * (1/sqrt(mean(x^2) + eps)) * w for every row.
// src_kind: 0 = fp32 rows [B][D] (cross-CTA data), 1 = fp16 embedding rows, 2 = f32 embedding rows.
__device__ void residual_norm(Ctx& c, const float* src, int src_kind, const float* add, float* dst, const float* w) {
  const PParams& p = c.p;
  const int D = p.D;
  const int own = ((D + c.nct - 1) / c.nct + 3) & ~3;
  const int r0 = c.cta * own, r1 = min(D, r0 + own);
  for (int b = 0; b < p.B; ++b) {
    float ss = 0.f;
    float* xs = c.s.xs + (size_t)b * D;
    for (int k = 4 * c.tid; k < D; k += 4 * kCThreads) {
      float4 x;
      if (src_kind == 0) {
        x = ldcg4(src + (size_t)b * D + k);
      } else {
        const int tok = p.tokens[b];
        if (src_kind == 1) {
          const __half* e = reinterpret_cast<const __half*>(p.embedding) + (size_t)tok * D + k;
          x = make_float4(__half2float(e[0]), __half2float(e[1]), __half2float(e[2]), __half2float(e[3]));
        } else {
          x = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.embedding) + (size_t)tok * D + k);
        }
      }
      if (add) {
        // addInto (generate.zig:3642).
        const float4 bv = ldcg4(add + (size_t)b * D + k);
        x.x = x.x + bv.x; x.y = x.y + bv.y; x.z = x.z + bv.z; x.w = x.w + bv.w;
      }
      *reinterpret_cast<float4*>(xs + k) = x;
      if (dst && k >= r0 && k < r1) *reinterpret_cast<float4*>(dst + (size_t)b * D + k) = x;
      ss = fmaf(x.x, x.x, ss);
      ss = fmaf(x.y, x.y, ss);
      ss = fmaf(x.z, x.z, ss);
      ss = fmaf(x.w, x.w, ss);
    }
    ss = csum(c, ss);
    const float inv = 1.0f / sqrtf(ss / (float)D + p.eps);  // rmsNormF32, kernels.zig:141
    for (int k = 4 * c.tid; k < D; k += 4 * kCThreads) {
      float4 x = *reinterpret_cast<float4*>(xs + k);
      const float4 wv = *reinterpret_cast<const float4*>(w + k);
      x = make_float4(x.x * inv * wv.x, x.y * inv * wv.y, x.z * inv * wv.z, x.w * inv * wv.w);
      *reinterpret_cast<float4*>(xs + k) = x;
    }
  }
  cbar();
}

// B fragments (x as fp16 hi + lo columns) of the 256-code stages this CTA
// needs for matrix m, from act(b, k) (k < K; 0 beyond).
template <typename Act>
__device__ void build_frags(Ctx& c, int m, Act act) {
  const PParams& p = c.p;
  const MatPlan& mp = p.mp[m];
  int s0, n;
  stage_range(mp, c.cta, s0, n);
  if (n == 0) return;
  const bool full = n >= mp.S;
  const int nslots = full ? mp.S : n, a = s0 % mp.S;
  const int flanes = 8 * p.B;
  for (int idx = c.tid; idx < nslots * 8 * flanes; idx += kCThreads) {
    const int slot = idx / (8 * flanes), rem = idx - slot * 8 * flanes;
    const int bl = rem / flanes, l = rem - bl * flanes;
    const int kst = full ? slot : (a + slot) % mp.S;
    const int nn = l >> 2, cq = l & 3, b = nn >> 1;
    const int k0 = kst * 256 + bl * 32 + 8 * cq;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (k0 + j < mp.K) ? act(b, k0 + j) : 0.f;
    __half h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __half hi = __float2half_rn(v[j]);
      h[j] = (nn & 1) ? __float2half_rn(v[j] - __half2float(hi)) : hi;
    }
    c.s.xfrag[idx] = make_uint4(pack_half2(h[0], h[4]), pack_half2(h[1], h[5]), pack_half2(h[2], h[6]),
                                pack_half2(h[3], h[7]));
  }
  cbar();
}

// Issues stage `seq` of this CTA's weight sequence (layer-major: qkv, o, gate/up,
// down of each layer, then the LM head) into its ring slot: the nibble tile
// and its fp16 scales, one mbarrier completion.  Past the end: nothing.
__device__ void issue_stage(const PParams& p, Smem& s, int cta, unsigned seq) {
  const int* ns = s.nstage;
  if (seq >= (unsigned)ns[5]) return;
  const int per_layer = ns[0] + ns[1] + ns[2] + ns[3];
  int l, m, i;
  if (seq < (unsigned)(p.L * per_layer)) {
    l = (int)seq / per_layer;
    i = (int)seq - l * per_layer;
    m = 0;
    while (i >= ns[m]) i -= ns[m++];
  } else {
    l = p.L;
    m = kLM;
    i = (int)seq - p.L * per_layer;
  }
  const MatPlan& mp = p.mp[m];
  const int st = cta * mp.per + i, tile = st / mp.S, kst = st - tile * mp.S;
  const CUtensorMap* mw = &p.maps[m == kLM ? 2 * 4 * p.L : 2 * (4 * l + m)];
  const int slot = (int)(seq % (unsigned)p.ring);
  uint8_t* dst = s.ring + (size_t)slot * kStage;
  const uint64_t pol = l2_evict_first_policy();
  mbar_arrive_expect_tx(&s.full[slot], kStage);
  tma_load_2d(dst, mw, kst * 128, tile * kTileRows, &s.full[slot], pol);
  tma_load_2d(dst + kNib, mw + 1, kst * 8, tile * kTileRows, &s.full[slot], pol);
  atomicMax(s.issued, seq + 1);
}

// Tile fixup by one warp of the CTA that finished a tile's K range last (the
// other warps keep streaming): every row of the tile is the sum of its
// 2 * nseg partial rows in order (segments in order, each one's two K-halves in
// order), written to out[m]; lane L takes rows L, L + 32, L + 64, L + 96.  For
// the LM head it also leaves the tile's best eligible logit per lane
// (argmaxEligible, sampling.zig:55-107: lowest index among equal values,
// eligible NaN flagged, eligible count).
__device__ void warp_fixup(Ctx& c, int m, int tile) {
  const PParams& p = c.p;
  const MatPlan& mp = p.mp[m];
  const int n = 2 * seg_count(mp, tile);
  const int rows = min(kTileRows, mp.M - tile * kTileRows);
  const size_t stride = (size_t)p.B * mp.M;
  __threadfence();  // acquire: the other warps' and CTAs' partial rows are published
  for (int b = 0; b < p.B; ++b) {
    const float* base = p.part[m] + (size_t)b * mp.M + tile * kTileRows;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j0 = 0; j0 < n; j0 += 4) {
      float t[4][4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int row = c.lane + 32 * r;
          t[u][r] = (j0 + u < n && row < rows) ? __ldcg(base + (size_t)(j0 + u) * stride + row) : 0.f;
        }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int r = 0; r < 4; ++r)
          if (j0 + u < n) v[r] += t[u][r];
    }
    Cand best{0.f, -1};
    int nan = 0, cnt = 0;
    const uint64_t* wr = p.words ? p.words + (size_t)b * p.word_count : nullptr;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int lr = c.lane + 32 * r;
      if (lr >= rows) continue;
      const int row = tile * kTileRows + lr;
      if (p.out[m]) p.out[m][(size_t)b * mp.M + row] = v[r];
      if (m == kLM && (!wr || ((wr[row >> 6] >> (row & 63)) & 1ull))) {
        ++cnt;
        if (v[r] != v[r]) nan = 1;
        else if (better(Cand{v[r], row}, best)) best = Cand{v[r], row};
      }
    }
    if (m == kLM) {
      best = warp_best(best);
      nan = __reduce_or_sync(0xffffffffu, nan);
      cnt = __reduce_add_sync(0xffffffffu, cnt);
      if (c.lane == 0) {
        const size_t o = (size_t)b * mp.T + tile;
        p.tw_v[o] = best.v;
        p.tw_i[o] = best.i;
        p.tw_f[2 * o] = nan;
        p.tw_f[2 * o + 1] = cnt;
      }
    }
  }
}

// This CTA's stages of matrix m from the ring: warp w takes 16 rows (w mod 8)
// and half of each stage's eight 32-code blocks (w / 8); the partials of each
// tile segment go to part[m][2 * segment + half][b][row].  A warp that ends a
// segment publishes its rows and counts itself in a per-CTA slot; the CTA's
// last such warp counts the CTA in the tile's global counter, and the warp
// that completes the tile's K range sums its partials (warp_fixup).  No other
// warp waits.
__device__ void gemv(Ctx& c, int m) {
  const PParams& p = c.p;
  const MatPlan& mp = p.mp[m];
  int s0, n;
  stage_range(mp, c.cta, s0, n);
  if (n == 0) return;
  const bool full = n >= mp.S;
  const int flanes = 8 * p.B;
  const int r = c.lane >> 2, cq = c.lane & 3;
  const bool bcol = c.lane < flanes;
  const uint32_t swz = (uint32_t)(r & 7);
  const int kh = c.warp >> 3;
  const int rho = 16 * (c.warp & 7) + r;
  float acc0 = 0.f, acc1 = 0.f;
  // Stage coordinates advance incrementally (no divisions in the loop).
  int tile = s0 / mp.S, kst = s0 - tile * mp.S;
  for (int i = 0; i < n; ++i) {
    const int slot = c.ring_slot;
    const uint32_t par = c.ring_par;
    if (!mbar_wait(&c.s.full[slot], par, p.err)) {
      c.ok = false;
      c.s.flag[1] = 1;
      return;
    }
    const uint8_t* stg = c.s.ring + (size_t)slot * kStage;
    const uint8_t* sstg = stg + kNib;
    // This half's four group scales of rows rho and rho + 8.
    const uint2 sc0 = *reinterpret_cast<const uint2*>(sstg + rho * 16 + kh * 8);
    const uint2 sc1 = *reinterpret_cast<const uint2*>(sstg + (rho + 8) * 16 + kh * 8);
    const uint8_t* rowbase = stg + rho * 128 + 4 * cq;
    const int xslot = full ? kst : i;  // slots hold stages a, a + 1, ... (mod S) in order
    const uint4* xf = c.s.xfrag + (size_t)xslot * 8 * flanes;
#pragma unroll
    for (int bb = 0; bb < 4; ++bb) {
      const int bl = 4 * kh + bb;
      const uint32_t off = ((uint32_t)bl ^ swz) << 4;
      const uint4 bf = bcol ? xf[bl * flanes + c.lane] : make_uint4(0, 0, 0, 0);
      const uint32_t w0 = *reinterpret_cast<const uint32_t*>(rowbase + off);
      const uint32_t w1 = *reinterpret_cast<const uint32_t*>(rowbase + 8 * 128 + off);
      uint32_t q0[4], q1[4];
      unpack8(w0, q0);
      unpack8(w1, q1);
      float ca[4];
      mma_16816_z(ca, q0[0], q1[0], q0[1], q1[1], bf.x, bf.y);
      mma_16816(ca, q0[2], q1[2], q0[3], q1[3], bf.z, bf.w);
      acc0 = fmaf(scale_of4(sc0, bb), ca[0] + ca[1], acc0);
      acc1 = fmaf(scale_of4(sc1, bb), ca[2] + ca[3], acc1);
    }
    __syncwarp();
    if (c.lane == 0) {
      // The last of the 16 warps to finish with the slot refills it (its reads of
      // the slot precede the asynchronous write).
      __threadfence_block();
      if (atomicAdd(&c.s.relcnt[slot], 1u) == (unsigned)kCW - 1) {
        c.s.relcnt[slot] = 0;
        __threadfence_block();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue_stage(p, c.s, c.cta, c.ring_pos + (unsigned)p.ring);
      }
    }
    ++c.ring_pos;
    if (++c.ring_slot == p.ring) {
      c.ring_slot = 0;
      c.ring_par ^= 1u;
    }
    if (i == n - 1 || kst == mp.S - 1) {  // the same stage for all 16 warps
      const int j = 2 * (c.cta - seg_first(mp, tile)) + kh;
      const int row = tile * kTileRows + rho;
      if (cq < p.B) {
        float* dst = p.part[m] + ((size_t)j * p.B + cq) * mp.M;
        if (row < mp.M) dst[row] = acc0;
        if (row + 8 < mp.M) dst[row + 8] = acc1;
      }
      acc0 = acc1 = 0.f;
      __syncwarp();
      int fix = 0;
      if (c.lane == 0) {
        __threadfence();  // this warp's partial rows, visible to every CTA
        unsigned* sc = &c.s.segcnt[c.seg_seq & (kSegSlots - 1)];
        if (atomicAdd(sc, 1u) == (unsigned)kCW - 1) {
          *sc = 0;
          const int nseg = seg_count(mp, tile);
          if (nseg == 1) {
            fix = 1;
          } else {
            unsigned* cnt = p.tilecnt + p.tile_off[m] + tile;
            if (atomicAdd(cnt, 1u) == (unsigned)nseg - 1) {
              *cnt = 0;  // ready for the next layer
              __threadfence();
              fix = 1;
            }
          }
        }
      }
      ++c.seg_seq;
      if (__shfl_sync(0xffffffffu, fix, 0)) warp_fixup(c, m, tile);
    }
    if (++kst == mp.S) {
      kst = 0;
      ++tile;
    }
  }
}

// One row of the fused q/k/v projection plus its bias.
__device__ __forceinline__ float qkv_val(const PParams& p, int b, int row, const float* bias) {
  return __ldcg(p.out[kQKV] + (size_t)b * p.mp[kQKV].M + row) + bias[row];
}

// Attention for every lane: items (lane, kv head, chunk of `cp` positions); this
// CTA takes items cta, cta + nct, ...  The CTA holding a (lane, kv head)'s last
// chunk first writes the rotated k and the v row of the new position into the
// page (the KV append).  Each warp takes a share of the chunk, two positions
// per step; the CTA merges its warps and leaves one partial (max, sum,
// unnormalised o) per query head; the CTA finishing a (lane, kv head) last
// merges the chunks, in chunk order, into attn_out.
template <int HD>
__device__ void attention(Ctx& c, int layer, const int* ctxs, const int* items_b, int total_items, int cp) {
  const PParams& p = c.p;
  constexpr int VD = HD / 32;
  constexpr float kLog2e = 1.4426950408889634f;
  const int G = p.H / p.Hkv, half = HD / 2;
  const int qd = p.H * HD, kvd = p.Hkv * HD;
  const float* bias = p.layers[layer].bqkv;
  for (int it = c.cta; it < total_items; it += c.nct) {
    int b = 0, base = 0;
    while (it >= base + p.Hkv * items_b[b]) {
      base += p.Hkv * items_b[b];
      ++b;
    }
    const int nb = items_b[b];
    const int kvh = (it - base) / nb, chunk = (it - base) - kvh * nb;
    const int ctx = ctxs[b], ps = ctx - 1;
    const int j0 = chunk * cp, j1 = min(ctx, j0 + cp);
    const float* ct = p.rope_cos + (size_t)ps * half;
    const float* st = p.rope_sin + (size_t)ps * half;
    // q of the G heads: bias, NeoX rotation, then 1/sqrt(hd) * log2(e) (softmax in base 2).
    for (int idx = c.tid; idx < G * half; idx += kCThreads) {
      const int g = idx / half, i = idx - g * half;
      const int r0 = (kvh * G + g) * HD + i;
      const float x0 = qkv_val(p, b, r0, bias), x1 = qkv_val(p, b, r0 + half, bias);
      const float cs = ct[i], sn = st[i];
      c.s.qs[g * HD + i] = (x0 * cs - x1 * sn) * p.qscale;
      c.s.qs[g * HD + i + half] = (x0 * sn + x1 * cs) * p.qscale;
    }
    if (j1 == ctx) {
      // KV append of the new position (paged_kv_cache.zig:1074): page slot (ps / 16, ps % 16).
      const int32_t page = p.block_tables[(size_t)b * p.max_pages + (ps >> 4)];
      float* kdst = p.pool + (size_t)page * p.page_floats + ((size_t)(layer * 2 + 0) * 16 + (ps & 15)) * kvd + kvh * HD;
      float* vdst = p.pool + (size_t)page * p.page_floats + ((size_t)(layer * 2 + 1) * 16 + (ps & 15)) * kvd + kvh * HD;
      for (int i = c.tid; i < half; i += kCThreads) {
        const int r0 = qd + kvh * HD + i;
        const float x0 = qkv_val(p, b, r0, bias), x1 = qkv_val(p, b, r0 + half, bias);
        const float cs = ct[i], sn = st[i];
        kdst[i] = x0 * cs - x1 * sn;
        kdst[i + half] = x0 * sn + x1 * cs;
      }
      for (int d = c.tid; d < HD; d += kCThreads) vdst[d] = qkv_val(p, b, qd + kvd + kvh * HD + d, bias);
    }
    cbar();
    // ---- each warp: a contiguous share of [j0, j1), two positions per step ----
    float mrun[kMaxG], lrun[kMaxG], o[kMaxG][VD];
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
      mrun[g] = -INFINITY;
      lrun[g] = 0.f;
#pragma unroll
      for (int i = 0; i < VD; ++i) o[g][i] = 0.f;
    }
    const int share = (j1 - j0 + kCW - 1) / kCW;
    const int w0 = j0 + c.warp * share, w1 = min(j1, w0 + share);
    const int gme = (c.lane >> 1) & 7, ume = c.lane >> 4;  // the (position, head) whose score this lane ends with
    for (int jj = w0; jj < w1; jj += 2) {
      float kv[2][VD], vv[2][VD];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int j = min(jj + u, w1 - 1);
        const int32_t page = p.block_tables[(size_t)b * p.max_pages + (j >> 4)];
        const float* kr = p.pool + (size_t)page * p.page_floats + ((size_t)(layer * 2 + 0) * 16 + (j & 15)) * kvd +
                          kvh * HD + c.lane * VD;
        const float* vr = kr + (size_t)16 * kvd;
        if constexpr (VD == 4) {
          const float4 a4 = __ldcg(reinterpret_cast<const float4*>(kr));
          const float4 b4 = __ldcg(reinterpret_cast<const float4*>(vr));
          kv[u][0] = a4.x; kv[u][1] = a4.y; kv[u][2] = a4.z; kv[u][3] = a4.w;
          vv[u][0] = b4.x; vv[u][1] = b4.y; vv[u][2] = b4.z; vv[u][3] = b4.w;
        } else {
          const float2 a2 = __ldcg(reinterpret_cast<const float2*>(kr));
          const float2 b2 = __ldcg(reinterpret_cast<const float2*>(vr));
          kv[u][0] = a2.x; kv[u][1] = a2.y;
          vv[u][0] = b2.x; vv[u][1] = b2.y;
        }
      }
      // Scores of 2 positions x 8 heads: 16 lane-partial dot products, reduced by a
      // transposing butterfly; lanes L and L ^ 1 end with value L >> 1 = 8 u + g.
      float v[16];
#pragma unroll
      for (int g = 0; g < kMaxG; ++g) {
        float q[VD];
        if (g < G) {
          if constexpr (VD == 4) {
            const float4 t = *reinterpret_cast<const float4*>(c.s.qs + g * HD + c.lane * 4);
            q[0] = t.x; q[1] = t.y; q[2] = t.z; q[3] = t.w;
          } else {
            const float2 t = *reinterpret_cast<const float2*>(c.s.qs + g * HD + c.lane * 2);
            q[0] = t.x; q[1] = t.y;
          }
        } else {
#pragma unroll
          for (int i = 0; i < VD; ++i) q[i] = 0.f;
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          float a = 0.f;
#pragma unroll
          for (int i = 0; i < VD; ++i) a = fmaf(q[i], kv[u][i], a);
          v[u * 8 + g] = a;
        }
      }
#pragma unroll
      for (int sh = 16; sh >= 2; sh >>= 1) {
        const int cnt = sh / 2;
        const bool upper = (c.lane & sh) != 0;
#pragma unroll
        for (int k = 0; k < cnt; ++k) {
          const float send = upper ? v[k] : v[k + cnt];
          const float keep = upper ? v[k + cnt] : v[k];
          v[k] = keep + __shfl_xor_sync(0xffffffffu, send, sh);
        }
      }
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
      const bool valid = (jj + ume < w1) && gme < G;
      const float sc = valid ? v[0] : -INFINITY;
      // Per head: max over the 2 positions (lanes 2g (+1) and 16 + 2g (+1)).
      const float mx = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 16));
      float mnew[kMaxG], alpha[kMaxG], mh = -INFINITY;
#pragma unroll
      for (int g = 0; g < kMaxG; ++g) {
        mnew[g] = fmaxf(mrun[g], __shfl_sync(0xffffffffu, mx, 2 * g));
        alpha[g] = mrun[g] == -INFINITY ? 0.f : ex2_approx(mrun[g] - mnew[g]);
        if (g == gme) mh = mnew[g];
      }
      const float e = (valid && mh != -INFINITY) ? ex2_approx(sc - mh) : 0.f;
      const float es = e + __shfl_xor_sync(0xffffffffu, e, 16);
#pragma unroll
      for (int g = 0; g < kMaxG; ++g) {
        lrun[g] = lrun[g] * alpha[g] + __shfl_sync(0xffffffffu, es, 2 * g);
        mrun[g] = mnew[g];
        const float p0 = __shfl_sync(0xffffffffu, e, 2 * g), p1 = __shfl_sync(0xffffffffu, e, 16 + 2 * g);
#pragma unroll
        for (int i = 0; i < VD; ++i) o[g][i] = fmaf(p1, vv[1][i], fmaf(p0, vv[0][i], o[g][i] * alpha[g]));
      }
    }
    // ---- warp partials -> one chunk partial: warps 8..15 fold into warps 0..7, then 8 merge ----
    float* wpo = c.s.wpo;  // [8][G][HD]
    float* wpm = c.s.wpm;  // [8][G][2]
    const int wl = c.warp & 7;
    auto put = [&]() {
#pragma unroll
      for (int g = 0; g < kMaxG; ++g)
        if (g < G) {
#pragma unroll
          for (int i = 0; i < VD; ++i) wpo[((size_t)wl * G + g) * HD + c.lane * VD + i] = o[g][i];
          if (c.lane == 0) {
            wpm[(wl * G + g) * 2 + 0] = mrun[g];
            wpm[(wl * G + g) * 2 + 1] = lrun[g];
          }
        }
    };
    if (c.warp >= 8) put();
    cbar();
    if (c.warp < 8) {
#pragma unroll
      for (int g = 0; g < kMaxG; ++g)
        if (g < G) {
          const float m2 = wpm[(wl * G + g) * 2 + 0], l2 = wpm[(wl * G + g) * 2 + 1];
          const float M = fmaxf(mrun[g], m2);
          const float f1 = mrun[g] == -INFINITY ? 0.f : ex2_approx(mrun[g] - M);
          const float f2 = m2 == -INFINITY ? 0.f : ex2_approx(m2 - M);
#pragma unroll
          for (int i = 0; i < VD; ++i)
            o[g][i] = o[g][i] * f1 + wpo[((size_t)wl * G + g) * HD + c.lane * VD + i] * f2;
          lrun[g] = lrun[g] * f1 + l2 * f2;
          mrun[g] = M;
        }
    }
    cbar();
    if (c.warp < 8) put();
    cbar();
    const size_t pbase = ((size_t)b * p.H + (size_t)kvh * G) * p.max_items + chunk;
    for (int idx = c.tid; idx < G * HD; idx += kCThreads) {
      const int g = idx / HD, d = idx - g * HD;
      float M = -INFINITY;
      for (int w = 0; w < 8; ++w) M = fmaxf(M, wpm[(w * G + g) * 2]);
      float acc = 0.f, L = 0.f;
      for (int w = 0; w < 8; ++w) {
        const float mw = wpm[(w * G + g) * 2];
        const float f = (mw == -INFINITY) ? 0.f : ex2_approx(mw - M);
        acc = fmaf(wpo[((size_t)w * G + g) * HD + d], f, acc);
        L = fmaf(wpm[(w * G + g) * 2 + 1], f, L);
      }
      p.part_o[(pbase + (size_t)g * p.max_items) * HD + d] = acc;
      if (d == 0) {
        p.part_ml[(pbase + (size_t)g * p.max_items) * 2 + 0] = M / kLog2e;  // natural-log units
        p.part_ml[(pbase + (size_t)g * p.max_items) * 2 + 1] = L;
      }
    }
    __threadfence();
    cbar();
    if (c.tid == 0) {
      unsigned* cnt = p.sync + 1 + b * p.Hkv + kvh;
      const unsigned prev = atomicAdd(cnt, 1u);
      const bool last = prev == (unsigned)nb - 1;
      if (last) {
        *cnt = 0;  // ready for the next layer
        __threadfence();
      }
      c.s.flag[2] = last ? 1 : 0;
    }
    cbar();
    if (c.s.flag[2]) {
      // out = sum_c o_c e^(m_c - M) / sum_c l_c e^(m_c - M), chunks in order.  A warp per
      // head turns the chunks' (max, sum) into normalised weights; then two threads per
      // 4 output values take the even and the odd chunks, loads batched by eight.
      float* wts = c.s.xs;  // [G][nb] (q and the warp partials are no longer needed)
      if (c.warp < G) {
        const int g = c.warp;
        const size_t hb = ((size_t)b * p.H + (size_t)kvh * G + g) * p.max_items;
        float M = -INFINITY;
        for (int ch = c.lane; ch < nb; ch += 32) M = fmaxf(M, __ldcg(p.part_ml + (hb + ch) * 2));
        M = warp_max(M);
        float L = 0.f;
        for (int ch = c.lane; ch < nb; ch += 32) {
          const float mc = __ldcg(p.part_ml + (hb + ch) * 2);
          const float f = mc == -INFINITY ? 0.f : expf(mc - M);
          L = fmaf(__ldcg(p.part_ml + (hb + ch) * 2 + 1), f, L);
          wts[g * nb + ch] = f;
        }
        L = warp_sum(L);
        const float inv = 1.0f / L;
        for (int ch = c.lane; ch < nb; ch += 32) wts[g * nb + ch] *= inv;
      }
      cbar();
      const int cols = G * HD / 4;
      float4* red4 = reinterpret_cast<float4*>(c.s.wpo);  // [cols] odd-chunk sums
      const int col = c.tid % cols, par = c.tid / cols;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      if (par < 2) {
        const int g = (4 * col) / HD, d = 4 * col - g * HD;
        const float* po = p.part_o + (((size_t)b * p.H + (size_t)kvh * G + g) * p.max_items) * HD + d;
        for (int c0 = par; c0 < nb; c0 += 16) {
          float4 t[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int ch = c0 + 2 * u;
            t[u] = ch < nb ? ldcg4(po + (size_t)ch * HD) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int ch = c0 + 2 * u;
            const float w = ch < nb ? wts[g * nb + ch] : 0.f;
            acc.x = fmaf(t[u].x, w, acc.x); acc.y = fmaf(t[u].y, w, acc.y);
            acc.z = fmaf(t[u].z, w, acc.z); acc.w = fmaf(t[u].w, w, acc.w);
          }
        }
        if (par == 1) red4[col] = acc;
      }
      cbar();
      if (par == 0) {
        const float4 t = red4[col];
        const int g = (4 * col) / HD, d = 4 * col - g * HD;
        *reinterpret_cast<float4*>(p.attn_out + (size_t)b * qd + (kvh * G + g) * HD + d) =
            make_float4(acc.x + t.x, acc.y + t.y, acc.z + t.z, acc.w + t.w);
      }
    }
    cbar();
  }
}

template <int HD>
__global__ void __launch_bounds__(kThreadsP, 1) persistent_decode_kernel(const __grid_constant__ PParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Smem s;
  const int G = p.H / p.Hkv;
  s.ring = base;
  uint8_t* q = base + (size_t)p.ring * kStage;
  s.full = reinterpret_cast<uint64_t*>(q);
  s.relcnt = reinterpret_cast<unsigned*>(s.full + p.ring);
  q += 2 * p.ring * sizeof(uint64_t);
  q = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(q) + 15) & ~uintptr_t(15));
  s.xfrag = reinterpret_cast<uint4*>(q);
  q += (size_t)p.slots * 8 * 8 * p.B * 16;
  s.xs = reinterpret_cast<float*>(q);
  // Attention scratch shares the space after the fragments with xs (phases do not overlap).
  const size_t xs_bytes = (size_t)p.B * p.D * 4;
  const size_t att_bytes = ((size_t)G * HD + (size_t)8 * G * HD + (size_t)8 * G * 2) * 4;
  s.qs = s.xs;
  s.wpo = s.qs + G * HD;
  s.wpm = s.wpo + 8 * G * HD;
  q += std::max(xs_bytes, att_bytes);
  s.red = reinterpret_cast<float*>(q);
  s.flag = reinterpret_cast<int*>(s.red + 64);
  s.nstage = s.flag + 4;
  s.issued = reinterpret_cast<unsigned*>(s.nstage + 6);
  s.segcnt = s.issued + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nct = gridDim.x, cta = blockIdx.x;

  // Lane contexts and input checks (every CTA decides identically).
  __shared__ int ctxs[kMaxB], items_b[kMaxB], sh_total, sh_cp, sh_bad;
  if (tid == 0) {
    int bad = 0, tot = 0;
    for (int b = 0; b < p.B; ++b) {
      const int ps = p.pos[b], tok = p.tokens[b];
      if (ps < 0 || ps >= p.positions || (ps >> 4) >= p.max_pages || tok < 0 || tok >= p.V) bad = 1;
      ctxs[b] = ps + 1;
      tot += ps + 1;
    }
    // Chunk length: about one (lane, kv head, chunk) item per two CTAs, a multiple of 16
    // positions (longer chunks keep the merge of a (lane, kv head) short).
    int cp = ((2 * p.Hkv * tot + nct - 1) / nct + 15) & ~15;
    cp = max(cp, 16);
    int total = 0;
    for (int b = 0; b < p.B; ++b) {
      items_b[b] = (ctxs[b] + cp - 1) / cp;
      if (items_b[b] > p.max_items) bad = 1;
      total += p.Hkv * items_b[b];
    }
    sh_total = total;
    sh_cp = cp;
    sh_bad = bad;
    for (int i = 0; i < p.ring; ++i) {
      mbar_init(&s.full[i], 1);
      s.relcnt[i] = 0;
    }
    fence_mbar_init();
    s.flag[0] = s.flag[1] = s.flag[2] = s.flag[3] = 0;
    int all = 0;
    for (int m = 0; m < kNumMats; ++m) {
      int s0, n;
      stage_range(p.mp[m], cta, s0, n);
      s.nstage[m] = n;
      all += m == kLM ? n : p.L * n;
    }
    s.nstage[5] = all;
    *s.issued = 0;
    for (int i = 0; i < kSegSlots; ++i) s.segcnt[i] = 0;
  }
  __syncthreads();
  if (sh_bad) {
    if (tid == 0 && cta == 0) {
      atomicExch(p.err, kErrBadInput);
      for (int b = 0; b < p.B; ++b) {
        p.tokens_out[b] = -1;
        if (p.status_out) p.status_out[b] = GLACIER_CUDA_EINVAL;
      }
    }
    return;
  }

  if (tid == 0)
    for (int i = 0; i < p.ring; ++i) issue_stage(p, s, cta, (unsigned)i);

  // ---------------- the step ----------------
  auto run = [&]() {
    Ctx c{p, s, cta, nct, tid, warp, lane, 0u, 0u, 0u, 0, 0u, true, 0ull};
    if (tid == 0 && cta == 0 && p.phase_ns) c.t_phase = globaltimer_ns();
    const int D = p.D, F = p.F;
    for (int l = 0; l < p.L; ++l) {
      const LayerPtrs Lp = p.layers[l];
      // A: x (+ down of the previous layer) -> x1; rmsnorm -> q/k/v projection.
      residual_norm(c, l == 0 ? nullptr : p.x0, l == 0 ? (p.emb_f32 ? 2 : 1) : 0,
                    l == 0 ? nullptr : p.out[kDN], p.x1, Lp.in_norm);
      build_frags(c, kQKV, [&](int b, int k) { return c.s.xs[b * D + k]; });
      gemv(c, kQKV);
      if (!grid_sync(c, 0)) return;
      // B: RoPE, KV append, attention.
      attention<HD>(c, l, ctxs, items_b, sh_total, sh_cp);
      if (!grid_sync(c, 1)) return;
      // C: o projection of the attention output.
      build_frags(c, kO, [&](int b, int k) { return __ldcg(p.attn_out + (size_t)b * p.H * p.hd + k); });
      gemv(c, kO);
      if (!grid_sync(c, 2)) return;
      // D: x1 + o -> x0; rmsnorm -> gate/up projection.
      residual_norm(c, p.x1, 0, p.out[kO], p.x0, Lp.post_norm);
      build_frags(c, kGU, [&](int b, int k) { return c.s.xs[b * D + k]; });
      gemv(c, kGU);
      if (!grid_sync(c, 3)) return;
      // E: silu(gate) * up (kernels.zig:465) -> down projection.
      build_frags(c, kDN, [&](int b, int k) {
        const float* gu = p.out[kGU] + (size_t)b * 2 * F;
        const float g = __ldcg(gu + k), u = __ldcg(gu + F + k);
        return g * (1.0f / (1.0f + expf(-g))) * u;
      });
      gemv(c, kDN);
      if (!grid_sync(c, 4)) return;
    }
    // F: final residual + rmsnorm -> LM head.
    residual_norm(c, p.x0, 0, p.out[kDN], nullptr, p.final_norm);
    build_frags(c, kLM, [&](int b, int k) { return c.s.xs[b * D + k]; });
    gemv(c, kLM);
    if (!grid_sync(c, 5)) return;
    // G: the greedy id of each lane from the LM head tiles' winners (CTA 0, a warp
    // per lane): argmaxEligible over the whole vocabulary (sampling.zig:55-107).
    if (cta == 0 && warp < p.B) {
      const int b = warp;
      const int T = p.mp[kLM].T;
      Cand bb{0.f, -1};
      int nan = 0;
      long long elig = 0;
      for (int t0 = lane; t0 < T; t0 += 32 * 4) {
        Cand tc[4];
        int fl[4], el[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int t = t0 + 32 * u;
          const size_t o = (size_t)b * T + t;
          tc[u] = t < T ? Cand{__ldcg(p.tw_v + o), __ldcg(p.tw_i + o)} : Cand{0.f, -1};
          fl[u] = t < T ? __ldcg(p.tw_f + 2 * o) : 0;
          el[u] = t < T ? __ldcg(p.tw_f + 2 * o + 1) : 0;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (better(tc[u], bb)) bb = tc[u];
          nan |= fl[u] & 1;
          elig += el[u];
        }
      }
      bb = warp_best(bb);
      nan = __reduce_or_sync(0xffffffffu, nan);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) elig += __shfl_xor_sync(0xffffffffu, elig, o);
      if (lane == 0) {
        // Tail bits past V in the mask's last word must be clear.
        const int V = p.V;
        const uint64_t* wr = p.words ? p.words + (size_t)b * p.word_count : nullptr;
        const bool tail = wr && (V & 63) && (wr[p.word_count - 1] & ~((1ull << (V & 63)) - 1));
        int st = GLACIER_CUDA_OK;
        if (wr && (tail || elig == 0)) st = GLACIER_CUDA_EMASK;
        else if (nan) st = GLACIER_CUDA_ENAN;
        else if (bb.i < 0) st = GLACIER_CUDA_EMASK;
        p.tokens_out[b] = st == GLACIER_CUDA_OK ? bb.i : -1;
        if (p.status_out) p.status_out[b] = st;
      }
    }
    if (tid == 0 && cta == 0 && p.phase_ns) {
      const unsigned long long t = globaltimer_ns();
      p.phase_ns[6] += t - c.t_phase;
      p.phase_n[6] += 1;
    }
  };
  run();
  // Leave no copy in flight (after a wait gave up, some stages were never consumed).
  __syncthreads();
  if (tid == 0) {
    const unsigned hi = *(volatile unsigned*)s.issued;
    for (unsigned i = hi > (unsigned)p.ring ? hi - p.ring : 0; i < hi; ++i)
      mbar_wait(&s.full[i % p.ring], (i / p.ring) & 1, p.err);
  }
}

MatPlan make_plan(size_t M, size_t K, int nct) {
  MatPlan mp;
  mp.M = (int)M;
  mp.K = (int)K;
  mp.S = (int)ceil_div(K, 256);
  mp.T = (int)ceil_div(M, kTileRows);
  mp.per = (int)ceil_div((size_t)mp.T * mp.S, (size_t)nct);
  return mp;
}

int seg_max(const MatPlan& mp) {
  int mx = 1;
  for (int t = 0; t < mp.T; ++t)
    mx = std::max(mx, ((t + 1) * mp.S - 1) / mp.per - (t * mp.S) / mp.per + 1);
  return mx;
}

struct DevMem {
  void* p = nullptr;
  ~DevMem() {
    if (p) cudaFree(p);
  }
  int alloc(size_t n) {
    if (cudaMalloc(&p, n) != cudaSuccess) {
      cudaGetLastError();
      p = nullptr;
      return set_error(GLACIER_CUDA_ENOMEM, "persistent step: cudaMalloc(%zu) failed", n);
    }
    return GLACIER_CUDA_OK;
  }
};

}  // namespace

struct PersistState {
  PParams prm;
  int device = 0;
  size_t smem = 0;
  int grid = 0;
  size_t max_lanes = 0, max_pages = 0;
  DevMem maps, layers, parts, outs, x, att_o, att_ml, attn_out, tiles, sync, stats;
  int tiles_total = 0;
  const void* kern = nullptr;
};

void persist_destroy(PersistState* s) { delete s; }

int persist_create(const PersistModel& pm, size_t max_lanes, size_t max_pages, PersistState** out) {
  *out = nullptr;
  if (max_lanes < 1 || max_lanes > 1) return GLACIER_CUDA_EUNSUPPORTED;
  if (pm.hd != 64 && pm.hd != 128) return GLACIER_CUDA_EUNSUPPORTED;
  if (pm.H % pm.Hkv != 0 || pm.H / pm.Hkv > kMaxG || pm.D % 4 != 0) return GLACIER_CUDA_EUNSUPPORTED;
  for (const Int4Weight* w : pm.w)
    if (!w || !w->tc || !w->f16 || w->nonfinite || w->group != 32) return GLACIER_CUDA_EUNSUPPORTED;
  auto st = std::make_unique<PersistState>();
  GLC_CHECK_CUDA(cudaGetDevice(&st->device));
  const int nct = sm_count();
  const int B = (int)max_lanes;
  PParams& p = st->prm;
  p = PParams{};
  p.B = B;
  p.L = pm.L;
  p.D = pm.D;
  p.F = pm.F;
  p.H = pm.H;
  p.Hkv = pm.Hkv;
  p.hd = pm.hd;
  p.V = pm.V;
  p.eps = pm.eps;
  p.qscale = (1.0f / sqrtf((float)pm.hd)) * 1.4426950408889634f;
  p.positions = pm.positions;
  p.emb_f32 = pm.emb_f32;
  p.embedding = pm.embedding;
  p.rope_cos = pm.rope_cos;
  p.rope_sin = pm.rope_sin;
  p.final_norm = pm.final_norm;
  const size_t qd = (size_t)pm.H * pm.hd, kvd = (size_t)pm.Hkv * pm.hd;
  const size_t Ms[kNumMats] = {qd + 2 * kvd, (size_t)pm.D, 2 * (size_t)pm.F, (size_t)pm.D, (size_t)pm.V};
  const size_t Ks[kNumMats] = {(size_t)pm.D, qd, (size_t)pm.D, (size_t)pm.F, (size_t)pm.D};
  size_t part_floats = 0, out_floats = 0;
  int slots = 1, tiles_total = 0;
  for (int m = 0; m < kNumMats; ++m) {
    if (Ms[m] % 4 != 0) return GLACIER_CUDA_EUNSUPPORTED;  // float4 partial rows
    p.mp[m] = make_plan(Ms[m], Ks[m], nct);
    part_floats += (size_t)2 * seg_max(p.mp[m]) * B * Ms[m];
    if (m != kLM) out_floats += (size_t)B * Ms[m];
    p.tile_off[m] = tiles_total;
    tiles_total += p.mp[m].T;
    slots = std::max(slots, std::min(p.mp[m].S, p.mp[m].per));
    GLC_REQUIRE(Ks[m] % 32 == 0, "persistent step: K %zu is not whole groups", Ks[m]);
  }
  p.slots = slots;
  // Shared memory: the ring takes what the rest leaves (at most 12 stages).
  const int G = pm.H / pm.Hkv;
  const size_t frag = (size_t)slots * 8 * 8 * B * 16;
  // The attention merge's weight table ([G][chunks]) also lives here.
  const size_t xs = std::max({(size_t)B * pm.D * 4, ((size_t)G * pm.hd * 9 + (size_t)8 * G * 2) * 4,
                              (size_t)G * max_pages * 4});
  const size_t fixed = 1024 + frag + xs + 64 * 4 + 16 + 64 + kSegSlots * 4;
  int dev_max = 0;
  GLC_CHECK_CUDA(cudaDeviceGetAttribute(&dev_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, st->device));
  const size_t avail = (size_t)dev_max - 1024;  // room for the kernel's static shared memory
  if (fixed + 4 * (kStage + 16) > avail)
    return set_error(GLACIER_CUDA_EUNSUPPORTED, "persistent step: %zu bytes of shared memory leave no ring", fixed);
  p.ring = (int)std::min<size_t>(12, (avail - fixed) / (kStage + 16));
  st->smem = fixed + (size_t)p.ring * (kStage + 16);
  // Device buffers.
  const size_t nmaps = (size_t)(4 * pm.L + 1) * 2;
  std::vector<CUtensorMap> hmaps(nmaps);
  for (size_t i = 0; i < pm.w.size(); ++i) {
    hmaps[2 * i] = pm.w[i]->tmap_w;
    hmaps[2 * i + 1] = pm.w[i]->tmap_s;
  }
  std::vector<LayerPtrs> hl(pm.L);
  for (int l = 0; l < pm.L; ++l) hl[l] = LayerPtrs{pm.bqkv[l], pm.in_norm[l], pm.post_norm[l]};
  p.max_items = (int)max_pages;  // chunks are at least 16 positions
  int rc;
  if ((rc = st->maps.alloc(nmaps * sizeof(CUtensorMap))) || (rc = st->layers.alloc(hl.size() * sizeof(LayerPtrs))) ||
      (rc = st->parts.alloc(part_floats * 4)) || (rc = st->x.alloc(2 * (size_t)B * pm.D * 4)) ||
      (rc = st->att_o.alloc((size_t)B * pm.H * p.max_items * pm.hd * 4)) ||
      (rc = st->att_ml.alloc((size_t)B * pm.H * p.max_items * 2 * 4)) ||
      (rc = st->attn_out.alloc((size_t)B * qd * 4)) || (rc = st->outs.alloc(out_floats * 4)) ||
      (rc = st->tiles.alloc((size_t)B * p.mp[kLM].T * 16)) ||
      (rc = st->sync.alloc(((size_t)1 + B * pm.Hkv + tiles_total) * 4)) || (rc = st->stats.alloc(16 * 8)))
    return rc;
  st->tiles_total = tiles_total;
  GLC_CHECK_CUDA(cudaMemcpy(st->maps.p, hmaps.data(), nmaps * sizeof(CUtensorMap), cudaMemcpyHostToDevice));
  GLC_CHECK_CUDA(cudaMemcpy(st->layers.p, hl.data(), hl.size() * sizeof(LayerPtrs), cudaMemcpyHostToDevice));
  GLC_CHECK_CUDA(cudaMemset(st->sync.p, 0, ((size_t)1 + B * pm.Hkv + tiles_total) * 4));
  GLC_CHECK_CUDA(cudaMemset(st->stats.p, 0, 16 * 8));
  p.maps = static_cast<const CUtensorMap*>(st->maps.p);
  p.layers = static_cast<const LayerPtrs*>(st->layers.p);
  float* part = static_cast<float*>(st->parts.p);
  for (int m = 0; m < kNumMats; ++m) {
    p.part[m] = part;
    part += (size_t)2 * seg_max(p.mp[m]) * B * Ms[m];
  }
  p.x0 = static_cast<float*>(st->x.p);
  p.x1 = p.x0 + (size_t)B * pm.D;
  p.part_o = static_cast<float*>(st->att_o.p);
  p.part_ml = static_cast<float*>(st->att_ml.p);
  p.attn_out = static_cast<float*>(st->attn_out.p);
  float* outs = static_cast<float*>(st->outs.p);
  for (int m = 0; m < kLM; ++m) {
    p.out[m] = outs;
    outs += (size_t)B * Ms[m];
  }
  p.out[kLM] = nullptr;  // set per step: the caller's logits buffer, or none
  p.tw_v = static_cast<float*>(st->tiles.p);
  p.tw_i = reinterpret_cast<int*>(p.tw_v + (size_t)B * p.mp[kLM].T);
  p.tw_f = p.tw_i + (size_t)B * p.mp[kLM].T;
  p.sync = static_cast<unsigned*>(st->sync.p);
  p.tilecnt = p.sync + 1 + (size_t)B * pm.Hkv;
  p.err = device_symbol_address(g_persist_error);
  GLC_REQUIRE(p.err != nullptr, "persistent step: device status word unavailable");
  st->kern = pm.hd == 128 ? (const void*)persistent_decode_kernel<128> : (const void*)persistent_decode_kernel<64>;
  if ((rc = allow_dynamic_smem(st->kern, (int)st->smem))) return rc;
  int occ = 0;
  GLC_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, st->kern, kThreadsP, st->smem));
  if (occ < 1)
    return set_error(GLACIER_CUDA_EUNSUPPORTED, "persistent step: a %d-thread CTA with %zu bytes of shared memory "
                     "does not fit on an SM", kThreadsP, st->smem);
  st->grid = nct;
  st->max_lanes = max_lanes;
  st->max_pages = max_pages;
  *out = st.release();
  return GLACIER_CUDA_OK;
}

int persist_step(PersistState* st, size_t lanes, const int32_t* tokens, const int32_t* positions,
                 const int32_t* block_tables, size_t max_pages, float* pool, size_t page_floats, bool profile,
                 const uint64_t* eligible, size_t eligible_words, int32_t* tokens_out, int32_t* status_out,
                 float* logits_out, cudaStream_t stream) {
  GLC_REQUIRE(st && lanes == (size_t)st->prm.B, "persistent step: %zu lanes, built for %d", lanes, st->prm.B);
  PParams p = st->prm;
  p.tokens = tokens;
  p.pos = positions;
  p.block_tables = block_tables;
  p.max_pages = (int)max_pages;
  p.pool = pool;
  p.page_floats = (long long)page_floats;
  GLC_REQUIRE(tokens_out, "persistent step: null token output");
  GLC_REQUIRE(!eligible || eligible_words == ceil_div((size_t)p.V, 64), "persistent step: eligible mask words");
  p.logits = logits_out;
  p.out[kLM] = logits_out;
  p.words = eligible;
  p.word_count = (int)eligible_words;
  p.tokens_out = tokens_out;
  p.status_out = status_out;
  unsigned long long* stats = static_cast<unsigned long long*>(st->stats.p);
  p.phase_ns = profile ? stats : nullptr;
  p.phase_n = profile ? stats + 8 : nullptr;
  GLC_CHECK_CUDA(cudaMemsetAsync(st->sync.p, 0, ((size_t)1 + p.B * p.Hkv + st->tiles_total) * 4, stream));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)st->grid);
  cfg.blockDim = dim3(kThreadsP);
  cfg.dynamicSmemBytes = st->smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once (grid barriers)
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (p.hd == 128)
    GLC_CHECK_CUDA(cudaLaunchKernelEx(&cfg, persistent_decode_kernel<128>, p));
  else
    GLC_CHECK_CUDA(cudaLaunchKernelEx(&cfg, persistent_decode_kernel<64>, p));
  note_launch();
  return GLACIER_CUDA_OK;
}

int persist_read_stats(PersistState* st, unsigned long long* ns, unsigned long long* n) {
  unsigned long long h[16];
  GLC_CHECK_CUDA(cudaMemcpy(h, st->stats.p, sizeof(h), cudaMemcpyDeviceToHost));
  GLC_CHECK_CUDA(cudaMemset(st->stats.p, 0, sizeof(h)));
  for (int i = 0; i < 8; ++i) {
    ns[i] = h[i];
    n[i] = h[8 + i];
  }
  return GLACIER_CUDA_OK;
}

int persist_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_persist_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_persist_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace glacier
