// Device-resident model, paged KV pool and the batched decode step.
//
// The step is the reference's cached decode (forwardLayerCached,
// src/generate.zig:1511-1967, and the loop at :5366-5450) for `lanes`
// independent requests at once, each with its own position and block table
// (decode_lane4.zig generalised to any lane count):
//
//   x = embed(token)                                  loadEmbeddingRow :3653
//   per layer:  h = rmsnorm(x + down_prev)            (fused residual add)
//               qkv = W_qkv h        (one GEMV over the fused [Wq; Wk; Wv])
//               q, k = rope(q, k, pos); pages <- k, v; q += bias, ...
//               a = paged_attention(q)                paged_attention.zig:108
//               h2 = rmsnorm(x + W_o a)
//               gu = W_gu h2         (one GEMV over the fused [Wgate; Wup])
//               down = W_d (silu(gate) * up)
//   logits = W_lm rmsnorm(x + down)  ->  eligible argmax  ->  token ids
//
// Row-major INT4 payloads concatenate by rows, so Q/K/V and gate/up are
// uploaded straight into one fused device matrix each (no re-layout of the
// codes).  Every buffer is reserved up front: a step allocates nothing and can
// be captured in a CUDA graph.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "persistent.cuh"

namespace glacier {

int add_rmsnorm(const float* a, size_t lda, const float* b, size_t ldb, size_t b_split_stride, int nb,
                float* residual, size_t ldr, const float* w, float eps, float* out, size_t ldo, size_t batch,
                size_t dim, cudaStream_t stream, SplitOut so = SplitOut());
int silu_mul(const float* gate, const float* up, size_t ld_in, float* out, size_t ld_out, size_t batch, size_t n,
             cudaStream_t stream, SplitOut so = SplitOut());
int embed_gather(const __half* table, size_t vocab, size_t dim, const int32_t* tokens, size_t batch, float* out,
                 size_t ldo, cudaStream_t stream);
int embed_gather(const float* table, size_t vocab, size_t dim, const int32_t* tokens, size_t batch, float* out,
                 size_t ldo, cudaStream_t stream);
int qkv_rope_append(const float* qkv, size_t ld, size_t split_stride, int nsplit, const float* bias,
                    const float* cos_t, const float* sin_t, size_t positions, const int32_t* pos, size_t batch,
                    size_t num_heads, size_t num_kv_heads, size_t head_dim, float* q_out, size_t ldq, float* pool,
                    size_t page_floats, const int32_t* block_tables, size_t max_pages, size_t layer,
                    cudaStream_t stream);
size_t attention_workspace_floats(size_t lanes, size_t num_heads, size_t head_dim, size_t nsplit);
int attention_segments(size_t lanes, size_t num_heads, size_t head_dim, size_t max_ctx);
int paged_attention(const float* q, size_t ldq, const float* pool, size_t page_floats, const int32_t* block_tables,
                    size_t max_pages, const int32_t* ctx_lens, size_t max_ctx, size_t lanes, size_t layer,
                    size_t num_heads, size_t num_kv_heads, size_t head_dim, float* out, size_t ldo, float* workspace,
                    size_t workspace_floats, int chunk, cudaStream_t stream, SplitOut so = SplitOut(),
                    StepProfiler* prof = nullptr, int combine_kind = -1);
size_t argmax_workspace_bytes(size_t batch, size_t n);
int argmax_rows(const float* logits, size_t ld, size_t batch, size_t n, const uint64_t* words, size_t word_count,
                glacier_argmax_result* out, int32_t* tokens, int32_t* status, void* workspace, size_t ws_bytes,
                cudaStream_t stream);

int tp_unique_id(void* out);
int tp_comm_create(void** comm, int rank, int world, const void* id_bytes);
void tp_comm_destroy(void* comm);
int tp_all_reduce(void* comm, float* buf, size_t count, cudaStream_t stream);
int reduce_splits(const float* part, size_t split_stride, int nsplit, float* y, size_t n, cudaStream_t stream);

size_t gemm_split_bytes(size_t np, size_t K);
bool gemm_tc_supported(const Int4Weight& w);
int split_activation(const float* x, size_t ldx, size_t n, size_t K, size_t np, __half* xs, float* xscale,
                     cudaStream_t stream);
int encode_split_map(CUtensorMap* map, const __half* xs, size_t np, size_t K);
int gemm_splits(size_t M, size_t K);

void StepProfiler::mark(int kind, cudaStream_t stream) {
  if (!on) return;
  if (used == events.size()) {
    cudaEvent_t e = nullptr;
    if (events.size() >= kMaxEvents || cudaEventCreate(&e) != cudaSuccess) {
      overflow = true;
      return;
    }
    events.push_back(e);
    kinds.push_back(-1);
  }
  if (cudaEventRecord(events[used], stream) != cudaSuccess) {
    overflow = true;
    return;
  }
  kinds[used++] = kind;
}

int StepProfiler::read(double* ms, uint64_t* regions, size_t kinds_n) {
  for (size_t k = 0; k < kinds_n; ++k) {
    ms[k] = 0.0;
    regions[k] = 0;
  }
  const bool lost = overflow;
  overflow = false;
  if (used > 0) GLC_CHECK_CUDA(cudaEventSynchronize(events[used - 1]));
  for (size_t i = 0; i + 1 < used; ++i) {
    const int k = kinds[i];
    if (k < 0 || (size_t)k >= kinds_n) continue;
    float t = 0.f;
    GLC_CHECK_CUDA(cudaEventElapsedTime(&t, events[i], events[i + 1]));
    ms[k] += t;
    regions[k] += 1;
  }
  used = 0;
  GLC_REQUIRE(!lost, "profile: more than %zu regions recorded between reads; some were dropped", kMaxEvents);
  return GLACIER_CUDA_OK;
}

StepProfiler::~StepProfiler() {
  for (cudaEvent_t e : events) cudaEventDestroy(e);
}

namespace {

// Row i of a prompt chunk: position first + i and a copy of the request's block table.
__global__ void prefill_rows_kernel(const int32_t* __restrict__ table, int max_pages, int first,
                                    int32_t* __restrict__ pos, int32_t* __restrict__ tables) {
  griddep_launch();
  griddep_wait();
  const int i = blockIdx.x;
  if (threadIdx.x == 0) pos[i] = first + i;
  for (int j = threadIdx.x; j < max_pages; j += blockDim.x) tables[(size_t)i * max_pages + j] = table[j];
}

// Attention context of each lane: position + 1.  With a lane split (tensor
// parallelism with more ranks than kv heads) a rank attends only the lanes
// b with b % groups == index; the others get context 0, so their attention
// output is zero and the all-reduce of o sums each lane's heads from its owners.
// Context length of each lane (position + 1; 0 for lanes another tensor-parallel
// rank attends).  A position outside [0, limit) -- past the RoPE table or the
// lane's block table -- gives context 0, so attention never reads past the
// block table, and raises the bad-input word (the RoPE / append kernel also
// skips that lane).
__global__ void ctx_from_pos_kernel(const int32_t* __restrict__ pos, int32_t* __restrict__ ctx, int n, int groups,
                                    int index, int limit, int* __restrict__ bad) {
  griddep_launch();
  griddep_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int p = pos[i];
  if (p < 0 || p >= limit) {
    ctx[i] = 0;
    atomicExch(bad, 1);
    return;
  }
  ctx[i] = (i % groups == index) ? p + 1 : 0;
}

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  int alloc(size_t n) {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
    if (n == 0) return GLACIER_CUDA_OK;
    if (cudaMalloc(&p, n) != cudaSuccess) {
      cudaGetLastError();
      return set_error(GLACIER_CUDA_ENOMEM, "cudaMalloc(%zu) failed", n);
    }
    bytes = n;
    return GLACIER_CUDA_OK;
  }
  template <typename T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

// Host -> device upload of weight bytes through two pinned bounce buffers: the
// host copy of one chunk overlaps the DMA of the previous one, where a pageable
// cudaMemcpy stages every byte itself.  Process-wide buffers under a mutex;
// synchronous for the caller.
int upload_h2d(void* dst, const void* src, size_t bytes) {
  constexpr size_t kChunk = (size_t)32 << 20;
  struct Bounce {
    std::mutex mu;
    void* buf[2] = {nullptr, nullptr};
    cudaStream_t st = nullptr;
    cudaEvent_t ev[2] = {nullptr, nullptr};
    int device = -1;
  };
  static Bounce bb;
  if (bytes < ((size_t)4 << 20)) {  // small tensors: one pageable copy
    GLC_CHECK_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
    return GLACIER_CUDA_OK;
  }
  std::lock_guard<std::mutex> lock(bb.mu);
  int dev = 0;
  GLC_CHECK_CUDA(cudaGetDevice(&dev));
  if (bb.device != dev) {  // streams and events belong to the device that made them
    if (bb.st) {
      cudaStreamDestroy(bb.st);
      for (auto& e : bb.ev) cudaEventDestroy(e);
    }
    bb.st = nullptr;
    GLC_CHECK_CUDA(cudaStreamCreateWithFlags(&bb.st, cudaStreamNonBlocking));
    for (auto& e : bb.ev) GLC_CHECK_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    for (auto& b : bb.buf)  // portable: pinned for every device's context, not only the first
      if (!b) GLC_CHECK_CUDA(cudaHostAlloc(&b, kChunk, cudaHostAllocPortable));
    bb.device = dev;
  }
  const uint8_t* s = static_cast<const uint8_t*>(src);
  uint8_t* d = static_cast<uint8_t*>(dst);
  for (size_t off = 0, i = 0; off < bytes; off += kChunk, ++i) {
    const size_t n = std::min(kChunk, bytes - off);
    const int k = (int)(i & 1);
    GLC_CHECK_CUDA(cudaEventSynchronize(bb.ev[k]));  // the DMA that last read this buffer is done
    memcpy(bb.buf[k], s + off, n);
    GLC_CHECK_CUDA(cudaMemcpyAsync(d + off, bb.buf[k], n, cudaMemcpyHostToDevice, bb.st));
    GLC_CHECK_CUDA(cudaEventRecord(bb.ev[k], bb.st));
  }
  GLC_CHECK_CUDA(cudaStreamSynchronize(bb.st));
  return GLACIER_CUDA_OK;
}

// Prepared runtime-image layouts back to row-major codes, on the device
// (int4_weights.zig:113-170 rows4_k16; :42-54 PairNibble).  One thread per
// (4-row tile t, 16-column block b).  In rows4_k16 the block is 32 contiguous
// bytes ordered [4-column chunk c][row lane l][byte p]; as 16-bit units h[4c + l]
// it is a 4 x 4 transpose: row l's 8 row-major bytes are h[l], h[4+l], h[8+l],
// h[12+l].  A PairNibble block is 64 bytes [c][l][byte pair p][lo, hi] holding
// gate codes in the low nibbles and up codes in the high ones.
__global__ void rows4_to_rows_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint64_t tiles,
                                     uint32_t blocks, uint64_t row_bytes) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= tiles * blocks) return;
  const uint64_t t = i / blocks, b = i % blocks;
  const uint4* s = reinterpret_cast<const uint4*>(src + t * 4 * row_bytes + b * 32);
  const uint4 a = s[0], c = s[1];
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
  auto h = [&](int k) { return (w[k >> 1] >> (16 * (k & 1))) & 0xFFFFu; };
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const uint2 v = make_uint2(h(l) | h(4 + l) << 16, h(8 + l) | h(12 + l) << 16);
    *reinterpret_cast<uint2*>(dst + (t * 4 + l) * row_bytes + b * 8) = v;
  }
}

__global__ void pair_nibble_split_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ gate,
                                         uint8_t* __restrict__ up, uint64_t tiles, uint32_t blocks,
                                         uint64_t row_bytes) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= tiles * blocks) return;
  const uint64_t t = i / blocks, b = i % blocks;
  const uint4* s = reinterpret_cast<const uint4*>(src + t * 4 * 2 * row_bytes + b * 64);
  uint8_t by[64];
#pragma unroll
  for (int q = 0; q < 4; ++q) *reinterpret_cast<uint4*>(by + 16 * q) = s[q];
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    uint32_t g[2] = {0, 0}, u[2] = {0, 0};
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const uint32_t lo = by[c * 16 + l * 4 + 2 * p], hi = by[c * 16 + l * 4 + 2 * p + 1];
        const int o = c * 2 + p;  // byte of the row's 8
        g[o >> 2] |= ((lo & 15u) | (hi & 15u) << 4) << (8 * (o & 3));
        u[o >> 2] |= ((lo >> 4) | (hi & 0xF0u)) << (8 * (o & 3));
      }
    *reinterpret_cast<uint2*>(gate + (t * 4 + l) * row_bytes + b * 8) = make_uint2(g[0], g[1]);
    *reinterpret_cast<uint2*>(up + (t * 4 + l) * row_bytes + b * 8) = make_uint2(u[0], u[1]);
  }
}

// A fused INT4 matrix whose row blocks are uploaded piece by piece.
struct FusedWeight {
  DevBuf packed, scales;
  Int4Weight w;
  std::vector<size_t> part_rows;   // rows of each part
  std::vector<bool> loaded;
  size_t scale_stride = 0;
  bool f16 = true;

  int init(const std::vector<size_t>& rows, size_t K, size_t group, bool scales_f16) {
    part_rows = rows;
    loaded.assign(rows.size(), false);
    size_t M = 0;
    for (size_t r : rows) M += r;
    f16 = scales_f16;
    const size_t esz = f16 ? 2 : 4;
    const size_t groups = ceil_div(K, group);
    scale_stride = ceil_div(groups * esz, 16) * 16 / esz;  // 16-byte aligned scale rows
    int rc = packed.alloc(M * K / 2);
    if (rc) return rc;
    rc = scales.alloc(M * scale_stride * esz);
    if (rc) return rc;
    GLC_CHECK_CUDA(cudaMemset(scales.p, 0, scales.bytes));
    w.packed = packed.as<uint8_t>();
    w.scales = scales.p;
    w.f16 = f16;
    w.scale_stride = scale_stride;
    w.M = M;
    w.K = K;
    w.group = group;
    return GLACIER_CUDA_OK;
  }

  size_t part_row0(size_t part) const {
    size_t row0 = 0;
    for (size_t i = 0; i < part; ++i) row0 += part_rows[i];
    return row0;
  }

  int check_part(size_t part, size_t pk_bytes, size_t sc_count) const {
    GLC_REQUIRE(part < part_rows.size(), "weight part %zu out of range", part);
    const size_t rows = part_rows[part], K = w.K, group = w.group;
    GLC_REQUIRE(K % 2 == 0 && K % group == 0, "weight rows must hold whole bytes and groups (K=%zu g=%zu)", K,
                group);
    GLC_REQUIRE(pk_bytes == rows * K / 2, "packed bytes %zu != %zu", pk_bytes, rows * K / 2);
    GLC_REQUIRE(sc_count == rows * (K / group), "scale count %zu != %zu", sc_count, rows * (K / group));
    return GLACIER_CUDA_OK;
  }

  // One part given in the reference's Int4WeightData form: row-major packed
  // codes and one f32 scale per group along the flat index.
  int load_part(size_t part, const uint8_t* pk, size_t pk_bytes, const float* sc, size_t sc_count) {
    int rc = check_part(part, pk_bytes, sc_count);
    if (rc) return rc;
    if ((rc = upload_h2d(packed.as<uint8_t>() + part_row0(part) * w.K / 2, pk, pk_bytes))) return rc;
    return load_scales(part, sc);
  }

  // The same with the codes in rows4_k16 order: uploaded as they are and put in
  // row-major order by the device (the host never permutes them).
  int load_part_rows4(size_t part, const uint8_t* pk, size_t pk_bytes, const float* sc, size_t sc_count) {
    int rc = check_part(part, pk_bytes, sc_count);
    if (rc) return rc;
    const size_t rows = part_rows[part], K = w.K;
    GLC_REQUIRE(rows % 4 == 0 && K % 16 == 0, "rows4_k16 needs rows %% 4 == 0 and K %% 16 == 0 (%zu x %zu)", rows,
                K);
    DevBuf stage;
    if ((rc = stage.alloc(pk_bytes))) return rc;
    if ((rc = upload_h2d(stage.p, pk, pk_bytes))) return rc;
    const uint64_t tiles = rows / 4, blocks = K / 16, n = tiles * blocks;
    rows4_to_rows_kernel<<<(unsigned)ceil_div(n, (size_t)256), 256>>>(
        stage.as<uint8_t>(), packed.as<uint8_t>() + part_row0(part) * K / 2, tiles, (uint32_t)blocks, K / 2);
    GLC_CHECK_LAUNCH();
    GLC_CHECK_CUDA(cudaDeviceSynchronize());  // the staging buffer is freed on return
    return load_scales(part, sc);
  }

  // A PairNibble record into parts 0 (gate) and 1 (up) of this fused matrix: the
  // pair bytes are uploaded as they are and split on the device.
  int load_pair(const uint8_t* pairs, size_t pair_bytes, const float* gate_sc, const float* up_sc, size_t sc_count) {
    GLC_REQUIRE(part_rows.size() == 2 && part_rows[0] == part_rows[1], "PairNibble needs a gate/up matrix");
    const size_t rows = part_rows[0], K = w.K;
    int rc = check_part(0, pair_bytes / 2, sc_count);
    if (rc) return rc;
    GLC_REQUIRE(pair_bytes == rows * K && rows % 4 == 0 && K % 16 == 0, "PairNibble geometry (%zu bytes, %zu x %zu)",
                pair_bytes, rows, K);
    DevBuf stage;
    if ((rc = stage.alloc(pair_bytes))) return rc;
    if ((rc = upload_h2d(stage.p, pairs, pair_bytes))) return rc;
    const uint64_t tiles = rows / 4, blocks = K / 16, n = tiles * blocks;
    uint8_t* gate = packed.as<uint8_t>();
    pair_nibble_split_kernel<<<(unsigned)ceil_div(n, (size_t)256), 256>>>(stage.as<uint8_t>(), gate,
                                                                          gate + rows * K / 2, tiles,
                                                                          (uint32_t)blocks, K / 2);
    GLC_CHECK_LAUNCH();
    GLC_CHECK_CUDA(cudaDeviceSynchronize());
    if ((rc = load_scales(0, gate_sc))) return rc;
    return load_scales(1, up_sc);
  }

  // Group scales of one part (f32, row-major): the fp16 mirror or the f32 copy.
  int load_scales(size_t part, const float* sc) {
    const size_t rows = part_rows[part], K = w.K, group = w.group;
    const size_t groups = K / group;
    const size_t row0 = part_row0(part);
    const size_t esz = f16 ? 2 : 4;
    std::vector<uint8_t> host(rows * scale_stride * esz, 0);
    // Rows spread over the host's cores (a 152064-row LM head has 17M scales).
    std::atomic<bool> nonfinite{false};
    auto convert = [&](size_t r0, size_t r1) {
      bool nf = false;
      for (size_t r = r0; r < r1; ++r)
        for (size_t g = 0; g < groups; ++g) {
          const float s = sc[r * groups + g];
          if (f16) {
            // Round-to-nearest-even fp16 mirror (int4_weights.zig:348-358 withF16Scales).
            const uint16_t h = __half_as_ushort(__float2half_rn(s));
            memcpy(&host[(r * scale_stride + g) * 2], &h, 2);
            nf = nf || half_bits_nonfinite(h);
          } else {
            memcpy(&host[(r * scale_stride + g) * 4], &s, 4);
          }
        }
      if (nf) nonfinite = true;
    };
    const unsigned nt = rows * groups < ((size_t)1 << 20)
                            ? 1u
                            : std::max(1u, std::min(std::thread::hardware_concurrency(), 32u));
    std::vector<std::thread> pool;
    for (unsigned t = 1; t < nt; ++t) pool.emplace_back(convert, rows * t / nt, rows * (t + 1) / nt);
    convert(0, rows / nt);
    for (auto& th : pool) th.join();
    if (nonfinite) w.nonfinite = true;
    const int rc = upload_h2d(scales.as<uint8_t>() + row0 * scale_stride * esz, host.data(), host.size());
    if (rc) return rc;
    loaded[part] = true;
    return GLACIER_CUDA_OK;
  }

  bool complete() const {
    for (bool b : loaded)
      if (!b) return false;
    return true;
  }
};

struct Layer {
  FusedWeight qkv, o, gu, d;
  DevBuf bqkv, in_norm, post_norm;
  bool has_bias[3] = {false, false, false};
  bool norm_loaded[2] = {false, false};
};

}  // namespace

}  // namespace glacier

using namespace glacier;

struct glacier_cuda_model {
  glacier_cuda_model_config cfg;
  int device = 0;
  size_t q_dim = 0, kv_dim = 0, qkv_dim = 0;
  std::vector<std::unique_ptr<Layer>> layers;
  FusedWeight lm;
  DevBuf embedding, final_norm, rope_cos, rope_sin;
  bool emb_loaded = false, emb_f32 = false, final_loaded = false, finalized = false;
  // Reserved step workspace.
  size_t max_lanes = 0, max_pages = 0;
  DevBuf x, hn, qkv, q, attn, proj, gu, act, down, logits, ctx, att_ws, arg_ws, status;
  // GEMV-mode LM head with the eligible argmax in its epilogue: per-tile winners.
  DevBuf lm_arg;
  size_t att_floats = 0, arg_bytes = 0;
  int att_segs = 0;
  // Tensor-core GEMM mode (more than 4 lanes): activations in split fp16 form.
  bool gemm = false;
  size_t np = 0;
  DevBuf xs_d, xs_q, xs_f, xscale;
  CUtensorMap map_d, map_q, map_f;
  int split_qkv = 1, split_o = 1, split_d = 1;
  DevBuf pf_pos, pf_bt;  // prompt-chunk positions and per-row block tables (prefill)
  // Tensor parallelism: this rank's NCCL communicator (nullptr: one GPU).
  void* tp_comm = nullptr;
  int tp_rank = 0, tp_world = 1;
  int tp_lane_groups = 1, tp_lane_index = 0;  // lanes this rank attends: b % groups == index
  // One-lane reservations: the whole decode step as one persistent kernel
  // (decode_persistent.cu) when switched on (glacier_cuda_model_persistent).
  PersistState* ps = nullptr;
  bool persistent = false;
  ~glacier_cuda_model() {
    tp_comm_destroy(tp_comm);
    persist_destroy(ps);
  }
  StepProfiler prof;  // optional per-kernel-class timing of decode steps
};

struct glacier_cuda_kv {
  size_t num_pages = 0, page_floats = 0;
  DevBuf pool;
};

namespace {

int load_qio(const uint8_t* payload, size_t bytes, size_t expect_elems, size_t expect_group,
             std::vector<float>& scales, const uint8_t** packed, size_t* packed_bytes) {
  // src/model/qio.zig:49-70 readQuantHeader and :116-160 decodePage layout.
  GLC_REQUIRE(payload && bytes >= 16, "qio: truncated header");
  uint32_t magic, n, g;
  memcpy(&magic, payload, 4);
  memcpy(&n, payload + 4, 4);
  memcpy(&g, payload + 8, 4);
  GLC_REQUIRE(magic == 0x514F4954u, "qio: bad magic 0x%08x", magic);
  GLC_REQUIRE(g != 0, "qio: zero group size");
  GLC_REQUIRE(payload[12] == 1, "qio: precision %u is not INT4", (unsigned)payload[12]);
  GLC_REQUIRE(n == expect_elems && g == expect_group, "qio: %u elements / group %u, expected %zu / %zu", n, g,
              expect_elems, expect_group);
  const size_t ngroups = ceil_div(n, g);
  const size_t pk = ceil_div(n, 2);
  GLC_REQUIRE(bytes >= 16 + ngroups * 4 + pk, "qio: truncated payload");
  scales.resize(ngroups);
  memcpy(scales.data(), payload + 16, ngroups * 4);
  *packed = payload + 16 + ngroups * 4;
  *packed_bytes = pk;
  return GLACIER_CUDA_OK;
}

FusedWeight* weight_slot(glacier_cuda_model* m, int layer, int kind, size_t* part) {
  *part = 0;
  if (kind == GLACIER_CUDA_W_LM_HEAD) return layer == -1 ? &m->lm : nullptr;
  if (layer < 0 || layer >= (int)m->layers.size()) return nullptr;
  Layer& L = *m->layers[layer];
  switch (kind) {
    case GLACIER_CUDA_W_Q: *part = 0; return &L.qkv;
    case GLACIER_CUDA_W_K: *part = 1; return &L.qkv;
    case GLACIER_CUDA_W_V: *part = 2; return &L.qkv;
    case GLACIER_CUDA_W_O: return &L.o;
    case GLACIER_CUDA_W_GATE: *part = 0; return &L.gu;
    case GLACIER_CUDA_W_UP: *part = 1; return &L.gu;
    case GLACIER_CUDA_W_DOWN: return &L.d;
    default: return nullptr;
  }
}

size_t weight_out_features(const glacier_cuda_model* m, int kind) {
  const auto& c = m->cfg;
  switch (kind) {
    case GLACIER_CUDA_W_Q: return m->q_dim;
    case GLACIER_CUDA_W_K: case GLACIER_CUDA_W_V: return m->kv_dim;
    case GLACIER_CUDA_W_O: case GLACIER_CUDA_W_DOWN: return c.dim;
    case GLACIER_CUDA_W_GATE: case GLACIER_CUDA_W_UP: return c.hidden;
    case GLACIER_CUDA_W_LM_HEAD: return c.vocab;
    default: return 0;
  }
}

size_t weight_in_features(const glacier_cuda_model* m, int kind) {
  switch (kind) {
    case GLACIER_CUDA_W_O: return m->q_dim;
    case GLACIER_CUDA_W_DOWN: return m->cfg.hidden;
    default: return m->cfg.dim;
  }
}

int bind_device(const glacier_cuda_model* m) {
  GLC_CHECK_CUDA(cudaSetDevice(m->device));
  return GLACIER_CUDA_OK;
}

}  // namespace

extern "C" {

glacier_cuda_model* glacier_cuda_model_create(const glacier_cuda_model_config* cfg) {
  if (!cfg) {
    set_error(GLACIER_CUDA_EINVAL, "model_create: null config");
    return nullptr;
  }
  const auto& c = *cfg;
  if (c.num_layers == 0 || c.dim == 0 || c.hidden == 0 || c.num_heads == 0 || c.num_kv_heads == 0 ||
      c.head_dim == 0 || c.vocab == 0 || c.group_size == 0 || c.num_heads % c.num_kv_heads != 0 ||
      c.head_dim % 2 != 0 || c.max_positions == 0) {
    set_error(GLACIER_CUDA_EINVAL, "model_create: invalid configuration");
    return nullptr;
  }
  auto m = std::make_unique<glacier_cuda_model>();
  m->cfg = c;
  if (cudaGetDevice(&m->device) != cudaSuccess) {
    set_error(GLACIER_CUDA_ECUDA, "model_create: no CUDA device");
    return nullptr;
  }
  m->q_dim = (size_t)c.num_heads * c.head_dim;
  m->kv_dim = (size_t)c.num_kv_heads * c.head_dim;
  m->qkv_dim = m->q_dim + 2 * m->kv_dim;
  const bool f16 = c.scales_f16 != 0;
  for (uint32_t l = 0; l < c.num_layers; ++l) {
    auto L = std::make_unique<Layer>();
    if (L->qkv.init({m->q_dim, m->kv_dim, m->kv_dim}, c.dim, c.group_size, f16) ||
        L->o.init({c.dim}, m->q_dim, c.group_size, f16) ||
        L->gu.init({c.hidden, c.hidden}, c.dim, c.group_size, f16) ||
        L->d.init({c.dim}, c.hidden, c.group_size, f16) || L->bqkv.alloc(m->qkv_dim * 4) ||
        L->in_norm.alloc((size_t)c.dim * 4) || L->post_norm.alloc((size_t)c.dim * 4))
      return nullptr;
    if (cudaMemset(L->bqkv.p, 0, L->bqkv.bytes) != cudaSuccess) {
      set_error(GLACIER_CUDA_ECUDA, "model_create: memset failed");
      return nullptr;
    }
    m->layers.push_back(std::move(L));
  }
  if (m->lm.init({c.vocab}, c.dim, c.group_size, f16) || m->final_norm.alloc((size_t)c.dim * 4))
    return nullptr;
  // RoPE table (generate.zig:791-808): angle = pos / theta^(2i/hd) in f32.
  const size_t half = c.head_dim / 2, P = c.max_positions;
  std::vector<float> cs(P * half), sn(P * half);
  for (size_t pos = 0; pos < P; ++pos)
    for (size_t i = 0; i < half; ++i) {
      const float exponent = (float)(2 * i) / (float)c.head_dim;
      const float freq = 1.0f / powf(c.rope_theta, exponent);
      const float angle = (float)pos * freq;
      cs[pos * half + i] = cosf(angle);
      sn[pos * half + i] = sinf(angle);
    }
  if (m->rope_cos.alloc(cs.size() * 4) || m->rope_sin.alloc(sn.size() * 4)) return nullptr;
  if (cudaMemcpy(m->rope_cos.p, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(m->rope_sin.p, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
    set_error(GLACIER_CUDA_ECUDA, "model_create: rope upload failed");
    return nullptr;
  }
  return m.release();
}

void glacier_cuda_model_destroy(glacier_cuda_model* m) { delete m; }

int glacier_cuda_model_load_int4(glacier_cuda_model* m, int layer, int kind, const uint8_t* packed,
                                 size_t packed_bytes, const float* scales, size_t scale_count) {
  GLC_REQUIRE(m && packed && scales, "model_load_int4: null argument");
  GLC_REQUIRE(!m->finalized, "model_load_int4: model already finalized");
  size_t part = 0;
  FusedWeight* fw = weight_slot(m, layer, kind, &part);
  GLC_REQUIRE(fw, "model_load_int4: bad layer %d / kind %d", layer, kind);
  const int rc = bind_device(m);
  if (rc) return rc;
  return fw->load_part(part, packed, packed_bytes, scales, scale_count);
}

int glacier_cuda_model_load_int4_rows4(glacier_cuda_model* m, int layer, int kind, const uint8_t* packed,
                                       size_t packed_bytes, const float* scales, size_t scale_count) {
  GLC_REQUIRE(m && packed && scales, "model_load_int4_rows4: null argument");
  GLC_REQUIRE(!m->finalized, "model_load_int4_rows4: model already finalized");
  size_t part = 0;
  FusedWeight* fw = weight_slot(m, layer, kind, &part);
  GLC_REQUIRE(fw, "model_load_int4_rows4: bad layer %d / kind %d", layer, kind);
  const int rc = bind_device(m);
  if (rc) return rc;
  return fw->load_part_rows4(part, packed, packed_bytes, scales, scale_count);
}

int glacier_cuda_model_load_pair_nibble(glacier_cuda_model* m, int layer, const uint8_t* pairs, size_t pair_bytes,
                                        const uint16_t* pair_scales, size_t scale_count) {
  GLC_REQUIRE(m && pairs && pair_scales, "model_load_pair_nibble: null argument");
  GLC_REQUIRE(!m->finalized, "model_load_pair_nibble: model already finalized");
  GLC_REQUIRE(layer >= 0 && layer < (int)m->layers.size(), "model_load_pair_nibble: bad layer %d", layer);
  const size_t F = m->cfg.hidden, D = m->cfg.dim, group = m->cfg.group_size;
  GLC_REQUIRE(F % 4 == 0 && D % group == 0 && scale_count == 2 * F * (D / group),
              "model_load_pair_nibble: %zu scales for a %zu x %zu pair (group %zu)", scale_count, F, D, group);
  // Scale grid [tile][group][branch][lane] (int4_weights.zig:322-331) to row-major f32 per branch.
  const size_t per_row = D / group;
  std::vector<float> gs(F * per_row), us(F * per_row);
  for (size_t t = 0; t < F / 4; ++t)
    for (size_t g = 0; g < per_row; ++g)
      for (size_t l = 0; l < 4; ++l) {
        const size_t base = (t * per_row + g) * 8;
        __half hg, hu;
        memcpy(&hg, &pair_scales[base + l], 2);
        memcpy(&hu, &pair_scales[base + 4 + l], 2);
        gs[(t * 4 + l) * per_row + g] = __half2float(hg);
        us[(t * 4 + l) * per_row + g] = __half2float(hu);
      }
  const int rc = bind_device(m);
  if (rc) return rc;
  return m->layers[layer]->gu.load_pair(pairs, pair_bytes, gs.data(), us.data(), gs.size());
}

int glacier_cuda_model_load_qio(glacier_cuda_model* m, int layer, int kind, const uint8_t* payload,
                                size_t payload_bytes) {
  GLC_REQUIRE(m, "model_load_qio: null model");
  const size_t out_f = weight_out_features(m, kind), in_f = weight_in_features(m, kind);
  GLC_REQUIRE(out_f > 0, "model_load_qio: bad kind %d", kind);
  std::vector<float> scales;
  const uint8_t* pk = nullptr;
  size_t pk_bytes = 0;
  const int rc = load_qio(payload, payload_bytes, out_f * in_f, m->cfg.group_size, scales, &pk, &pk_bytes);
  if (rc) return rc;
  return glacier_cuda_model_load_int4(m, layer, kind, pk, pk_bytes, scales.data(), scales.size());
}

int glacier_cuda_model_load_f32(glacier_cuda_model* m, int layer, int kind, const float* data, size_t count) {
  GLC_REQUIRE(m && data, "model_load_f32: null argument");
  GLC_REQUIRE(!m->finalized, "model_load_f32: model already finalized");
  int rc = bind_device(m);
  if (rc) return rc;
  const auto& c = m->cfg;
  if (kind == GLACIER_CUDA_N_FINAL) {
    GLC_REQUIRE(layer == -1 && count == c.dim, "model_load_f32: final norm needs %u values", c.dim);
    GLC_CHECK_CUDA(cudaMemcpy(m->final_norm.p, data, count * 4, cudaMemcpyHostToDevice));
    m->final_loaded = true;
    return GLACIER_CUDA_OK;
  }
  GLC_REQUIRE(layer >= 0 && layer < (int)c.num_layers, "model_load_f32: bad layer %d", layer);
  Layer& L = *m->layers[layer];
  switch (kind) {
    case GLACIER_CUDA_B_Q:
    case GLACIER_CUDA_B_K:
    case GLACIER_CUDA_B_V: {
      const int part = kind - GLACIER_CUDA_B_Q;
      const size_t off = part == 0 ? 0 : part == 1 ? m->q_dim : m->q_dim + m->kv_dim;
      const size_t n = part == 0 ? m->q_dim : m->kv_dim;
      GLC_REQUIRE(count == n, "model_load_f32: bias needs %zu values", n);
      GLC_CHECK_CUDA(cudaMemcpy(L.bqkv.as<float>() + off, data, n * 4, cudaMemcpyHostToDevice));
      L.has_bias[part] = true;
      return GLACIER_CUDA_OK;
    }
    case GLACIER_CUDA_N_INPUT:
    case GLACIER_CUDA_N_POST_ATTN: {
      GLC_REQUIRE(count == c.dim, "model_load_f32: norm needs %u values", c.dim);
      DevBuf& dst = kind == GLACIER_CUDA_N_INPUT ? L.in_norm : L.post_norm;
      GLC_CHECK_CUDA(cudaMemcpy(dst.p, data, count * 4, cudaMemcpyHostToDevice));
      L.norm_loaded[kind == GLACIER_CUDA_N_INPUT ? 0 : 1] = true;
      return GLACIER_CUDA_OK;
    }
    default:
      return set_error(GLACIER_CUDA_EINVAL, "model_load_f32: bad kind %d", kind);
  }
}

int glacier_cuda_model_load_embedding_f16(glacier_cuda_model* m, const uint16_t* table, size_t count) {
  GLC_REQUIRE(m && table, "model_load_embedding: null argument");
  GLC_REQUIRE(count == (size_t)m->cfg.vocab * m->cfg.dim, "model_load_embedding: %zu values, expected %zu", count,
              (size_t)m->cfg.vocab * m->cfg.dim);
  GLC_REQUIRE(!m->finalized, "model_load_embedding: model already finalized");
  int rc = bind_device(m);
  if (rc) return rc;
  if (m->embedding.bytes != count * 2 && (rc = m->embedding.alloc(count * 2))) return rc;
  GLC_CHECK_CUDA(cudaMemcpy(m->embedding.p, table, count * 2, cudaMemcpyHostToDevice));
  m->emb_loaded = true;
  m->emb_f32 = false;
  return GLACIER_CUDA_OK;
}

int glacier_cuda_model_load_embedding_f32(glacier_cuda_model* m, const float* table, size_t count) {
  GLC_REQUIRE(m && table, "model_load_embedding_f32: null argument");
  GLC_REQUIRE(!m->finalized, "model_load_embedding_f32: model already finalized");
  GLC_REQUIRE(count == (size_t)m->cfg.vocab * m->cfg.dim, "model_load_embedding_f32: %zu values, expected %zu",
              count, (size_t)m->cfg.vocab * m->cfg.dim);
  int rc = bind_device(m);
  if (rc) return rc;
  if (m->embedding.bytes != count * 4 && (rc = m->embedding.alloc(count * 4))) return rc;
  GLC_CHECK_CUDA(cudaMemcpy(m->embedding.p, table, count * 4, cudaMemcpyHostToDevice));
  m->emb_loaded = true;
  m->emb_f32 = true;
  return GLACIER_CUDA_OK;
}

int glacier_cuda_model_finalize(glacier_cuda_model* m) {
  GLC_REQUIRE(m, "model_finalize: null model");
  int rc = bind_device(m);
  if (rc) return rc;
  for (size_t l = 0; l < m->layers.size(); ++l) {
    Layer& L = *m->layers[l];
    GLC_REQUIRE(L.qkv.complete() && L.o.complete() && L.gu.complete() && L.d.complete(),
                "model_finalize: layer %zu is missing a weight", l);
    GLC_REQUIRE(L.norm_loaded[0] && L.norm_loaded[1], "model_finalize: layer %zu is missing a norm", l);
    for (FusedWeight* fw : {&L.qkv, &L.o, &L.gu, &L.d})
      if ((rc = int4_weight_prepare(fw->w))) return rc;
  }
  GLC_REQUIRE(m->lm.complete() && m->emb_loaded && m->final_loaded,
              "model_finalize: LM head, embedding or final norm missing");
  if ((rc = int4_weight_prepare(m->lm.w))) return rc;
  m->finalized = true;
  return GLACIER_CUDA_OK;
}

int glacier_cuda_model_reserve(glacier_cuda_model* m, size_t max_lanes, size_t max_pages) {
  GLC_REQUIRE(m && m->finalized, "model_reserve: model not finalized");
  GLC_REQUIRE(max_lanes > 0 && max_pages > 0, "model_reserve: empty reservation");
  GLC_REQUIRE(max_pages * 16 <= m->cfg.max_positions, "model_reserve: %zu pages exceed %u RoPE positions",
              max_pages, m->cfg.max_positions);
  int rc = bind_device(m);
  if (rc) return rc;
  const auto& c = m->cfg;
  const size_t L = max_lanes;
  m->att_segs = attention_segments(L, c.num_heads, c.head_dim, max_pages * 16);
  const size_t nsplit = (size_t)m->att_segs;
  m->att_floats = attention_workspace_floats(L, c.num_heads, c.head_dim, nsplit);
  m->arg_bytes = argmax_workspace_bytes(L, c.vocab);
  if ((rc = m->x.alloc(L * c.dim * 4)) || (rc = m->hn.alloc(L * c.dim * 4)) ||
      (rc = m->qkv.alloc(L * m->qkv_dim * 4)) || (rc = m->q.alloc(L * m->q_dim * 4)) ||
      (rc = m->attn.alloc(L * m->q_dim * 4)) || (rc = m->proj.alloc(L * c.dim * 4)) ||
      (rc = m->gu.alloc(L * 2 * (size_t)c.hidden * 4)) || (rc = m->act.alloc(L * (size_t)c.hidden * 4)) ||
      (rc = m->down.alloc(L * c.dim * 4)) || (rc = m->logits.alloc(L * (size_t)c.vocab * 4)) ||
      (rc = m->ctx.alloc(L * 4)) || (rc = m->att_ws.alloc(m->att_floats * 4)) ||
      (rc = m->arg_ws.alloc(m->arg_bytes)) || (rc = m->status.alloc(L * 4)) || (rc = m->pf_pos.alloc(L * 4)) ||
      (rc = m->pf_bt.alloc(L * max_pages * 4)) || (rc = m->lm_arg.alloc(argmax_records_bytes(L, c.vocab))))
    return rc;
  m->max_lanes = max_lanes;
  m->max_pages = max_pages;
  persist_destroy(m->ps);
  m->ps = nullptr;
  if (max_lanes == 1) {
    PersistModel pm;
    pm.L = (int)c.num_layers;
    pm.D = (int)c.dim;
    pm.F = (int)c.hidden;
    pm.H = (int)c.num_heads;
    pm.Hkv = (int)c.num_kv_heads;
    pm.hd = (int)c.head_dim;
    pm.V = (int)c.vocab;
    pm.positions = (int)c.max_positions;
    pm.emb_f32 = m->emb_f32 ? 1 : 0;
    pm.eps = c.rms_eps;
    for (auto& Lp : m->layers) {
      for (FusedWeight* fw : {&Lp->qkv, &Lp->o, &Lp->gu, &Lp->d}) pm.w.push_back(&fw->w);
      pm.bqkv.push_back(Lp->bqkv.as<float>());
      pm.in_norm.push_back(Lp->in_norm.as<float>());
      pm.post_norm.push_back(Lp->post_norm.as<float>());
    }
    pm.w.push_back(&m->lm.w);
    pm.final_norm = m->final_norm.as<float>();
    pm.embedding = m->embedding.p;
    pm.rope_cos = m->rope_cos.as<float>();
    pm.rope_sin = m->rope_sin.as<float>();
    rc = persist_create(pm, max_lanes, max_pages, &m->ps);
    if (rc && rc != GLACIER_CUDA_EUNSUPPORTED) return rc;
  }
  m->gemm = max_lanes > 4 && gemm_tc_supported(m->layers[0]->qkv.w) && gemm_tc_supported(m->layers[0]->o.w) &&
            gemm_tc_supported(m->layers[0]->d.w) && gemm_tc_supported(m->lm.w);
  if (m->gemm) {
    GLC_REQUIRE(max_lanes <= 128, "model_reserve: at most 128 lanes per GPU in tensor-core mode");
    const size_t np = ceil_div(max_lanes, 16) * 16;
    m->np = np;
    m->split_qkv = gemm_splits(m->qkv_dim, c.dim);
    m->split_o = gemm_splits(c.dim, m->q_dim);
    m->split_d = gemm_splits(c.dim, c.hidden);
    if ((rc = m->xs_d.alloc(gemm_split_bytes(np, c.dim))) || (rc = m->xs_q.alloc(gemm_split_bytes(np, m->q_dim))) ||
        (rc = m->xs_f.alloc(gemm_split_bytes(np, c.hidden))) ||
        (rc = m->qkv.alloc((size_t)m->split_qkv * L * m->qkv_dim * 4)) ||
        (rc = m->proj.alloc((size_t)m->split_o * L * c.dim * 4)) ||
        (rc = m->down.alloc((size_t)m->split_d * L * c.dim * 4)))
      return rc;
    // Padding rows of the split activations stay zero.
    GLC_CHECK_CUDA(cudaMemset(m->xs_d.p, 0, m->xs_d.bytes));
    GLC_CHECK_CUDA(cudaMemset(m->xs_q.p, 0, m->xs_q.bytes));
    GLC_CHECK_CUDA(cudaMemset(m->xs_f.p, 0, m->xs_f.bytes));
    if ((rc = encode_split_map(&m->map_d, m->xs_d.as<__half>(), np, c.dim)) ||
        (rc = encode_split_map(&m->map_q, m->xs_q.as<__half>(), np, m->q_dim)) ||
        (rc = encode_split_map(&m->map_f, m->xs_f.as<__half>(), np, c.hidden)))
      return rc;
  }
  return GLACIER_CUDA_OK;
}

glacier_cuda_kv* glacier_cuda_kv_create(const glacier_cuda_model* m, size_t num_pages) {
  if (!m || num_pages == 0) {
    set_error(GLACIER_CUDA_EINVAL, "kv_create: null model or zero pages");
    return nullptr;
  }
  if (bind_device(m)) return nullptr;
  auto kv = std::make_unique<glacier_cuda_kv>();
  kv->num_pages = num_pages;
  // One page = 16 positions of K and V for every layer (paged_kv_cache.zig:1-16).
  kv->page_floats = (size_t)m->cfg.num_layers * 2 * 16 * m->kv_dim;
  if (kv->pool.alloc(num_pages * kv->page_floats * 4)) return nullptr;
  if (cudaMemset(kv->pool.p, 0, kv->pool.bytes) != cudaSuccess) {
    set_error(GLACIER_CUDA_ECUDA, "kv_create: memset failed");
    return nullptr;
  }
  return kv.release();
}

void glacier_cuda_kv_destroy(glacier_cuda_kv* kv) { delete kv; }

float* glacier_cuda_kv_pages(glacier_cuda_kv* kv) { return kv ? kv->pool.as<float>() : nullptr; }

size_t glacier_cuda_kv_page_floats(const glacier_cuda_kv* kv) { return kv ? kv->page_floats : 0; }

// How a step ends: every row through the LM head and argmax (decode), no head
// (a prompt chunk before the last), or the head for the last row only (the
// last prompt chunk).
enum StepHead { kHeadAllRows, kHeadNone, kHeadLastRow };

// One batched pass of `lanes` rows through every layer (validated by the caller).
static int step_impl(glacier_cuda_model* m, glacier_cuda_kv* kv, size_t lanes, const int32_t* tokens,
                     const int32_t* positions, const int32_t* block_tables, size_t max_pages, const uint64_t* eligible,
                     size_t eligible_words, int32_t* tokens_out, int32_t* status_out, float* logits_out,
                     cudaStream_t st, StepHead head) {
  const auto& c = m->cfg;
  const size_t D = c.dim, F = c.hidden, B = lanes;
  const size_t max_ctx = max_pages * 16;
  int rc;
  // One lane, greedy step, one GPU: the persistent kernel runs the whole step.
  if (m->ps && m->persistent && head == kHeadAllRows && lanes == 1 && !m->tp_comm)
    return persist_step(m->ps, lanes, tokens, positions, block_tables, max_pages, kv->pool.as<float>(),
                        kv->page_floats, m->prof.on, eligible, eligible_words, tokens_out,
                        status_out ? status_out : m->status.as<int32_t>(), logits_out, st);
  float* x = m->x.as<float>();
  float* hn = m->hn.as<float>();
  StepProfiler* prof = m->prof.on ? &m->prof : nullptr;
  auto mark = [&](int kind) {
    if (prof) prof->mark(kind, st);
  };
  mark(GLACIER_CUDA_STEP_EMBED);
  const int pos_limit = (int)std::min<size_t>(max_ctx, c.max_positions);
  if ((rc = launch_pdl(ctx_from_pos_kernel, dim3((unsigned)ceil_div(B, 128)), dim3(128), 0, st, 1, positions,
                       m->ctx.as<int32_t>(), (int)B, m->tp_lane_groups, m->tp_lane_index, pos_limit,
                       ops_error_word())))
    return rc;
  int32_t* st_out = status_out ? status_out : m->status.as<int32_t>();
  // The LM head's epilogue picks the tokens (no argmax pass over the logits,
  // which are written only when the caller asks for them).
  ArgmaxEpi ae;
  ae.words = eligible;
  ae.word_count = (int)eligible_words;
  ae.tokens = tokens_out;
  ae.status = st_out;
  ae.partials = m->lm_arg.as<int4>();
  auto lm_head_argmax = [&](const float* xin, size_t rows) -> int {
    return int4_linear_argmax(m->lm.w, xin, D, rows, logits_out, c.vocab, ae, st);
  };
  if ((rc = m->emb_f32 ? embed_gather(m->embedding.as<float>(), c.vocab, D, tokens, B, x, D, st)
                       : embed_gather(m->embedding.as<__half>(), c.vocab, D, tokens, B, x, D, st)))
    return rc;
  // Split-form destinations of the GEMM inputs (tensor-core mode only).
  auto split_of = [&](DevBuf& xs, size_t K) {
    SplitOut so;
    if (m->gemm) {
      so.xs = xs.as<__half>();
      so.xscale = reinterpret_cast<float*>(so.xs + 2 * m->np * K);
      so.np = (int)m->np;
    }
    return so;
  };
  const SplitOut so_d = split_of(m->xs_d, D), so_q = split_of(m->xs_q, m->q_dim), so_f = split_of(m->xs_f, F);
  // One projection: GEMV on fp32 activations (up to 4 lanes) or the tensor-core
  // GEMM on the split activations its producer wrote.
  auto project = [&](const Int4Weight& w, const float* xin, size_t K, const SplitOut& so, const CUtensorMap& map,
                     float* y, size_t ldy, int nsplit) -> int {
    if (!m->gemm) return int4_linear(w, xin, K, B, nullptr, y, ldy, st);
    return gemm_int4_tc(w, map, so.xscale, B, m->np, y, ldy, nsplit, B * ldy, nullptr, st);
  };
  const int sq = m->gemm ? m->split_qkv : 1, so_gemm = m->gemm ? m->split_o : 1, sd_gemm = m->gemm ? m->split_d : 1;
  // Partials the o / down consumers sum: with tensor parallelism the split-K
  // partials are summed locally and all-reduced as one buffer.
  const int so_ = m->tp_comm ? 1 : so_gemm, sd = m->tp_comm ? 1 : sd_gemm;
  auto tp_reduce = [&](float* buf, int nsplit) -> int {
    int r;
    mark(GLACIER_CUDA_STEP_ALL_REDUCE);
    if (nsplit > 1 && (r = reduce_splits(buf, B * D, nsplit, buf, B * D, st))) return r;
    return tp_all_reduce(m->tp_comm, buf, B * D, st);
  };
  for (size_t l = 0; l < c.num_layers; ++l) {
    Layer& L = *m->layers[l];
    // x (+ previous layer's down projection, its split-K partials summed in order) -> x, normed hn
    mark(GLACIER_CUDA_STEP_NORM);
    if ((rc = add_rmsnorm(x, D, l ? m->down.as<float>() : nullptr, D, B * D, l ? sd : 0, x, D, L.in_norm.as<float>(),
                          c.rms_eps, m->gemm ? nullptr : hn, D, B, D, st, so_d)))
      return rc;
    mark(GLACIER_CUDA_STEP_PROJ_QKV);
    if ((rc = project(L.qkv.w, hn, D, so_d, m->map_d, m->qkv.as<float>(), m->qkv_dim, sq))) return rc;
    mark(GLACIER_CUDA_STEP_ROPE_APPEND);
    if ((rc = qkv_rope_append(m->qkv.as<float>(), m->qkv_dim, B * m->qkv_dim, sq, L.bqkv.as<float>(),
                              m->rope_cos.as<float>(), m->rope_sin.as<float>(), c.max_positions, positions, B,
                              c.num_heads, c.num_kv_heads, c.head_dim, m->q.as<float>(), m->q_dim,
                              kv->pool.as<float>(), kv->page_floats, block_tables, max_pages, l, st)))
      return rc;
    mark(GLACIER_CUDA_STEP_ATTENTION);
    if ((rc = paged_attention(m->q.as<float>(), m->q_dim, kv->pool.as<float>(), kv->page_floats, block_tables,
                              max_pages, m->ctx.as<int32_t>(), max_ctx, B, l, c.num_heads, c.num_kv_heads, c.head_dim,
                              m->gemm ? nullptr : m->attn.as<float>(), m->q_dim, m->att_ws.as<float>(), m->att_floats,
                              m->att_segs, st, so_q, prof, GLACIER_CUDA_STEP_ATTN_COMBINE)))
      return rc;
    mark(GLACIER_CUDA_STEP_PROJ_O);
    if ((rc = project(L.o.w, m->attn.as<float>(), m->q_dim, so_q, m->map_q, m->proj.as<float>(), D, so_gemm)))
      return rc;
    // Tensor parallel: o summed over the ranks' head slices.
    if (m->tp_comm && (rc = tp_reduce(m->proj.as<float>(), so_gemm))) return rc;
    mark(GLACIER_CUDA_STEP_NORM);
    if ((rc = add_rmsnorm(x, D, m->proj.as<float>(), D, B * D, so_, x, D, L.post_norm.as<float>(), c.rms_eps,
                          m->gemm ? nullptr : hn, D, B, D, st, so_d)))
      return rc;
    mark(GLACIER_CUDA_STEP_PROJ_GATE_UP);
    if ((rc = project(L.gu.w, hn, D, so_d, m->map_d, m->gu.as<float>(), 2 * F, 1))) return rc;
    // GEMV mode: the down projection's activation loads compute silu(gate) * up
    // themselves (no SiLU launch); otherwise the SiLU kernel writes the split
    // (GEMM) or fp32 activations first.
    rc = m->gemm ? GLACIER_CUDA_EUNSUPPORTED : GLACIER_CUDA_OK;
    if (!m->gemm) {
      mark(GLACIER_CUDA_STEP_PROJ_DOWN);
      rc = int4_linear_swiglu(L.d.w, m->gu.as<float>(), m->gu.as<float>() + F, 2 * F, B, nullptr,
                              m->down.as<float>(), D, st);
      if (rc && rc != GLACIER_CUDA_EUNSUPPORTED) return rc;
    }
    if (rc == GLACIER_CUDA_EUNSUPPORTED) {
      mark(GLACIER_CUDA_STEP_SILU);
      if ((rc = silu_mul(m->gu.as<float>(), m->gu.as<float>() + F, 2 * F, m->gemm ? nullptr : m->act.as<float>(), F,
                         B, F, st, so_f)))
        return rc;
      mark(GLACIER_CUDA_STEP_PROJ_DOWN);
      if ((rc = project(L.d.w, m->act.as<float>(), F, so_f, m->map_f, m->down.as<float>(), D, sd_gemm))) return rc;
    }
    // Tensor parallel: down summed over the ranks' FFN slices.
    if (m->tp_comm && (rc = tp_reduce(m->down.as<float>(), sd_gemm))) return rc;
  }
  if (head == kHeadNone) {
    mark(-1);
    return GLACIER_CUDA_OK;
  }
  if (head == kHeadLastRow) {
    // Final residual + RMSNorm of the last row only (fp32), its LM-head GEMV and argmax.
    const size_t r = B - 1;
    mark(GLACIER_CUDA_STEP_NORM);
    if ((rc = add_rmsnorm(x + r * D, D, m->down.as<float>() + r * D, D, B * D, sd, x + r * D, D,
                          m->final_norm.as<float>(), c.rms_eps, hn, D, 1, D, st)))
      return rc;
    mark(GLACIER_CUDA_STEP_LM_HEAD);
    rc = lm_head_argmax(hn, 1);
    if (rc != GLACIER_CUDA_EUNSUPPORTED) {
      mark(-1);
      return rc;
    }
    float* logits = logits_out ? logits_out : m->logits.as<float>();
    if ((rc = int4_linear(m->lm.w, hn, D, 1, nullptr, logits, c.vocab, st))) return rc;
    mark(GLACIER_CUDA_STEP_ARGMAX);
    rc = argmax_rows(logits, c.vocab, 1, c.vocab, eligible, eligible_words, nullptr, tokens_out, st_out,
                     m->arg_ws.p, m->arg_bytes, st);
    mark(-1);
    return rc;
  }
  mark(GLACIER_CUDA_STEP_NORM);
  if ((rc = add_rmsnorm(x, D, m->down.as<float>(), D, B * D, sd, x, D, m->final_norm.as<float>(), c.rms_eps,
                        m->gemm ? nullptr : hn, D, B, D, st, so_d)))
    return rc;
  mark(GLACIER_CUDA_STEP_LM_HEAD);
  // GEMV mode: the argmax runs in the LM head's epilogue.  The tcgen05 GEMM
  // writes the logits and the two-pass argmax reads them: an epilogue argmax
  // there (64 cross-row warp reductions per tile) doubled the LM head's time.
  if (!m->gemm) {
    rc = lm_head_argmax(hn, B);
    if (rc != GLACIER_CUDA_EUNSUPPORTED) {
      mark(-1);
      return rc;
    }
  }
  float* logits = logits_out ? logits_out : m->logits.as<float>();
  if ((rc = project(m->lm.w, hn, D, so_d, m->map_d, logits, c.vocab, 1))) return rc;
  mark(GLACIER_CUDA_STEP_ARGMAX);
  rc = argmax_rows(logits, c.vocab, B, c.vocab, eligible, eligible_words, nullptr, tokens_out, st_out,
                   m->arg_ws.p, m->arg_bytes, st);
  mark(-1);
  return rc;
}

int glacier_cuda_decode_step(glacier_cuda_model* m, glacier_cuda_kv* kv, size_t lanes, const int32_t* tokens,
                             const int32_t* positions, const int32_t* block_tables, size_t max_pages,
                             const uint64_t* eligible, size_t eligible_words, int32_t* tokens_out,
                             int32_t* status_out, float* logits_out, void* stream_ptr) {
  GLC_REQUIRE(m && kv && m->finalized, "decode_step: model not finalized");
  GLC_REQUIRE(lanes > 0 && lanes <= m->max_lanes, "decode_step: %zu lanes, %zu reserved", lanes, m->max_lanes);
  GLC_REQUIRE(max_pages > 0 && max_pages <= m->max_pages, "decode_step: %zu pages per lane, %zu reserved", max_pages,
              m->max_pages);
  GLC_REQUIRE(tokens && positions && block_tables && tokens_out, "decode_step: null argument");
  if (eligible)
    GLC_REQUIRE(eligible_words == ceil_div(m->cfg.vocab, 64), "decode_step: eligible mask needs %zu words per lane",
                ceil_div(m->cfg.vocab, 64));
  return step_impl(m, kv, lanes, tokens, positions, block_tables, max_pages, eligible, eligible_words, tokens_out,
                   status_out, logits_out, (cudaStream_t)stream_ptr, kHeadAllRows);
}

int glacier_cuda_prefill(glacier_cuda_model* m, glacier_cuda_kv* kv, const int32_t* tokens, size_t count,
                         int32_t start, const int32_t* block_table, size_t max_pages, const uint64_t* eligible,
                         size_t eligible_words, int32_t* token_out, int32_t* status_out, float* logits_out,
                         void* stream_ptr) {
  GLC_REQUIRE(m && kv && m->finalized && m->max_lanes > 0, "prefill: model not finalized and reserved");
  GLC_REQUIRE(tokens && block_table && token_out && count > 0 && start >= 0, "prefill: null or empty argument");
  GLC_REQUIRE(max_pages > 0 && max_pages <= m->max_pages, "prefill: %zu pages, %zu reserved", max_pages,
              m->max_pages);
  GLC_REQUIRE((size_t)start + count <= max_pages * 16, "prefill: positions %d..%zu exceed the block table", start,
              (size_t)start + count - 1);
  if (eligible)
    GLC_REQUIRE(eligible_words == ceil_div(m->cfg.vocab, 64), "prefill: eligible mask needs %zu words",
                ceil_div(m->cfg.vocab, 64));
  cudaStream_t st = (cudaStream_t)stream_ptr;
  const size_t chunk = m->max_lanes;
  int32_t* pos = m->pf_pos.as<int32_t>();
  int32_t* bt = m->pf_bt.as<int32_t>();
  for (size_t b0 = 0; b0 < count; b0 += chunk) {
    const size_t nb = std::min(chunk, count - b0);
    // Positions start + b0 + i and the request's block table for every row of the chunk.
    int rc = launch_pdl(prefill_rows_kernel, dim3((unsigned)nb), dim3(256), 0, st, 1, block_table, (int)max_pages,
                        start + (int)b0, pos, bt);
    if (rc) return rc;
    const bool last = b0 + nb == count;
    rc = step_impl(m, kv, nb, tokens + b0, pos, bt, max_pages, eligible, eligible_words, token_out, status_out,
                   logits_out, st, last ? kHeadLastRow : kHeadNone);
    if (rc) return rc;
  }
  return GLACIER_CUDA_OK;
}

int glacier_cuda_tp_unique_id(void* id_out) { return tp_unique_id(id_out); }

int glacier_cuda_model_tp_init(glacier_cuda_model* m, int rank, int world, const void* id) {
  GLC_REQUIRE(m && m->finalized, "model_tp_init: model not finalized");
  GLC_REQUIRE(!m->tp_comm, "model_tp_init: tensor parallelism already set up");
  const int rc = bind_device(m);
  if (rc) return rc;
  void* comm = nullptr;
  const int r = tp_comm_create(&comm, rank, world, id);
  if (r) return r;
  m->tp_comm = comm;
  m->tp_rank = rank;
  m->tp_world = world;
  return GLACIER_CUDA_OK;
}

int glacier_cuda_model_tp_lanes(glacier_cuda_model* m, int groups, int index) {
  GLC_REQUIRE(m && m->tp_comm, "model_tp_lanes: tensor parallelism not set up");
  GLC_REQUIRE(groups >= 1 && index >= 0 && index < groups, "model_tp_lanes: lane group %d of %d", index, groups);
  m->tp_lane_groups = groups;
  m->tp_lane_index = index;
  return GLACIER_CUDA_OK;
}

int glacier_cuda_model_profile(glacier_cuda_model* m, int enable) {
  GLC_REQUIRE(m, "model_profile: null model");
  m->prof.on = enable != 0;
  return GLACIER_CUDA_OK;
}

int glacier_cuda_model_profile_read(glacier_cuda_model* m, double* ms, uint64_t* regions, size_t kinds) {
  GLC_REQUIRE(m && ms && regions && kinds > 0, "model_profile_read: null argument");
  int rc = bind_device(m);
  if (rc) return rc;
  if ((rc = m->prof.read(ms, regions, kinds))) return rc;
  if (m->ps) {
    // Phases of the persistent step, filed under the kernel classes they replace.
    unsigned long long ns[8], n[8];
    if ((rc = persist_read_stats(m->ps, ns, n))) return rc;
    const int kind_of[7] = {GLACIER_CUDA_STEP_PROJ_QKV, GLACIER_CUDA_STEP_ATTENTION,  GLACIER_CUDA_STEP_PROJ_O,
                            GLACIER_CUDA_STEP_PROJ_GATE_UP, GLACIER_CUDA_STEP_PROJ_DOWN, GLACIER_CUDA_STEP_LM_HEAD,
                            GLACIER_CUDA_STEP_ARGMAX};
    for (int i = 0; i < 7; ++i) {
      const size_t k = (size_t)kind_of[i];
      if (k >= kinds || n[i] == 0) continue;
      ms[k] += (double)ns[i] * 1e-6;
      regions[k] += n[i];
    }
  }
  return GLACIER_CUDA_OK;
}

int glacier_cuda_model_persistent(glacier_cuda_model* m, int enable) {
  GLC_REQUIRE(m, "model_persistent: null model");
  m->persistent = enable != 0;
  return m->ps ? 1 : 0;
}

}  // extern "C"

namespace glacier {
const glacier_cuda_model_config* model_config(const glacier_cuda_model* m) { return &m->cfg; }
}  // namespace glacier

