// Kernel (e): on-device greedy selection, so only token ids leave the GPU.
//
// Semantics of argmaxEligible (src/sampling.zig:55-107) per batch row:
//  * the eligibility bitset has exactly ceil(n/64) words per row (checked on
//    the host), keeps every bit >= n clear and has at least one set bit;
//    otherwise the row's status is InvalidEligibleMask;
//  * only set bits are read; an eligible NaN makes the status EligibleLogitNaN;
//  * infinities are valid scores; equal scores resolve to the lowest index.
// Without a bitset every row is eligible (greedy argmax, sampling.zig:194-207,
// first maximum wins), and a NaN logit is reported the way the reference's
// logitless greedy kernel does (int4_neon.c:1075-1254: saw_nan, not valid).
//
// Two deterministic passes: per-(row, chunk) partial winners, then a per-row
// reduction in chunk order.
#include <mutex>

#include "common.cuh"

namespace glacier {

namespace {

constexpr int kArgThreads = 256;
constexpr int kArgChunk = 8192;  // logits per partial

struct Cand {
  float v;
  int i;  // -1: none
};

// a beats b: larger value, or equal value with the lower index.
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

__global__ void __launch_bounds__(kArgThreads) argmax_partial_kernel(
    const float* __restrict__ logits, size_t ld, int n, const uint64_t* __restrict__ words, int word_count,
    float* __restrict__ pv, int* __restrict__ pi, int* __restrict__ pflags, int nchunks) {
  griddep_launch();
  griddep_wait();
  const int row = blockIdx.y, chunk = blockIdx.x;
  const int c0 = chunk * kArgChunk, c1 = min(n, c0 + kArgChunk);
  const float* lg = logits + row * ld;
  const uint64_t* wr = words ? words + (size_t)row * word_count : nullptr;
  Cand best{0.f, -1};
  int nan = 0, eligible = 0, tail_bad = 0;
  for (int k = c0 + threadIdx.x; k < c1; k += blockDim.x) {
    bool ok = true;
    if (wr) ok = (wr[k >> 6] >> (k & 63)) & 1ull;
    if (!ok) continue;
    ++eligible;
    const float v = lg[k];
    if (v != v) {
      nan = 1;
      continue;
    }
    Cand c{v, k};
    if (better(c, best)) best = c;
  }
  // Tail bits of the last word must be clear (checked once, by chunk 0).
  if (wr && chunk == 0 && threadIdx.x == 0 && (n & 63)) {
    const uint64_t valid = (1ull << (n & 63)) - 1;
    if (wr[word_count - 1] & ~valid) tail_bad = 1;
  }
  __shared__ Cand sb[kArgThreads / 32];
  __shared__ int sf[kArgThreads / 32][2];
  best = warp_best(best);
  nan = __reduce_or_sync(0xffffffffu, nan);
  eligible = __reduce_add_sync(0xffffffffu, eligible);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sb[w] = best;
    sf[w][0] = nan;
    sf[w][1] = eligible;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    Cand b = sb[0];
    int fl = sf[0][0], el = sf[0][1];
    for (int i = 1; i < kArgThreads / 32; ++i) {
      if (better(sb[i], b)) b = sb[i];
      fl |= sf[i][0];
      el += sf[i][1];
    }
    const size_t o = (size_t)row * nchunks + chunk;
    pv[o] = b.v;
    pi[o] = b.i;
    // flags: bit0 NaN seen among eligible rows, bit1 tail bits set; count above.
    pflags[2 * o] = fl | (tail_bad << 1);
    pflags[2 * o + 1] = el;
  }
}

__global__ void argmax_final_kernel(const float* __restrict__ pv, const int* __restrict__ pi,
                                    const int* __restrict__ pflags, int nchunks, int masked,
                                    glacier_argmax_result* __restrict__ out, int32_t* __restrict__ tokens,
                                    int32_t* __restrict__ status) {
  griddep_launch();
  griddep_wait();
  const int row = blockIdx.x;
  if (threadIdx.x != 0) return;
  Cand b{0.f, -1};
  int nan = 0, tail = 0;
  long long eligible = 0;
  for (int c = 0; c < nchunks; ++c) {
    const size_t o = (size_t)row * nchunks + c;
    Cand t{pv[o], pi[o]};
    if (better(t, b)) b = t;
    nan |= pflags[2 * o] & 1;
    tail |= (pflags[2 * o] >> 1) & 1;
    eligible += pflags[2 * o + 1];
  }
  int st = GLACIER_CUDA_OK;
  if (masked && (tail || eligible == 0)) st = GLACIER_CUDA_EMASK;
  else if (nan) st = GLACIER_CUDA_ENAN;
  else if (b.i < 0) st = GLACIER_CUDA_EMASK;
  if (out) {
    out[row].value = b.i >= 0 ? b.v : -INFINITY;
    out[row].index = b.i >= 0 ? (size_t)b.i : 0;
    out[row].valid = st == GLACIER_CUDA_OK;
    out[row].saw_nan = nan;
  }
  if (tokens) tokens[row] = st == GLACIER_CUDA_OK ? b.i : -1;
  if (status) status[row] = st;
}

}  // namespace

size_t argmax_workspace_bytes(size_t batch, size_t n) {
  const size_t chunks = ceil_div(n, kArgChunk);
  return batch * chunks * (sizeof(float) + 3 * sizeof(int)) + 64;
}

int argmax_rows(const float* logits, size_t ld, size_t batch, size_t n, const uint64_t* words, size_t word_count,
                glacier_argmax_result* out, int32_t* tokens, int32_t* status, void* workspace, size_t ws_bytes,
                cudaStream_t stream) {
  GLC_REQUIRE(logits && batch > 0 && n > 0 && n < (1u << 31), "argmax: empty or null argument");
  if (words) GLC_REQUIRE(word_count == ceil_div(n, 64), "argmax: eligible mask needs %zu words per row, got %zu",
                         ceil_div(n, 64), word_count);
  GLC_REQUIRE(workspace && ws_bytes >= argmax_workspace_bytes(batch, n), "argmax: workspace too small");
  const int chunks = (int)ceil_div(n, kArgChunk);
  float* pv = static_cast<float*>(workspace);
  int* pi = reinterpret_cast<int*>(pv + batch * chunks);
  int* pf = pi + batch * chunks;
  int rc = launch_pdl(argmax_partial_kernel, dim3(chunks, (unsigned)batch), dim3(kArgThreads), 0, stream, 1, logits,
                      ld, (int)n, words, (int)word_count, pv, pi, pf, chunks);
  if (rc) return rc;
  rc = launch_pdl(argmax_final_kernel, dim3((unsigned)batch), dim3(32), 0, stream, 1, (const float*)pv, (const int*)pi,
                  (const int*)pf, chunks, (int)(words != nullptr), out, tokens, status);
  if (rc) return rc;
  return GLACIER_CUDA_OK;
}

}  // namespace glacier

// ---------------------------------------------------------------------------
// Allocation-free variant: glacier_cuda_argmax_eligible_f32_noalloc.
//
// Some callers cannot allocate device memory at the point where they pick the
// next token: a host runtime that budgets every byte of GPU memory when it
// admits a request, or a plugin that is handed buffers but no allocator.
// cudaMalloc can also synchronise the device and fail under memory pressure.
// This entry point therefore takes no workspace. Its partial winners live in
// one fixed array of device memory that is part of the library image.
//
// Limits and sharing:
//  * the array holds GLACIER_CUDA_ARGMAX_NOALLOC_SCRATCH_BYTES (64 KiB); calls
//    whose batch and vocabulary need more are rejected before any launch;
//  * every GPU that loads the library keeps its copy of the array until the
//    process exits;
//  * all calls on a device share the one array, so calls that overlap on the
//    GPU (different streams, or host threads racing) corrupt each other's
//    partial results. Order them on one stream or serialise them;
//  * the array keeps the previous call's contents. Nothing needs clearing:
//    the first pass writes every partial slot that the second pass reads;
//  * the first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current and caches it. Make that
//    first call before any stream capture begins on the device. The cached
//    address is valid while the CUDA context that first loaded the library on
//    the device lives: after cudaDeviceReset the module is reloaded elsewhere,
//    so a process that resets a device must not call this entry point on it
//    again.
// ---------------------------------------------------------------------------

static_assert(GLACIER_CUDA_ARGMAX_NOALLOC_SCRATCH_BYTES % 256 == 0, "scratch size must keep 256-byte alignment");
static __device__ __align__(256) unsigned char g_argmax_scratch[GLACIER_CUDA_ARGMAX_NOALLOC_SCRATCH_BYTES];

namespace glacier {
namespace {

constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_address[kMaxScratchDevices];  // device address of g_argmax_scratch, per device

// Host code cannot use g_argmax_scratch's name as a device address: on the
// host it names a shadow variable. Ask the runtime once per device, with that
// device current, and cache the answer.
int scratch_for_current_device(void** out) {
  int dev = -1;
  GLC_CHECK_CUDA(cudaGetDevice(&dev));
  GLC_REQUIRE(dev >= 0 && dev < kMaxScratchDevices, "argmax_noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_address[dev]) {
    void* p = nullptr;
    GLC_CHECK_CUDA(cudaGetSymbolAddress(&p, g_argmax_scratch));
    GLC_REQUIRE(p != nullptr && (reinterpret_cast<uintptr_t>(p) & 255) == 0,
                "argmax_noalloc: scratch address is not 256-byte aligned");
    g_scratch_address[dev] = p;
  }
  *out = g_scratch_address[dev];
  return GLACIER_CUDA_OK;
}

}  // namespace

}  // namespace glacier

extern "C" int glacier_cuda_argmax_eligible_f32_noalloc(const float* logits, size_t batch, size_t n,
                                                        const uint64_t* words, size_t word_count, int32_t* tokens,
                                                        int32_t* status, glacier_argmax_result* results,
                                                        void* stream) {
  using namespace glacier;
  GLC_REQUIRE(logits && batch > 0 && n > 0 && n < (1u << 31), "argmax_noalloc: empty or null argument");
  const size_t need = argmax_workspace_bytes(batch, n);
  GLC_REQUIRE(need <= GLACIER_CUDA_ARGMAX_NOALLOC_SCRATCH_BYTES,
              "argmax_noalloc: batch %zu x %zu logits needs %zu bytes of scratch, the fixed scratch holds %d; "
              "use glacier_cuda_argmax_eligible_f32 with a workspace",
              batch, n, need, GLACIER_CUDA_ARGMAX_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != GLACIER_CUDA_OK) return rc;
  return argmax_rows(logits, n, batch, n, words, word_count, results, tokens, status, scratch,
                     GLACIER_CUDA_ARGMAX_NOALLOC_SCRATCH_BYTES, (cudaStream_t)stream);
}
