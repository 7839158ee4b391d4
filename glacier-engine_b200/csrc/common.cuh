// Shared helpers for the Glacier B200 INT4 decode library (sm_100a only).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <vector>

#include "glacier_cuda.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "glacier_cuda targets sm_100a only"
#endif

namespace glacier {

// Records a message for glacier_cuda_last_error(); returns the status code.
int set_error(int code, const char* fmt, ...);

#define GLC_CHECK_CUDA(expr)                                                        \
  do {                                                                              \
    cudaError_t _e = (expr);                                                        \
    if (_e != cudaSuccess)                                                          \
      return ::glacier::set_error(GLACIER_CUDA_ECUDA, "%s failed: %s (%s:%d)", #expr, \
                                  cudaGetErrorString(_e), __FILE__, __LINE__);      \
  } while (0)

#define GLC_REQUIRE(cond, ...)                                                      \
  do {                                                                              \
    if (!(cond)) return ::glacier::set_error(GLACIER_CUDA_EINVAL, __VA_ARGS__);     \
  } while (0)

// Counts every kernel this library launches (process-wide, all devices).
void note_launch();

// Launch-error check after a kernel launch (no device synchronisation).
#define GLC_CHECK_LAUNCH()      \
  do {                          \
    ::glacier::note_launch();   \
    GLC_CHECK_CUDA(cudaGetLastError()); \
  } while (0)

__host__ __device__ inline size_t ceil_div(size_t a, size_t b) { return (a + b - 1) / b; }

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue now; wait until the previous kernel's writes are visible.
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Number of SMs of the current device (cached per device).
int sm_count();

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda
// link dependency).  Returns a GLACIER_CUDA_* status.
int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                   uint64_t outer, uint64_t outer_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                   CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo);

// Device address of a library __device__ variable on the current device, looked
// up once per (variable, device) (host code cannot use the variable's name as
// an address).  Returns nullptr on failure.  The cached address is valid while
// the CUDA context that first loaded the library on that device lives (a
// cudaDeviceReset reloads the module, and the library is not used after one).
void* device_symbol_address_raw(const void* symbol);
template <typename T>
inline T* device_symbol_address(const T& symbol) {
  return static_cast<T*>(device_symbol_address_raw(static_cast<const void*>(&symbol)));
}

// Allows `bytes` of dynamic shared memory for `kernel` on the current device
// (the attribute is set once per kernel, device and larger size).
int allow_dynamic_smem(const void* kernel, int bytes);

// Launch with programmatic dependent launch allowed (and an optional cluster
// size): the kernel may start while its stream predecessor is still running,
// and every kernel of this library calls griddep_wait() before it touches
// memory that a predecessor writes, so results are as if serialised.
template <typename Kern, typename... Args>
inline int launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, int cluster,
                      Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  GLC_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...));
  note_launch();
  return GLACIER_CUDA_OK;
}

// Optional per-kernel-class timing of a multi-kernel step: while `on`, mark()
// records a CUDA event on the launching stream that closes the open region and
// opens one of `kind` (kind < 0 only closes).  The events are read back later,
// so the step is never synchronised.  Host-side only; one owner per instance.
struct StepProfiler {
  static constexpr size_t kMaxEvents = 1 << 16;
  bool on = false;
  bool overflow = false;
  size_t used = 0;
  std::vector<cudaEvent_t> events;
  std::vector<int> kinds;
  void mark(int kind, cudaStream_t stream);
  // Sums region times per kind into ms[kind] / regions[kind] (kind < kinds_n),
  // waiting for the last event; then forgets the records.
  int read(double* ms, uint64_t* regions, size_t kinds_n);
  ~StepProfiler();
};

// A device-resident INT4 weight: the reference's exact nibble packing plus one
// scale row per output row (fp16 mirror or the original fp32), with the TMA
// descriptors of the tensor-core GEMV encoded once.
struct Int4Weight {
  const uint8_t* packed = nullptr;  // [M, K/2] (or the flat packing when !row_groups)
  const void* scales = nullptr;     // [M, scale_stride] or flat [ceil(M*K/group)]
  bool f16 = true;
  size_t scale_stride = 0;          // elements per scale row; 0 = flat reference array
  size_t M = 0, K = 0, group = 0;
  bool tc = false;                  // tensor-core GEMV eligible (group 32, maps valid)
  bool tcg = false;                 // tensor-core GEMM maps valid (group 8, 16 or 32)
  bool nonfinite = false;           // fp16 scales hold an infinity or NaN: exact-conversion kernels
  CUtensorMap tmap_w, tmap_s;
};

// Validates the layout and encodes TMA maps when the tensor-core path applies.
int int4_weight_prepare(Int4Weight& w);

// y[b, :] = x[b, :] * dequant(W)^T + bias for b < batch (row strides ldx, ldy).
int int4_linear(const Int4Weight& w, const float* x, size_t ldx, size_t batch, const float* bias, float* y,
                size_t ldy, cudaStream_t stream);

// The Q8-activation form (linearInt4WeightQ8 on a non-AArch64 host): bit-identical
// to the reference's portable path; LM-head-sized outputs and long inputs run int4_linear.
int int4_linear_q8(const Int4Weight& w, const float* x, size_t ldx, size_t batch, const float* bias, float* y,
                   size_t ldy, cudaStream_t stream);

// y[b, :] = (silu(gate[b, :]) * up[b, :]) * dequant(W)^T + bias on the tensor-core
// GEMV with the SwiGLU folded into its activation loads (gate and up share the
// row stride ld); GLACIER_CUDA_EUNSUPPORTED when that kernel does not apply.
int int4_linear_swiglu(const Int4Weight& w, const float* gate, const float* up, size_t ld, size_t batch,
                       const float* bias, float* y, size_t ldy, cudaStream_t stream);

// Epilogue of the LM head's GEMV (up to 4 rows): the eligible argmax of each
// activation row (the semantics of argmax_rows).  Every warp reduces the 32
// output columns it produced to one winner record {value, index, NaN seen,
// eligible count} at partials[row * records + column / 32]; a one-CTA-per-row
// kernel (argmax_records_reduce) reduces the records.  `partials` holds
// argmax_records_bytes(rows, M) bytes.
struct ArgmaxEpi {
  const uint64_t* words = nullptr;  // eligibility bitset rows of word_count words, or null
  int word_count = 0;
  int32_t* tokens = nullptr;
  int32_t* status = nullptr;
  glacier_argmax_result* results = nullptr;  // optional per-row records
  int4* partials = nullptr;
};

// y = x W^T on the tensor-core GEMV (up to 4 rows, no bias; y may be null: no
// logits), then the eligible argmax of each row into a.tokens / a.status.
// GLACIER_CUDA_EUNSUPPORTED when the tensor-core GEMV does not apply.
int int4_linear_argmax(const Int4Weight& w, const float* x, size_t ldx, size_t batch, float* y, size_t ldy,
                       const ArgmaxEpi& a, cudaStream_t stream);
size_t argmax_records_bytes(size_t rows, size_t M);

// The tcgen05 GEMM on split-form activations (int4_gemm_tc.cu): y[b, :] for the
// n live rows of np, nsplit K-split partials split_stride apart.
int gemm_int4_tc(const Int4Weight& w, const CUtensorMap& xmap, const float* xscale, size_t n, size_t np, float* y,
                 size_t ldy, int nsplit, size_t split_stride, const float* bias, cudaStream_t stream);
// Tokens, statuses and records of `rows` rows from their `records` winner records each.
int argmax_records_reduce(const ArgmaxEpi& a, size_t rows, size_t records, size_t n, cudaStream_t stream);
int* ops_error_word();

// Destination of an activation block that feeds the tensor-core GEMM: rows of
// fp16 hi / lo parts ([2*np, K]: hi rows 0..np-1, lo rows np..2np-1) in the
// per-8 code order (0,4,1,5,2,6,3,7), plus one power-of-two scale per row
// (x = scale * (hi + lo)).  xs == nullptr selects a plain fp32 destination.
struct SplitOut {
  __half* xs = nullptr;
  float* xscale = nullptr;
  int np = 0;
};

// Device-side error words (written by kernels that give up waiting).
enum DeviceError : int { kErrNone = 0, kErrTimeout = 1 };

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

// Streaming 128-bit load of read-once weight bytes: bypass L1, evict early
// from L2 so the activations and KV stay resident.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint4 ld_stream_u4(const void* p, uint64_t policy) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(policy));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t d;
  // (a & mask) | orv  -> LUT 0xEA
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(orv));
  return d;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier ----------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// try_wait with a suspend-time hint: a waiting thread sleeps in hardware until
// the phase completes (or ~1 ms passes) instead of spinning on the issue port.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}
// Bounded wait: returns false (and raises *err) when the phase does not
// complete within kSpinLimitCycles SM clock cycles (about two seconds); the
// cycle counter is checked every 8 (hardware-suspended) polls.
constexpr long long kSpinLimitCycles = 4000000000ll;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
#pragma unroll 1
  for (int it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 7) == 0 && clock64() - t0 > kSpinLimitCycles) {
      if (err) atomicExch(err, kErrTimeout);
      return false;
    }
  }
}

// True in exactly one lane of a converged warp.
__device__ __forceinline__ bool elect_one() {
  uint32_t p;
  asm volatile("{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\tselp.u32 %0, 1, 0, P;\n\t}" : "=r"(p));
  return p != 0;
}

// Non-blocking probe of a phase (no suspension), for the one thread on a
// pipeline's critical path: a satisfied try_wait costs it hundreds of cycles.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded polling wait built on mbar_test_wait (same limit as mbar_wait).
__device__ __forceinline__ bool mbar_wait_poll(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_test_wait(bar, parity)) return true;
  const long long t0 = clock64();
#pragma unroll 1
  for (int it = 1;; ++it) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((it & 63) == 0 && clock64() - t0 > kSpinLimitCycles) {
      if (err) atomicExch(err, kErrTimeout);
      return false;
    }
  }
}

// ---- TMA ---------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---- clusters ----------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// Power-of-two scale s with max|x| / s in [2^14, 2^15) (1 for an all-zero row).
__device__ __forceinline__ float split_scale(float m) {
  if (!(m > 0.f) || !isfinite(m)) return 1.f;
  int e;
  frexpf(m, &e);
  return ldexpf(1.f, e - 15);
}

// (sum, max) over the row: block reduction, then the cluster's CTAs through DSMEM.
__device__ __forceinline__ float2 row_sum_max(float s, float m, float2* sh, float2* xch) {
  s = warp_sum(s);
  m = warp_max(m);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  if (l == 0) sh[w] = make_float2(s, m);
  __syncthreads();
  if (w == 0) {
    float2 t = l < nw ? sh[l] : make_float2(0.f, 0.f);
    t.x = warp_sum(t.x);
    t.y = warp_max(t.y);
    if (l == 0) *xch = t;
  }
  const uint32_t cn = cluster_nctarank();
  if (cn == 1) {
    __syncthreads();
    return *xch;
  }
  cluster_sync_all();
  const uint32_t a = smem_u32(xch);
  float2 r = make_float2(0.f, 0.f);
  for (uint32_t q = 0; q < cn; ++q) {
    const uint32_t pa = mapa_shared(a, q);
    r.x += ld_dsmem_f32(pa);
    r.y = fmaxf(r.y, ld_dsmem_f32(pa + 4));
  }
  return r;
}

__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Writes 8 consecutive values (k = base..base+7 of row r) in split form.
__device__ __forceinline__ void store_split8(const SplitOut& so, int r, size_t K, size_t base, const float (&v)[8],
                                             float inv_scale) {
  __half h[8], l[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float x = v[(i & 1) ? 4 + (i >> 1) : (i >> 1)] * inv_scale;  // order (0,4,1,5,2,6,3,7)
    h[i] = __float2half_rn(x);
    l[i] = __float2half_rn(x - __half2float(h[i]));
  }
  *reinterpret_cast<uint4*>(so.xs + (size_t)r * K + base) = *reinterpret_cast<uint4*>(h);
  *reinterpret_cast<uint4*>(so.xs + ((size_t)so.np + r) * K + base) = *reinterpret_cast<uint4*>(l);
}

// fp16 bits (low 16 bits of h) to the equal fp32 value without the conversion
// unit: the magnitude bits shifted into an fp32 field give the value times
// 2^-112 for normal and subnormal inputs alike (the fp32 result of a subnormal
// input is itself subnormal), and the power-of-two product is exact.  Finite
// inputs only: weights whose fp16 scales hold an infinity or NaN are flagged at
// load (Int4Weight::nonfinite) and read through the conversion instruction.  In
// hot loops this keeps the fp16 -> fp32 scale conversions off the narrow
// special-function pipe.
__device__ __forceinline__ float half_to_float_bits(uint32_t h) {
  const uint32_t b = ((h & 0x8000u) << 16) | ((h & 0x7FFFu) << 13);
  return __uint_as_float(b) * 0x1p112f;
}

// Argmax candidate order of argmaxEligible (sampling.zig:55-107): larger value,
// equal values to the lower index; i < 0 is "none".
__device__ __forceinline__ bool arg_better(float av, int ai, float bv, int bi) {
  if (ai < 0) return false;
  if (bi < 0) return true;
  return av > bv || (av == bv && ai < bi);
}

__device__ __forceinline__ void arg_warp_reduce(float& v, int& i, int& nan, int& elig) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float tv = __shfl_xor_sync(0xffffffffu, v, o);
    const int ti = __shfl_xor_sync(0xffffffffu, i, o);
    if (arg_better(tv, ti, v, i)) {
      v = tv;
      i = ti;
    }
    nan |= __shfl_xor_sync(0xffffffffu, nan, o);
    elig += __shfl_xor_sync(0xffffffffu, elig, o);
  }
}

// fp16 scale bits with exponent 31 (infinity or NaN).
__host__ __device__ inline bool half_bits_nonfinite(uint16_t h) { return (h & 0x7C00u) == 0x7C00u; }

// Scale loads: the library keeps fp16 scale mirrors (as the reference's
// int4_weights.withF16Scales does) but also accepts fp32 scales.
__device__ __forceinline__ float load_scale(const __half* s, size_t i) { return __half2float(s[i]); }
__device__ __forceinline__ float load_scale(const float* s, size_t i) { return s[i]; }

}  // namespace glacier
