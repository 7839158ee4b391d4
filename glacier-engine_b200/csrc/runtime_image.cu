// Host-side reader for the prepared runtime image (`.glrt`) and the loader
// that uploads one into a device-resident model.
//
// Image (src/model/runtime_image.zig, docs/RUNTIME_IMAGE.md; little-endian):
//   [0, 512)              header: config snapshot, fingerprints, CRCs (:206-292)
//   [512, +count*rsize)   records, 128 bytes (v1) or 160 bytes (v2) (:308-430)
//   [data_offset, size)   64-byte aligned streams per record, in the order
//                         packed_weights, scales_f32, scales_f16, scales_f16_rows4, raw
// A record is one tensor (raw f32, or INT4 in row-major or rows4_k16 nibble
// order) or, in v2, one MLP gate/up PairNibble artifact.
//
// Admission mirrors MappedImage.openOwnedFileWithOptionsV1 (:828-850):
// Header.decode, validateHeaderBytes (:1336-1376), then per record in index
// order its descriptor and bounds (:432-578), identity and overlap against
// every earlier record, and its payload CRC and v2 SHA-256 digest
// (validateIndexAndRecords, :1005-1056).  Content checks run on all host cores;
// the failure reported is the one the sequential walk meets first.
//
// Loading mirrors loader.zig loadPreparedOwnedFileWithOptionsV1 (:216-385)
// with its schema checks (validatePreparedConfig :618-652,
// validatePreparedRecordSet :656-714, isExpectedPreparedRecord :730-766,
// preparedRaw :785-809, preparedInt4 :811-868, inspectPreparedPairNibble
// :871-912).  rows4_k16 codes, rows4 fp16 scale grids and PairNibble pairs are
// put back into row-major form on the host (int4_weights.zig packedNibbleIndex
// :153-170, withRows4F16Scales :362-386, pairRows4K16 :251-346 read in reverse)
// so the same GEMV/GEMM kernels serve every prepared layout.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "common.cuh"

namespace glacier {

const glacier_cuda_model_config* model_config(const glacier_cuda_model* m);
int32_t* format_error_slot();
uint32_t crc32_ieee(uint32_t crc, const uint8_t* p, size_t n);

namespace {

constexpr uint64_t kHeader = 512, kRecV1 = 128, kRecV2 = 160, kAlign = 64;
constexpr uint32_t kGlobalLayer = 0xFFFFFFFFu;
enum : uint16_t { ENC_RAW = 0, ENC_INT4 = 1, ENC_PAIR = 2 };
enum : uint16_t { LAY_ROW_MAJOR = 0, LAY_ROWS4 = 1, LAY_NONE = 0xFFFF };
enum : uint16_t { ROLE_TENSOR = 0, ROLE_PAIR = 1 };
enum : uint16_t { PAIR_ROWS4 = 0, PAIR_NONE = 0xFFFF };
enum : uint32_t {
  K_EMBEDDING = 0, K_Q = 1, K_K = 2, K_V = 3, K_O = 4, K_UP = 5, K_DOWN = 6, K_GATE = 7, K_INPUT_NORM = 8,
  K_LM_HEAD = 9, K_FINAL_NORM = 10, K_POST_NORM = 11, K_BQ = 12, K_BK = 13, K_BV = 14, K_BO = 15, K_OTHER = 255
};
constexpr int kStreams = 5;  // packed, scales_f32, scales_f16, scales_f16_rows4, raw
enum { S_PACKED = 0, S_F32 = 1, S_F16 = 2, S_ROWS4 = 3, S_RAW = 4 };

// Execution-ABI fingerprints by (version, policy): the SHA-256 values the
// runtime image specification lists for the AArch64 and portable preparation
// policies (docs/RUNTIME_IMAGE.md, "Execution ABI fingerprints").
const char* const kAbiHex[2][2] = {
    {"0c1f185ceff5e9d366a920c8b0046f1543290f85965fbd7cb13f21fe2eec42b6",   // v1 portable
     "dc5fe778a28150235c6f11c53bbf876e130dde0804c3b7a492f4de7e059bc7ad"},  // v1 aarch64
    {"8f291472be36fab2d8e32bfbb87671ebbb18a982036a2d17dc06cbe2907ec890",   // v2 portable
     "d0d7df06350af6b2d48e282f65ff873a3cf95bd6397b1d2d26cc6e679304e06f"}};  // v2 aarch64

bool hex_eq(const char* hex, const uint8_t* bytes) {
  for (int i = 0; i < 32; ++i) {
    unsigned v;
    if (sscanf(hex + 2 * i, "%2x", &v) != 1 || v != bytes[i]) return false;
  }
  return true;
}

int fail(int32_t reason, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int32_t reason, const char* fmt, ...) {
  char buf[400];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  *format_error_slot() = reason;
  return set_error(GLACIER_CUDA_EFORMAT, "runtime image: %s", buf);
}

template <typename T>
T rd(const uint8_t* p) {
  T v;
  memcpy(&v, p, sizeof(T));
  return v;
}

bool all_zero(const uint8_t* p, size_t n) {
  for (size_t i = 0; i < n; ++i)
    if (p[i]) return false;
  return true;
}

uint32_t crc32_of(const uint8_t* p, size_t n, uint32_t crc = 0) { return crc32_ieee(crc, p, n); }

// ------------------------------------------------------------- SHA-256 ----
// FIPS 180-4 SHA-256.
struct Sha256 {
  uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  uint8_t buf[64];
  size_t fill = 0;
  uint64_t total = 0;

  static uint32_t rotr(uint32_t x, int n) { return x >> n | x << (32 - n); }

  void block(const uint8_t* p) {
    static const uint32_t K[64] = {
        0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
        0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
        0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
        0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
        0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
        0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
        0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
        0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + K[i] + w[i];
      const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      hh = g, g = f, f = e, e = d + t1, d = c, c = b, b = a, a = t1 + t2;
    }
    h[0] += a, h[1] += b, h[2] += c, h[3] += d, h[4] += e, h[5] += f, h[6] += g, h[7] += hh;
  }
  void update(const uint8_t* p, size_t n) {
    total += n;
    if (fill) {
      const size_t k = std::min(n, 64 - fill);
      memcpy(buf + fill, p, k);
      fill += k, p += k, n -= k;
      if (fill < 64) return;
      block(buf);
      fill = 0;
    }
    for (; n >= 64; p += 64, n -= 64) block(p);
    memcpy(buf, p, n);
    fill = n;
  }
  void final(uint8_t out[32]) {
    const uint64_t bits = total * 8;
    const uint8_t pad = 0x80;
    update(&pad, 1);
    const uint8_t zero[64] = {};
    update(zero, (fill <= 56 ? 56 : 120) - fill);
    uint8_t len[8];
    for (int i = 0; i < 8; ++i) len[i] = (uint8_t)(bits >> (56 - 8 * i));
    update(len, 8);
    for (int i = 0; i < 8; ++i)
      for (int k = 0; k < 4; ++k) out[4 * i + k] = (uint8_t)(h[i] >> (24 - 8 * k));
  }
};

// --------------------------------------------------------------- records ----
struct Range {
  uint64_t off, len;
};

struct Rec {
  uint32_t layer, kind, group, out_f, in_f, flags, crc;
  uint16_t encoding, layout, role, pair_layout;
  uint64_t n;
  Range s[kStreams];
  uint8_t digest[32];
  const uint8_t* desc;  // the record's bytes in the image
};

struct Image {
  const uint8_t* b;
  uint64_t len;
  uint16_t version;
  uint32_t policy;  // 1 portable, 2 aarch64
  uint64_t count, data_off;
  glacier_cuda_glrt_info info;
  std::vector<Rec> recs;
};

// Header.decode (runtime_image.zig:258-291) and ConfigSnapshot.validate (:191-203).
int decode_header(const uint8_t* b, uint64_t len, Image* im) {
  if (len < kHeader) return fail(GLACIER_CUDA_FMT_TRUNCATED_HEADER, "file of %llu bytes", (unsigned long long)len);
  if (memcmp(b, "GLRT", 4)) return fail(GLACIER_CUDA_FMT_BAD_MAGIC, "magic is not GLRT");
  const uint16_t version = rd<uint16_t>(b + 4);
  if (version != 1 && version != 2) return fail(GLACIER_CUDA_FMT_BAD_VERSION, "version %u", version);
  if (rd<uint16_t>(b + 6) != kHeader) return fail(GLACIER_CUDA_FMT_BAD_HEADER_SIZE, "header_size %u", rd<uint16_t>(b + 6));
  if (rd<uint16_t>(b + 8) != (version == 1 ? kRecV1 : kRecV2))
    return fail(GLACIER_CUDA_FMT_BAD_RECORD_SIZE, "record_size %u for version %u", rd<uint16_t>(b + 8), version);
  if (rd<uint16_t>(b + 10) != kAlign) return fail(GLACIER_CUDA_FMT_BAD_ALIGNMENT, "data_alignment %u", rd<uint16_t>(b + 10));
  if (b[140] > 1) return fail(GLACIER_CUDA_FMT_BAD_CONFIG, "tie_embeddings byte %u", b[140]);
  if (!all_zero(b + 141, 3) || !all_zero(b + 160, kHeader - 160))
    return fail(GLACIER_CUDA_FMT_BAD_RESERVED_FIELD, "reserved header bytes set");
  glacier_cuda_glrt_info& in = im->info;
  memset(&in, 0, sizeof(in));
  in.version = version;
  in.record_count = rd<uint64_t>(b + 16);
  in.data_offset = rd<uint64_t>(b + 32);
  in.file_size = rd<uint64_t>(b + 40);
  memcpy(in.source_fingerprint, b + 48, 32);
  memcpy(in.abi_fingerprint, b + 80, 32);
  in.dim = rd<uint32_t>(b + 112);
  in.hidden = rd<uint32_t>(b + 116);
  in.num_layers = rd<uint32_t>(b + 120);
  in.vocab = rd<uint32_t>(b + 124);
  in.num_heads = rd<uint32_t>(b + 128);
  in.head_dim = rd<uint32_t>(b + 132);
  in.num_kv_heads = rd<uint32_t>(b + 136);
  in.tie_embeddings = b[140];
  in.rms_eps = rd<float>(b + 144);
  in.rope_theta = rd<float>(b + 148);
  if (!in.dim || !in.hidden || !in.num_layers || !in.vocab || !in.num_heads || !in.head_dim || !in.num_kv_heads)
    return fail(GLACIER_CUDA_FMT_BAD_CONFIG, "zero model dimension");
  if (!std::isfinite(in.rms_eps) || in.rms_eps <= 0 || !std::isfinite(in.rope_theta) || in.rope_theta <= 0)
    return fail(GLACIER_CUDA_FMT_BAD_CONFIG, "rms_eps / rope_theta not positive and finite");
  im->version = version;
  im->count = in.record_count;
  im->data_off = in.data_offset;
  return GLACIER_CUDA_OK;
}

// validateHeaderBytes (runtime_image.zig:1336-1376).
int validate_header(const uint8_t* b, uint64_t len, Image* im, const glacier_cuda_glrt_options& o) {
  uint8_t h[kHeader];
  memcpy(h, b, kHeader);
  memset(h + 156, 0, 4);
  if (crc32_of(h, kHeader) != rd<uint32_t>(b + 156)) return fail(GLACIER_CUDA_FMT_HEADER_CRC_MISMATCH, "header CRC");
  if (im->version == 1 && o.reject_v1) return fail(GLACIER_CUDA_FMT_LEGACY_VERSION_DISABLED, "v1 image refused");
  if (rd<uint32_t>(b + 12) != 0 || im->count == 0) return fail(GLACIER_CUDA_FMT_BAD_HEADER, "flags set or no records");
  if (rd<uint64_t>(b + 24) != kHeader || im->info.file_size != len)
    return fail(GLACIER_CUDA_FMT_BAD_BOUNDS, "index offset or file size disagrees with the file");
  uint64_t index_len, index_end;
  if (__builtin_mul_overflow(im->count, (uint64_t)(im->version == 1 ? kRecV1 : kRecV2), &index_len) ||
      __builtin_add_overflow((uint64_t)kHeader, index_len, &index_end))
    return fail(GLACIER_CUDA_FMT_BAD_BOUNDS, "index size overflows");
  if (im->data_off < index_end || im->data_off % kAlign || im->data_off > im->info.file_size)
    return fail(GLACIER_CUDA_FMT_BAD_ALIGNMENT, "data_offset %llu", (unsigned long long)im->data_off);
  if (o.expected_source_fingerprint && memcmp(o.expected_source_fingerprint, b + 48, 32))
    return fail(GLACIER_CUDA_FMT_SOURCE_FINGERPRINT_MISMATCH, "source fingerprint");
  im->policy = 0;
  for (uint32_t p = 0; p < 2; ++p)
    if (hex_eq(kAbiHex[im->version - 1][p], b + 80)) im->policy = p + 1;
  if (!im->policy || (o.abi_policy && o.abi_policy != im->policy))
    return fail(GLACIER_CUDA_FMT_ABI_FINGERPRINT_MISMATCH, "execution ABI fingerprint is not the expected policy");
  im->info.abi_policy = im->policy;
  return GLACIER_CUDA_OK;
}

// Record.decode (runtime_image.zig:383-430).
int decode_record(const uint8_t* r, uint16_t version, uint64_t index, Rec* x) {
  const unsigned long long ix = index;
  if (version == 1 ? !all_zero(r + 120, 8) : !all_zero(r + 124, 4))
    return fail(GLACIER_CUDA_FMT_BAD_RESERVED_FIELD, "record %llu: reserved bytes set", ix);
  x->desc = r;
  x->layer = rd<uint32_t>(r);
  x->kind = rd<uint32_t>(r + 4);
  if (x->kind > K_BO && x->kind != K_OTHER) return fail(GLACIER_CUDA_FMT_BAD_TENSOR_KIND, "record %llu: kind %u", ix, x->kind);
  x->encoding = rd<uint16_t>(r + 8);
  if (x->encoding > ENC_PAIR) return fail(GLACIER_CUDA_FMT_BAD_ENCODING, "record %llu: encoding %u", ix, x->encoding);
  x->layout = rd<uint16_t>(r + 10);
  if (x->layout > LAY_ROWS4 && x->layout != LAY_NONE)
    return fail(GLACIER_CUDA_FMT_BAD_PACKED_LAYOUT, "record %llu: packed layout %u", ix, x->layout);
  x->role = version == 1 ? (uint16_t)ROLE_TENSOR : rd<uint16_t>(r + 120);
  if (x->role > ROLE_PAIR) return fail(GLACIER_CUDA_FMT_BAD_ROLE, "record %llu: role %u", ix, x->role);
  x->pair_layout = version == 1 ? (uint16_t)PAIR_NONE : rd<uint16_t>(r + 122);
  if (x->pair_layout != PAIR_ROWS4 && x->pair_layout != PAIR_NONE)
    return fail(GLACIER_CUDA_FMT_BAD_PAIR_NIBBLE_LAYOUT, "record %llu: pair layout %u", ix, x->pair_layout);
  x->group = rd<uint32_t>(r + 12);
  x->out_f = rd<uint32_t>(r + 16);
  x->in_f = rd<uint32_t>(r + 20);
  x->flags = rd<uint32_t>(r + 24);
  x->crc = rd<uint32_t>(r + 28);
  x->n = rd<uint64_t>(r + 32);
  for (int s = 0; s < kStreams; ++s) x->s[s] = {rd<uint64_t>(r + 40 + 16 * s), rd<uint64_t>(r + 48 + 16 * s)};
  if (version == 2)
    memcpy(x->digest, r + 128, 32);
  else
    memset(x->digest, 0, 32);
  return GLACIER_CUDA_OK;
}

// Record.validateDescriptor (runtime_image.zig:432-554).
int validate_descriptor(const Rec& x, uint16_t version, uint64_t index) {
  const unsigned long long ix = index;
  auto shape = [&](const char* why) { return fail(GLACIER_CUDA_FMT_BAD_TENSOR_SHAPE, "record %llu: %s", ix, why); };
  auto enc = [&](const char* why) { return fail(GLACIER_CUDA_FMT_BAD_ENCODING, "record %llu: %s", ix, why); };
  if (x.flags) return fail(GLACIER_CUDA_FMT_BAD_FLAGS, "record %llu: flags set", ix);
  if (version == 1) {
    if (x.role != ROLE_TENSOR || x.pair_layout != PAIR_NONE || !all_zero(x.digest, 32))
      return fail(GLACIER_CUDA_FMT_BAD_VERSIONED_RECORD, "record %llu: v2 fields in a v1 record", ix);
    if (x.encoding == ENC_PAIR) return enc("PairNibble in a v1 image");
  } else if (all_zero(x.digest, 32)) {
    return fail(GLACIER_CUDA_FMT_MISSING_DIGEST, "record %llu: no digest", ix);
  }
  if (!x.out_f || !x.in_f || !x.n) return shape("empty shape");
  if ((uint64_t)x.out_f * x.in_f != x.n) return shape("num_elements is not out_f * in_f");
  const Range* s = x.s;
  switch (x.encoding) {
    case ENC_RAW: {
      if (x.role != ROLE_TENSOR || x.layout != LAY_NONE || x.pair_layout != PAIR_NONE || x.group)
        return enc("raw f32 record with a layout, role or group");
      if (!s[S_RAW].len || s[S_PACKED].len || s[S_F32].len || s[S_F16].len || s[S_ROWS4].len)
        return enc("raw f32 record streams");
      uint64_t bytes;
      if (__builtin_mul_overflow(x.n, (uint64_t)4, &bytes) || s[S_RAW].len != bytes) return shape("raw length");
      return GLACIER_CUDA_OK;
    }
    case ENC_INT4: {
      if (x.role != ROLE_TENSOR || x.pair_layout != PAIR_NONE || x.layout == LAY_NONE || !x.group ||
          !s[S_PACKED].len || s[S_RAW].len)
        return enc("INT4 record fields");
      if (s[S_PACKED].len != x.n / 2 + x.n % 2) return shape("packed length");
      const uint64_t groups = x.n / x.group + (x.n % x.group != 0);
      if ((s[S_F32].len && s[S_F32].len != groups * 4) || (s[S_F16].len && s[S_F16].len != groups * 2) ||
          (s[S_ROWS4].len && s[S_ROWS4].len != groups * 2))
        return shape("scale stream length");
      if (!s[S_F32].len && !s[S_F16].len && !s[S_ROWS4].len)
        return fail(GLACIER_CUDA_FMT_MISSING_SCALES, "record %llu: no scale stream", ix);
      if (x.layout == LAY_ROWS4 && (x.out_f % 4 || x.in_f % 16 || !s[S_ROWS4].len))
        return fail(GLACIER_CUDA_FMT_BAD_PACKED_LAYOUT, "record %llu: rows4_k16 geometry", ix);
      return GLACIER_CUDA_OK;
    }
    default: {  // PairNibble
      if (version != 2 || x.role != ROLE_PAIR) return fail(GLACIER_CUDA_FMT_BAD_ROLE, "record %llu: pair role", ix);
      if (x.layout != LAY_NONE || x.pair_layout != PAIR_ROWS4)
        return fail(GLACIER_CUDA_FMT_BAD_PAIR_NIBBLE_LAYOUT, "record %llu: pair layout", ix);
      if ((x.group != 8 && x.group != 16) || x.out_f % 4 || x.in_f % 16 || x.in_f % x.group)
        return shape("PairNibble geometry");
      if (s[S_RAW].len || s[S_F32].len || s[S_F16].len) return enc("PairNibble streams");
      if (s[S_PACKED].len != x.n) return shape("pair byte count");
      if (s[S_ROWS4].len != (uint64_t)x.out_f * (x.in_f / x.group) * 2 * 2) return shape("pair scale count");
      return GLACIER_CUDA_OK;
    }
  }
}

bool overlap(const Range& a, const Range& b) { return a.off < b.off + b.len && b.off < a.off + a.len; }

// validateBoundsForVersion (runtime_image.zig:556-590).
int validate_bounds(const Rec& x, const Image& im, uint64_t index) {
  int rc = validate_descriptor(x, im.version, index);
  if (rc) return rc;
  const unsigned long long ix = index;
  for (int s = 0; s < kStreams; ++s) {
    const Range& r = x.s[s];
    if ((r.off == 0) != (r.len == 0)) return fail(GLACIER_CUDA_FMT_BAD_BOUNDS, "record %llu: stream %d empty/offset", ix, s);
    if (!r.len) continue;
    if (r.off < im.data_off || r.off % kAlign)
      return fail(GLACIER_CUDA_FMT_BAD_ALIGNMENT, "record %llu: stream %d at %llu", ix, s, (unsigned long long)r.off);
    uint64_t end;
    if (__builtin_add_overflow(r.off, r.len, &end) || end > im.info.file_size)
      return fail(GLACIER_CUDA_FMT_BAD_BOUNDS, "record %llu: stream %d past the end", ix, s);
  }
  for (int a = 0; a < kStreams; ++a)
    for (int c = a + 1; c < kStreams; ++c)
      if (x.s[a].len && x.s[c].len && overlap(x.s[a], x.s[c]))
        return fail(GLACIER_CUDA_FMT_OVERLAPPING_PAYLOAD, "record %llu: streams %d and %d overlap", ix, a, c);
  return GLACIER_CUDA_OK;
}

bool identity_eq(const Rec& a, const Rec& b) {
  if (a.layer != b.layer || a.role != b.role) return false;
  return a.role != ROLE_TENSOR || a.kind == b.kind;
}

// Payload CRC over the streams in canonical order, and the v2 digest over the
// descriptor's first 128 bytes followed by the same streams.  0 when good.
int content_status(const Image& im, const Rec& x, bool crc, bool digest) {
  if (crc) {
    uint32_t c = 0;
    for (int s = 0; s < kStreams; ++s)
      if (x.s[s].len) c = crc32_of(im.b + x.s[s].off, x.s[s].len, c);
    if (c != x.crc) return 1;
  }
  if (digest && im.version == 2) {
    Sha256 h;
    h.update(x.desc, 128);
    for (int s = 0; s < kStreams; ++s)
      if (x.s[s].len) h.update(im.b + x.s[s].off, x.s[s].len);
    uint8_t d[32];
    h.final(d);
    if (memcmp(d, x.digest, 32)) return 2;
  }
  return 0;
}

int admit(const uint8_t* b, uint64_t len, const glacier_cuda_glrt_options* opts, Image* im) {
  *format_error_slot() = 0;
  GLC_REQUIRE(b || !len, "runtime image: null buffer");
  glacier_cuda_glrt_options o = {};
  if (opts) o = *opts;
  im->b = b;
  im->len = len;
  int rc = decode_header(b, len, im);
  if (rc || (rc = validate_header(b, len, im, o))) return rc;
  const uint64_t rsize = im->version == 1 ? kRecV1 : kRecV2;
  if (kHeader + im->count * rsize > len) return fail(GLACIER_CUDA_FMT_BAD_BOUNDS, "index past the end");
  if (crc32_of(b + kHeader, im->count * rsize) != rd<uint32_t>(b + 152))
    return fail(GLACIER_CUDA_FMT_INDEX_CRC_MISMATCH, "index CRC");
  // Structure of every record in index order; the first structural failure
  // ends the walk, after the content of the records before it is checked.
  im->recs.resize(im->count);
  uint64_t bad = im->count;
  int bad_rc = 0;
  for (uint64_t i = 0; i < im->count && bad == im->count; ++i) {
    Rec& x = im->recs[i];
    int r = decode_record(b + kHeader + i * rsize, im->version, i, &x);
    if (!r) r = validate_bounds(x, *im, i);
    for (uint64_t j = 0; !r && j < i; ++j) {
      const Rec& p = im->recs[j];
      if (identity_eq(x, p)) {
        r = fail(GLACIER_CUDA_FMT_DUPLICATE_RECORD, "record %llu repeats record %llu", (unsigned long long)i,
                 (unsigned long long)j);
        break;
      }
      for (int s = 0; !r && s < kStreams; ++s)
        for (int t = 0; !r && t < kStreams; ++t)
          if (x.s[s].len && p.s[t].len && overlap(x.s[s], p.s[t]))
            r = fail(GLACIER_CUDA_FMT_OVERLAPPING_PAYLOAD, "record %llu overlaps record %llu",
                     (unsigned long long)i, (unsigned long long)j);
    }
    if (r) bad = i, bad_rc = r;
  }
  char saved_msg[512];
  const int32_t saved_reason = *format_error_slot();
  snprintf(saved_msg, sizeof(saved_msg), "%s", glacier_cuda_last_error());
  const bool crc = !o.skip_payload_crc, dig = !o.skip_payload_digest;
  if (crc || dig) {
    uint64_t bytes = 0;
    for (uint64_t i = 0; i < bad; ++i)
      for (int s = 0; s < kStreams; ++s) bytes += im->recs[i].s[s].len;
    unsigned nt = std::max(1u, std::min(std::thread::hardware_concurrency(), 64u));
    if (bytes < (32ull << 20)) nt = 1;
    std::atomic<uint64_t> next{0};
    std::vector<int> status(bad, 0);
    auto work = [&] {
      for (uint64_t i; (i = next.fetch_add(1)) < bad;) status[i] = content_status(*im, im->recs[i], crc, dig);
    };
    std::vector<std::thread> pool;
    for (unsigned t = 1; t < nt; ++t) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
    for (uint64_t i = 0; i < bad; ++i)
      if (status[i] == 1) return fail(GLACIER_CUDA_FMT_CRC_MISMATCH, "record %llu: payload CRC", (unsigned long long)i);
      else if (status[i] == 2)
        return fail(GLACIER_CUDA_FMT_DIGEST_MISMATCH, "record %llu: payload digest", (unsigned long long)i);
  }
  if (bad < im->count) {
    *format_error_slot() = saved_reason;
    set_error(bad_rc, "%s", saved_msg);
    return bad_rc;
  }
  return GLACIER_CUDA_OK;
}

// ------------------------------------------------------------- layouts ----
uint8_t nib(const uint8_t* p, uint64_t i) { return (p[i >> 1] >> ((i & 1) * 4)) & 15; }
// Physical nibble of (row, col) in a rows4_k16 stream (int4_weights.zig:153-170):
//   (row/4)*(4*in_f) + (col/16)*64 + ((col%16)/4)*16 + (row%4)*4 + col%4.

float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000) << 16, exp = (h >> 10) & 0x1F, man = h & 0x3FF;
  uint32_t bits;
  if (exp == 0x1F) {
    bits = sign | 0x7F800000u | man << 13;
  } else if (exp) {
    bits = sign | (exp + 112) << 23 | man << 13;
  } else if (man) {
    int e = -1;
    uint32_t m = man;
    do {
      m <<= 1;
      ++e;
    } while (!(m & 0x400));
    bits = sign | (uint32_t)(112 - e) << 23 | (m & 0x3FF) << 13;
  } else {
    bits = sign;
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

// Runs f(tile) for every 4-row tile, spread over the host's cores for large tensors.
template <typename F>
void for_each_tile(uint64_t tiles, uint64_t bytes_per_tile, const F& f) {
  unsigned nt = std::max(1u, std::min(std::thread::hardware_concurrency(), 32u));
  if (tiles * bytes_per_tile < (8ull << 20)) nt = 1;
  std::atomic<uint64_t> next{0};
  auto work = [&] {
    for (uint64_t t0; (t0 = next.fetch_add(64)) < tiles;)
      for (uint64_t t = t0; t < std::min(tiles, t0 + 64); ++t) f(t);
  };
  std::vector<std::thread> pool;
  for (unsigned i = 1; i < nt; ++i) pool.emplace_back(work);
  work();
  for (auto& th : pool) th.join();
}

// rows4_k16 -> row-major as a byte permutation.  Inside a 4-row tile, the
// 16-column block b is 32 contiguous bytes ordered [chunk c][row lane l][pair p]
// (nibbles c*16 + l*4 + 2p and 2p+1), and that byte is exactly row l's byte for
// columns 16b + 4c + 2p and +1 in row-major order.
void rows4_to_row_major(const uint8_t* src, uint8_t* dst, uint64_t out_f, uint64_t in_f) {
  const uint64_t rb = in_f / 2;
  for_each_tile(out_f / 4, 4 * rb, [&](uint64_t t) {
    const uint8_t* s = src + t * 4 * rb;
    uint8_t* d = dst + t * 4 * rb;
    for (uint64_t b = 0; b < in_f / 16; ++b)
      for (int c = 0; c < 4; ++c)
        for (int l = 0; l < 4; ++l) {
          d[l * rb + b * 8 + c * 2] = s[b * 32 + c * 8 + l * 2];
          d[l * rb + b * 8 + c * 2 + 1] = s[b * 32 + c * 8 + l * 2 + 1];
        }
  });
}

// One INT4 record's row-major f32 scales.  Scale choice: the f32 stream when
// present (the portable numerics), else the row-major fp16 mirror, else the
// rows4 fp16 grid; fp16 widens to f32 exactly.
void int4_scales(const Image& im, const Rec& x, std::vector<float>* scales) {
  const uint64_t groups = x.n / x.group + (x.n % x.group != 0);
  scales->resize(groups);
  if (x.s[S_F32].len) {
    memcpy(scales->data(), im.b + x.s[S_F32].off, groups * 4);
  } else if (x.s[S_F16].len) {
    for (uint64_t g = 0; g < groups; ++g) (*scales)[g] = half_to_float(rd<uint16_t>(im.b + x.s[S_F16].off + 2 * g));
  } else {  // rows4 grid [tile][group][lane]; rows hold whole groups here
    const uint64_t per_row = x.in_f / x.group;
    const uint8_t* s4 = im.b + x.s[S_ROWS4].off;
    for (uint64_t t = 0; t < x.out_f / 4; ++t)
      for (uint64_t g = 0; g < per_row; ++g)
        for (uint64_t l = 0; l < 4; ++l)
          (*scales)[(t * 4 + l) * per_row + g] = half_to_float(rd<uint16_t>(s4 + 2 * ((t * per_row + g) * 4 + l)));
  }
}

// One INT4 record as row-major codes (permuted on the host) and row-major f32 scales.
void int4_row_major(const Image& im, const Rec& x, std::vector<uint8_t>* packed, std::vector<float>* scales) {
  const uint8_t* pk = im.b + x.s[S_PACKED].off;
  packed->resize(x.n / 2 + x.n % 2);
  if (x.layout == LAY_ROW_MAJOR)
    memcpy(packed->data(), pk, packed->size());
  else
    rows4_to_row_major(pk, packed->data(), x.out_f, x.in_f);
  int4_scales(im, x, scales);
}

// A PairNibble record split into row-major gate and up tensors: the byte at
// coefficient position of (r, c) in rows4_k16 order holds gate in its low nibble and up
// in its high nibble, and the scale grid is [tile][group][branch][lane]
// (int4_weights.zig:42-54, :322-331).  Columns 2j and 2j+1 of a row sit in
// adjacent pair bytes, so each output byte comes from two input bytes.
void pair_split(const uint8_t* pairs, const uint8_t* scale_bits, uint64_t out_f, uint64_t in_f, uint64_t group,
                uint8_t* gate, uint8_t* up, float* gate_scales, float* up_scales) {
  const uint64_t rb = in_f / 2;
  for_each_tile(out_f / 4, 4 * in_f, [&](uint64_t t) {
    const uint8_t* s = pairs + t * 4 * in_f;
    for (uint64_t b = 0; b < in_f / 16; ++b)
      for (int c = 0; c < 4; ++c)
        for (int l = 0; l < 4; ++l)
          for (int p = 0; p < 2; ++p) {
            const uint8_t lo = s[b * 64 + c * 16 + l * 4 + 2 * p], hi = s[b * 64 + c * 16 + l * 4 + 2 * p + 1];
            const uint64_t o = (t * 4 + l) * rb + b * 8 + c * 2 + p;
            gate[o] = (uint8_t)((lo & 15) | (hi & 15) << 4);
            up[o] = (uint8_t)((lo >> 4) | (hi & 0xF0));
          }
  });
  const uint64_t per_row = in_f / group;
  for (uint64_t t = 0; t < out_f / 4; ++t)
    for (uint64_t g = 0; g < per_row; ++g)
      for (uint64_t l = 0; l < 4; ++l) {
        const uint64_t base = (t * per_row + g) * 8;
        gate_scales[(t * 4 + l) * per_row + g] = half_to_float(rd<uint16_t>(scale_bits + 2 * (base + l)));
        up_scales[(t * 4 + l) * per_row + g] = half_to_float(rd<uint16_t>(scale_bits + 2 * (base + 4 + l)));
      }
}

// ------------------------------------------------------ prepared schema ----
const Rec* find(const Image& im, uint32_t layer, uint32_t kind) {
  for (const Rec& x : im.recs)
    if (x.role == ROLE_TENSOR && x.layer == layer && x.kind == kind) return &x;
  return nullptr;
}

const Rec* find_pair(const Image& im, uint32_t layer) {
  for (const Rec& x : im.recs)
    if (x.role == ROLE_PAIR && x.layer == layer) return &x;
  return nullptr;
}

int bad_payload(const char* fmt, ...) __attribute__((format(printf, 1, 2)));
int bad_payload(const char* fmt, ...) {
  char buf[300];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return fail(GLACIER_CUDA_FMT_BAD_PAYLOAD, "%s", buf);
}

// validatePreparedConfig (loader.zig:618-652).
int check_config(const glacier_cuda_glrt_info& c) {
  if ((uint64_t)c.num_heads * c.head_dim != c.dim || c.num_kv_heads > c.num_heads || c.num_heads % c.num_kv_heads)
    return bad_payload("config: heads * head_dim must equal dim and kv_heads divide heads");
  return GLACIER_CUDA_OK;
}

// isExpectedPreparedRecord (loader.zig:730-766).
bool expected_record(const glacier_cuda_glrt_info& c, const Rec& x) {
  if (x.role == ROLE_PAIR) return x.layer != kGlobalLayer && x.layer < c.num_layers;
  if (x.layer == kGlobalLayer)
    return x.kind == K_FINAL_NORM || x.kind == K_EMBEDDING || (x.kind == K_LM_HEAD && !c.tie_embeddings);
  if (x.layer >= c.num_layers) return false;
  return x.kind <= K_BO && x.kind != K_EMBEDDING && x.kind != K_LM_HEAD && x.kind != K_FINAL_NORM;
}

// preparedRaw (loader.zig:785-809); *out is null for an absent optional record.
int prepared_raw(const Image& im, uint32_t layer, uint32_t kind, uint64_t n, bool required, const Rec** out) {
  *out = find(im, layer, kind);
  if (!*out) return required ? fail(GLACIER_CUDA_FMT_MISSING_TENSOR, "layer %d has no tensor kind %u", (int)layer, kind)
                             : GLACIER_CUDA_OK;
  const Rec& x = **out;
  if (x.encoding != ENC_RAW || x.layout != LAY_NONE || x.group || x.out_f != 1 || x.in_f != n || x.n != n)
    return bad_payload("layer %d kind %u: raw tensor of %llu values expected", (int)layer, kind, (unsigned long long)n);
  return GLACIER_CUDA_OK;
}

// preparedInt4 (loader.zig:811-868).
int prepared_int4(const Image& im, uint32_t layer, uint32_t kind, uint64_t out_f, uint64_t in_f, bool need_f32,
                  const Rec** out) {
  *out = find(im, layer, kind);
  if (!*out) return fail(GLACIER_CUDA_FMT_MISSING_TENSOR, "layer %d has no tensor kind %u", (int)layer, kind);
  const Rec& x = **out;
  if (x.encoding != ENC_INT4 || !x.group || x.out_f != out_f || x.in_f != in_f || x.n != out_f * in_f)
    return bad_payload("layer %d kind %u: INT4 [%llu x %llu] expected", (int)layer, kind, (unsigned long long)out_f,
                       (unsigned long long)in_f);
  const uint64_t groups = x.n / x.group + (x.n % x.group != 0);
  if (need_f32 && x.s[S_F32].len != groups * 4) return bad_payload("kind %u needs f32 scales", kind);
  if (x.layout == LAY_ROWS4 && (out_f % 4 || in_f % 16 || x.s[S_ROWS4].len != groups * 2))
    return bad_payload("kind %u: rows4_k16 geometry", kind);
  if (x.layout == LAY_NONE) return bad_payload("kind %u: INT4 without a packed layout", kind);
  return GLACIER_CUDA_OK;
}

// inspectPreparedPairNibble (loader.zig:871-912); *out is null when absent.
int prepared_pair(const Image& im, uint32_t layer, uint64_t out_f, uint64_t in_f, const Rec** out) {
  *out = find_pair(im, layer);
  if (!*out) return GLACIER_CUDA_OK;
  const Rec& x = **out;
  if (x.encoding != ENC_PAIR || x.layout != LAY_NONE || x.pair_layout != PAIR_ROWS4 || x.out_f != out_f ||
      x.in_f != in_f || x.n != out_f * in_f)
    return bad_payload("layer %u: PairNibble [%llu x %llu] expected", layer, (unsigned long long)out_f,
                       (unsigned long long)in_f);
  return GLACIER_CUDA_OK;
}

// validatePreparedRecordSet (loader.zig:656-714): every record expected, and
// per layer either one PairNibble role or both separate branches, the same
// form in every layer.  Returns 1 separate / 2 pair in *layout.
int check_record_set(const Image& im, uint32_t* layout) {
  const auto& c = im.info;
  for (const Rec& x : im.recs)
    if (!expected_record(c, x))
      return bad_payload("unexpected record: layer %d kind %u role %u", (int)x.layer, x.kind, x.role);
  *layout = 0;
  for (uint32_t l = 0; l < c.num_layers; ++l) {
    const bool gate = find(im, l, K_GATE), up = find(im, l, K_UP);
    const Rec* pair = find_pair(im, l);
    uint32_t mine;
    int rc;
    if (pair) {
      if (gate || up) return bad_payload("layer %u has both a PairNibble record and separate branches", l);
      if ((rc = prepared_pair(im, l, c.hidden, c.dim, &pair))) return rc;
      mine = 2;
    } else {
      if (!gate || !up) return fail(GLACIER_CUDA_FMT_MISSING_TENSOR, "layer %u lacks a gate or up branch", l);
      const Rec* r;
      if ((rc = prepared_int4(im, l, K_GATE, c.hidden, c.dim, false, &r)) ||
          (rc = prepared_int4(im, l, K_UP, c.hidden, c.dim, false, &r)))
        return rc;
      mine = 1;
    }
    if (*layout && *layout != mine) return bad_payload("layer %u: MLP form differs from earlier layers", l);
    *layout = mine;
  }
  if (!*layout) return fail(GLACIER_CUDA_FMT_NO_LAYERS, "no layers");
  return GLACIER_CUDA_OK;
}

// The INT4 records the model uses, with their group sizes; one group size
// across the model is what this decode path's kernels take.
int uniform_group(const Image& im, uint32_t* group) {
  *group = 0;
  for (const Rec& x : im.recs) {
    if (x.encoding == ENC_RAW) continue;
    if (*group && x.group != *group)
      return set_error(GLACIER_CUDA_EUNSUPPORTED, "runtime image: INT4 groups %u and %u in one model", *group, x.group);
    *group = x.group;
  }
  return GLACIER_CUDA_OK;
}

int prepared_model(const uint8_t* b, uint64_t len, const glacier_cuda_glrt_options* opts, Image* im) {
  int rc = admit(b, len, opts, im);
  if (rc || (rc = check_config(im->info)) || (rc = check_record_set(*im, &im->info.mlp_layout)) ||
      (rc = uniform_group(*im, &im->info.group_size)))
    return rc;
  return GLACIER_CUDA_OK;
}

}  // namespace
}  // namespace glacier

using namespace glacier;

extern "C" {

int glacier_cuda_glrt_open(const uint8_t* bytes, uint64_t len, const glacier_cuda_glrt_options* opts,
                           glacier_cuda_glrt_info* info) {
  Image im;
  const int rc = admit(bytes, len, opts, &im);
  if (!rc && info) *info = im.info;
  return rc;
}

int glacier_cuda_glrt_records(const uint8_t* bytes, uint64_t len, glacier_cuda_glrt_entry* out, uint64_t capacity,
                              uint64_t* count) {
  GLC_REQUIRE(count && (out || capacity == 0), "glrt_records: null output");
  glacier_cuda_glrt_options o = {};
  o.skip_payload_crc = o.skip_payload_digest = 1;
  Image im;
  const int rc = admit(bytes, len, &o, &im);
  if (rc) return rc;
  *count = im.recs.size();
  for (uint64_t i = 0; i < std::min<uint64_t>(capacity, im.recs.size()); ++i) {
    const Rec& x = im.recs[i];
    glacier_cuda_glrt_entry& e = out[i];
    e.layer_idx = x.layer;
    e.tensor_kind = x.kind;
    e.encoding = x.encoding;
    e.packed_layout = x.layout;
    e.role = x.role;
    e.pair_nibble_layout = x.pair_layout;
    e.group_size = x.group;
    e.out_f = x.out_f;
    e.in_f = x.in_f;
    e.payload_crc32 = x.crc;
    e.num_elements = x.n;
    for (int s = 0; s < kStreams; ++s) {
      e.stream_offset[s] = x.s[s].off;
      e.stream_len[s] = x.s[s].len;
    }
    memcpy(e.payload_digest, x.digest, 32);
  }
  return GLACIER_CUDA_OK;
}

int glacier_cuda_glrt_record(const uint8_t* bytes, uint64_t len, uint64_t index, glacier_cuda_glrt_entry* out) {
  GLC_REQUIRE(out, "glrt_record: null output");
  std::vector<glacier_cuda_glrt_entry> all;
  uint64_t n = 0;
  int rc = glacier_cuda_glrt_records(bytes, len, nullptr, 0, &n);
  if (rc) return rc;
  GLC_REQUIRE(index < n, "glrt_record: record %llu of %llu", (unsigned long long)index, (unsigned long long)n);
  all.resize(n);
  if ((rc = glacier_cuda_glrt_records(bytes, len, all.data(), n, &n))) return rc;
  *out = all[index];
  return GLACIER_CUDA_OK;
}

int glacier_cuda_glrt_model_info(const uint8_t* bytes, uint64_t len, const glacier_cuda_glrt_options* opts,
                                 glacier_cuda_glrt_info* info) {
  GLC_REQUIRE(info, "glrt_model_info: null output");
  Image im;
  const int rc = prepared_model(bytes, len, opts, &im);
  if (!rc) *info = im.info;
  return rc;
}

int glacier_cuda_rows4_k16_to_row_major(const uint8_t* src, uint8_t* dst, size_t out_f, size_t in_f) {
  GLC_REQUIRE(src && dst && out_f % 4 == 0 && in_f % 16 == 0, "rows4_k16: bad arguments");
  rows4_to_row_major(src, dst, out_f, in_f);
  return GLACIER_CUDA_OK;
}

int glacier_cuda_rows4_scales_to_row_major(const uint16_t* src, float* dst, size_t out_f, size_t groups_per_row) {
  GLC_REQUIRE(src && dst && out_f % 4 == 0, "rows4 scales: bad arguments");
  for (size_t t = 0; t < out_f / 4; ++t)
    for (size_t g = 0; g < groups_per_row; ++g)
      for (size_t l = 0; l < 4; ++l) dst[(t * 4 + l) * groups_per_row + g] = half_to_float(src[(t * groups_per_row + g) * 4 + l]);
  return GLACIER_CUDA_OK;
}

int glacier_cuda_pair_nibble_split(const uint8_t* pairs, const uint16_t* pair_scales, size_t out_f, size_t in_f,
                                   size_t group, uint8_t* gate, uint8_t* up, float* gate_scales, float* up_scales) {
  GLC_REQUIRE(pairs && pair_scales && gate && up && gate_scales && up_scales, "pair_nibble_split: null argument");
  GLC_REQUIRE(out_f % 4 == 0 && in_f % 16 == 0 && (group == 8 || group == 16) && in_f % group == 0,
              "pair_nibble_split: geometry");
  pair_split(pairs, reinterpret_cast<const uint8_t*>(pair_scales), out_f, in_f, group, gate, up, gate_scales,
             up_scales);
  return GLACIER_CUDA_OK;
}

int glacier_cuda_model_load_glrt(glacier_cuda_model* model, const uint8_t* bytes, uint64_t len,
                                 const glacier_cuda_glrt_options* opts) {
  GLC_REQUIRE(model, "model_load_glrt: null model");
  const glacier_cuda_model_config& mc = *model_config(model);
  Image im;
  int rc = prepared_model(bytes, len, opts, &im);
  if (rc) return rc;
  const auto& c = im.info;
  GLC_REQUIRE(mc.dim == c.dim && mc.hidden == c.hidden && mc.num_layers == c.num_layers && mc.vocab == c.vocab &&
                  mc.num_heads == c.num_heads && mc.head_dim == c.head_dim && mc.num_kv_heads == c.num_kv_heads &&
                  mc.group_size == c.group_size,
              "model_load_glrt: the model was created with a config other than the image's");
  GLC_REQUIRE(!memcmp(&mc.rms_eps, &c.rms_eps, 4) && !memcmp(&mc.rope_theta, &c.rope_theta, 4),
              "model_load_glrt: rms_eps / rope_theta differ from the image's");
  const uint64_t D = c.dim, F = c.hidden, KV = (uint64_t)c.num_kv_heads * c.head_dim;

  std::vector<uint8_t> pk;
  std::vector<float> sc;
  // Codes go up as the image stores them; rows4_k16 is put in row-major order on the device.
  auto upload_int4 = [&](const Rec* r, int layer, int kind) {
    int4_scales(im, *r, &sc);
    const uint8_t* codes = bytes + r->s[S_PACKED].off;
    const size_t nbytes = r->n / 2 + r->n % 2;
    if (r->layout == LAY_ROW_MAJOR)
      return glacier_cuda_model_load_int4(model, layer, kind, codes, nbytes, sc.data(), sc.size());
    return glacier_cuda_model_load_int4_rows4(model, layer, kind, codes, nbytes, sc.data(), sc.size());
  };
  auto upload_raw = [&](const Rec* r, int layer, int kind) {
    return glacier_cuda_model_load_f32(model, layer, kind, reinterpret_cast<const float*>(bytes + r->s[S_RAW].off),
                                       r->n);
  };

  for (uint32_t l = 0; l < c.num_layers; ++l) {
    const Rec *in, *post, *bq, *bk, *bv, *bo, *q, *k, *v, *o, *gate = nullptr, *up = nullptr, *pair = nullptr, *down;
    if ((rc = prepared_raw(im, l, K_INPUT_NORM, D, true, &in)) || (rc = prepared_raw(im, l, K_BQ, D, false, &bq)) ||
        (rc = prepared_raw(im, l, K_BK, KV, false, &bk)) || (rc = prepared_raw(im, l, K_BV, KV, false, &bv)) ||
        (rc = prepared_raw(im, l, K_BO, D, false, &bo)) || (rc = prepared_raw(im, l, K_POST_NORM, D, true, &post)) ||
        (rc = prepared_int4(im, l, K_Q, D, D, false, &q)) || (rc = prepared_int4(im, l, K_K, KV, D, false, &k)) ||
        (rc = prepared_int4(im, l, K_V, KV, D, false, &v)) || (rc = prepared_int4(im, l, K_O, D, D, false, &o)))
      return rc;
    if (c.mlp_layout == 1) {
      if ((rc = prepared_int4(im, l, K_GATE, F, D, false, &gate)) || (rc = prepared_int4(im, l, K_UP, F, D, false, &up)))
        return rc;
    } else {
      if ((rc = prepared_pair(im, l, F, D, &pair))) return rc;
      if (!pair) return fail(GLACIER_CUDA_FMT_MISSING_TENSOR, "layer %u has no PairNibble record", l);
    }
    if ((rc = prepared_int4(im, l, K_DOWN, D, F, false, &down))) return rc;
    if (bo)
      return set_error(GLACIER_CUDA_EUNSUPPORTED, "model_load_glrt: layer %u carries an attention output bias", l);

    const int L = (int)l;
    if ((rc = upload_raw(in, L, GLACIER_CUDA_N_INPUT)) || (rc = upload_raw(post, L, GLACIER_CUDA_N_POST_ATTN)) ||
        (bq && (rc = upload_raw(bq, L, GLACIER_CUDA_B_Q))) || (bk && (rc = upload_raw(bk, L, GLACIER_CUDA_B_K))) ||
        (bv && (rc = upload_raw(bv, L, GLACIER_CUDA_B_V))) || (rc = upload_int4(q, L, GLACIER_CUDA_W_Q)) ||
        (rc = upload_int4(k, L, GLACIER_CUDA_W_K)) || (rc = upload_int4(v, L, GLACIER_CUDA_W_V)) ||
        (rc = upload_int4(o, L, GLACIER_CUDA_W_O)) || (rc = upload_int4(down, L, GLACIER_CUDA_W_DOWN)))
      return rc;
    if (pair) {
      // The pair bytes go up as stored and are split into gate and up rows on the device.
      if ((rc = glacier_cuda_model_load_pair_nibble(
               model, L, bytes + pair->s[S_PACKED].off, F * D,
               reinterpret_cast<const uint16_t*>(bytes + pair->s[S_ROWS4].off), 2 * F * D / pair->group)))
        return rc;
    } else if ((rc = upload_int4(gate, L, GLACIER_CUDA_W_GATE)) || (rc = upload_int4(up, L, GLACIER_CUDA_W_UP))) {
      return rc;
    }
  }

  const Rec *fin, *emb, *head;
  if ((rc = prepared_raw(im, kGlobalLayer, K_FINAL_NORM, D, true, &fin)) ||
      (rc = prepared_int4(im, kGlobalLayer, K_EMBEDDING, c.vocab, D, true, &emb)))
    return rc;
  if (!c.tie_embeddings && (rc = prepared_int4(im, kGlobalLayer, K_LM_HEAD, c.vocab, D, false, &head))) return rc;
  if ((rc = upload_raw(fin, -1, GLACIER_CUDA_N_FINAL))) return rc;
  // Embedding rows dequantize as dequantizeRow (int4_matmul.zig:3166-3196):
  // code offset times the f32 group scale, through the record's nibble layout.
  int4_row_major(im, *emb, &pk, &sc);
  std::vector<float> table(emb->n);
  for (uint64_t i = 0; i < emb->n; ++i) table[i] = (float)((int)nib(pk.data(), i) - 7) * sc[i / emb->group];
  if ((rc = glacier_cuda_model_load_embedding_f32(model, table.data(), table.size()))) return rc;
  // A tied head is the embedding's INT4 data (loader.zig:351-361).
  if (c.tie_embeddings)
    return glacier_cuda_model_load_int4(model, -1, GLACIER_CUDA_W_LM_HEAD, pk.data(), pk.size(), sc.data(), sc.size());
  return upload_int4(head, -1, GLACIER_CUDA_W_LM_HEAD);
}

}  // extern "C"
