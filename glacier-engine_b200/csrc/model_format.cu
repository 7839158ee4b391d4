// Host-side reader for the portable `.glacier` model container and the loader
// that turns one into a device-resident model.
//
// Container (src/model/format.zig:1-14, all little-endian):
//   [0, 256)                  header (format.zig:67-139)
//   [256, 256+meta_len)       metadata: one JSON object (format.zig:432-440)
//   [meta_end, +64*num_pages) page index, 64-byte entries (format.zig:141-202)
//   [index_end, file_end)     page payloads, back to back in page order
// A page covers the flat element range [row_start, row_end) of one
// (layer, tensor_kind) tensor.  Raw pages (fp32/fp16/bf16) hold the elements
// verbatim; INT8/INT4 pages hold a 16-byte qio sub-header, one f32 scale per
// group of the page's own elements, then the packed codes (src/model/qio.zig:1-22).
//
// Admission follows FileReader.openFile (format.zig:407-478): header fields,
// layout, metadata JSON, every entry's reserved fields / kind / precision, then
// the page walk (ids, ranges, geometry, contiguity, no trailing bytes).  The
// per-page payload schema and CRC-32 are checked on demand, as
// validateAllPageCrcs (format.zig:497-534) and readPage (:488-495) do.
//
// Loading follows loader.zig loadWithOptions (:1214-1540) with compact INT4:
// pages grouped by (layer, kind) in page-id order; an all-INT4 group of a
// projection, the LM head or the embedding is concatenated in packed form
// (concatInt4Pages, :1633-1730); every other group is decoded to f32 and
// concatenated.  Nothing here touches the GPU until the final uploads through
// the glacier_cuda_model_load_* entries.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"

namespace glacier {

const glacier_cuda_model_config* model_config(const glacier_cuda_model* m);

namespace {

constexpr uint64_t kHeaderSize = 256;
constexpr uint32_t kPageSizeLog2 = 18;
constexpr uint64_t kPageSizeBytes = 1ull << kPageSizeLog2;
constexpr uint64_t kEntrySize = 64;
constexpr uint64_t kMaxMetadata = 16ull << 20;  // format.zig:34
constexpr uint64_t kMaxPages = 1ull << 20;      // format.zig:35
constexpr uint32_t kQioMagic = 0x514F4954u;     // "QOIT", qio.zig:27
constexpr uint64_t kQioHeader = 16;

enum Precision : uint8_t { P_FP16 = 0, P_BF16 = 1, P_INT8 = 2, P_INT4 = 3, P_INT2 = 4, P_TRI = 5, P_FP32 = 6 };
enum Kind : uint32_t {
  K_EMBEDDING = 0, K_Q = 1, K_K = 2, K_V = 3, K_O = 4, K_UP = 5, K_DOWN = 6, K_GATE = 7, K_INPUT_NORM = 8,
  K_LM_HEAD = 9, K_FINAL_NORM = 10, K_POST_NORM = 11, K_BQ = 12, K_BK = 13, K_BV = 14, K_BO = 15, K_OTHER = 255
};

thread_local int32_t g_format_error = 0;

struct Header {
  uint64_t meta_offset, meta_len, num_pages, index_offset, data_offset;
};

// A format failure: the reason code (GLACIER_CUDA_FMT_*) and a message.
int fail(int32_t reason, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int32_t reason, const char* fmt, ...) {
  char buf[400];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_format_error = reason;
  return set_error(GLACIER_CUDA_EFORMAT, "glacier format: %s", buf);
}

template <typename T>
T rd(const uint8_t* p) {
  T v;
  memcpy(&v, p, sizeof(T));  // the container is little-endian, like every supported host
  return v;
}

bool add_ok(uint64_t a, uint64_t b, uint64_t* out) { return !__builtin_add_overflow(a, b, out); }
bool mul_ok(uint64_t a, uint64_t b, uint64_t* out) { return !__builtin_mul_overflow(a, b, out); }
uint64_t cdiv(uint64_t a, uint64_t b) { return a / b + (a % b != 0); }

// ---------------------------------------------------------------- CRC-32 ----
// CRC-32/ISO-HDLC (reflected polynomial 0xEDB88320, init and xor-out all ones),
// the checksum std.hash.Crc32 computes; slicing-by-8 tables built at first use.
struct CrcTables {
  uint32_t t[8][256];
  CrcTables() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c >> 1) ^ (0xEDB88320u & (0u - (c & 1u)));
      t[0][i] = c;
    }
    for (uint32_t i = 0; i < 256; ++i)
      for (int s = 1; s < 8; ++s) t[s][i] = (t[s - 1][i] >> 8) ^ t[0][t[s - 1][i] & 0xFF];
  }
};

const CrcTables& crc_tables() {
  static const CrcTables tables;
  return tables;
}

uint32_t crc32_update(uint32_t crc, const uint8_t* p, size_t n) {
  const auto& T = crc_tables().t;
  crc = ~crc;
  while (n >= 8) {
    const uint32_t lo = rd<uint32_t>(p) ^ crc, hi = rd<uint32_t>(p + 4);
    crc = T[7][lo & 0xFF] ^ T[6][(lo >> 8) & 0xFF] ^ T[5][(lo >> 16) & 0xFF] ^ T[4][lo >> 24] ^ T[3][hi & 0xFF] ^
          T[2][(hi >> 8) & 0xFF] ^ T[1][(hi >> 16) & 0xFF] ^ T[0][hi >> 24];
    p += 8;
    n -= 8;
  }
  while (n--) crc = (crc >> 8) ^ T[0][(crc ^ *p++) & 0xFF];
  return ~crc;
}

// ------------------------------------------------------------------ JSON ----
// Metadata admission parses the blob as a std.json Value with default options
// and requires an object (format.zig:432-440).  This is an RFC 8259 syntax
// check with the same acceptance: UTF-8 strings without raw control
// characters, paired \u surrogates, strict numbers, one value and only
// whitespace around it, and duplicate member names rejected (std.json's
// default duplicate_field_behavior is an error).  Containers nest on an
// explicit stack, so deep nesting cannot exhaust the host stack.
class JsonCheck {
 public:
  JsonCheck(const uint8_t* s, size_t n) : s_(s), n_(n) {}

  bool object_document() {
    ws();
    if (i_ >= n_ || s_[i_] != '{') return false;
    if (!value()) return false;
    ws();
    return i_ == n_;
  }

 private:
  struct Frame {
    bool object;
    std::set<std::string> keys;
  };
  const uint8_t* s_;
  size_t n_, i_ = 0;

  void ws() {
    while (i_ < n_ && (s_[i_] == ' ' || s_[i_] == '\t' || s_[i_] == '\n' || s_[i_] == '\r')) ++i_;
  }
  bool lit(const char* w) {
    const size_t k = strlen(w);
    if (n_ - i_ < k || memcmp(s_ + i_, w, k)) return false;
    i_ += k;
    return true;
  }
  bool digits() {
    const size_t b = i_;
    while (i_ < n_ && s_[i_] >= '0' && s_[i_] <= '9') ++i_;
    return i_ > b;
  }
  bool number() {
    if (s_[i_] == '-') ++i_;
    if (i_ >= n_) return false;
    if (s_[i_] == '0') {
      ++i_;
    } else if (!digits()) {
      return false;
    }
    if (i_ < n_ && s_[i_] == '.') {
      ++i_;
      if (!digits()) return false;
    }
    if (i_ < n_ && (s_[i_] == 'e' || s_[i_] == 'E')) {
      ++i_;
      if (i_ < n_ && (s_[i_] == '+' || s_[i_] == '-')) ++i_;
      if (!digits()) return false;
    }
    return true;
  }
  bool hex4(uint32_t* v) {
    if (n_ - i_ < 4) return false;
    *v = 0;
    for (int k = 0; k < 4; ++k) {
      const uint8_t c = s_[i_++];
      const int d = c >= '0' && c <= '9' ? c - '0' : c >= 'a' && c <= 'f' ? c - 'a' + 10
                                                   : c >= 'A' && c <= 'F' ? c - 'A' + 10 : -1;
      if (d < 0) return false;
      *v = *v << 4 | (uint32_t)d;
    }
    return true;
  }
  static void put_utf8(std::string* out, uint32_t cp) {
    if (cp < 0x80) {
      out->push_back((char)cp);
    } else if (cp < 0x800) {
      out->push_back((char)(0xC0 | cp >> 6));
      out->push_back((char)(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
      out->push_back((char)(0xE0 | cp >> 12));
      out->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
      out->push_back((char)(0x80 | (cp & 0x3F)));
    } else {
      out->push_back((char)(0xF0 | cp >> 18));
      out->push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
      out->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
      out->push_back((char)(0x80 | (cp & 0x3F)));
    }
  }
  // One well-formed UTF-8 sequence (no overlong forms, no encoded surrogates,
  // nothing above U+10FFFF), appended to out.
  bool utf8(std::string* out) {
    const uint8_t c = s_[i_];
    int len;
    uint32_t cp, min;
    if (c < 0x80) {
      len = 1, cp = c, min = 0;
    } else if ((c & 0xE0) == 0xC0) {
      len = 2, cp = c & 0x1F, min = 0x80;
    } else if ((c & 0xF0) == 0xE0) {
      len = 3, cp = c & 0x0F, min = 0x800;
    } else if ((c & 0xF8) == 0xF0) {
      len = 4, cp = c & 0x07, min = 0x10000;
    } else {
      return false;
    }
    if (n_ - i_ < (size_t)len) return false;
    for (int k = 1; k < len; ++k) {
      const uint8_t cc = s_[i_ + k];
      if ((cc & 0xC0) != 0x80) return false;
      cp = cp << 6 | (cc & 0x3F);
    }
    if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    out->append((const char*)s_ + i_, len);
    i_ += len;
    return true;
  }
  bool string(std::string* out) {
    ++i_;  // opening quote
    while (true) {
      if (i_ >= n_) return false;
      const uint8_t c = s_[i_];
      if (c == '"') {
        ++i_;
        return true;
      }
      if (c < 0x20) return false;
      if (c != '\\') {
        if (!utf8(out)) return false;
        continue;
      }
      if (++i_ >= n_) return false;
      const uint8_t e = s_[i_++];
      switch (e) {
        case '"': out->push_back('"'); break;
        case '\\': out->push_back('\\'); break;
        case '/': out->push_back('/'); break;
        case 'b': out->push_back('\b'); break;
        case 'f': out->push_back('\f'); break;
        case 'n': out->push_back('\n'); break;
        case 'r': out->push_back('\r'); break;
        case 't': out->push_back('\t'); break;
        case 'u': {
          uint32_t cp;
          if (!hex4(&cp)) return false;
          if (cp >= 0xDC00 && cp <= 0xDFFF) return false;  // low surrogate first
          if (cp >= 0xD800 && cp <= 0xDBFF) {
            uint32_t lo;
            if (n_ - i_ < 2 || s_[i_] != '\\' || s_[i_ + 1] != 'u') return false;
            i_ += 2;
            if (!hex4(&lo) || lo < 0xDC00 || lo > 0xDFFF) return false;
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(out, cp);
          break;
        }
        default:
          return false;
      }
    }
  }
  // Parses one value starting at s_[i_] (whitespace already skipped).
  bool value() {
    std::vector<Frame> stack;
    bool need_value = true;
    while (true) {
      if (need_value) {
        ws();
        if (i_ >= n_) return false;
        const uint8_t c = s_[i_];
        if (c == '{' || c == '[') {
          ++i_;
          stack.push_back(Frame{c == '{', {}});
          ws();
          if (i_ < n_ && s_[i_] == (c == '{' ? '}' : ']')) {
            ++i_;
            stack.pop_back();
            need_value = false;
          } else if (c == '{') {
            if (!member_key(&stack.back())) return false;
          }
          continue;
        }
        std::string scratch;
        if (c == '"') {
          if (!string(&scratch)) return false;
        } else if (c == 't') {
          if (!lit("true")) return false;
        } else if (c == 'f') {
          if (!lit("false")) return false;
        } else if (c == 'n') {
          if (!lit("null")) return false;
        } else if (c == '-' || (c >= '0' && c <= '9')) {
          if (!number()) return false;
        } else {
          return false;
        }
        need_value = false;
      }
      // A value just completed: continue or close the enclosing container.
      if (stack.empty()) return true;
      ws();
      if (i_ >= n_) return false;
      Frame& f = stack.back();
      const uint8_t c = s_[i_++];
      if (c == ',') {
        if (f.object && !member_key(&f)) return false;
        need_value = true;
      } else if (c == (f.object ? '}' : ']')) {
        stack.pop_back();
      } else {
        return false;
      }
    }
  }
  // `"name" :` inside an object; duplicate names are rejected.
  bool member_key(Frame* f) {
    ws();
    if (i_ >= n_ || s_[i_] != '"') return false;
    std::string key;
    if (!string(&key)) return false;
    if (!f->keys.insert(key).second) return false;
    ws();
    if (i_ >= n_ || s_[i_] != ':') return false;
    ++i_;
    return true;
  }
};

// ------------------------------------------------------------- admission ----
struct Container {
  Header h;
  std::vector<glacier_cuda_page_entry> pages;
};

// Header.readFrom (format.zig:103-138) then validateHeaderLayoutV1 (:216-249).
int read_header(const uint8_t* b, uint64_t len, Header* h) {
  if (len < kHeaderSize) return fail(GLACIER_CUDA_FMT_TRUNCATED_HEADER, "file of %llu bytes", (unsigned long long)len);
  if (memcmp(b, "GLAC", 4)) return fail(GLACIER_CUDA_FMT_BAD_MAGIC, "magic is not GLAC");
  if (rd<uint16_t>(b + 4) != 1) return fail(GLACIER_CUDA_FMT_BAD_VERSION, "version %u", rd<uint16_t>(b + 4));
  if (rd<uint16_t>(b + 6) != kHeaderSize)
    return fail(GLACIER_CUDA_FMT_BAD_HEADER_SIZE, "header_size %u", rd<uint16_t>(b + 6));
  h->meta_offset = rd<uint64_t>(b + 8);
  h->meta_len = rd<uint64_t>(b + 16);
  h->num_pages = rd<uint64_t>(b + 24);
  h->index_offset = rd<uint64_t>(b + 32);
  h->data_offset = rd<uint64_t>(b + 40);
  if (rd<uint32_t>(b + 48) != kPageSizeLog2)
    return fail(GLACIER_CUDA_FMT_BAD_PAGE_SIZE, "page_size_log2 %u", rd<uint32_t>(b + 48));
  for (uint64_t k = 52; k < kHeaderSize; ++k)
    if (b[k]) return fail(GLACIER_CUDA_FMT_BAD_RESERVED_FIELD, "header byte %llu is not zero", (unsigned long long)k);

  if (h->meta_offset != kHeaderSize) return fail(GLACIER_CUDA_FMT_BAD_LAYOUT, "meta_offset is not 256");
  if (h->meta_len > kMaxMetadata) return fail(GLACIER_CUDA_FMT_METADATA_TOO_LARGE, "meta_len above 16 MiB");
  if (h->num_pages > kMaxPages) return fail(GLACIER_CUDA_FMT_INDEX_TOO_LARGE, "more than 2^20 pages");
  const uint64_t meta_end = h->meta_offset + h->meta_len;  // both bounded above: no overflow
  if (h->index_offset != meta_end) return fail(GLACIER_CUDA_FMT_BAD_LAYOUT, "page index does not follow metadata");
  const uint64_t index_end = h->index_offset + h->num_pages * kEntrySize;
  if (h->data_offset != index_end) return fail(GLACIER_CUDA_FMT_BAD_LAYOUT, "page data does not follow the index");
  if (meta_end > len) return fail(GLACIER_CUDA_FMT_TRUNCATED_META, "metadata runs past the end");
  if (index_end > len) return fail(GLACIER_CUDA_FMT_TRUNCATED_INDEX, "page index runs past the end");
  return GLACIER_CUDA_OK;
}

// PageEntry.readFrom (format.zig:169-201).
int read_entry(const uint8_t* e, uint64_t index, glacier_cuda_page_entry* p) {
  p->page_id = rd<uint64_t>(e);
  p->layer_idx = rd<uint32_t>(e + 8);
  p->tensor_kind = rd<uint32_t>(e + 12);
  p->row_start = rd<uint64_t>(e + 16);
  p->row_end = rd<uint64_t>(e + 24);
  p->precision = e[32];
  p->quant_group = e[33];
  p->reserved = 0;
  p->data_offset = rd<uint64_t>(e + 36);
  p->data_len = rd<uint64_t>(e + 44);
  p->crc32 = rd<uint32_t>(e + 52);
  if (rd<uint16_t>(e + 34) || rd<uint32_t>(e + 56) || rd<uint32_t>(e + 60))
    return fail(GLACIER_CUDA_FMT_BAD_RESERVED_FIELD, "page %llu: reserved field set", (unsigned long long)index);
  if (p->tensor_kind > K_BO && p->tensor_kind != K_OTHER)
    return fail(GLACIER_CUDA_FMT_BAD_TENSOR_KIND, "page %llu: tensor kind %u", (unsigned long long)index,
                p->tensor_kind);
  if (p->precision > P_FP32)
    return fail(GLACIER_CUDA_FMT_BAD_PRECISION, "page %llu: precision %u", (unsigned long long)index,
                (unsigned)p->precision);
  return GLACIER_CUDA_OK;
}

// validatePageGeometryV1 (format.zig:279-345): the payload length a page's
// precision, element count and quantization group imply, and the V1 bounds.
int check_geometry(const glacier_cuda_page_entry& p, uint64_t index) {
  const unsigned long long ix = index;
  const uint64_t n = p.row_end - p.row_start;
  uint64_t expect = 0;
  switch (p.precision) {
    case P_FP32:
    case P_FP16:
    case P_BF16:
      if (p.quant_group) return fail(GLACIER_CUDA_FMT_BAD_QUANT_GROUP, "page %llu: raw page with a group", ix);
      if (!mul_ok(n, p.precision == P_FP32 ? 4 : 2, &expect))
        return fail(GLACIER_CUDA_FMT_LAYOUT_OVERFLOW, "page %llu: byte count overflows", ix);
      break;
    case P_INT8:
    case P_INT4: {
      if (!p.quant_group) return fail(GLACIER_CUDA_FMT_BAD_QUANT_GROUP, "page %llu: quantized page without a group", ix);
      if (n > kPageSizeBytes / 4)
        return fail(GLACIER_CUDA_FMT_PAGE_GEOMETRY_TOO_LARGE, "page %llu: %llu quantized elements", ix,
                    (unsigned long long)n);
      const uint64_t packed = p.precision == P_INT8 ? n : cdiv(n, 2);
      expect = kQioHeader + cdiv(n, p.quant_group) * 4 + packed;
      break;
    }
    default:
      return fail(GLACIER_CUDA_FMT_UNSUPPORTED_PRECISION, "page %llu: precision %u is not supported", ix,
                  (unsigned)p.precision);
  }
  if (expect != p.data_len)
    return fail(GLACIER_CUDA_FMT_BAD_PAGE_GEOMETRY, "page %llu: data_len %llu, geometry implies %llu", ix,
                (unsigned long long)p.data_len, (unsigned long long)expect);
  if ((p.precision == P_FP32 || p.precision == P_FP16 || p.precision == P_BF16) && expect > kPageSizeBytes)
    return fail(GLACIER_CUDA_FMT_PAGE_GEOMETRY_TOO_LARGE, "page %llu: raw payload above 256 KiB", ix);
  return GLACIER_CUDA_OK;
}

// FileReader.openFile (format.zig:407-478) on an in-memory image.
int admit(const uint8_t* b, uint64_t len, Container* c) {
  g_format_error = 0;
  if (!b && len) return set_error(GLACIER_CUDA_EINVAL, "glacier format: null buffer");
  int rc = read_header(b, len, &c->h);
  if (rc) return rc;
  const Header& h = c->h;
  if (!JsonCheck(b + h.meta_offset, h.meta_len).object_document())
    return fail(GLACIER_CUDA_FMT_BAD_METADATA, "metadata is not one JSON object");
  c->pages.resize(h.num_pages);
  for (uint64_t i = 0; i < h.num_pages; ++i)
    if ((rc = read_entry(b + h.index_offset + i * kEntrySize, i, &c->pages[i]))) return rc;
  // validatePagesV1 (format.zig:251-277).
  uint64_t expect = h.data_offset;
  for (uint64_t i = 0; i < h.num_pages; ++i) {
    const auto& p = c->pages[i];
    const unsigned long long ix = i;
    if (p.page_id != i) return fail(GLACIER_CUDA_FMT_BAD_PAGE_ID, "entry %llu has page_id %llu", ix,
                                    (unsigned long long)p.page_id);
    if (p.row_end <= p.row_start) return fail(GLACIER_CUDA_FMT_BAD_ROW_RANGE, "page %llu: empty row range", ix);
    if (p.data_len == 0) return fail(GLACIER_CUDA_FMT_EMPTY_PAGE, "page %llu: no payload", ix);
    if ((rc = check_geometry(p, i))) return rc;
    if (p.data_offset != expect)
      return fail(GLACIER_CUDA_FMT_NON_CONTIGUOUS_PAYLOAD, "page %llu: payload at %llu, expected %llu", ix,
                  (unsigned long long)p.data_offset, (unsigned long long)expect);
    if (!add_ok(p.data_offset, p.data_len, &expect))
      return fail(GLACIER_CUDA_FMT_LAYOUT_OVERFLOW, "page %llu: payload end overflows", ix);
    if (expect > len) return fail(GLACIER_CUDA_FMT_TRUNCATED_PAGE, "page %llu runs past the end", ix);
  }
  if (expect != len)
    return fail(GLACIER_CUDA_FMT_TRAILING_BYTES, "%llu bytes after the last page",
                (unsigned long long)(len - expect));
  return GLACIER_CUDA_OK;
}

// validatePayloadSchemaV1 (format.zig:347-375): a quantized payload's
// sub-header must describe the entry's own element count, group and precision.
int check_schema(const uint8_t* b, const glacier_cuda_page_entry& p, uint64_t index) {
  if (p.precision != P_INT8 && p.precision != P_INT4) return GLACIER_CUDA_OK;
  const uint8_t* q = b + p.data_offset;
  const unsigned long long ix = index;
  if (q[13] || q[14] || q[15]) return fail(GLACIER_CUDA_FMT_BAD_QUANT_PAYLOAD, "page %llu: sub-header byte set", ix);
  const uint32_t magic = rd<uint32_t>(q), n = rd<uint32_t>(q + 4), g = rd<uint32_t>(q + 8);
  if (magic != kQioMagic || g == 0 || q[12] > 1)
    return fail(GLACIER_CUDA_FMT_BAD_QUANT_PAYLOAD, "page %llu: bad qio sub-header", ix);
  if (n != p.row_end - p.row_start || g != p.quant_group || q[12] != (p.precision == P_INT8 ? 0 : 1))
    return fail(GLACIER_CUDA_FMT_BAD_QUANT_PAYLOAD, "page %llu: sub-header disagrees with the entry", ix);
  return GLACIER_CUDA_OK;
}

int check_crc(const uint8_t* b, const glacier_cuda_page_entry& p, uint64_t index) {
  const uint32_t got = crc32_update(0, b + p.data_offset, p.data_len);
  if (got != p.crc32)
    return fail(GLACIER_CUDA_FMT_CRC_MISMATCH, "page %llu: crc32 %08x, entry says %08x", (unsigned long long)index,
                got, p.crc32);
  return GLACIER_CUDA_OK;
}

// Schema and CRC of every page, spread over the host's cores; the first
// failing page in page order is the one reported.  validateAllPageCrcs checks
// each page's quantized sub-header, then its CRC (format.zig:503-534).  The
// model loader reads pages through readPage, which checks the CRC first
// (:488-495), and a sub-header it cannot use fails the load as BadPayload
// (loader.zig:1697-1700); `loader` selects that order and naming.
bool schema_ok(const uint8_t* b, const glacier_cuda_page_entry& p) {
  if (p.precision != P_INT8 && p.precision != P_INT4) return true;
  const uint8_t* q = b + p.data_offset;
  return !q[13] && !q[14] && !q[15] && rd<uint32_t>(q) == kQioMagic && rd<uint32_t>(q + 4) == p.row_end - p.row_start &&
         rd<uint32_t>(q + 8) == p.quant_group && q[12] == (p.precision == P_INT8 ? 0 : 1);
}

int check_all_pages(const uint8_t* b, const Container& c, bool loader) {
  const uint64_t n = c.pages.size();
  unsigned nt = std::max(1u, std::min(std::thread::hardware_concurrency(), 64u));
  uint64_t bytes = 0;
  for (const auto& p : c.pages) bytes += p.data_len;
  if (bytes < (64ull << 20)) nt = 1;
  std::atomic<uint64_t> next{0}, first_bad{UINT64_MAX};
  auto work = [&] {
    for (uint64_t i; (i = next.fetch_add(1)) < n;) {
      const auto& p = c.pages[i];
      if (schema_ok(b, p) && crc32_update(0, b + p.data_offset, p.data_len) == p.crc32) continue;
      uint64_t cur = first_bad.load();
      while (i < cur && !first_bad.compare_exchange_weak(cur, i)) {
      }
    }
  };
  std::vector<std::thread> pool;
  for (unsigned t = 1; t < nt; ++t) pool.emplace_back(work);
  work();
  for (auto& t : pool) t.join();
  const uint64_t bad = first_bad.load();
  if (bad == UINT64_MAX) return GLACIER_CUDA_OK;
  const auto& p = c.pages[bad];
  if (loader) {
    const int rc = check_crc(b, p, bad);
    return rc ? rc : fail(GLACIER_CUDA_FMT_BAD_PAYLOAD, "page %llu: quantized sub-header does not match the entry",
                          (unsigned long long)bad);
  }
  const int rc = check_schema(b, p, bad);
  return rc ? rc : check_crc(b, p, bad);
}

// IEEE binary16 -> binary32, exact for every input (normal, subnormal, zero,
// infinity, NaN with its payload).
float half_bits_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  const uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF;
  uint32_t bits;
  if (exp == 0x1F) {
    bits = sign | 0x7F800000u | man << 13;
  } else if (exp) {
    bits = sign | (exp + 112) << 23 | man << 13;
  } else if (man) {  // subnormal: man * 2^-24, exactly representable
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

// readPageDequant(f32) (format.zig:638-662): raw pages widen exactly
// (decodeRawPageV1, :675-716); quantized pages dequantize as
// core/quant.zig:114-160 does, (code - qmax) * scale in f32 with qmax 7 for
// INT4 and 127 for INT8.  The page must have passed admission.
void decode_f32(const uint8_t* b, const glacier_cuda_page_entry& p, float* out) {
  const uint8_t* d = b + p.data_offset;
  const uint64_t n = p.row_end - p.row_start;
  switch (p.precision) {
    case P_FP32:
      memcpy(out, d, n * 4);
      return;
    case P_FP16:
      for (uint64_t i = 0; i < n; ++i) out[i] = half_bits_to_float(rd<uint16_t>(d + 2 * i));
      return;
    case P_BF16:
      for (uint64_t i = 0; i < n; ++i) {
        const uint32_t bits = (uint32_t)rd<uint16_t>(d + 2 * i) << 16;
        memcpy(out + i, &bits, 4);
      }
      return;
    default: {
      const uint32_t g = p.quant_group;
      const uint8_t* codes = d + kQioHeader + cdiv(n, g) * 4;
      for (uint64_t i = 0; i < n; ++i) {
        const int q = p.precision == P_INT8 ? (int)codes[i] - 127 : (int)((codes[i >> 1] >> ((i & 1) * 4)) & 15) - 7;
        out[i] = (float)q * rd<float>(d + kQioHeader + (i / g) * 4);
      }
    }
  }
}

// ---------------------------------------------------------------- loader ----
// loader.zig:1224-1260: geometry from page metadata.  Norm pages are raw, so
// their largest row_end is dim; MLP and vocabulary tensors are quantized over
// their flat element ranges, so hidden and vocab are the largest row_end
// divided by dim.  The group size is the first INT4 page's.
void geometry(const Container& c, glacier_cuda_file_geometry* g) {
  memset(g, 0, sizeof(*g));
  uint64_t dim = 0, hidden = 0, vocab = 0;
  for (const auto& p : c.pages) {
    g->num_layers = std::max<uint32_t>(g->num_layers, p.layer_idx + 1);
    switch (p.tensor_kind) {
      case K_INPUT_NORM: case K_POST_NORM: case K_FINAL_NORM: dim = std::max(dim, p.row_end); break;
      case K_UP: case K_GATE: case K_DOWN: hidden = std::max(hidden, p.row_end); break;
      case K_EMBEDDING: case K_LM_HEAD: vocab = std::max(vocab, p.row_end); break;
      default: break;
    }
    if (p.precision == P_INT4 && !g->group_size) g->group_size = p.quant_group;
    if (p.tensor_kind == K_LM_HEAD) g->has_lm_head = 1;
    if (p.tensor_kind == K_BQ || p.tensor_kind == K_BK || p.tensor_kind == K_BV) g->has_qkv_bias = 1;
  }
  if (dim > 0) {
    if (hidden > dim) hidden /= dim;
    if (vocab > dim) vocab /= dim;
  } else {
    dim = hidden > 0 ? hidden / 4 : 16;
    hidden = 4 * dim;
  }
  g->dim = dim;
  g->hidden = hidden;
  g->vocab = vocab;
}

struct Tensor {
  std::vector<const glacier_cuda_page_entry*> pages;  // page-id order
};

// concatInt4Pages (loader.zig:1633-1730): one packed tensor from INT4 pages
// quantized one page at a time.  Every page but the last covers whole groups,
// so the pages' scales laid end to end are the tensor's flat group scales.
int int4_layout(const Tensor& t, uint32_t* group, uint64_t* elements) {
  uint32_t g = 0;
  uint64_t total = 0, nscales = 0;
  for (size_t k = 0; k < t.pages.size(); ++k) {
    const auto& p = *t.pages[k];
    if (!g) g = p.quant_group;
    const uint64_t n = p.row_end - p.row_start;
    if (p.quant_group != g || (k + 1 < t.pages.size() && n % g))
      return fail(GLACIER_CUDA_FMT_BAD_PAYLOAD, "page %llu: INT4 pages of one tensor split a group",
                  (unsigned long long)p.page_id);
    total += n;
    nscales += cdiv(n, g);
  }
  if (nscales != cdiv(total, g)) return fail(GLACIER_CUDA_FMT_BAD_PAYLOAD, "INT4 tensor scale count mismatch");
  *group = g;
  *elements = total;
  return GLACIER_CUDA_OK;
}

int concat_int4(const uint8_t* b, const Tensor& t, std::vector<uint8_t>* packed, std::vector<float>* scales,
                uint32_t* group) {
  uint64_t total = 0;
  int rc = int4_layout(t, group, &total);
  if (rc) return rc;
  const uint32_t g = *group;
  packed->assign(cdiv(total, 2), 0);
  scales->resize(cdiv(total, g));
  uint64_t at = 0, sat = 0;
  for (const auto* pp : t.pages) {
    const auto& p = *pp;
    const uint64_t n = p.row_end - p.row_start, ns = cdiv(n, g);
    const uint8_t* d = b + p.data_offset;
    memcpy(scales->data() + sat, d + kQioHeader, ns * 4);
    const uint8_t* codes = d + kQioHeader + ns * 4;
    if (at % 2 == 0 && n % 2 == 0) {
      memcpy(packed->data() + at / 2, codes, n / 2);
    } else {
      for (uint64_t i = 0; i < n; ++i) {
        const uint8_t v = (codes[i >> 1] >> ((i & 1) * 4)) & 15;
        uint8_t& dst = (*packed)[(at + i) >> 1];
        dst = ((at + i) & 1) ? (uint8_t)((dst & 0x0F) | v << 4) : (uint8_t)((dst & 0xF0) | v);
      }
    }
    at += n;
    sat += ns;
  }
  return GLACIER_CUDA_OK;
}

std::vector<float> concat_f32(const uint8_t* b, const Tensor& t) {
  uint64_t total = 0;
  for (const auto* p : t.pages) total += p->row_end - p->row_start;
  std::vector<float> out(total);
  uint64_t at = 0;
  for (const auto* p : t.pages) {
    decode_f32(b, *p, out.data() + at);
    at += p->row_end - p->row_start;
  }
  return out;
}

bool all_int4(const Tensor& t) {
  for (const auto* p : t.pages)
    if (p->precision != P_INT4) return false;
  return !t.pages.empty();
}

bool is_packed_kind(uint32_t kind) {  // isCompactTensorKind, loader.zig:1593-1607
  return kind == K_EMBEDDING || (kind >= K_Q && kind <= K_GATE) || kind == K_LM_HEAD;
}

int int4_kind_to_model(uint32_t kind) {
  switch (kind) {
    case K_Q: return GLACIER_CUDA_W_Q;
    case K_K: return GLACIER_CUDA_W_K;
    case K_V: return GLACIER_CUDA_W_V;
    case K_O: return GLACIER_CUDA_W_O;
    case K_GATE: return GLACIER_CUDA_W_GATE;
    case K_UP: return GLACIER_CUDA_W_UP;
    case K_DOWN: return GLACIER_CUDA_W_DOWN;
    default: return -1;
  }
}

}  // namespace

// Shared with the runtime-image reader: the CRC and this thread's format reason.
uint32_t crc32_ieee(uint32_t crc, const uint8_t* p, size_t n) { return crc32_update(crc, p, n); }
int32_t* format_error_slot() { return &g_format_error; }

}  // namespace glacier

using namespace glacier;

extern "C" {

int32_t glacier_cuda_format_error(void) { return g_format_error; }

uint32_t glacier_cuda_crc32(const uint8_t* data, size_t len) { return data ? crc32_update(0, data, len) : 0; }

int glacier_cuda_glacier_open(const uint8_t* bytes, uint64_t len, glacier_cuda_file_info* info) {
  GLC_REQUIRE(info, "glacier_open: null info");
  Container c;
  const int rc = admit(bytes, len, &c);
  if (rc) return rc;
  info->container_bytes = len;
  info->meta_offset = c.h.meta_offset;
  info->meta_len = c.h.meta_len;
  info->num_pages = c.h.num_pages;
  info->page_index_offset = c.h.index_offset;
  info->page_data_offset = c.h.data_offset;
  return GLACIER_CUDA_OK;
}

int glacier_cuda_glacier_validate_pages(const uint8_t* bytes, uint64_t len) {
  Container c;
  const int rc = admit(bytes, len, &c);
  return rc ? rc : check_all_pages(bytes, c, false);
}

int glacier_cuda_glacier_pages(const uint8_t* bytes, uint64_t len, glacier_cuda_page_entry* out, uint64_t capacity,
                               uint64_t* count) {
  GLC_REQUIRE(count && (out || capacity == 0), "glacier_pages: null output");
  Container c;
  const int rc = admit(bytes, len, &c);
  if (rc) return rc;
  *count = c.pages.size();
  std::copy(c.pages.begin(), c.pages.begin() + std::min<uint64_t>(capacity, c.pages.size()), out);
  return GLACIER_CUDA_OK;
}

int glacier_cuda_glacier_page(const uint8_t* bytes, uint64_t len, uint64_t index, glacier_cuda_page_entry* out) {
  GLC_REQUIRE(out, "glacier_page: null output");
  Container c;
  const int rc = admit(bytes, len, &c);
  if (rc) return rc;
  GLC_REQUIRE(index < c.pages.size(), "glacier_page: page %llu of %zu", (unsigned long long)index, c.pages.size());
  *out = c.pages[index];
  return GLACIER_CUDA_OK;
}

int glacier_cuda_glacier_page_decode_f32(const uint8_t* bytes, uint64_t len, uint64_t index, float* out,
                                         uint64_t count) {
  GLC_REQUIRE(out, "glacier_page_decode: null output");
  Container c;
  int rc = admit(bytes, len, &c);
  if (rc) return rc;
  GLC_REQUIRE(index < c.pages.size(), "glacier_page_decode: page %llu of %zu", (unsigned long long)index,
              c.pages.size());
  const auto& p = c.pages[index];
  if (count != p.row_end - p.row_start)
    return fail(GLACIER_CUDA_FMT_SIZE_MISMATCH, "page %llu holds %llu elements, output has %llu",
                (unsigned long long)index, (unsigned long long)(p.row_end - p.row_start),
                (unsigned long long)count);
  // readPage checks the CRC before any decode (format.zig:488-495).
  if ((rc = check_crc(bytes, p, index)) || (rc = check_schema(bytes, p, index))) return rc;
  decode_f32(bytes, p, out);
  return GLACIER_CUDA_OK;
}

int glacier_cuda_glacier_geometry(const uint8_t* bytes, uint64_t len, glacier_cuda_file_geometry* out) {
  GLC_REQUIRE(out, "glacier_geometry: null output");
  Container c;
  const int rc = admit(bytes, len, &c);
  if (rc) return rc;
  if (c.pages.empty()) return fail(GLACIER_CUDA_FMT_NO_LAYERS, "the container has no pages");
  geometry(c, out);
  return GLACIER_CUDA_OK;
}

int glacier_cuda_model_load_glacier(glacier_cuda_model* model, const uint8_t* bytes, uint64_t len,
                                    int tie_word_embeddings) {
  GLC_REQUIRE(model, "model_load_glacier: null model");
  const glacier_cuda_model_config& cfg = *model_config(model);
  Container c;
  int rc = admit(bytes, len, &c);
  if (rc) return rc;
  if (c.pages.empty()) return fail(GLACIER_CUDA_FMT_NO_LAYERS, "the container has no pages");
  // Every page is read through readPage in the reference loader, so every
  // payload's CRC (and quantized sub-header) is checked before any upload.
  if ((rc = check_all_pages(bytes, c, true))) return rc;

  glacier_cuda_file_geometry geo;
  geometry(c, &geo);
  GLC_REQUIRE(geo.num_layers == cfg.num_layers, "model_load_glacier: file has %u layers, model %u", geo.num_layers,
              cfg.num_layers);

  std::map<std::pair<uint32_t, uint32_t>, Tensor> groups;  // (layer, kind) -> pages in id order
  for (const auto& p : c.pages) groups[{p.layer_idx, p.tensor_kind}].pages.push_back(&p);

  auto find = [&](uint32_t layer, uint32_t kind) -> const Tensor* {
    auto it = groups.find({layer, kind});
    return it == groups.end() ? nullptr : &it->second;
  };
  auto missing = [&](uint32_t layer, const char* what) {
    return fail(GLACIER_CUDA_FMT_MISSING_TENSOR, "layer %u has no %s", layer, what);
  };
  auto upload_int4 = [&](const Tensor& t, int layer, int kind, const char* what) -> int {
    if (!all_int4(t))
      return set_error(GLACIER_CUDA_EUNSUPPORTED, "model_load_glacier: %s is not INT4 (dense projections are not "
                       "part of this decode path)", what);
    std::vector<uint8_t> packed;
    std::vector<float> scales;
    uint32_t g = 0;
    int r = concat_int4(bytes, t, &packed, &scales, &g);
    if (r) return r;
    if (g != cfg.group_size)
      return fail(GLACIER_CUDA_FMT_BAD_PAYLOAD, "%s has group %u, model %u", what, g, cfg.group_size);
    return glacier_cuda_model_load_int4(model, layer, kind, packed.data(), packed.size(), scales.data(),
                                        scales.size());
  };
  auto upload_f32 = [&](const Tensor& t, int layer, int kind) -> int {
    const std::vector<float> v = concat_f32(bytes, t);
    return glacier_cuda_model_load_f32(model, layer, kind, v.data(), v.size());
  };

  // The reference loader materialises every group, so a packed group that
  // splits a quantization group fails the load even when nothing uses it.
  for (const auto& kv : groups) {
    uint32_t g;
    uint64_t n;
    if (is_packed_kind(kv.first.second) && all_int4(kv.second) && (rc = int4_layout(kv.second, &g, &n))) return rc;
  }

  for (uint32_t l = 0; l < cfg.num_layers; ++l) {
    static const struct { uint32_t kind; const char* name; } projections[] = {
        {K_Q, "attn_q"}, {K_K, "attn_k"}, {K_V, "attn_v"}, {K_O, "attn_o"},
        {K_GATE, "mlp_gate"}, {K_UP, "mlp_up"}, {K_DOWN, "mlp_down"}};
    for (const auto& pr : projections) {
      const Tensor* t = find(l, pr.kind);
      if (!t) return missing(l, pr.name);
      if ((rc = upload_int4(*t, (int)l, int4_kind_to_model(pr.kind), pr.name))) return rc;
    }
    const Tensor* in = find(l, K_INPUT_NORM);
    const Tensor* post = find(l, K_POST_NORM);
    if (!in) return missing(l, "input_norm");
    if (!post) return missing(l, "post_attn_norm");
    if ((rc = upload_f32(*in, (int)l, GLACIER_CUDA_N_INPUT)) || (rc = upload_f32(*post, (int)l, GLACIER_CUDA_N_POST_ATTN)))
      return rc;
    static const struct { uint32_t kind; int model_kind; } biases[] = {
        {K_BQ, GLACIER_CUDA_B_Q}, {K_BK, GLACIER_CUDA_B_K}, {K_BV, GLACIER_CUDA_B_V}};
    for (const auto& bi : biases)
      if (const Tensor* t = find(l, bi.kind))
        if ((rc = upload_f32(*t, (int)l, bi.model_kind))) return rc;
    if (find(l, K_BO))
      return set_error(GLACIER_CUDA_EUNSUPPORTED, "model_load_glacier: layer %u carries an attention output bias", l);
  }

  // Global tensors live at layer 0 (loader.zig:1510-1523).
  const Tensor* fin = find(0, K_FINAL_NORM);
  if (!fin) return missing(0, "final_norm");
  if ((rc = upload_f32(*fin, -1, GLACIER_CUDA_N_FINAL))) return rc;

  const Tensor* emb = find(0, K_EMBEDDING);
  if (!emb) return missing(0, "embedding");
  bool all_f16 = true;
  for (const auto* p : emb->pages) all_f16 = all_f16 && p->precision == P_FP16;
  if (all_f16) {
    // fp16 pages go up as they are: the table keeps the file's bits.
    uint64_t n = 0;
    for (const auto* p : emb->pages) n += p->row_end - p->row_start;
    std::vector<uint16_t> table(n);
    uint64_t at = 0;
    for (const auto* p : emb->pages) {
      memcpy(table.data() + at, bytes + p->data_offset, p->data_len);
      at += p->row_end - p->row_start;
    }
    rc = glacier_cuda_model_load_embedding_f16(model, table.data(), table.size());
  } else {
    // INT4 rows dequantize as int4_matmul.zig dequantizeRow (:3166-3196),
    // code offset times the f32 group scale; other precisions widen exactly.
    const std::vector<float> table = concat_f32(bytes, *emb);
    rc = glacier_cuda_model_load_embedding_f32(model, table.data(), table.size());
  }
  if (rc) return rc;

  if (tie_word_embeddings) {
    // A tied head is the embedding's own INT4 data (loader.zig:1521-1523).
    if (!all_int4(*emb))
      return set_error(GLACIER_CUDA_EUNSUPPORTED, "model_load_glacier: a tied LM head needs an INT4 embedding");
    return upload_int4(*emb, -1, GLACIER_CUDA_W_LM_HEAD, "embedding (tied LM head)");
  }
  const Tensor* head = find(0, K_LM_HEAD);
  if (!head) return missing(0, "lm_head");
  return upload_int4(*head, -1, GLACIER_CUDA_W_LM_HEAD, "lm_head");
}

}  // extern "C"
