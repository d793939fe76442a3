// zcblk.cu -- ZCBLK01 tensor blocks, the ZCINF01 model manifest with its shard
// map and experts pack index, and the expert loader that streams FP4 expert
// blocks from disk into HBM.  Host code only: block bytes move on the copy
// engines, from pinned staging buffers that reader threads fill with pread.
#include <errno.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cctype>
#include <set>
#include <thread>

namespace {

constexpr uint64_t kAlign2M = 2ull << 20;
constexpr uint64_t kBlockHeader = 40;  // QUANT_BLOCK_HEADER_SIZE (src/model_format.rs:14)
constexpr uint64_t kRecord = 52;       // QUANT_TENSOR_RECORD_SIZE (src/model_format.rs:15)
constexpr uint16_t kQuantFp4 = 2402;   // QUANT_DEEPSEEK_FP4_E2M1_PACKED (src/deepseek_v4.rs:43)
constexpr uint16_t kQuantUe8m0 = 2403; // QUANT_DEEPSEEK_UE8M0_SCALE (src/deepseek_v4.rs:44)
constexpr uint64_t kPlace = 256;       // device placement of each expert tensor

#define WH_TRY(call)                 \
  do {                               \
    wh_status s_ = (call);           \
    if (s_ != WH_OK) return s_;      \
  } while (0)

bool add_ovf(uint64_t a, uint64_t b, uint64_t* r) { return __builtin_add_overflow(a, b, r); }
bool mul_ovf(uint64_t a, uint64_t b, uint64_t* r) { return __builtin_mul_overflow(a, b, r); }
uint64_t round_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

struct Blk {
  const uint8_t* p;
  uint64_t n;
};

// read_le_bytes (src/compute.rs:7199-7214); the host is little-endian
template <typename T>
wh_status rd(const Blk& b, uint64_t off, const char* field, T* out) {
  uint64_t end;
  if (add_ovf(off, sizeof(T), &end)) return fail(WH_ERR_BLOCK_INVALID, "read range overflow");
  if (end > b.n) return fail(WH_ERR_BLOCK_TRUNCATED, field);
  memcpy(out, b.p + off, sizeof(T));
  return WH_OK;
}

// parse_quant_block (src/compute.rs:1099-1147)
wh_status parse_block(const Blk& b, wh_zcblk_header* h) {
  if (b.n < kBlockHeader) return fail(WH_ERR_BLOCK_TRUNCATED, "block header");
  if (memcmp(b.p, "ZCBLK01\0", 8) != 0) return fail(WH_ERR_BLOCK_MAGIC, "invalid ZCBLK magic");
  uint32_t version, count, qf, flags;
  uint64_t rto, nmo;
  WH_TRY(rd(b, 8, "block.version", &version));
  if (version != 1)
    return fail(WH_ERR_BLOCK_VERSION, "unsupported ZCBLK version: " + std::to_string(version));
  WH_TRY(rd(b, 12, "block.tensor_count", &count));
  WH_TRY(rd(b, 16, "block.quant_format", &qf));
  WH_TRY(rd(b, 20, "block.flags", &flags));
  WH_TRY(rd(b, 24, "block.record_table_offset", &rto));
  WH_TRY(rd(b, 32, "block.names_offset", &nmo));
  uint64_t rec_end;
  if (add_ovf(rto, uint64_t(count) * kRecord, &rec_end))
    return fail(WH_ERR_BLOCK_INVALID, "record table range overflow");
  if (rto < kBlockHeader || rec_end > b.n) return fail(WH_ERR_BLOCK_TRUNCATED, "record table");
  if (nmo > b.n) return fail(WH_ERR_BLOCK_TRUNCATED, "names blob");
  *h = wh_zcblk_header{count, qf, flags, 0, rto, nmo};
  return WH_OK;
}

// QuantBlockLayout::tensor (src/compute.rs:545-595) with read_name_blob and
// read_shape_layout (src/compute.rs:7136-7178)
wh_status tensor_at(const Blk& b, const wh_zcblk_header& h, uint64_t index, wh_zcblk_tensor* t) {
  if (index >= h.tensor_count)
    return fail(WH_ERR_TENSOR_INDEX, "tensor index out of range: index=" +
                                         std::to_string(index) +
                                         ", count=" + std::to_string(h.tensor_count));
  uint64_t ro, ro_end;
  if (add_ovf(h.record_table_offset, index * kRecord, &ro))
    return fail(WH_ERR_BLOCK_INVALID, "record offset overflow");
  if (add_ovf(ro, kRecord, &ro_end) || ro_end > b.n)
    return fail(WH_ERR_BLOCK_TRUNCATED, "tensor record");
  const uint8_t* r = b.p + ro;
  uint64_t name_off, shape_off, data_off, data_len;
  *t = wh_zcblk_tensor{};
  memcpy(&t->dtype_original, r + 0, 2);
  memcpy(&t->quant_format, r + 2, 2);
  memcpy(&t->rank, r + 4, 4);
  memcpy(&t->flags, r + 8, 4);
  memcpy(&name_off, r + 12, 8);
  memcpy(&shape_off, r + 20, 8);
  memcpy(&data_off, r + 28, 8);
  memcpy(&data_len, r + 36, 8);
  memcpy(&t->scale, r + 44, 4);
  memcpy(&t->zero_point, r + 48, 4);

  uint64_t absolute, name_end;
  if (add_ovf(h.names_offset, name_off, &absolute))
    return fail(WH_ERR_BLOCK_INVALID, "name offset overflow");
  uint16_t name_len;
  WH_TRY(rd(b, absolute, "name.len", &name_len));
  if (add_ovf(absolute + 2, name_len, &name_end))
    return fail(WH_ERR_BLOCK_INVALID, "name end overflow");
  if (name_end > b.n) return fail(WH_ERR_BLOCK_TRUNCATED, "name blob");
  t->name_pos = absolute + 2;
  t->name_len = name_len;

  uint32_t rank;
  WH_TRY(rd(b, shape_off, "shape.rank", &rank));
  if (rank != t->rank) return fail(WH_ERR_BLOCK_INVALID, "shape rank mismatch");
  uint64_t shape_end;
  if (add_ovf(shape_off, 4 + uint64_t(rank) * 8, &shape_end))
    return fail(WH_ERR_BLOCK_INVALID, "shape end overflow");
  if (shape_end > b.n) return fail(WH_ERR_BLOCK_TRUNCATED, "shape blob");
  t->shape_pos = shape_off;

  uint64_t data_end;
  if (add_ovf(data_off, data_len, &data_end))
    return fail(WH_ERR_BLOCK_INVALID, "tensor data range overflow");
  if (data_end > b.n) return fail(WH_ERR_BLOCK_TRUNCATED, "tensor data");
  t->data_pos = data_off;
  t->data_len = data_len;
  return WH_OK;
}

// ShapeLayout::dim (src/compute.rs:514-520)
wh_status tensor_dim(const Blk& b, const wh_zcblk_tensor& t, uint64_t index, uint64_t* out) {
  if (index >= t.rank) return fail(WH_ERR_BLOCK_INVALID, "shape dim index out of range");
  return rd(b, t.shape_pos + 4 + index * 8, "shape.dim", out);
}

// find_tensor_by_suffix (src/compute.rs:1149-1169)
wh_status find_suffix(const Blk& b, const wh_zcblk_header& h, const char* suffix,
                      wh_zcblk_tensor* out) {
  const size_t sl = strlen(suffix);
  bool found = false;
  for (uint64_t i = 0; i < h.tensor_count; ++i) {
    wh_zcblk_tensor t;
    WH_TRY(tensor_at(b, h, i, &t));
    if (t.name_len >= sl && memcmp(b.p + t.name_pos + t.name_len - sl, suffix, sl) == 0) {
      if (found) return fail(WH_ERR_BLOCK_INVALID, "duplicate DeepSeek expert tensor suffix");
      *out = t;
      found = true;
    }
  }
  if (!found) return fail(WH_ERR_BLOCK_INVALID, "missing DeepSeek expert tensor suffix");
  return WH_OK;
}

// deepseek_fp4_matvec_from_tensors (src/compute.rs:1199-1247)
wh_status fp4_view(const Blk& b, const wh_zcblk_tensor& w, const wh_zcblk_tensor& s,
                   wh_zcblk_fp4_view* v) {
  if (w.quant_format != kQuantFp4)
    return fail(WH_ERR_BLOCK_INVALID, "DeepSeek expert weight is not FP4 E2M1 packed");
  if (s.quant_format != kQuantUe8m0)
    return fail(WH_ERR_BLOCK_INVALID, "DeepSeek expert scale is not UE8M0");
  if (w.rank != 2 || s.rank != 2) return fail(WH_ERR_INVALID_SHAPE, "DeepSeek FP4 expert rank");
  uint64_t rows, packed, srows, scols;
  WH_TRY(tensor_dim(b, w, 0, &rows));
  WH_TRY(tensor_dim(b, w, 1, &packed));
  WH_TRY(tensor_dim(b, s, 0, &srows));
  WH_TRY(tensor_dim(b, s, 1, &scols));
  if (rows == 0 || packed == 0 || scols == 0 || srows != rows)
    return fail(WH_ERR_INVALID_SHAPE, "DeepSeek FP4 expert shape");
  uint64_t cols, need_w, need_s;
  if (mul_ovf(packed, 2, &cols)) return fail(WH_ERR_INVALID_SHAPE, "DeepSeek FP4 expert cols overflow");
  if (mul_ovf(rows, packed, &need_w))
    return fail(WH_ERR_INVALID_SHAPE, "DeepSeek FP4 expert weight overflow");
  if (w.data_len < need_w) return fail(WH_ERR_BLOCK_TRUNCATED, "DeepSeek FP4 expert weight");
  if (mul_ovf(rows, scols, &need_s))
    return fail(WH_ERR_INVALID_SHAPE, "DeepSeek FP4 expert scale overflow");
  if (s.data_len < need_s) return fail(WH_ERR_BLOCK_TRUNCATED, "DeepSeek FP4 expert scale");
  *v = wh_zcblk_fp4_view{w.data_pos, need_w, s.data_pos, need_s, rows, cols, scols};
  return WH_OK;
}

// parse_quant_block + deepseek_v4_fp4_expert_from_quant_block (src/compute.rs:1249-1267)
wh_status fp4_expert_view(const Blk& b, wh_zcblk_fp4_expert_view* out) {
  wh_zcblk_header h;
  WH_TRY(parse_block(b, &h));
  wh_zcblk_fp4_view* v[3] = {&out->w1, &out->w3, &out->w2};
  const char* names[3][2] = {{".w1.weight", ".w1.scale"},
                             {".w3.weight", ".w3.scale"},
                             {".w2.weight", ".w2.scale"}};
  for (int k = 0; k < 3; ++k) {
    wh_zcblk_tensor w, s;
    WH_TRY(find_suffix(b, h, names[k][0], &w));
    WH_TRY(find_suffix(b, h, names[k][1], &s));
    WH_TRY(fp4_view(b, w, s, v[k]));
  }
  if (out->w1.cols != out->w3.cols || out->w1.rows != out->w3.rows ||
      out->w2.cols != out->w1.rows)
    return fail(WH_ERR_INVALID_SHAPE, "DeepSeek FP4 expert projection");
  return WH_OK;
}

uint64_t expert_device_bytes(uint64_t payload) { return round_up(payload + 6 * kPlace, kPlace); }

// The six tensors of a parsed expert, in placement order: (block position,
// length) pairs and the device specs they become at `dst`.
wh_status place_expert(const wh_zcblk_fp4_expert_view& v, uint8_t* dst, uint64_t dst_bytes,
                       uint64_t src_pos[6], uint64_t len[6], wh_fp4_expert* out) {
  const wh_zcblk_fp4_view* m[3] = {&v.w1, &v.w3, &v.w2};
  wh_fp4_matvec_spec* o[3] = {&out->w1, &out->w3, &out->w2};
  uint64_t off = 0;
  for (int k = 0; k < 3; ++k) {
    src_pos[2 * k] = m[k]->weight_pos;
    len[2 * k] = m[k]->weight_len;
    src_pos[2 * k + 1] = m[k]->scale_pos;
    len[2 * k + 1] = m[k]->scale_len;
    o[k]->packed_weight = dst + off;
    o[k]->packed_len = m[k]->weight_len;
    off = round_up(off + m[k]->weight_len, kPlace);
    o[k]->ue8m0_scales = dst + off;
    o[k]->scales_len = m[k]->scale_len;
    off = round_up(off + m[k]->scale_len, kPlace);
    o[k]->rows = m[k]->rows;
    o[k]->cols = m[k]->cols;
    o[k]->scale_cols = m[k]->scale_cols;
  }
  if (off > dst_bytes)
    return fail(WH_ERR_OUTPUT_TOO_SMALL, "expert slot too small: required=" +
                                             std::to_string(off) +
                                             ", actual=" + std::to_string(dst_bytes));
  return WH_OK;
}

wh_status queue_expert_copies(const uint8_t* block, const uint64_t src_pos[6],
                              const uint64_t len[6], const wh_fp4_expert& e, cudaStream_t s) {
  const wh_fp4_matvec_spec* o[3] = {&e.w1, &e.w3, &e.w2};
  for (int k = 0; k < 3; ++k) {
    WH_CUDA(cudaMemcpyAsync(const_cast<uint8_t*>(o[k]->packed_weight), block + src_pos[2 * k],
                            len[2 * k], cudaMemcpyHostToDevice, s));
    WH_CUDA(cudaMemcpyAsync(const_cast<uint8_t*>(o[k]->ue8m0_scales), block + src_pos[2 * k + 1],
                            len[2 * k + 1], cudaMemcpyHostToDevice, s));
  }
  return WH_OK;
}

// --------------------------------------------------------------------------
// A small JSON reader for the shard map and the experts pack index (the
// reference deserialises them with serde_json into ShardMapDisk /
// ExpertPackDisk, src/model_format.rs:307-337,438-461).  Numbers keep their
// token so that u32/u64 fields convert exactly.
struct JVal {
  enum Type { Null, Bool, Num, Str, Arr, Obj } t = Null;
  bool b = false;
  std::string s;  // Str: the decoded string; Num: the token
  std::vector<JVal> a;
  std::vector<std::pair<std::string, JVal>> o;
};

struct JParser {
  const char* p;
  const char* e;
  std::string err;

  void ws() {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool fail_at(const char* why) {
    if (err.empty()) err = why;
    return false;
  }
  static void utf8(std::string& out, uint32_t cp) {
    if (cp < 0x80) {
      out += char(cp);
    } else if (cp < 0x800) {
      out += char(0xC0 | (cp >> 6));
      out += char(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      out += char(0xE0 | (cp >> 12));
      out += char(0x80 | ((cp >> 6) & 0x3F));
      out += char(0x80 | (cp & 0x3F));
    } else {
      out += char(0xF0 | (cp >> 18));
      out += char(0x80 | ((cp >> 12) & 0x3F));
      out += char(0x80 | ((cp >> 6) & 0x3F));
      out += char(0x80 | (cp & 0x3F));
    }
  }
  bool hex4(uint32_t* v) {
    if (e - p < 4) return fail_at("truncated \\u escape");
    *v = 0;
    for (int i = 0; i < 4; ++i) {
      char c = *p++;
      *v <<= 4;
      if (c >= '0' && c <= '9') *v |= c - '0';
      else if (c >= 'a' && c <= 'f') *v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') *v |= c - 'A' + 10;
      else return fail_at("invalid \\u escape");
    }
    return true;
  }
  bool str(std::string& out) {
    ++p;  // opening quote
    while (p < e && *p != '"') {
      unsigned char c = *p;
      if (c < 0x20) return fail_at("control character in string");
      if (c != '\\') {
        out += char(c);
        ++p;
        continue;
      }
      if (++p >= e) return fail_at("truncated escape");
      char x = *p++;
      switch (x) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          uint32_t cp;
          if (!hex4(&cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00) {
            uint32_t lo;
            if (e - p < 2 || p[0] != '\\' || p[1] != 'u') return fail_at("lone surrogate");
            p += 2;
            if (!hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return fail_at("lone surrogate");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            return fail_at("lone surrogate");
          }
          utf8(out, cp);
          break;
        }
        default: return fail_at("invalid escape");
      }
    }
    if (p >= e) return fail_at("unterminated string");
    ++p;
    return true;
  }
  bool num(JVal& v) {
    const char* s = p;
    if (p < e && *p == '-') ++p;
    if (p >= e || !isdigit((unsigned char)*p)) return fail_at("invalid number");
    if (*p == '0') ++p;
    else while (p < e && isdigit((unsigned char)*p)) ++p;
    if (p < e && *p == '.') {
      ++p;
      if (p >= e || !isdigit((unsigned char)*p)) return fail_at("invalid number");
      while (p < e && isdigit((unsigned char)*p)) ++p;
    }
    if (p < e && (*p == 'e' || *p == 'E')) {
      ++p;
      if (p < e && (*p == '+' || *p == '-')) ++p;
      if (p >= e || !isdigit((unsigned char)*p)) return fail_at("invalid number");
      while (p < e && isdigit((unsigned char)*p)) ++p;
    }
    v.t = JVal::Num;
    v.s.assign(s, p);
    return true;
  }
  bool lit(const char* w, size_t n) {
    if (size_t(e - p) < n || memcmp(p, w, n) != 0) return fail_at("invalid literal");
    p += n;
    return true;
  }
  bool value(JVal& v, int depth) {
    if (depth > 64) return fail_at("nesting too deep");
    ws();
    if (p >= e) return fail_at("unexpected end of input");
    char c = *p;
    if (c == '{') {
      v.t = JVal::Obj;
      ++p;
      ws();
      if (p < e && *p == '}') {
        ++p;
        return true;
      }
      for (;;) {
        ws();
        if (p >= e || *p != '"') return fail_at("expected a key");
        std::string k;
        if (!str(k)) return false;
        ws();
        if (p >= e || *p != ':') return fail_at("expected ':'");
        ++p;
        v.o.emplace_back(std::move(k), JVal{});
        if (!value(v.o.back().second, depth + 1)) return false;
        ws();
        if (p < e && *p == ',') {
          ++p;
          continue;
        }
        if (p < e && *p == '}') {
          ++p;
          return true;
        }
        return fail_at("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.t = JVal::Arr;
      ++p;
      ws();
      if (p < e && *p == ']') {
        ++p;
        return true;
      }
      for (;;) {
        v.a.emplace_back();
        if (!value(v.a.back(), depth + 1)) return false;
        ws();
        if (p < e && *p == ',') {
          ++p;
          continue;
        }
        if (p < e && *p == ']') {
          ++p;
          return true;
        }
        return fail_at("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.t = JVal::Str;
      return str(v.s);
    }
    if (c == 't') {
      v.t = JVal::Bool;
      v.b = true;
      return lit("true", 4);
    }
    if (c == 'f') {
      v.t = JVal::Bool;
      return lit("false", 5);
    }
    if (c == 'n') return lit("null", 4);
    return num(v);
  }
};

wh_status json_parse(const std::string& text, JVal* out) {
  JParser jp{text.data(), text.data() + text.size(), {}};
  if (!jp.value(*out, 0)) return fail(WH_ERR_SHARD_MAP, jp.err);
  jp.ws();
  if (jp.p != jp.e) return fail(WH_ERR_SHARD_MAP, "trailing characters");
  return WH_OK;
}

// A struct field: absent -> `has` false; present twice -> serde's duplicate
// field error.
wh_status json_field(const JVal& obj, const char* key, const JVal** out) {
  *out = nullptr;
  for (const auto& kv : obj.o) {
    if (kv.first != key) continue;
    if (*out) return fail(WH_ERR_SHARD_MAP, std::string("duplicate field `") + key + "`");
    *out = &kv.second;
  }
  return WH_OK;
}

// An unsigned integer field of `bits` bits (serde's u32 / u64)
wh_status json_uint(const JVal& obj, const char* key, int bits, bool has_default, uint64_t* out) {
  const JVal* v;
  WH_TRY(json_field(obj, key, &v));
  if (!v) {
    if (!has_default) return fail(WH_ERR_SHARD_MAP, std::string("missing field `") + key + "`");
    *out = 0;
    return WH_OK;
  }
  const std::string bad = std::string("invalid value for `") + key + "`";
  if (v->t != JVal::Num || v->s.empty() || v->s[0] == '-' ||
      v->s.find_first_of(".eE") != std::string::npos)
    return fail(WH_ERR_SHARD_MAP, bad);
  uint64_t x = 0;
  for (char c : v->s) {
    if (mul_ovf(x, 10, &x) || add_ovf(x, uint64_t(c - '0'), &x)) return fail(WH_ERR_SHARD_MAP, bad);
  }
  if (bits < 64 && (x >> bits) != 0) return fail(WH_ERR_SHARD_MAP, bad);
  *out = x;
  return WH_OK;
}

wh_status json_string(const JVal& obj, const char* key, bool has_default, std::string* out) {
  const JVal* v;
  WH_TRY(json_field(obj, key, &v));
  if (!v) {
    if (!has_default) return fail(WH_ERR_SHARD_MAP, std::string("missing field `") + key + "`");
    out->clear();
    return WH_OK;
  }
  if (v->t != JVal::Str) return fail(WH_ERR_SHARD_MAP, std::string("invalid type for `") + key + "`");
  *out = v->s;
  return WH_OK;
}

wh_status json_array(const JVal& obj, const char* key, const std::vector<JVal>** out) {
  static const std::vector<JVal> empty;
  const JVal* v;
  WH_TRY(json_field(obj, key, &v));
  if (!v) {
    *out = &empty;
    return WH_OK;
  }
  if (v->t != JVal::Arr) return fail(WH_ERR_SHARD_MAP, std::string("invalid type for `") + key + "`");
  *out = &v->a;
  return WH_OK;
}

// --------------------------------------------------------------------------
// Files
std::string io_detail(const std::string& path, int err) { return path + ": " + strerror(err); }

wh_status read_file(const std::string& path, std::string* out) {
  int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) return fail(WH_ERR_IO, io_detail(path, errno));
  out->clear();
  char buf[1 << 16];
  for (;;) {
    ssize_t r = read(fd, buf, sizeof(buf));
    if (r < 0) {
      if (errno == EINTR) continue;
      int e = errno;
      close(fd);
      return fail(WH_ERR_IO, io_detail(path, e));
    }
    if (r == 0) break;
    out->append(buf, size_t(r));
  }
  close(fd);
  return WH_OK;
}

// pread until `n` bytes or end of file; *got receives the byte count
wh_status pread_full(int fd, const std::string& path, void* dst, uint64_t n, uint64_t off,
                     uint64_t* got) {
  uint64_t done = 0;
  while (done < n) {
    ssize_t r = pread(fd, static_cast<uint8_t*>(dst) + done, size_t(n - done), off_t(off + done));
    if (r < 0) {
      if (errno == EINTR) continue;
      return fail(WH_ERR_IO, io_detail(path, errno));
    }
    if (r == 0) break;
    done += uint64_t(r);
  }
  *got = done;
  return WH_OK;
}

wh_status read_exact_at(int fd, const std::string& path, void* dst, uint64_t n, uint64_t off) {
  uint64_t got;
  WH_TRY(pread_full(fd, path, dst, n, off, &got));
  if (got != n) return fail(WH_ERR_IO, path + ": failed to fill whole buffer");
  return WH_OK;
}

bool file_exists(const std::string& p) {
  struct stat st;
  return stat(p.c_str(), &st) == 0;
}

// Path::parent (empty for a bare file name) and Path::join
std::string parent_dir(const std::string& p) {
  size_t k = p.find_last_of('/');
  if (k == std::string::npos) return "";
  return k == 0 ? "/" : p.substr(0, k);
}
std::string join_path(const std::string& dir, const std::string& rel) {
  if (!rel.empty() && rel[0] == '/') return rel;
  if (dir.empty()) return rel;
  return dir.back() == '/' ? dir + rel : dir + "/" + rel;
}
// Path::with_extension: replace the file name's last extension (a leading dot
// does not start one) or add one
std::string with_extension(const std::string& p, const std::string& ext) {
  size_t k = p.find_last_of('/');
  size_t name = k == std::string::npos ? 0 : k + 1;
  size_t dot = p.find_last_of('.');
  std::string stem = (dot != std::string::npos && dot > name) ? p.substr(0, dot) : p;
  return stem + "." + ext;
}

wh_status validate_aligned(const char* field, uint64_t v) {
  if (v & (kAlign2M - 1)) return fail(WH_ERR_UNALIGNED, field);
  return WH_OK;
}

struct ShardRef {
  std::string path;
  uint64_t disk_bytes, payload_bytes, checksum;
};
struct PackEntry {
  uint64_t offset, disk_bytes, payload_bytes;
};
struct ModelLayer {
  wh_model_layer d;
  std::vector<wh_model_expert> experts;
};

}  // namespace

struct wh_model {
  std::string path, base_dir, pack_file;
  wh_engine_header hdr{};
  std::vector<ModelLayer> layers;
  std::map<std::pair<uint32_t, uint32_t>, ShardRef> shards;
  std::map<std::pair<uint32_t, uint32_t>, PackEntry> pack;
  bool has_pack = false;
};

namespace {

// load_optional_shard_map (src/model_format.rs:339-436)
wh_status load_shard_map(wh_model* m, bool merge) {
  const std::string sp = with_extension(m->path, "shards.json");
  if (!file_exists(sp)) return WH_OK;
  std::string text;
  JVal root;
  WH_TRY(read_file(sp, &text));
  WH_TRY(json_parse(text, &root));
  if (root.t != JVal::Obj) return fail(WH_ERR_SHARD_MAP, "shard map is not an object");
  std::string format;
  const std::vector<JVal>* experts;
  WH_TRY(json_string(root, "format", true, &format));
  WH_TRY(json_array(root, "experts", &experts));
  struct Disk {
    uint64_t layer_id, expert_id, disk_bytes, payload_bytes, dequant_bytes, quant_format, checksum;
    std::string path;
  };
  std::vector<Disk> disk;
  for (const JVal& e : *experts) {
    if (e.t != JVal::Obj) return fail(WH_ERR_SHARD_MAP, "invalid type for expert entry");
    Disk d;
    WH_TRY(json_uint(e, "layer_id", 32, false, &d.layer_id));
    WH_TRY(json_uint(e, "expert_id", 32, false, &d.expert_id));
    WH_TRY(json_string(e, "path", false, &d.path));
    WH_TRY(json_uint(e, "disk_bytes", 64, false, &d.disk_bytes));
    WH_TRY(json_uint(e, "payload_bytes", 64, false, &d.payload_bytes));
    WH_TRY(json_uint(e, "dequant_bytes", 64, true, &d.dequant_bytes));
    WH_TRY(json_uint(e, "quant_format", 32, true, &d.quant_format));
    WH_TRY(json_uint(e, "checksum", 64, true, &d.checksum));
    disk.push_back(std::move(d));
  }
  // "zeroclaw-..." is the format's earlier name, still valid on disk
  if (format != "wohper-sharded-experts" && format != "zeroclaw-sharded-experts")
    return fail(WH_ERR_SHARD_MAP, "unsupported shard map format in " + sp + ": " + format);
  std::set<std::pair<uint32_t, uint32_t>> known;
  for (const auto& L : m->layers)
    for (const auto& x : L.experts) known.insert({x.layer_id, x.expert_id});
  int merged = 0;
  for (const Disk& d : disk) {
    const std::pair<uint32_t, uint32_t> key{uint32_t(d.layer_id), uint32_t(d.expert_id)};
    const bool in_manifest = known.count(key) != 0;
    if (!in_manifest && !merge) continue;
    WH_TRY(validate_aligned("expert_shard.disk_bytes", d.disk_bytes));
    if (!in_manifest) {
      ModelLayer* target = nullptr;
      for (auto& L : m->layers)
        if ((L.d.flags & 0xff) == 0 && L.d.layer_id == key.first) {
          target = &L;
          break;
        }
      if (!target) continue;
      const uint32_t tmpl = target->experts.empty() ? 0 : target->experts[0].quant_format;
      wh_model_expert x{};
      x.layer_id = key.first;
      x.expert_id = key.second;
      x.disk_offset = 0;
      x.disk_bytes = d.disk_bytes;
      x.payload_bytes = d.payload_bytes;
      x.dequant_bytes = d.dequant_bytes;
      x.quant_format = d.quant_format ? uint32_t(d.quant_format) : tmpl;
      x.route_rank_hint = key.second;
      x.checksum = d.checksum;
      target->experts.push_back(x);
      ++merged;
    }
    m->shards[key] = ShardRef{join_path(m->base_dir, d.path), d.disk_bytes, d.payload_bytes,
                              d.checksum};
  }
  if (merged) {
    for (auto& L : m->layers) {
      std::stable_sort(L.experts.begin(), L.experts.end(),
                       [](const wh_model_expert& a, const wh_model_expert& b) {
                         return a.expert_id < b.expert_id;
                       });
      L.d.num_experts = uint32_t(L.experts.size());
    }
  }
  return WH_OK;
}

// load_optional_expert_pack (src/model_format.rs:463-505)
wh_status load_pack(wh_model* m) {
  const std::string ip = with_extension(m->path, "experts_pack.index.json");
  if (!file_exists(ip)) return WH_OK;
  std::string text;
  JVal root;
  WH_TRY(read_file(ip, &text));
  WH_TRY(json_parse(text, &root));
  if (root.t != JVal::Obj) return fail(WH_ERR_SHARD_MAP, "pack index is not an object");
  std::string format, pack_name;
  const std::vector<JVal>* entries;
  WH_TRY(json_string(root, "format", true, &format));
  WH_TRY(json_string(root, "pack_file", true, &pack_name));
  WH_TRY(json_array(root, "entries", &entries));
  std::vector<std::pair<std::pair<uint32_t, uint32_t>, PackEntry>> disk;
  for (const JVal& e : *entries) {
    if (e.t != JVal::Obj) return fail(WH_ERR_SHARD_MAP, "invalid type for pack entry");
    uint64_t lid, eid;
    PackEntry pe;
    WH_TRY(json_uint(e, "layer_id", 32, false, &lid));
    WH_TRY(json_uint(e, "expert_id", 32, false, &eid));
    WH_TRY(json_uint(e, "offset", 64, false, &pe.offset));
    WH_TRY(json_uint(e, "disk_bytes", 64, false, &pe.disk_bytes));
    WH_TRY(json_uint(e, "payload_bytes", 64, false, &pe.payload_bytes));
    disk.push_back({{uint32_t(lid), uint32_t(eid)}, pe});
  }
  if (format != "wohper-experts-pack" && format != "zeroclaw-experts-pack")
    return fail(WH_ERR_SHARD_MAP, "unsupported experts pack format in " + ip + ": " + format);
  const std::string pf = join_path(parent_dir(ip), pack_name);
  if (!file_exists(pf)) return fail(WH_ERR_SHARD_MAP, "experts pack file missing: " + pf);
  for (const auto& kv : disk) {
    WH_TRY(validate_aligned("expert_pack.offset", kv.second.offset));
    WH_TRY(validate_aligned("expert_pack.disk_bytes", kv.second.disk_bytes));
    m->pack[kv.first] = kv.second;
  }
  m->pack_file = pf;
  m->has_pack = true;
  return WH_OK;
}

// ModelManifest::load (src/model_format.rs:193-263) with validate_header,
// validate_layer and validate_expert (:507-541)
wh_status load_model(wh_model* m, bool merge) {
  int fd = open(m->path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) return fail(WH_ERR_IO, io_detail(m->path, errno));
  struct Closer {
    int fd;
    ~Closer() { close(fd); }
  } closer{fd};
  static_assert(sizeof(wh_engine_header) == 128, "EngineHeader is 128 bytes");
  wh_engine_header& h = m->hdr;
  WH_TRY(read_exact_at(fd, m->path, &h, sizeof(h), 0));
  if (memcmp(h.magic, "ZCINF01\0", 8) != 0) return fail(WH_ERR_MODEL_MAGIC, "invalid magic");
  if (h.version != 1)
    return fail(WH_ERR_MODEL_VERSION, "unsupported version: " + std::to_string(h.version));
  if (h.block_alignment != kAlign2M) return fail(WH_ERR_UNALIGNED, "block_alignment");
  WH_TRY(validate_aligned("manifest_offset", h.manifest_offset));
  WH_TRY(validate_aligned("tokenizer_offset", h.tokenizer_offset));
  WH_TRY(validate_aligned("router_metadata_offset", h.router_metadata_offset));

  struct ManifestHeader {
    uint32_t layer_count, expert_count, tensor_count, reserved;
    uint64_t layer_desc_offset, expert_desc_offset, tensor_desc_offset;
  } mh;
  static_assert(sizeof(ManifestHeader) == 40, "ManifestHeader is 40 bytes");
  WH_TRY(read_exact_at(fd, m->path, &mh, sizeof(mh), h.manifest_offset));
  if (mh.layer_count != h.num_layers)
    return fail(WH_ERR_LAYER_COUNT, "invalid layer count: header=" + std::to_string(h.num_layers) +
                                        ", manifest=" + std::to_string(mh.layer_count));
  struct LayerDisk {
    uint32_t layer_id, flags;
    uint64_t dense_offset, dense_disk_bytes, dense_payload_bytes, dense_dequant_bytes;
    uint32_t tensor_count, first_tensor_index, first_expert_index, num_experts, quant_format,
        checksum_kind;
    uint64_t checksum;
  };
  static_assert(sizeof(LayerDisk) == 72, "LayerBlockDescDisk is 72 bytes");
  static_assert(sizeof(wh_model_expert) == 56, "ExpertBlockDescDisk is 56 bytes");
  std::vector<LayerDisk> layers(mh.layer_count);
  std::vector<wh_model_expert> experts(mh.expert_count);
  uint64_t lo, eo;
  if (add_ovf(h.manifest_offset, mh.layer_desc_offset, &lo) ||
      add_ovf(h.manifest_offset, mh.expert_desc_offset, &eo))
    return fail(WH_ERR_IO, m->path + ": invalid seek to a negative or overflowing position");
  WH_TRY(read_exact_at(fd, m->path, layers.data(), layers.size() * sizeof(LayerDisk), lo));
  WH_TRY(read_exact_at(fd, m->path, experts.data(), experts.size() * sizeof(wh_model_expert), eo));
  for (const LayerDisk& d : layers) {
    WH_TRY(validate_aligned("dense_offset", d.dense_offset));
    WH_TRY(validate_aligned("dense_disk_bytes", d.dense_disk_bytes));
    const uint64_t start = d.first_expert_index, end = start + uint64_t(d.num_experts);
    if (end > experts.size())
      return fail(WH_ERR_EXPERT_TABLE, "invalid expert table for layer " + std::to_string(d.layer_id));
    ModelLayer L;
    L.d = wh_model_layer{d.layer_id, d.flags, d.dense_offset, d.dense_disk_bytes,
                         d.dense_payload_bytes, d.dense_dequant_bytes, d.num_experts, 0};
    for (uint64_t i = start; i < end; ++i) {
      const wh_model_expert& x = experts[i];
      if (x.disk_offset == 0) {
        // external expert shards are resolved through MODEL.shards.json
        WH_TRY(validate_aligned("expert.disk_bytes", x.disk_bytes));
      } else {
        WH_TRY(validate_aligned("expert.disk_offset", x.disk_offset));
        WH_TRY(validate_aligned("expert.disk_bytes", x.disk_bytes));
      }
      if (x.layer_id != d.layer_id)
        return fail(WH_ERR_EXPERT_TABLE,
                    "invalid expert table for layer " + std::to_string(d.layer_id));
      L.experts.push_back(x);
    }
    m->layers.push_back(std::move(L));
  }
  m->base_dir = parent_dir(m->path);
  WH_TRY(load_shard_map(m, merge));
  WH_TRY(load_pack(m));
  return WH_OK;
}

// MoEIoScheduler::enqueue_expert_read (src/scheduler.rs:148-193)
wh_status expert_source(const wh_model* m, int layer_index, uint32_t expert_id,
                        wh_expert_source* out) {
  if (layer_index < 0 || size_t(layer_index) >= m->layers.size())
    return fail(WH_ERR_INVALID_SHAPE, "layer index out of range");
  const ModelLayer& L = m->layers[layer_index];
  const wh_model_expert* x = nullptr;
  for (const auto& e : L.experts)
    if (e.expert_id == expert_id) {
      x = &e;
      break;
    }
  if (!x)
    return fail(WH_ERR_INVALID_EXPERT, "invalid expert: layer=" + std::to_string(L.d.layer_id) +
                                           ", expert=" + std::to_string(expert_id));
  const std::pair<uint32_t, uint32_t> key{L.d.layer_id, expert_id};
  *out = wh_expert_source{};
  auto pk = m->pack.find(key);
  if (pk != m->pack.end()) {
    *out = wh_expert_source{m->pack_file.c_str(), pk->second.offset, pk->second.disk_bytes,
                            pk->second.payload_bytes, WH_SOURCE_PACK, 0};
    return WH_OK;
  }
  auto sh = m->shards.find(key);
  if (sh != m->shards.end())
    *out = wh_expert_source{sh->second.path.c_str(), x->disk_offset, x->disk_bytes,
                            x->payload_bytes, WH_SOURCE_SHARD, 0};
  else
    *out = wh_expert_source{m->path.c_str(), x->disk_offset, x->disk_bytes, x->payload_bytes,
                            WH_SOURCE_MODEL, 0};
  return WH_OK;
}

constexpr uint64_t kDirectAlign = 4096;

struct LoaderSlot {
  uint8_t* buf = nullptr;
  cudaEvent_t free_ev = nullptr;  // the copies out of buf have finished
};
struct LoaderWorker {
  cudaStream_t stream = nullptr;
  cudaEvent_t done = nullptr;
  LoaderSlot slot[2];
};

}  // namespace

struct wh_expert_loader {
  wh_ctx* ctx = nullptr;
  const wh_model* model = nullptr;
  bool direct = false;
  uint64_t slot_bytes = 0;
  std::vector<LoaderWorker> workers;
};

extern "C" {

wh_status wh_zcblk_parse(const uint8_t* block, size_t len, wh_zcblk_header* out) {
  if (!block || !out) return fail(WH_ERR_INVALID_POINTER, "block or out is null");
  return parse_block(Blk{block, len}, out);
}

wh_status wh_zcblk_tensor_at(const uint8_t* block, size_t len, uint32_t index,
                             wh_zcblk_tensor* out) {
  if (!block || !out) return fail(WH_ERR_INVALID_POINTER, "block or out is null");
  wh_zcblk_header h;
  WH_TRY(parse_block(Blk{block, len}, &h));
  return tensor_at(Blk{block, len}, h, index, out);
}

wh_status wh_zcblk_tensor_dim(const uint8_t* block, size_t len, const wh_zcblk_tensor* tensor,
                              uint32_t index, uint64_t* out) {
  if (!block || !tensor || !out) return fail(WH_ERR_INVALID_POINTER, "null argument");
  return tensor_dim(Blk{block, len}, *tensor, index, out);
}

wh_status wh_zcblk_find_suffix(const uint8_t* block, size_t len, const char* suffix,
                               wh_zcblk_tensor* out) {
  if (!block || !suffix || !out) return fail(WH_ERR_INVALID_POINTER, "null argument");
  wh_zcblk_header h;
  WH_TRY(parse_block(Blk{block, len}, &h));
  return find_suffix(Blk{block, len}, h, suffix, out);
}

wh_status wh_zcblk_fp4_expert(const uint8_t* block, size_t len, wh_zcblk_fp4_expert_view* out) {
  if (!block || !out) return fail(WH_ERR_INVALID_POINTER, "block or out is null");
  return fp4_expert_view(Blk{block, len}, out);
}

size_t wh_fp4_expert_device_bytes(uint64_t payload_bytes) {
  return size_t(expert_device_bytes(payload_bytes));
}

wh_status wh_fp4_expert_upload(wh_ctx* ctx, const uint8_t* block, size_t len, void* dst,
                               size_t dst_bytes, wh_fp4_expert* out, wh_stream_t stream) {
  if (!ctx || !block || !dst || !out) return fail(WH_ERR_INVALID_POINTER, "null argument");
  if (device_reach(dst) != 0) return fail(WH_ERR_INVALID_POINTER, "dst is not device memory");
  if (!aligned(dst, kPlace)) return fail(WH_ERR_INVALID_POINTER, "dst is not 256-byte aligned");
  wh_zcblk_fp4_expert_view v;
  WH_TRY(fp4_expert_view(Blk{block, len}, &v));
  uint64_t pos[6], n[6];
  wh_fp4_expert e;
  WH_TRY(place_expert(v, static_cast<uint8_t*>(dst), dst_bytes, pos, n, &e));
  WH_TRY(queue_expert_copies(block, pos, n, e, (cudaStream_t)stream));
  *out = e;
  return WH_OK;
}

wh_status wh_model_open(const char* path, int merge_sidecar_experts, wh_model** out) {
  if (!path || !out) return fail(WH_ERR_INVALID_POINTER, "path or out is null");
  *out = nullptr;
  wh_model* m = new wh_model();
  m->path = path;
  wh_status st = load_model(m, merge_sidecar_experts != 0);
  if (st != WH_OK) {
    delete m;
    return st;
  }
  *out = m;
  return WH_OK;
}

void wh_model_close(wh_model* model) { delete model; }

wh_status wh_model_get_header(const wh_model* model, wh_engine_header* out) {
  if (!model || !out) return fail(WH_ERR_INVALID_POINTER, "model or out is null");
  *out = model->hdr;
  return WH_OK;
}

int wh_model_layer_count(const wh_model* model) {
  return model ? int(model->layers.size()) : 0;
}

wh_status wh_model_get_layer(const wh_model* model, int layer_index, wh_model_layer* out) {
  if (!model || !out) return fail(WH_ERR_INVALID_POINTER, "model or out is null");
  if (layer_index < 0 || size_t(layer_index) >= model->layers.size())
    return fail(WH_ERR_INVALID_SHAPE, "layer index out of range");
  *out = model->layers[layer_index].d;
  out->num_experts = uint32_t(model->layers[layer_index].experts.size());
  return WH_OK;
}

wh_status wh_model_get_expert(const wh_model* model, int layer_index, int expert_index,
                              wh_model_expert* out) {
  if (!model || !out) return fail(WH_ERR_INVALID_POINTER, "model or out is null");
  if (layer_index < 0 || size_t(layer_index) >= model->layers.size())
    return fail(WH_ERR_INVALID_SHAPE, "layer index out of range");
  const auto& ex = model->layers[layer_index].experts;
  if (expert_index < 0 || size_t(expert_index) >= ex.size())
    return fail(WH_ERR_INVALID_SHAPE, "expert index out of range");
  *out = ex[expert_index];
  return WH_OK;
}

wh_status wh_model_expert_source(const wh_model* model, int layer_index, uint32_t expert_id,
                                 wh_expert_source* out) {
  if (!model || !out) return fail(WH_ERR_INVALID_POINTER, "model or out is null");
  return expert_source(model, layer_index, expert_id, out);
}

wh_status wh_expert_arena_bytes(const wh_model* model, int layer_index,
                                const uint32_t* expert_ids, int n, size_t* out) {
  if (!model || !out || (n > 0 && !expert_ids)) return fail(WH_ERR_INVALID_POINTER, "null argument");
  if (n < 0) return fail(WH_ERR_INVALID_SHAPE, "n < 0");
  uint64_t total = 0;
  for (int i = 0; i < n; ++i) {
    wh_expert_source s;
    WH_TRY(expert_source(model, layer_index, expert_ids[i], &s));
    total += expert_device_bytes(s.payload_bytes);
  }
  *out = size_t(total);
  return WH_OK;
}

void wh_expert_loader_destroy(wh_expert_loader* l) {
  if (!l) return;
  cudaSetDevice(l->ctx->device);
  for (auto& w : l->workers) {
    for (auto& s : w.slot) {
      if (s.free_ev) {
        cudaEventSynchronize(s.free_ev);
        cudaEventDestroy(s.free_ev);
      }
      if (s.buf) cudaFreeHost(s.buf);
    }
    if (w.done) cudaEventDestroy(w.done);
    if (w.stream) cudaStreamDestroy(w.stream);
  }
  delete l;
}

wh_status wh_expert_loader_create(wh_ctx* ctx, const wh_model* model, int threads, int direct_io,
                                  wh_expert_loader** out) {
  if (!ctx || !model || !out) return fail(WH_ERR_INVALID_POINTER, "null argument");
  *out = nullptr;
  if (threads <= 0) threads = 8;
  threads = std::min(threads, 64);
  wh_expert_loader* l = new wh_expert_loader();
  l->ctx = ctx;
  l->model = model;
  l->direct = direct_io != 0;
  // a staging slot holds the largest block any expert of the model reads
  uint64_t most = 0;
  for (int li = 0; li < int(model->layers.size()); ++li)
    for (const auto& x : model->layers[li].experts) {
      wh_expert_source s;
      if (expert_source(model, li, x.expert_id, &s) != WH_OK) continue;
      most = std::max(most, l->direct ? round_up(s.payload_bytes, kDirectAlign) : s.payload_bytes);
    }
  l->slot_bytes = std::max<uint64_t>(round_up(most, kDirectAlign), kDirectAlign);
  l->workers.resize(threads);
  auto cleanup = [&](wh_status st) {
    wh_expert_loader_destroy(l);
    return st;
  };
  cudaSetDevice(ctx->device);
  for (auto& w : l->workers) {
    cudaError_t e = cudaStreamCreateWithFlags(&w.stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&w.done, cudaEventDisableTiming);
    for (auto& s : w.slot) {
      if (e == cudaSuccess) e = cudaHostAlloc(&s.buf, l->slot_bytes, cudaHostAllocDefault);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.free_ev, cudaEventDisableTiming);
    }
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "expert loader staging"));
  }
  *out = l;
  return WH_OK;
}

wh_status wh_expert_loader_load(wh_expert_loader* l, int layer_index, const uint32_t* expert_ids,
                                int n, void* arena, size_t arena_bytes, wh_fp4_expert* out,
                                wh_stream_t stream) {
  if (!l || (n > 0 && (!expert_ids || !arena || !out)))
    return fail(WH_ERR_INVALID_POINTER, "null argument");
  if (n < 0) return fail(WH_ERR_INVALID_SHAPE, "n < 0");
  if (n == 0) return WH_OK;
  if (device_reach(arena) != 0) return fail(WH_ERR_INVALID_POINTER, "arena is not device memory");
  if (!aligned(arena, kPlace)) return fail(WH_ERR_INVALID_POINTER, "arena is not 256-byte aligned");
  std::vector<wh_expert_source> src(n);
  std::vector<uint64_t> slot_off(n);
  uint64_t need = 0;
  for (int i = 0; i < n; ++i) {
    WH_TRY(expert_source(l->model, layer_index, expert_ids[i], &src[i]));
    slot_off[i] = need;
    need += expert_device_bytes(src[i].payload_bytes);
  }
  if (need > arena_bytes)
    return fail(WH_ERR_OUTPUT_TOO_SMALL, "arena too small: required=" + std::to_string(need) +
                                             ", actual=" + std::to_string(arena_bytes));
  cudaSetDevice(l->ctx->device);
  std::atomic<int> next{0};
  std::atomic<bool> failed{false};
  std::mutex mu;
  wh_status err = WH_OK;
  std::string err_detail;
  auto record = [&](wh_status st) {
    std::lock_guard<std::mutex> g(mu);
    if (err == WH_OK) {
      err = st;
      err_detail = g_detail;
    }
    failed = true;
  };
  uint8_t* base = static_cast<uint8_t*>(arena);
  auto work = [&](LoaderWorker& w) {
    cudaSetDevice(l->ctx->device);
    int k = 0;
    for (;;) {
      const int i = next.fetch_add(1);
      if (i >= n || failed) break;
      LoaderSlot& slot = w.slot[k++ & 1];
      cudaError_t ce = cudaEventSynchronize(slot.free_ev);
      if (ce != cudaSuccess) return record(cuda_fail(ce, "staging slot wait"));
      const wh_expert_source& s = src[i];
      const uint64_t want = l->direct ? round_up(s.payload_bytes, kDirectAlign) : s.payload_bytes;
      if (want > l->slot_bytes) return record(fail(WH_ERR_IO, "block larger than the staging slot"));
      int fd = -1;
      bool direct = false;
      if (l->direct) {
        fd = open(s.path, O_RDONLY | O_CLOEXEC | O_DIRECT);
        direct = fd >= 0;
      }
      if (fd < 0) fd = open(s.path, O_RDONLY | O_CLOEXEC);
      if (fd < 0) return record(fail(WH_ERR_IO, io_detail(s.path, errno)));
      uint64_t got = 0;
      wh_status st = pread_full(fd, s.path, slot.buf, direct ? want : s.payload_bytes, s.offset, &got);
      close(fd);
      if (st != WH_OK) return record(st);
      if (got < s.payload_bytes)
        return record(fail(WH_ERR_IO, std::string(s.path) + ": failed to fill whole buffer"));
      wh_zcblk_fp4_expert_view v;
      st = fp4_expert_view(Blk{slot.buf, s.payload_bytes}, &v);
      uint64_t pos[6], len[6];
      if (st == WH_OK)
        st = place_expert(v, base + slot_off[i], expert_device_bytes(s.payload_bytes), pos, len,
                          &out[i]);
      if (st != WH_OK) return record(st);
      st = queue_expert_copies(slot.buf, pos, len, out[i], w.stream);
      // the slot is reused only after whatever was queued out of it has run
      ce = cudaEventRecord(slot.free_ev, w.stream);
      if (st != WH_OK) return record(st);
      if (ce != cudaSuccess) return record(cuda_fail(ce, "staging slot record"));
    }
  };
  const int T = std::min<int>(int(l->workers.size()), n);
  std::vector<std::thread> pool;
  pool.reserve(T);
  for (int t = 0; t < T; ++t) pool.emplace_back(work, std::ref(l->workers[t]));
  for (auto& th : pool) th.join();
  // the caller's stream waits for every worker's copies, also after an error
  // (the staging slots stay guarded by their events either way)
  for (int t = 0; t < T; ++t) {
    LoaderWorker& w = l->workers[t];
    WH_CUDA(cudaEventRecord(w.done, w.stream));
    WH_CUDA(cudaStreamWaitEvent((cudaStream_t)stream, w.done, 0));
  }
  if (err != WH_OK) return fail(err, err_detail);
  return WH_OK;
}

}  // extern "C"
