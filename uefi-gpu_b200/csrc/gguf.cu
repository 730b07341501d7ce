// gguf.cu -- GGUF v3 directory parsing and decoder binding (host code only).
//
// The reference reads its model from GGUF files with a bounded zero-copy directory parser
// (frontier_gguf.rs:145-200 Shard::parse, :84-104 Tensor::rows / expert, :106-140 ModelIndex)
// and maps tensor bodies from storage.  Here the directory is parsed with the same limits and
// checks, in the same order, so a malformed file fails with the same error; tensor bodies stay
// with the caller, who copies them to the device and binds a decoder to them through
// ugb_gguf_model_weights.  The file format itself (magic, version, key/value table, tensor infos,
// aligned data section) is GGUF's, so the field order here is the format's.
#include <algorithm>
#include <cstring>
#include <new>
#include <set>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "internal.hpp"

namespace {

struct MetaItem {
  std::string key;
  uint32_t kind;
  std::vector<uint8_t> data;  // the value's bytes as stored (after the kind)
};

struct TensorItem {
  std::string name;
  uint64_t dims[4];
  uint32_t rank, kind;
  uint64_t offset, bytes, row_bytes;
};

// Bounded little-endian reader over a byte range.
struct Reader {
  const uint8_t *data;
  size_t len, pos;
  int32_t take(size_t n, const uint8_t **out) {
    if (n > SIZE_MAX - pos) return UGB_GGUF_OVERFLOW;
    if (pos + n > len) return UGB_GGUF_TRUNCATED;
    *out = data + pos;
    pos += n;
    return UGB_GGUF_OK;
  }
  int32_t u32(uint32_t *v) {
    const uint8_t *p;
    const int32_t e = take(4, &p);
    if (e) return e;
    std::memcpy(v, p, 4);
    return UGB_GGUF_OK;
  }
  int32_t u64(uint64_t *v) {
    const uint8_t *p;
    const int32_t e = take(8, &p);
    if (e) return e;
    std::memcpy(v, p, 8);
    return UGB_GGUF_OK;
  }
  // GGUF string: u64 length + bytes, at most 16 MiB, valid UTF-8.
  int32_t str(const uint8_t **s, size_t *n);
  // Skip one value of `kind`; arrays may not nest.
  int32_t skip(uint32_t kind, bool nested);
};

bool valid_utf8(const uint8_t *s, size_t n) {
  size_t i = 0;
  while (i < n) {
    const uint8_t c = s[i];
    size_t extra;
    uint32_t cp;
    if (c < 0x80) {
      ++i;
      continue;
    } else if ((c & 0xE0) == 0xC0) {
      extra = 1;
      cp = c & 0x1F;
    } else if ((c & 0xF0) == 0xE0) {
      extra = 2;
      cp = c & 0x0F;
    } else if ((c & 0xF8) == 0xF0) {
      extra = 3;
      cp = c & 0x07;
    } else {
      return false;
    }
    if (i + extra >= n) return false;  // the sequence runs past the string
    for (size_t k = 1; k <= extra; ++k) {
      if ((s[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (s[i + k] & 0x3F);
    }
    // overlong forms, surrogates and values past U+10FFFF are not UTF-8
    if ((extra == 1 && cp < 0x80) || (extra == 2 && cp < 0x800) || (extra == 3 && cp < 0x10000) ||
        (cp >= 0xD800 && cp <= 0xDFFF) || cp > 0x10FFFF)
      return false;
    i += extra + 1;
  }
  return true;
}

int32_t Reader::str(const uint8_t **s, size_t *n) {
  uint64_t len64;
  int32_t e = u64(&len64);
  if (e) return e;
  if (len64 > 16ull * 1024 * 1024) return UGB_GGUF_LIMIT;
  e = take(static_cast<size_t>(len64), s);
  if (e) return e;
  if (!valid_utf8(*s, static_cast<size_t>(len64))) return UGB_GGUF_UTF8;
  *n = static_cast<size_t>(len64);
  return UGB_GGUF_OK;
}

int32_t Reader::skip(uint32_t kind, bool nested) {
  const uint8_t *p;
  switch (kind) {
    case 0: case 1: case 7: return take(1, &p);   // u8, i8, bool
    case 2: case 3: return take(2, &p);           // u16, i16
    case 4: case 5: case 6: return take(4, &p);   // u32, i32, f32
    case 10: case 11: case 12: return take(8, &p);  // u64, i64, f64
    case 8: {
      size_t n;
      return str(&p, &n);
    }
    case 9: {
      if (nested) return UGB_GGUF_TYPE;
      uint32_t elem;
      uint64_t count;
      int32_t e = u32(&elem);
      if (!e) e = u64(&count);
      if (e) return e;
      if (count > 1000000) return UGB_GGUF_LIMIT;
      for (uint64_t i = 0; i < count; ++i) {
        e = skip(elem, true);
        if (e) return e;
      }
      return UGB_GGUF_OK;
    }
    default: return UGB_GGUF_TYPE;
  }
}

// Bytes of one row of n elements of `kind`: the library's table (ugb_row_bytes) plus F16.
int32_t gguf_row_bytes(uint32_t kind, uint64_t n, uint64_t *out) {
  uint64_t block, bytes;
  switch (kind) {
    case 0: block = 1; bytes = 4; break;      // F32
    case 1: block = 1; bytes = 2; break;      // F16
    case 8: block = 32; bytes = 34; break;    // Q8_0
    case 11: block = 256; bytes = 110; break; // Q3_K
    case 12: block = 256; bytes = 144; break; // Q4_K
    case 14: block = 256; bytes = 210; break; // Q6_K
    case 18: block = 256; bytes = 98; break;  // IQ3_XXS
    case 20: block = 32; bytes = 18; break;   // IQ4_NL
    case 23: block = 256; bytes = 136; break; // IQ4_XS
    case 30: block = 1; bytes = 2; break;     // BF16
    default: return UGB_GGUF_TYPE;
  }
  if (n == 0 || n % block != 0) return UGB_GGUF_SHAPE;
  const uint64_t nb = n / block;
  if (nb > UINT64_MAX / bytes) return UGB_GGUF_OVERFLOW;
  *out = nb * bytes;
  return UGB_GGUF_OK;
}

bool mul_ok(uint64_t a, uint64_t b, uint64_t *out) {
  if (a != 0 && b > UINT64_MAX / a) return false;
  *out = a * b;
  return true;
}

bool add_ok(uint64_t a, uint64_t b, uint64_t *out) {
  if (b > UINT64_MAX - a) return false;
  *out = a + b;
  return true;
}

}  // namespace

struct ugb_gguf {
  std::vector<MetaItem> meta;
  std::vector<TensorItem> tensors;
  std::unordered_map<std::string, size_t> by_name;
  uint64_t data_offset = 0, logical_bytes = 0, split_no = 0, split_count = 1, total_tensors = 0;

  const MetaItem *find(const char *key) const {
    for (const MetaItem &m : meta)
      if (m.key == key) return &m;
    return nullptr;
  }
};

namespace {

// Unsigned value of kind u8 / u16 / u32 / u64 (Value::unsigned, frontier_gguf.rs:44-51).
int32_t value_unsigned(uint32_t kind, const uint8_t *p, size_t n, uint64_t *v) {
  size_t w = kind == 0 ? 1 : kind == 2 ? 2 : kind == 4 ? 4 : kind == 10 ? 8 : 0;
  if (!w) return UGB_GGUF_TYPE;
  if (n < w) return UGB_GGUF_TRUNCATED;
  uint64_t x = 0;
  std::memcpy(&x, p, w);
  *v = x;
  return UGB_GGUF_OK;
}

}  // namespace

extern "C" {

int32_t ugb_gguf_parse(const uint8_t *prefix, size_t prefix_len, uint64_t logical_bytes, ugb_gguf **out) {
  if (!out) return UGB_GGUF_MISSING;
  *out = nullptr;
  if (!prefix && prefix_len) return UGB_GGUF_TRUNCATED;
  if (prefix_len > 16u * 1024 * 1024) return UGB_GGUF_LIMIT;
  Reader r{prefix, prefix_len, 0};
  const uint8_t *p;
  int32_t e = r.take(4, &p);
  if (e) return e;
  if (std::memcmp(p, "GGUF", 4) != 0) return UGB_GGUF_MAGIC;
  uint32_t version;
  if ((e = r.u32(&version))) return e;
  if (version != 3) return UGB_GGUF_VERSION;
  uint64_t nt, nk;
  if ((e = r.u64(&nt)) || (e = r.u64(&nk))) return e;
  if (nt > 4096 || nk > 1024) return UGB_GGUF_LIMIT;
  ugb_gguf *g = new (std::nothrow) ugb_gguf();
  if (!g) return UGB_GGUF_LIMIT;
  auto fail = [&](int32_t code) {
    delete g;
    return code;
  };
  g->meta.reserve(nk);
  for (uint64_t i = 0; i < nk; ++i) {
    const uint8_t *ks;
    size_t kn;
    if ((e = r.str(&ks, &kn))) return fail(e);
    if (kn > 256) return fail(UGB_GGUF_LIMIT);
    std::string key(reinterpret_cast<const char *>(ks), kn);
    if (g->find(key.c_str())) return fail(UGB_GGUF_DUPLICATE);
    uint32_t kind;
    if ((e = r.u32(&kind))) return fail(e);
    const size_t start = r.pos;
    if ((e = r.skip(kind, false))) return fail(e);
    g->meta.push_back(MetaItem{std::move(key), kind, std::vector<uint8_t>(prefix + start, prefix + r.pos)});
  }
  g->logical_bytes = logical_bytes;
  g->total_tensors = nt;
  uint64_t v;
  if (const MetaItem *m = g->find("split.no")) {
    if ((e = value_unsigned(m->kind, m->data.data(), m->data.size(), &v))) return fail(e);
    g->split_no = v;
  }
  if (const MetaItem *m = g->find("split.count")) {
    if ((e = value_unsigned(m->kind, m->data.data(), m->data.size(), &v))) return fail(e);
    g->split_count = v;
  }
  if (const MetaItem *m = g->find("split.tensors.count")) {
    if (m->kind == 5) {  // int32 in the standard split files
      int32_t n32;
      if (m->data.size() != 4) return fail(UGB_GGUF_TYPE);
      std::memcpy(&n32, m->data.data(), 4);
      if (n32 < 0) return fail(UGB_GGUF_SPLIT);
      g->total_tensors = static_cast<uint64_t>(n32);
    } else {
      if ((e = value_unsigned(m->kind, m->data.data(), m->data.size(), &v))) return fail(e);
      g->total_tensors = v;
    }
  }
  if (g->split_count == 0 || g->split_count > 64 || g->split_no >= g->split_count || g->total_tensors < nt ||
      g->total_tensors > 65536)
    return fail(UGB_GGUF_SPLIT);
  uint64_t alignment = 32;
  if (const MetaItem *m = g->find("general.alignment")) {
    if ((e = value_unsigned(m->kind, m->data.data(), m->data.size(), &alignment))) return fail(e);
  }
  if (alignment == 0 || (alignment & (alignment - 1)) || alignment > 4096) return fail(UGB_GGUF_ALIGNMENT);
  g->tensors.reserve(nt);
  for (uint64_t i = 0; i < nt; ++i) {
    const uint8_t *ns;
    size_t nn;
    if ((e = r.str(&ns, &nn))) return fail(e);
    if (nn > 256) return fail(UGB_GGUF_LIMIT);
    TensorItem t{};
    t.name.assign(reinterpret_cast<const char *>(ns), nn);
    if (g->by_name.count(t.name)) return fail(UGB_GGUF_DUPLICATE);
    uint32_t rank;
    if ((e = r.u32(&rank))) return fail(e);
    if (rank < 1 || rank > 4) return fail(UGB_GGUF_SHAPE);
    t.rank = rank;
    for (int d = 0; d < 4; ++d) t.dims[d] = 1;
    for (uint32_t d = 0; d < rank; ++d) {
      if ((e = r.u64(&t.dims[d]))) return fail(e);
      if (t.dims[d] == 0) return fail(UGB_GGUF_SHAPE);
    }
    if ((e = r.u32(&t.kind)) || (e = r.u64(&t.offset))) return fail(e);
    if (t.offset % alignment != 0) return fail(UGB_GGUF_ALIGNMENT);
    if ((e = gguf_row_bytes(t.kind, t.dims[0], &t.row_bytes))) return fail(e);
    t.bytes = t.row_bytes;
    for (uint32_t d = 1; d < rank; ++d)
      if (!mul_ok(t.bytes, t.dims[d], &t.bytes)) return fail(UGB_GGUF_OVERFLOW);
    g->by_name.emplace(t.name, g->tensors.size());
    g->tensors.push_back(std::move(t));
  }
  uint64_t data_offset;
  if (!add_ok(r.pos, alignment - 1, &data_offset)) return fail(UGB_GGUF_OVERFLOW);
  data_offset &= ~(alignment - 1);
  if (data_offset > logical_bytes) return fail(UGB_GGUF_TENSOR_BOUNDS);
  g->data_offset = data_offset;
  std::vector<std::pair<uint64_t, uint64_t>> ranges;
  ranges.reserve(g->tensors.size());
  for (TensorItem &t : g->tensors) {
    uint64_t end;
    if (!add_ok(t.offset, data_offset, &t.offset) || !add_ok(t.offset, t.bytes, &end)) return fail(UGB_GGUF_OVERFLOW);
    if (end > logical_bytes) return fail(UGB_GGUF_TENSOR_BOUNDS);
    ranges.emplace_back(t.offset, end);
  }
  std::sort(ranges.begin(), ranges.end());
  for (size_t i = 1; i < ranges.size(); ++i)
    if (ranges[i - 1].second > ranges[i].first) return fail(UGB_GGUF_OVERLAP);
  *out = g;
  return UGB_GGUF_OK;
}

void ugb_gguf_free(ugb_gguf *g) { delete g; }

int32_t ugb_gguf_info(const ugb_gguf *g, uint64_t *data_offset, uint64_t *split_no, uint64_t *split_count,
                      uint64_t *total_tensors, int64_t *n_tensors) {
  if (!g) return UGB_GGUF_MISSING;
  if (data_offset) *data_offset = g->data_offset;
  if (split_no) *split_no = g->split_no;
  if (split_count) *split_count = g->split_count;
  if (total_tensors) *total_tensors = g->total_tensors;
  if (n_tensors) *n_tensors = static_cast<int64_t>(g->tensors.size());
  return UGB_GGUF_OK;
}

static void fill_tensor(const TensorItem &t, ugb_gguf_tensor *out) {
  out->name = t.name.c_str();
  for (int d = 0; d < 4; ++d) out->dims[d] = t.dims[d];
  out->rank = t.rank;
  out->kind = t.kind;
  out->offset = t.offset;
  out->bytes = t.bytes;
  out->row_bytes = t.row_bytes;
}

int32_t ugb_gguf_tensor_at(const ugb_gguf *g, int64_t index, ugb_gguf_tensor *out) {
  if (!g || !out) return UGB_GGUF_MISSING;
  if (index < 0 || static_cast<size_t>(index) >= g->tensors.size()) return UGB_GGUF_MISSING;
  fill_tensor(g->tensors[static_cast<size_t>(index)], out);
  return UGB_GGUF_OK;
}

int32_t ugb_gguf_find_tensor(const ugb_gguf *g, const char *name, ugb_gguf_tensor *out) {
  if (!g || !name || !out) return UGB_GGUF_MISSING;
  auto it = g->by_name.find(name);
  if (it == g->by_name.end()) return UGB_GGUF_MISSING;
  fill_tensor(g->tensors[it->second], out);
  return UGB_GGUF_OK;
}

int32_t ugb_gguf_tensor_rows(const ugb_gguf_tensor *t, uint64_t start, uint64_t count, uint64_t *offset,
                             uint64_t *bytes) {
  if (!t || !t->row_bytes) return UGB_GGUF_MISSING;
  const uint64_t total = t->bytes / t->row_bytes;
  uint64_t end, rel, len;
  if (!add_ok(start, count, &end)) return UGB_GGUF_OVERFLOW;
  if (count == 0 || end > total) return UGB_GGUF_TENSOR_BOUNDS;
  if (!mul_ok(start, t->row_bytes, &rel) || !mul_ok(count, t->row_bytes, &len)) return UGB_GGUF_OVERFLOW;
  uint64_t off;
  if (!add_ok(t->offset, rel, &off)) return UGB_GGUF_OVERFLOW;
  if (offset) *offset = off;
  if (bytes) *bytes = len;
  return UGB_GGUF_OK;
}

int32_t ugb_gguf_tensor_expert(const ugb_gguf_tensor *t, uint32_t id, uint64_t *offset, uint64_t *bytes) {
  if (!t) return UGB_GGUF_MISSING;
  if (t->rank != 3 || id >= t->dims[2]) return UGB_GGUF_SHAPE;
  uint64_t start;
  if (!mul_ok(id, t->dims[1], &start)) return UGB_GGUF_OVERFLOW;
  return ugb_gguf_tensor_rows(t, start, t->dims[1], offset, bytes);
}

int32_t ugb_gguf_meta_kind(const ugb_gguf *g, const char *key, uint32_t *kind) {
  const MetaItem *m = g && key ? g->find(key) : nullptr;
  if (!m) return UGB_GGUF_MISSING;
  if (kind) *kind = m->kind;
  return UGB_GGUF_OK;
}

int32_t ugb_gguf_meta_unsigned(const ugb_gguf *g, const char *key, uint64_t *value) {
  const MetaItem *m = g && key ? g->find(key) : nullptr;
  if (!m) return UGB_GGUF_MISSING;
  uint64_t v;
  const int32_t e = value_unsigned(m->kind, m->data.data(), m->data.size(), &v);
  if (!e && value) *value = v;
  return e;
}

int32_t ugb_gguf_meta_float(const ugb_gguf *g, const char *key, float *value) {
  const MetaItem *m = g && key ? g->find(key) : nullptr;
  if (!m) return UGB_GGUF_MISSING;
  if (m->kind != 6 || m->data.size() != 4) return UGB_GGUF_TYPE;
  if (value) std::memcpy(value, m->data.data(), 4);
  return UGB_GGUF_OK;
}

}  // extern "C"

namespace {

// The string at `p` (u64 length + bytes, validated at parse time) into buf.
int32_t copy_string(const uint8_t *p, char *buf, size_t cap, size_t *len) {
  uint64_t n;
  std::memcpy(&n, p, 8);
  if (len) *len = static_cast<size_t>(n);
  if (buf && cap) {
    const size_t c = std::min<size_t>(cap, static_cast<size_t>(n));
    std::memcpy(buf, p + 8, c);
  }
  return UGB_GGUF_OK;
}

// Element `index` of the array value m: its kind and bytes.
int32_t array_element(const MetaItem *m, uint64_t index, uint32_t *kind, const uint8_t **elem, size_t *n) {
  if (m->kind != 9) return UGB_GGUF_TYPE;
  Reader r{m->data.data(), m->data.size(), 0};
  uint32_t ek;
  uint64_t count;
  int32_t e = r.u32(&ek);
  if (!e) e = r.u64(&count);
  if (e) return e;
  if (index >= count) return UGB_GGUF_MISSING;
  for (uint64_t i = 0; i <= index; ++i) {
    const size_t start = r.pos;
    if ((e = r.skip(ek, true))) return e;
    if (i == index) {
      *kind = ek;
      *elem = m->data.data() + start;
      *n = r.pos - start;
    }
  }
  return UGB_GGUF_OK;
}

}  // namespace

extern "C" {

int32_t ugb_gguf_meta_string(const ugb_gguf *g, const char *key, char *buf, size_t cap, size_t *len) {
  const MetaItem *m = g && key ? g->find(key) : nullptr;
  if (!m) return UGB_GGUF_MISSING;
  if (m->kind != 8) return UGB_GGUF_TYPE;
  return copy_string(m->data.data(), buf, cap, len);
}

int32_t ugb_gguf_meta_array(const ugb_gguf *g, const char *key, uint32_t *elem_kind, uint64_t *count) {
  const MetaItem *m = g && key ? g->find(key) : nullptr;
  if (!m) return UGB_GGUF_MISSING;
  if (m->kind != 9) return UGB_GGUF_TYPE;
  if (elem_kind) std::memcpy(elem_kind, m->data.data(), 4);
  if (count) std::memcpy(count, m->data.data() + 4, 8);
  return UGB_GGUF_OK;
}

int32_t ugb_gguf_meta_array_unsigned(const ugb_gguf *g, const char *key, uint64_t index, uint64_t *value) {
  const MetaItem *m = g && key ? g->find(key) : nullptr;
  if (!m) return UGB_GGUF_MISSING;
  uint32_t kind;
  const uint8_t *p;
  size_t n;
  int32_t e = array_element(m, index, &kind, &p, &n);
  if (e) return e;
  uint64_t v;
  e = value_unsigned(kind, p, n, &v);
  if (!e && value) *value = v;
  return e;
}

int32_t ugb_gguf_meta_array_string(const ugb_gguf *g, const char *key, uint64_t index, char *buf, size_t cap,
                                   size_t *len) {
  const MetaItem *m = g && key ? g->find(key) : nullptr;
  if (!m) return UGB_GGUF_MISSING;
  uint32_t kind;
  const uint8_t *p;
  size_t n;
  const int32_t e = array_element(m, index, &kind, &p, &n);
  if (e) return e;
  if (kind != 8) return UGB_GGUF_TYPE;
  return copy_string(p, buf, cap, len);
}

int32_t ugb_gguf_check_index(ugb_gguf *const *shards, int32_t count) {
  if (!shards || count < 1) return UGB_GGUF_SPLIT;
  std::vector<const ugb_gguf *> s(shards, shards + count);
  for (const ugb_gguf *g : s)
    if (!g) return UGB_GGUF_SPLIT;
  std::sort(s.begin(), s.end(), [](const ugb_gguf *a, const ugb_gguf *b) { return a->split_no < b->split_no; });
  const uint64_t total = s[0]->total_tensors;
  std::set<std::string> names;
  for (size_t i = 0; i < s.size(); ++i) {
    if (s[i]->split_no != i || s[i]->split_count != s.size() || s[i]->total_tensors != total) return UGB_GGUF_SPLIT;
    for (const TensorItem &t : s[i]->tensors)
      if (!names.insert(t.name).second) return UGB_GGUF_DUPLICATE;
  }
  if (names.size() != total) return UGB_GGUF_SPLIT;
  return UGB_GGUF_OK;
}

int32_t ugb_gguf_inventory(ugb_gguf *const *shards, int32_t count, uint64_t *counts) {
  if (!shards || count < 1 || !counts) return UGB_GGUF_SPLIT;
  uint64_t c[3] = {0, 0, 0};
  for (int32_t i = 0; i < count; ++i) {
    if (!shards[i]) return UGB_GGUF_SPLIT;
    for (const TensorItem &t : shards[i]->tensors) {
      const size_t n = t.name.size();
      const int cat = t.name == "per_layer_token_embd.weight"
                          ? 1
                          : (n >= 12 && t.name.compare(n - 12, 12, "_exps.weight") == 0 ? 2 : 0);
      if (!add_ok(c[cat], t.bytes, &c[cat])) return UGB_GGUF_OVERFLOW;
    }
  }
  for (int k = 0; k < 3; ++k) counts[k] = c[k];
  return UGB_GGUF_OK;
}

}  // extern "C"

namespace {

struct Located {
  const ugb_gguf *g = nullptr;
  int shard = -1;
  TensorItem t{};
};

// The tensor `name` in any shard.
bool locate(ugb_gguf *const *shards, int32_t count, const std::string &name, Located &out) {
  for (int32_t i = 0; i < count; ++i) {
    auto it = shards[i]->by_name.find(name);
    if (it != shards[i]->by_name.end()) {
      out.g = shards[i];
      out.shard = i;
      out.t = shards[i]->tensors[it->second];
      return true;
    }
  }
  return false;
}

// First shard holding `key`.
const MetaItem *find_meta(ugb_gguf *const *shards, int32_t count, const std::string &key) {
  for (int32_t i = 0; i < count; ++i)
    if (const MetaItem *m = shards[i]->find(key.c_str())) return m;
  return nullptr;
}

int32_t meta_u32(ugb_gguf *const *shards, int32_t count, const std::string &key, int32_t *out, bool required) {
  const MetaItem *m = find_meta(shards, count, key);
  if (!m) return required ? UGB_GGUF_MISSING : UGB_GGUF_OK;
  uint64_t v;
  int32_t e;
  if (m->kind == 5 && m->data.size() == 4) {  // i32
    int32_t x;
    std::memcpy(&x, m->data.data(), 4);
    if (x < 0) return UGB_GGUF_SHAPE;
    v = static_cast<uint64_t>(x);
  } else if ((e = value_unsigned(m->kind, m->data.data(), m->data.size(), &v))) {
    return e;
  }
  if (v > 0x7fffffff) return UGB_GGUF_SHAPE;
  *out = static_cast<int32_t>(v);
  return UGB_GGUF_OK;
}

int32_t meta_f32(ugb_gguf *const *shards, int32_t count, const std::string &key, float *out, bool required) {
  const MetaItem *m = find_meta(shards, count, key);
  if (!m) return required ? UGB_GGUF_MISSING : UGB_GGUF_OK;
  if (m->kind != 6 || m->data.size() != 4) return UGB_GGUF_TYPE;
  std::memcpy(out, m->data.data(), 4);
  return UGB_GGUF_OK;
}

}  // namespace

extern "C" {

int32_t ugb_gguf_decoder_config(ugb_gguf *const *shards, int32_t count, ugb_decoder_config *cfg) {
  if (!cfg) return UGB_GGUF_MISSING;
  int32_t e = ugb_gguf_check_index(shards, count);
  if (e) return e;
  const MetaItem *arch_m = find_meta(shards, count, "general.architecture");
  if (!arch_m) return UGB_GGUF_MISSING;
  if (arch_m->kind != 8) return UGB_GGUF_TYPE;
  uint64_t n;
  std::memcpy(&n, arch_m->data.data(), 8);
  const std::string arch(reinterpret_cast<const char *>(arch_m->data.data() + 8), static_cast<size_t>(n));
  ugb_decoder_config c{};
  const std::string a = arch + ".";
  if ((e = meta_u32(shards, count, a + "block_count", &c.n_layer, true)) ||
      (e = meta_u32(shards, count, a + "embedding_length", &c.n_embd, true)) ||
      (e = meta_u32(shards, count, a + "attention.head_count", &c.n_head, true)))
    return e;
  c.n_head_kv = c.n_head;
  int32_t key_length = 0, ctx_len = 4096;
  if ((e = meta_u32(shards, count, a + "attention.head_count_kv", &c.n_head_kv, false)) ||
      (e = meta_u32(shards, count, a + "attention.key_length", &key_length, false)) ||
      (e = meta_u32(shards, count, a + "context_length", &ctx_len, false)) ||
      (e = meta_u32(shards, count, a + "feed_forward_length", &c.n_ff, false)) ||
      (e = meta_u32(shards, count, a + "expert_count", &c.n_expert, false)) ||
      (e = meta_u32(shards, count, a + "expert_used_count", &c.top_k, false)) ||
      (e = meta_u32(shards, count, a + "expert_feed_forward_length", &c.n_ff_expert, false)))
    return e;
  c.head_dim = key_length ? key_length : (c.n_head ? c.n_embd / c.n_head : 0);
  c.n_ctx = std::min(ctx_len, 32768);
  c.rope_theta = 10000.f;
  c.norm_eps = 1e-6f;
  if ((e = meta_f32(shards, count, a + "rope.freq_base", &c.rope_theta, false)) ||
      (e = meta_f32(shards, count, a + "attention.layer_norm_rms_epsilon", &c.norm_eps, false)))
    return e;
  Located emb, q, head, ex;
  if (!locate(shards, count, "token_embd.weight", emb) || !locate(shards, count, "blk.0.attn_q.weight", q))
    return UGB_GGUF_MISSING;
  if (emb.t.rank != 2 || emb.t.dims[0] != static_cast<uint64_t>(c.n_embd)) return UGB_GGUF_SHAPE;
  c.n_vocab = static_cast<int32_t>(std::min<uint64_t>(emb.t.dims[1], 0x7fffffff));
  c.kind = q.t.kind;
  c.head_kind = locate(shards, count, "output.weight", head) ? head.t.kind : emb.t.kind;
  if (c.n_expert > 0) {
    if (!locate(shards, count, "blk.0.ffn_gate_exps.weight", ex)) return UGB_GGUF_MISSING;
    c.expert_kind = ex.t.kind;
    c.n_ff = 0;
  }
  c.batch = 1;
  c.kv_type = UGB_F32;
  *cfg = c;
  return UGB_GGUF_OK;
}

int32_t ugb_gguf_model_weights(ugb_gguf *const *shards, int32_t count, const void *const *dev_bases,
                               const uint64_t *base_offsets, const uint64_t *dev_sizes,
                               const ugb_decoder_config *cfg, ugb_model_weights *weights,
                               ugb_layer_weights *layers) {
  if (!dev_bases || !base_offsets || !dev_sizes || !cfg || !weights || !layers) return UGB_GGUF_MISSING;
  int32_t e = ugb_gguf_check_index(shards, count);
  if (e) return e;
  const ugb_decoder_config &c = *cfg;
  const int64_t E = c.n_embd, Q = static_cast<int64_t>(c.n_head) * c.head_dim,
                KV = static_cast<int64_t>(c.n_head_kv) * c.head_dim;
  // Device address of rows [row0, ...) of `name`; checks rank / row length / rows / kind.
  auto bind = [&](const std::string &name, uint32_t kind, int64_t k, int64_t rows, int64_t rows_total,
                  int64_t row0, const void **out) -> int32_t {
    Located L;
    if (!locate(shards, count, name, L)) return UGB_GGUF_MISSING;
    const TensorItem &t = L.t;
    if (t.kind != kind) return UGB_GGUF_TYPE;
    uint64_t all = 1;
    for (uint32_t d = 1; d < t.rank; ++d) all *= t.dims[d];
    if (t.dims[0] != static_cast<uint64_t>(k) || all != static_cast<uint64_t>(rows_total) || row0 < 0 ||
        row0 + rows > rows_total)
      return UGB_GGUF_SHAPE;
    const uint64_t off = t.offset + static_cast<uint64_t>(row0) * t.row_bytes;
    const uint64_t len = static_cast<uint64_t>(rows) * t.row_bytes;
    const uint64_t base = base_offsets[L.shard];
    if (off < base || off - base > dev_sizes[L.shard] || len > dev_sizes[L.shard] - (off - base))
      return UGB_GGUF_TENSOR_BOUNDS;
    *out = static_cast<const uint8_t *>(dev_bases[L.shard]) + (off - base);
    return UGB_GGUF_OK;
  };
  auto optional = [&](const std::string &name, uint32_t kind, int64_t k, const void **out) -> int32_t {
    Located L;
    *out = nullptr;
    if (!locate(shards, count, name, L)) return UGB_GGUF_OK;
    return bind(name, kind, k, 1, 1, 0, out);
  };
  ugb_model_weights w{};
  const int vocab_local = c.n_vocab_local ? c.n_vocab_local : c.n_vocab;
  if ((e = bind("token_embd.weight", UGB_Q8_0, E, c.n_vocab, c.n_vocab, 0, &w.tok_embd)) ||
      (e = bind("output_norm.weight", UGB_F32, E, 1, 1, 0, &w.output_norm)))
    return e;
  Located head;
  if (locate(shards, count, "output.weight", head))
    e = bind("output.weight", c.head_kind, E, vocab_local, c.n_vocab, c.vocab0, &w.output);
  else
    e = bind("token_embd.weight", c.head_kind, E, vocab_local, c.n_vocab, c.vocab0, &w.output);
  if (e) return e;
  const int n_local = c.n_expert ? (c.n_expert_local ? c.n_expert_local : c.n_expert) : 0;
  for (int l = 0; l < c.n_layer; ++l) {
    ugb_layer_weights L{};
    const std::string b = "blk." + std::to_string(l) + ".";
    if ((e = bind(b + "attn_norm.weight", UGB_F32, E, 1, 1, 0, &L.attn_norm)) ||
        (e = bind(b + "ffn_norm.weight", UGB_F32, E, 1, 1, 0, &L.ffn_norm)) ||
        (e = bind(b + "attn_q.weight", c.kind, E, Q, Q, 0, &L.wq)) ||
        (e = bind(b + "attn_k.weight", c.kind, E, KV, KV, 0, &L.wk)) ||
        (e = bind(b + "attn_v.weight", c.kind, E, KV, KV, 0, &L.wv)) ||
        (e = bind(b + "attn_output.weight", c.kind, Q, E, E, 0, &L.wo)) ||
        (e = optional(b + "attn_q.bias", UGB_F32, Q, &L.bq)) || (e = optional(b + "attn_k.bias", UGB_F32, KV, &L.bk)) ||
        (e = optional(b + "attn_v.bias", UGB_F32, KV, &L.bv)))
      return e;
    if (c.n_expert) {
      const int64_t ffe = c.n_ff_expert, ne = c.n_expert;
      if ((e = bind(b + "ffn_gate_inp.weight", c.kind, E, ne, ne, 0, &L.router)) ||
          (e = bind(b + "ffn_gate_exps.weight", c.expert_kind, E, ffe * n_local, ffe * ne, ffe * c.expert0, &L.gate_exps)) ||
          (e = bind(b + "ffn_up_exps.weight", c.expert_kind, E, ffe * n_local, ffe * ne, ffe * c.expert0, &L.up_exps)) ||
          (e = bind(b + "ffn_down_exps.weight", c.expert_kind, ffe, E * n_local, E * ne, E * c.expert0, &L.down_exps)))
        return e;
    } else {
      if ((e = bind(b + "ffn_gate.weight", c.kind, E, c.n_ff, c.n_ff, 0, &L.w_gate)) ||
          (e = bind(b + "ffn_up.weight", c.kind, E, c.n_ff, c.n_ff, 0, &L.w_up)) ||
          (e = bind(b + "ffn_down.weight", c.kind, c.n_ff, E, E, 0, &L.w_down)))
        return e;
    }
    layers[l] = L;
  }
  w.layers = layers;
  *weights = w;
  return UGB_GGUF_OK;
}

}  // extern "C"
