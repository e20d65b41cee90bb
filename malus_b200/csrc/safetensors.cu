// SafeTensors files for named sets of tensors: the exchange format malus's
// interop spec names for weights (docs/spec/08-interop.md, "SafeTensors [v1]":
// `load(path)` gives a name -> tensor mapping placed on the GPU, `save(tensors,
// path)` writes a set of named tensors).
//
// Format (the published SafeTensors layout): an 8-byte little-endian header
// length N, N bytes of UTF-8 JSON, then the data region.  The JSON object
// maps each name to {"dtype": "F32" | "I32" | "I64", "shape": [...],
// "data_offsets": [begin, end]} (byte offsets into the data region, row-major
// little-endian values) and may hold a "__metadata__" object of strings.
// Writers here lay the tensors out in the order given, back to back from
// offset 0, and pad the header with spaces to a multiple of 8 bytes.
//
// The host-only entry points (…_host) need no GPU; the others move tensors
// between files and device memory (a view or deferred result is materialised
// first, as for any raw read).
#include "common.cuh"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace malus {
namespace {

const char* st_dtype_name(int32_t dt) {
  switch (dt) {
    case MALUS_F32: return "F32";
    case MALUS_I32: return "I32";
    case MALUS_I64: return "I64";
    default: return nullptr;
  }
}
int32_t st_dtype_code(const std::string& s) {
  if (s == "F32") return MALUS_F32;
  if (s == "I32") return MALUS_I32;
  if (s == "I64") return MALUS_I64;
  return -1;
}

void json_string(std::string& out, const char* s) {
  out += '"';
  for (const unsigned char* p = (const unsigned char*)s; *p; ++p) {
    if (*p == '"' || *p == '\\') {
      out += '\\';
      out += (char)*p;
    } else if (*p < 0x20) {
      char b[8];
      snprintf(b, sizeof b, "\\u%04x", *p);
      out += b;
    } else {
      out += (char)*p;
    }
  }
  out += '"';
}

// ---- a small JSON reader for the header: objects, arrays, strings, integers ----
struct JVal {
  enum Kind { kNull, kNum, kStr, kArr, kObj } kind = kNull;
  int64_t num = 0;
  bool num_ok = true;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
};

struct JParser {
  const char* p;
  const char* end;
  int depth = 0;
  void ws() { while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p; }
  bool lit(const char* s) {
    const size_t n = strlen(s);
    if ((size_t)(end - p) >= n && memcmp(p, s, n) == 0) { p += n; return true; }
    return false;
  }
  bool str(std::string& out) {
    if (p >= end || *p != '"') return false;
    ++p;
    while (p < end && *p != '"') {
      if (*p == '\\') {
        if (++p >= end) return false;
        const char c = *p++;
        if (c == 'u') {
          if (end - p < 4) return false;
          unsigned v = 0;
          for (int i = 0; i < 4; ++i) {
            const char h = *p++;
            int d = -1;
            if (h >= '0' && h <= '9') d = h - '0';
            else if (h >= 'a' && h <= 'f') d = h - 'a' + 10;
            else if (h >= 'A' && h <= 'F') d = h - 'A' + 10;
            if (d < 0) return false;
            v = v * 16 + (unsigned)d;
          }
          if (v < 0x80) out += (char)v;                       // names here are ASCII or raw UTF-8
          else if (v < 0x800) { out += (char)(0xC0 | (v >> 6)); out += (char)(0x80 | (v & 0x3F)); }
          else { out += (char)(0xE0 | (v >> 12)); out += (char)(0x80 | ((v >> 6) & 0x3F)); out += (char)(0x80 | (v & 0x3F)); }
        } else {
          const char* m = strchr("\"\\/bfnrt", c);
          if (!c || !m) return false;
          static const char rep[] = "\"\\/\b\f\n\r\t";
          out += rep[m - "\"\\/bfnrt"];
        }
      } else {
        out += *p++;
      }
    }
    if (p >= end) return false;
    ++p;
    return true;
  }
  bool value(JVal& v) {
    if (++depth > 16) return false;   // the header nests three levels deep
    ws();
    if (p >= end) return false;
    bool r = true;
    if (*p == '{') {
      v.kind = JVal::kObj;
      ++p;
      ws();
      if (p < end && *p == '}') { ++p; --depth; return true; }
      while (r) {
        ws();
        std::string k;
        JVal x;
        r = str(k);
        ws();
        r = r && p < end && *p == ':';
        if (r) ++p;
        r = r && value(x);
        if (r) v.obj.emplace_back(std::move(k), std::move(x));
        ws();
        if (!r || p >= end) return false;
        if (*p == ',') { ++p; continue; }
        if (*p == '}') { ++p; break; }
        return false;
      }
    } else if (*p == '[') {
      v.kind = JVal::kArr;
      ++p;
      ws();
      if (p < end && *p == ']') { ++p; --depth; return true; }
      while (r) {
        JVal x;
        r = value(x);
        if (r) v.arr.push_back(std::move(x));
        ws();
        if (!r || p >= end) return false;
        if (*p == ',') { ++p; continue; }
        if (*p == ']') { ++p; break; }
        return false;
      }
    } else if (*p == '"') {
      v.kind = JVal::kStr;
      r = str(v.str);
    } else if (*p == '-' || (*p >= '0' && *p <= '9')) {
      v.kind = JVal::kNum;
      bool neg = *p == '-';
      if (neg) ++p;
      if (p >= end || *p < '0' || *p > '9') return false;
      uint64_t n = 0;
      while (p < end && *p >= '0' && *p <= '9') {
        const uint64_t d = (uint64_t)(*p++ - '0');
        if (n > (UINT64_MAX - d) / 10) v.num_ok = false;
        n = n * 10 + d;
      }
      if (p < end && (*p == '.' || *p == 'e' || *p == 'E')) v.num_ok = false;   // sizes are integers
      while (p < end && (*p == '.' || *p == 'e' || *p == 'E' || *p == '+' || *p == '-' || (*p >= '0' && *p <= '9'))) ++p;
      if (n > (uint64_t)INT64_MAX) v.num_ok = false;
      v.num = neg ? -(int64_t)n : (int64_t)n;
    } else if (lit("null")) {
      v.kind = JVal::kNull;
    } else if (lit("true") || lit("false")) {
      v.kind = JVal::kNull;
    } else {
      return false;
    }
    --depth;
    return r;
  }
};

struct StEntry {
  std::string name;
  int32_t dtype;
  std::vector<size_t> shape;
  uint64_t begin, end;   // offsets in the data region
};

// Parse a file's header.  Returns 0 and fills `entries` and `data_start`, or a
// negative code: -1 open/read, -2 header length, -3 JSON, -4 a field, -5
// offsets (outside the file, not matching the shape, or overlapping).
int st_parse(const char* path, std::vector<StEntry>* entries, uint64_t* data_start, uint64_t* file_size) {
  FILE* f = fopen(path, "rb");
  if (!f) return -1;
  unsigned char lenb[8];
  if (fread(lenb, 1, 8, f) != 8) { fclose(f); return -2; }
  uint64_t n = 0;
  for (int i = 7; i >= 0; --i) n = (n << 8) | lenb[i];
  if (fseek(f, 0, SEEK_END) != 0) { fclose(f); return -1; }
  const long fs = ftell(f);
  if (fs < 8 || n > (uint64_t)fs - 8 || n > ((uint64_t)1 << 30)) { fclose(f); return -2; }
  std::string hdr((size_t)n, '\0');
  if (fseek(f, 8, SEEK_SET) != 0 || (n && fread(&hdr[0], 1, (size_t)n, f) != (size_t)n)) { fclose(f); return -1; }
  fclose(f);
  JParser jp{hdr.data(), hdr.data() + hdr.size()};
  JVal root;
  if (!jp.value(root) || root.kind != JVal::kObj) return -3;
  jp.ws();
  if (jp.p != jp.end) return -3;
  const uint64_t data_len = (uint64_t)fs - 8 - n;
  std::vector<StEntry> out;
  for (auto& kv : root.obj) {
    if (kv.first == "__metadata__") continue;
    const JVal& o = kv.second;
    if (o.kind != JVal::kObj) return -4;
    const JVal *dt = nullptr, *sh = nullptr, *off = nullptr;
    for (auto& f2 : o.obj) {
      if (f2.first == "dtype") dt = &f2.second;
      else if (f2.first == "shape") sh = &f2.second;
      else if (f2.first == "data_offsets") off = &f2.second;
    }
    if (!dt || dt->kind != JVal::kStr || !sh || sh->kind != JVal::kArr || !off || off->kind != JVal::kArr ||
        off->arr.size() != 2 || sh->arr.size() > (size_t)kMaxRank)
      return -4;
    StEntry e;
    e.name = kv.first;
    e.dtype = st_dtype_code(dt->str);
    if (e.dtype < 0) return -4;
    uint64_t count = 1;
    for (auto& d : sh->arr) {
      if (d.kind != JVal::kNum || !d.num_ok || d.num < 0) return -4;
      e.shape.push_back((size_t)d.num);
      if (d.num && count > UINT64_MAX / (uint64_t)d.num) return -5;
      count *= (uint64_t)d.num;
    }
    for (auto& d : off->arr)
      if (d.kind != JVal::kNum || !d.num_ok || d.num < 0) return -4;
    e.begin = (uint64_t)off->arr[0].num;
    e.end = (uint64_t)off->arr[1].num;
    if (e.end < e.begin || e.end > data_len || count > UINT64_MAX / dtype_size(e.dtype) ||
        e.end - e.begin != count * dtype_size(e.dtype))
      return -5;
    out.push_back(std::move(e));
  }
  // no two tensors may share bytes
  std::vector<std::pair<uint64_t, uint64_t>> iv;
  for (auto& e : out) if (e.end > e.begin) iv.emplace_back(e.begin, e.end);
  std::sort(iv.begin(), iv.end());
  for (size_t i = 1; i < iv.size(); ++i)
    if (iv[i].first < iv[i - 1].second) return -5;
  *entries = std::move(out);
  *data_start = 8 + n;
  *file_size = (uint64_t)fs;
  return 0;
}

// Write the header and the tensors' bytes; `data[i]` holds tensor i's
// row-major values on the host.
int st_write(const char* path, size_t n, const char* const* names, const int32_t* dtypes,
             const std::vector<std::vector<size_t>>& shapes, const void* const* data) {
  std::map<std::string, int> seen;
  std::string hdr = "{";
  uint64_t off = 0;
  std::vector<uint64_t> bytes(n);
  for (size_t i = 0; i < n; ++i) {
    if (!names[i] || !*names[i] || strcmp(names[i], "__metadata__") == 0 || seen.count(names[i])) return -4;
    seen[names[i]] = 1;
    const char* dn = st_dtype_name(dtypes[i]);
    if (!dn) return -4;
    uint64_t count = 1;
    for (size_t d : shapes[i]) count *= d;
    bytes[i] = count * dtype_size(dtypes[i]);
    if (i) hdr += ',';
    json_string(hdr, names[i]);
    hdr += ":{\"dtype\":\"";
    hdr += dn;
    hdr += "\",\"shape\":[";
    for (size_t d = 0; d < shapes[i].size(); ++d) {
      if (d) hdr += ',';
      hdr += std::to_string(shapes[i][d]);
    }
    hdr += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + bytes[i]) + "]}";
    off += bytes[i];
  }
  hdr += ",\"__metadata__\":{\"format\":\"pt\",\"writer\":\"malus_b200\"}}";
  if (n == 0) hdr = "{\"__metadata__\":{\"format\":\"pt\",\"writer\":\"malus_b200\"}}";
  while (hdr.size() % 8) hdr += ' ';
  FILE* f = fopen(path, "wb");
  if (!f) return -1;
  unsigned char lenb[8];
  uint64_t hl = hdr.size();
  for (int i = 0; i < 8; ++i) lenb[i] = (unsigned char)(hl >> (8 * i));
  bool ok = fwrite(lenb, 1, 8, f) == 8 && fwrite(hdr.data(), 1, hdr.size(), f) == hdr.size();
  for (size_t i = 0; i < n && ok; ++i)
    if (bytes[i]) ok = fwrite(data[i], 1, (size_t)bytes[i], f) == (size_t)bytes[i];
  ok = (fclose(f) == 0) && ok;
  return ok ? 0 : -1;
}

int st_read_bytes(const char* path, uint64_t at, void* dst, uint64_t bytes) {
  if (!bytes) return 0;
  FILE* f = fopen(path, "rb");
  if (!f) return -1;
  const bool ok = fseek(f, (long)at, SEEK_SET) == 0 && fread(dst, 1, (size_t)bytes, f) == (size_t)bytes;
  fclose(f);
  return ok ? 0 : -1;
}

}  // namespace
}  // namespace malus

extern "C" {

// Write n named tensors held in host memory.  dtypes: 0 f32, 5 i32, 6 i64;
// shapes[i] has ndims[i] dims.  Returns 0, or -1 (I/O), -4 (an empty,
// duplicate or reserved name, an unsupported dtype, or a rank above 8).
int32_t malus_safetensors_write_host(const char* path, size_t n, const char* const* names, const int32_t* dtypes,
                                     const size_t* const* shapes, const size_t* ndims, const void* const* data) {
  using namespace malus;
  std::vector<std::vector<size_t>> sh(n);
  for (size_t i = 0; i < n; ++i) {
    if (ndims[i] > (size_t)kMaxRank) return -4;
    sh[i].assign(shapes[i], shapes[i] + ndims[i]);
  }
  return st_write(path, n, names, dtypes, sh, data);
}

// The file's tensor names, newline-separated in header order, into buf
// (NUL-terminated, truncated at cap); returns the length the whole list needs,
// or a negative code of the header check (-1 I/O, -2 length, -3 JSON, -4 a
// field, -5 offsets).
int32_t malus_safetensors_names(const char* path, char* buf, int32_t cap) {
  using namespace malus;
  std::vector<StEntry> es;
  uint64_t ds = 0, fs = 0;
  const int r = st_parse(path, &es, &ds, &fs);
  if (r < 0) return r;
  std::string text;
  for (auto& e : es) text += e.name + "\n";
  if (buf && cap > 0) {
    const size_t k = std::min(text.size(), (size_t)cap - 1);
    memcpy(buf, text.data(), k);
    buf[k] = 0;
  }
  return (int32_t)text.size();
}

// One tensor of a file into host memory: its dtype, rank and shape (up to 8
// dims) always; its bytes when `cap` holds them.  Returns the byte count, -6
// when the name is absent, or a negative code of the header check.
int64_t malus_safetensors_read_host(const char* path, const char* name, int32_t* dtype, size_t* shape,
                                    size_t* ndim, void* data, size_t cap) {
  using namespace malus;
  std::vector<StEntry> es;
  uint64_t ds = 0, fs = 0;
  const int r = st_parse(path, &es, &ds, &fs);
  if (r < 0) return r;
  for (auto& e : es) {
    if (e.name != name) continue;
    if (dtype) *dtype = e.dtype;
    if (ndim) *ndim = e.shape.size();
    if (shape) for (size_t i = 0; i < e.shape.size(); ++i) shape[i] = e.shape[i];
    const uint64_t bytes = e.end - e.begin;
    if (data && cap >= bytes && st_read_bytes(path, ds + e.begin, data, bytes) != 0) return -1;
    return (int64_t)bytes;
  }
  return -6;
}

// Save tensors (handles) under the given names: each is copied to the host
// (views and deferred results materialised) and written in order.  Returns 0
// or a negative code as malus_safetensors_write_host.
int32_t malus_save_safetensors(const char* path, size_t n, const char* const* names, const int64_t* handles) {
  using namespace malus;
  std::vector<std::vector<unsigned char>> host(n);
  std::vector<const void*> ptrs(n);
  std::vector<int32_t> dts(n);
  std::vector<std::vector<size_t>> sh(n);
  for (size_t i = 0; i < n; ++i) {
    TensorBuffer* t = tb(handles[i]);
    dts[i] = t->dtype;
    sh[i].assign(t->shape, t->shape + t->ndim);
    host[i].resize(t->len * dtype_size(t->dtype));
    if (!host[i].empty())
      MALUS_CUDA(cudaMemcpyAsync(host[i].data(), vptr(handles[i]), host[i].size(), cudaMemcpyDeviceToHost, stream()));
    ptrs[i] = host[i].data();
  }
  gpu_barrier();
  return st_write(path, n, names, dts.data(), sh, ptrs.data());
}

// Load one tensor of a file onto the GPU as a new handle (refcount 1), or 0
// when the name is absent or the file is not a valid SafeTensors file (the
// reason goes to stderr).
int64_t malus_load_safetensors(const char* path, const char* name) {
  using namespace malus;
  std::vector<StEntry> es;
  uint64_t ds = 0, fs = 0;
  const int r = st_parse(path, &es, &ds, &fs);
  if (r < 0) {
    fprintf(stderr, "malus: %s is not a readable SafeTensors file (code %d)\n", path, r);
    return 0;
  }
  for (auto& e : es) {
    if (e.name != name) continue;
    std::vector<unsigned char> host((size_t)(e.end - e.begin));
    if (st_read_bytes(path, ds + e.begin, host.data(), host.size()) != 0) {
      fprintf(stderr, "malus: reading %s from %s failed\n", name, path);
      return 0;
    }
    const int64_t h = alloc(e.dtype, e.shape.data(), (int)e.shape.size());
    if (!host.empty()) MALUS_CUDA(cudaMemcpyAsync(vptr(h), host.data(), host.size(), cudaMemcpyHostToDevice, stream()));
    gpu_barrier();   // the host staging buffer is released on return
    return h;
  }
  fprintf(stderr, "malus: %s holds no tensor named %s\n", path, name);
  return 0;
}

}  // extern "C"
