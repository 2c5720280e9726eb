// Reader for .safetensors files, the container of the reference's packed
// checkpoints (read by src/safetensors.h; written by
// convert_to_b1_0_packed.py): an 8-byte little-endian header length, a JSON
// header {"name": {"dtype": "...", "shape": [...], "data_offsets": [b, e]},
// "__metadata__": {...}}, then the tensor bytes, offsets relative to the end
// of the header.  Only the index is parsed here; tensors are read on demand
// with st_read, so a 1.6 GB checkpoint never has to sit in host memory whole.
// GGUF files (recognised by their magic) are indexed into the same view.
#include "../../include/bonsai_cuda.h"
#include "internal.cuh"

#include <cctype>
#include <cstring>

namespace bonsai {
namespace {

// Minimal JSON cursor for the safetensors header (objects, arrays, strings,
// integers; anything else is skipped by skip_value).
struct Json {
  const std::string& s;
  size_t p = 0;
  std::string err;
  explicit Json(const std::string& str) : s(str) {}

  void ws() {
    while (p < s.size() && std::isspace((unsigned char)s[p])) ++p;
  }
  bool eat(char c) {
    ws();
    if (p < s.size() && s[p] == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool expect(char c) {
    if (eat(c)) return true;
    err = std::string("expected '") + c + "' at offset " + std::to_string(p);
    return false;
  }
  bool str(std::string& out) {
    ws();
    if (p >= s.size() || s[p] != '"') {
      err = "expected a string at offset " + std::to_string(p);
      return false;
    }
    ++p;
    out.clear();
    while (p < s.size() && s[p] != '"') {
      if (s[p] == '\\') {
        if (p + 1 >= s.size()) break;
        const char e = s[p + 1];
        if (e == 'u') {  // keep \uXXXX escapes verbatim (names are ASCII in practice)
          out += s.substr(p, 6);
          p += 6;
          continue;
        }
        out += (e == 'n') ? '\n' : (e == 't') ? '\t' : e;
        p += 2;
        continue;
      }
      out += s[p++];
    }
    if (p >= s.size()) {
      err = "unterminated string";
      return false;
    }
    ++p;
    return true;
  }
  bool integer(long long& v) {
    ws();
    size_t q = p;
    if (q < s.size() && (s[q] == '-' || s[q] == '+')) ++q;
    if (q >= s.size() || !std::isdigit((unsigned char)s[q])) {
      err = "expected an integer at offset " + std::to_string(p);
      return false;
    }
    v = std::strtoll(s.c_str() + p, nullptr, 10);
    p = q;
    while (p < s.size() && std::isdigit((unsigned char)s[p])) ++p;
    return true;
  }
  bool int_array(std::vector<long long>& v) {
    v.clear();
    if (!expect('[')) return false;
    if (eat(']')) return true;
    do {
      long long x;
      if (!integer(x)) return false;
      v.push_back(x);
    } while (eat(','));
    return expect(']');
  }
  bool skip_value() {
    ws();
    if (p >= s.size()) {
      err = "unexpected end of header";
      return false;
    }
    const char c = s[p];
    if (c == '"') {
      std::string t;
      return str(t);
    }
    if (c == '{' || c == '[') {
      const char close = c == '{' ? '}' : ']';
      ++p;
      if (eat(close)) return true;
      do {
        if (c == '{') {
          std::string k;
          if (!str(k) || !expect(':')) return false;
        }
        if (!skip_value()) return false;
      } while (eat(','));
      return expect(close);
    }
    while (p < s.size() && s[p] != ',' && s[p] != '}' && s[p] != ']') ++p;  // number / literal
    return true;
  }
};

}  // namespace

StFile::~StFile() {
  if (f) fclose(f);
}

namespace {

// ---------------------------------------------------------------- GGUF
// The GGUF container (the published format the reference's
// convert_to_b1_0.py writes through the gguf package, B1_0 as tensor type
// 100 with 6-byte blocks of 32 weights): "GGUF", u32 version (2 or 3), u64
// tensor count, u64 key/value count, typed key/values, tensor infos (name,
// u32 n_dims, u64 dims innermost first, u32 type, u64 offset), then the data
// at the next multiple of general.alignment (default 32).  Tensors are
// exposed under the reference's safetensors names (the converter's renaming
// undone) in the safetensors view: B1_0 as U8 [out][in/32*6], F32 / F16 with
// row-major shapes.
enum GgufKv : uint32_t {
  KV_U8 = 0, KV_I8 = 1, KV_U16 = 2, KV_I16 = 3, KV_U32 = 4, KV_I32 = 5, KV_F32 = 6,
  KV_BOOL = 7, KV_STRING = 8, KV_ARRAY = 9, KV_U64 = 10, KV_I64 = 11, KV_F64 = 12,
};
constexpr uint32_t kGgmlF32 = 0, kGgmlF16 = 1, kGgmlB1_0 = 100;

bool rd(FILE* f, void* p, size_t n) { return fread(p, 1, n, f) == n; }

bool rd_str(FILE* f, std::string& s, long long limit) {
  uint64_t n = 0;
  if (!rd(f, &n, 8) || n > (uint64_t)limit || n > (1u << 20)) return false;
  s.assign((size_t)n, '\0');
  return n == 0 || rd(f, &s[0], (size_t)n);
}

long long kv_size(uint32_t t) {
  switch (t) {
    case KV_U8: case KV_I8: case KV_BOOL: return 1;
    case KV_U16: case KV_I16: return 2;
    case KV_U32: case KV_I32: case KV_F32: return 4;
    case KV_U64: case KV_I64: case KV_F64: return 8;
    default: return -1;
  }
}

bool skip_kv(FILE* f, uint32_t t, long long limit, int depth = 0) {
  if (t == KV_STRING) {
    std::string s;
    return rd_str(f, s, limit);
  }
  if (t == KV_ARRAY) {
    uint32_t et = 0;
    uint64_t n = 0;
    if (depth > 4 || !rd(f, &et, 4) || !rd(f, &n, 8) || n > (uint64_t)limit) return false;
    const long long es = kv_size(et);
    if (es > 0) return fseeko(f, (off_t)(n * (uint64_t)es), SEEK_CUR) == 0;
    for (uint64_t i = 0; i < n; ++i)
      if (!skip_kv(f, et, limit, depth + 1)) return false;
    return true;
  }
  const long long sz = kv_size(t);
  return sz > 0 && fseeko(f, sz, SEEK_CUR) == 0;
}

// Undo convert_to_b1_0.py's map_tensor_name.
std::string reference_name(std::string n) {
  if (n.compare(0, 4, "blk.") == 0) n = "single_transformer_blocks." + n.substr(4);
  if (n.compare(0, 14, "double_stream_") == 0 && n.compare(0, 25, "double_stream_modulation_") != 0)
    n = "double_stream_modulation_" + n.substr(14);
  return n;
}

int gguf_parse(StFile& out) {
  FILE* f = out.f;
  const long long limit = out.file_size;
  uint32_t version = 0;
  uint64_t n_tensors = 0, n_kv = 0;
  fseeko(f, 4, SEEK_SET);
  if (!rd(f, &version, 4) || !rd(f, &n_tensors, 8) || !rd(f, &n_kv, 8))
    return fail(BONSAI_ERR_ARG, "gguf: truncated header");
  if (version < 2 || version > 3)
    return fail(BONSAI_ERR_UNSUPPORTED, "gguf: version " + std::to_string(version) + " (2 or 3 supported)");
  if (n_tensors > (uint64_t)limit || n_kv > (uint64_t)limit) return fail(BONSAI_ERR_ARG, "gguf: invalid counts");
  uint64_t alignment = 32;
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key;
    uint32_t t = 0;
    if (!rd_str(f, key, limit) || !rd(f, &t, 4)) return fail(BONSAI_ERR_ARG, "gguf: truncated key/value");
    if (key == "general.alignment" && t == KV_U32) {
      uint32_t a = 0;
      if (!rd(f, &a, 4)) return fail(BONSAI_ERR_ARG, "gguf: truncated key/value");
      if (a == 0 || (a & (a - 1))) return fail(BONSAI_ERR_ARG, "gguf: alignment must be a power of two");
      alignment = a;
    } else if (!skip_kv(f, t, limit)) {
      return fail(BONSAI_ERR_ARG, "gguf: bad value of key " + key);
    }
  }
  struct Info {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type;
    uint64_t offset;
  };
  std::vector<Info> infos((size_t)n_tensors);
  for (auto& ti : infos) {
    uint32_t nd = 0;
    if (!rd_str(f, ti.name, limit) || !rd(f, &nd, 4) || nd == 0 || nd > 4)
      return fail(BONSAI_ERR_ARG, "gguf: bad tensor info");
    ti.dims.resize(nd);
    for (auto& d : ti.dims)
      if (!rd(f, &d, 8)) return fail(BONSAI_ERR_ARG, "gguf: truncated tensor info");
    if (!rd(f, &ti.type, 4) || !rd(f, &ti.offset, 8)) return fail(BONSAI_ERR_ARG, "gguf: truncated tensor info");
  }
  const long long pos = (long long)ftello(f);
  out.data_start = (long long)(((uint64_t)pos + alignment - 1) / alignment * alignment);
  for (const auto& ti : infos) {
    uint64_t numel = 1;
    for (uint64_t d : ti.dims) {
      // overflow guard only; the byte range is checked against the file below
      if (d == 0 || numel > (1ull << 50) / d) return fail(BONSAI_ERR_ARG, "gguf: bad dims of " + ti.name);
      numel *= d;
    }
    StTensor t;
    long long bytes = 0;
    if (ti.type == kGgmlF32 || ti.type == kGgmlF16) {
      t.dtype = ti.type == kGgmlF32 ? "F32" : "F16";
      for (size_t i = ti.dims.size(); i-- > 0;) t.shape.push_back((long long)ti.dims[i]);
      bytes = (long long)numel * (ti.type == kGgmlF32 ? 4 : 2);
    } else if (ti.type == kGgmlB1_0) {
      if (ti.dims[0] % 32 != 0) return fail(BONSAI_ERR_ARG, "gguf: B1_0 tensor " + ti.name + " with ne0 % 32 != 0");
      t.dtype = "U8";
      t.shape = {(long long)(numel / ti.dims[0]), (long long)(ti.dims[0] / 32 * 6)};
      bytes = (long long)(numel / 32 * 6);
    } else {
      continue;  // a tensor type this engine never loads; not listed
    }
    t.begin = (long long)ti.offset;
    t.end = t.begin + bytes;
    if (t.begin < 0 || out.data_start + t.end > out.file_size)
      return fail(BONSAI_ERR_ARG, "gguf: tensor " + ti.name + " lies outside the file");
    out.tensors[reference_name(ti.name)] = t;
  }
  return 0;
}

}  // namespace

int st_open(const char* path, StFile& out) {
  if (!path) return fail(BONSAI_ERR_ARG, "safetensors: null path");
  out.f = fopen(path, "rb");
  if (!out.f) return fail(BONSAI_ERR_ARG, std::string("safetensors: cannot open ") + path);
  if (fseeko(out.f, 0, SEEK_END) != 0) return fail(BONSAI_ERR_ARG, "safetensors: seek failed");
  out.file_size = (long long)ftello(out.f);
  fseeko(out.f, 0, SEEK_SET);
  unsigned char lenb[8];
  if (out.file_size < 8 || fread(lenb, 1, 8, out.f) != 8)
    return fail(BONSAI_ERR_ARG, "safetensors: file shorter than its 8-byte header length");
  if (memcmp(lenb, "GGUF", 4) == 0) return gguf_parse(out);
  unsigned long long hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | lenb[i];
  if (hlen == 0 || hlen > (unsigned long long)(out.file_size - 8) || hlen > (1ull << 30))
    return fail(BONSAI_ERR_ARG, "safetensors: invalid header length");
  std::string header((size_t)hlen, '\0');
  if (fread(&header[0], 1, (size_t)hlen, out.f) != (size_t)hlen)
    return fail(BONSAI_ERR_ARG, "safetensors: truncated header");
  out.data_start = 8 + (long long)hlen;

  Json j(header);
  if (!j.expect('{')) return fail(BONSAI_ERR_ARG, "safetensors header: " + j.err);
  if (!j.eat('}')) {
    do {
      std::string name;
      if (!j.str(name) || !j.expect(':')) return fail(BONSAI_ERR_ARG, "safetensors header: " + j.err);
      if (name == "__metadata__") {
        if (!j.skip_value()) return fail(BONSAI_ERR_ARG, "safetensors header: " + j.err);
        continue;
      }
      StTensor t;
      bool have_offsets = false;
      if (!j.expect('{')) return fail(BONSAI_ERR_ARG, "safetensors header: " + j.err);
      if (!j.eat('}')) {
        do {
          std::string key;
          if (!j.str(key) || !j.expect(':')) return fail(BONSAI_ERR_ARG, "safetensors header: " + j.err);
          bool ok = true;
          if (key == "dtype") {
            ok = j.str(t.dtype);
          } else if (key == "shape") {
            ok = j.int_array(t.shape);
          } else if (key == "data_offsets") {
            std::vector<long long> o;
            ok = j.int_array(o);
            if (ok && o.size() != 2) {
              j.err = "data_offsets of " + name + " must have two entries";
              ok = false;
            }
            if (ok) {
              t.begin = o[0];
              t.end = o[1];
              have_offsets = true;
            }
          } else {
            ok = j.skip_value();
          }
          if (!ok) return fail(BONSAI_ERR_ARG, "safetensors header: " + j.err);
        } while (j.eat(','));
        if (!j.expect('}')) return fail(BONSAI_ERR_ARG, "safetensors header: " + j.err);
      }
      if (!have_offsets || t.dtype.empty())
        return fail(BONSAI_ERR_ARG, "safetensors header: tensor " + name + " lacks dtype or data_offsets");
      if (t.begin < 0 || t.end < t.begin || out.data_start + t.end > out.file_size)
        return fail(BONSAI_ERR_ARG, "safetensors: tensor " + name + " lies outside the file");
      out.tensors[name] = t;
    } while (j.eat(','));
    if (!j.expect('}')) return fail(BONSAI_ERR_ARG, "safetensors header: " + j.err);
  }
  return 0;
}

int st_read(StFile& f, const StTensor& t, void* dst, long long bytes) {
  if (!f.f) return fail(BONSAI_ERR_ARG, "safetensors: file not open");
  if (bytes != t.end - t.begin) return fail(BONSAI_ERR_ARG, "safetensors: size mismatch on read");
  if (fseeko(f.f, (off_t)(f.data_start + t.begin), SEEK_SET) != 0)
    return fail(BONSAI_ERR_ARG, "safetensors: seek failed");
  if (bytes > 0 && fread(dst, 1, (size_t)bytes, f.f) != (size_t)bytes)
    return fail(BONSAI_ERR_ARG, "safetensors: short read");
  return 0;
}

}  // namespace bonsai

extern "C" int bonsai_safetensors_list(const char* path, char* out, int cap) {
  bonsai::StFile f;
  const int rc = bonsai::st_open(path, f);
  if (rc) return rc;
  std::string txt;
  for (const auto& kv : f.tensors) {
    txt += kv.first + "\t" + kv.second.dtype + "\t";
    for (size_t i = 0; i < kv.second.shape.size(); ++i)
      txt += (i ? "," : "") + std::to_string(kv.second.shape[i]);
    txt += "\t" + std::to_string(kv.second.begin) + "\t" + std::to_string(kv.second.end) + "\n";
  }
  if (out && cap > 0) {
    const size_t n = std::min<size_t>(txt.size(), (size_t)cap - 1);
    memcpy(out, txt.data(), n);
    out[n] = 0;
  }
  return (int)std::min<size_t>(txt.size(), 0x7fffffff);
}
