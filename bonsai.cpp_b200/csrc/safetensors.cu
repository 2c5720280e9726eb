// Reader for .safetensors files, the container of the reference's packed
// checkpoints (read by src/safetensors.h; written by
// convert_to_b1_0_packed.py): an 8-byte little-endian header length, a JSON
// header {"name": {"dtype": "...", "shape": [...], "data_offsets": [b, e]},
// "__metadata__": {...}}, then the tensor bytes, offsets relative to the end
// of the header.  Only the index is parsed here; tensors are read on demand
// with st_read, so a 1.6 GB checkpoint never has to sit in host memory whole.
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
