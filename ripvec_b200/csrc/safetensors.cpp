// rv_load_safetensors: reads a .safetensors file (the weight format the reference loads through
// the `safetensors` crate, backend/driver/cpu.rs:521-616 and backend/cpu.rs:633-704) and feeds
// every tensor of the model through rv_set_weight.  F32, BF16 and F16 tensors are accepted and
// widened to f32 on the host.
//
// Format: 8-byte little-endian header length N, N bytes of JSON
// {"name": {"dtype": "F32", "shape": [..], "data_offsets": [begin, end]}, "__metadata__": {..}},
// then the data section the offsets index.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/ripvec_b200.h"
#include "engine.h"

namespace {

struct Entry {
  std::string name, dtype;
  uint64_t begin = 0, end = 0;
};

// Minimal JSON walker for the safetensors header (objects, strings, numbers, arrays).
struct Parser {
  const std::string& s;
  size_t i = 0;
  bool ok = true;
  explicit Parser(const std::string& str) : s(str) {}
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\t' || s[i] == '\r')) ++i;
  }
  bool eat(char c) {
    ws();
    if (i < s.size() && s[i] == c) {
      ++i;
      return true;
    }
    return false;
  }
  std::string str() {
    ws();
    std::string out;
    if (i >= s.size() || s[i] != '"') {
      ok = false;
      return out;
    }
    ++i;
    while (i < s.size() && s[i] != '"') {
      if (s[i] == '\\' && i + 1 < s.size()) {
        out.push_back(s[i + 1]);
        i += 2;
      } else {
        out.push_back(s[i++]);
      }
    }
    if (i >= s.size()) ok = false;
    ++i;
    return out;
  }
  uint64_t num() {
    ws();
    uint64_t v = 0;
    bool any = false;
    while (i < s.size() && s[i] >= '0' && s[i] <= '9') {
      v = v * 10 + uint64_t(s[i++] - '0');
      any = true;
    }
    if (!any) ok = false;
    return v;
  }
  void skip() {  // skips any JSON value
    ws();
    if (i >= s.size()) {
      ok = false;
      return;
    }
    if (s[i] == '"') {
      str();
    } else if (s[i] == '{' || s[i] == '[') {
      const char open = s[i], close = open == '{' ? '}' : ']';
      int depth = 0;
      bool in_str = false;
      for (; i < s.size(); ++i) {
        const char c = s[i];
        if (in_str) {
          if (c == '\\') ++i;
          else if (c == '"') in_str = false;
        } else if (c == '"') {
          in_str = true;
        } else if (c == open) {
          ++depth;
        } else if (c == close && --depth == 0) {
          ++i;
          return;
        }
      }
      ok = false;
    } else {
      while (i < s.size() && s[i] != ',' && s[i] != '}' && s[i] != ']') ++i;
    }
  }
};

bool parse_header(const std::string& h, std::vector<Entry>* out) {
  Parser p(h);
  if (!p.eat('{')) return false;
  if (p.eat('}')) return true;
  do {
    const std::string name = p.str();
    if (!p.ok || !p.eat(':')) return false;
    if (name == "__metadata__") {
      p.skip();
      continue;
    }
    Entry e;
    e.name = name;
    if (!p.eat('{')) return false;
    do {
      const std::string key = p.str();
      if (!p.ok || !p.eat(':')) return false;
      if (key == "dtype") {
        e.dtype = p.str();
      } else if (key == "data_offsets") {
        if (!p.eat('[')) return false;
        e.begin = p.num();
        if (!p.eat(',')) return false;
        e.end = p.num();
        if (!p.eat(']')) return false;
      } else {
        p.skip();
      }
    } while (p.ok && p.eat(','));
    if (!p.eat('}')) return false;
    out->push_back(e);
  } while (p.ok && p.eat(','));
  return p.ok && p.eat('}');
}

float half_to_f32(uint16_t h) {
  const uint32_t sign = uint32_t(h & 0x8000) << 16;
  int exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      exp = 1;
      while (!(man & 0x400)) {
        man <<= 1;
        --exp;
      }
      man &= 0x3ff;
      bits = sign | uint32_t(exp + 127 - 15) << 23 | man << 13;
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | man << 13;
  } else {
    bits = sign | uint32_t(exp + 127 - 15) << 23 | man << 13;
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

}  // namespace

extern "C" int rv_load_safetensors(rv_ctx* c, const char* path) {
  if (!c || !path) return RV_E_INVALID;
  FILE* f = std::fopen(path, "rb");
  if (!f) {
    c->err = std::string("cannot open ") + path;
    return RV_E_IO;
  }
  uint64_t hlen = 0;
  std::string header;
  std::vector<Entry> entries;
  bool ok = std::fread(&hlen, 8, 1, f) == 1 && hlen < (uint64_t(1) << 30);
  if (ok) {
    header.resize(hlen);
    ok = std::fread(&header[0], 1, hlen, f) == hlen && parse_header(header, &entries);
  }
  if (!ok) {
    std::fclose(f);
    c->err = std::string("malformed safetensors header in ") + path;
    return RV_E_IO;
  }
  const long data0 = long(8 + hlen);
  std::vector<unsigned char> raw;
  std::vector<float> vals;
  for (const Entry& e : entries) {
    const uint64_t nbytes = e.end - e.begin;
    int es = e.dtype == "F32" ? 4 : (e.dtype == "BF16" || e.dtype == "F16") ? 2 : 0;
    if (es == 0 || e.end < e.begin || nbytes % es) continue;  // not a weight this library uses
    raw.resize(nbytes);
    if (std::fseek(f, data0 + long(e.begin), SEEK_SET) != 0 || std::fread(raw.data(), 1, nbytes, f) != nbytes) {
      std::fclose(f);
      c->err = "short read of tensor " + e.name;
      return RV_E_IO;
    }
    const size_t n = nbytes / es;
    vals.resize(n);
    if (es == 4) {
      std::memcpy(vals.data(), raw.data(), nbytes);
    } else if (e.dtype == "BF16") {
      for (size_t i = 0; i < n; ++i) {
        uint32_t b = uint32_t(raw[2 * i] | (raw[2 * i + 1] << 8)) << 16;
        std::memcpy(&vals[i], &b, 4);
      }
    } else {
      for (size_t i = 0; i < n; ++i) vals[i] = half_to_f32(uint16_t(raw[2 * i] | (raw[2 * i + 1] << 8)));
    }
    const int rc = rv_set_weight(c, e.name.c_str(), vals.data(), int64_t(n));
    if (rc == RV_E_INVALID && c->err.rfind("unknown weight name", 0) == 0) continue;  // e.g. pooler
    if (rc != RV_OK) {
      std::fclose(f);
      return rc;
    }
  }
  std::fclose(f);
  return RV_OK;
}
