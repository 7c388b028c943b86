// ltx25-safetensors.cc -- see ltx25-safetensors.h.
#include "ltx25-safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace ltx25 {

namespace {

bool fail(std::string* err, const std::string& m)
{
  if (err != nullptr) *err = m;
  return false;
}

// A strict reader of the JSON the format's header uses: objects, arrays,
// strings (with escapes), integers; other scalars (floats, true / false /
// null) are skipped where a value may be anything.
struct Json {
  const char* p;
  const char* e;
  std::string err;
  int depth = 0;

  void ws()
  {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool eat(char c)
  {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool bad(const std::string& m)
  {
    if (err.empty()) err = m;
    return false;
  }
  static void utf8(uint32_t cp, std::string* out)
  {
    if (cp < 0x80) {
      out->push_back((char)cp);
    } else if (cp < 0x800) {
      out->push_back((char)(0xC0 | (cp >> 6)));
      out->push_back((char)(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
      out->push_back((char)(0xE0 | (cp >> 12)));
      out->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
      out->push_back((char)(0x80 | (cp & 0x3F)));
    } else {
      out->push_back((char)(0xF0 | (cp >> 18)));
      out->push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
      out->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
      out->push_back((char)(0x80 | (cp & 0x3F)));
    }
  }
  bool hex4(uint32_t* v)
  {
    if (e - p < 4) return bad("short \\u escape");
    uint32_t x = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p++;
      x <<= 4;
      if (c >= '0' && c <= '9') x |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') x |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') x |= (uint32_t)(c - 'A' + 10);
      else return bad("bad \\u escape");
    }
    *v = x;
    return true;
  }
  bool str(std::string* out)
  {
    ws();
    if (p >= e || *p != '"') return bad("expected a string");
    ++p;
    out->clear();
    while (p < e && *p != '"') {
      if ((unsigned char)*p < 0x20) return bad("control character in a string");
      if (*p != '\\') {
        out->push_back(*p++);
        continue;
      }
      if (++p >= e) return bad("unterminated escape");
      const char c = *p++;
      switch (c) {
        case '"': out->push_back('"'); break;
        case '\\': out->push_back('\\'); break;
        case '/': out->push_back('/'); break;
        case 'b': out->push_back('\b'); break;
        case 'f': out->push_back('\f'); break;
        case 'n': out->push_back('\n'); break;
        case 'r': out->push_back('\r'); break;
        case 't': out->push_back('\t'); break;
        case 'u': {
          uint32_t cp = 0;
          if (!hex4(&cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00) {   // a surrogate pair
            uint32_t lo = 0;
            if (e - p < 6 || p[0] != '\\' || p[1] != 'u') return bad("lone surrogate");
            p += 2;
            if (!hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return bad("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          utf8(cp, out);
          break;
        }
        default: return bad("bad escape");
      }
    }
    if (p >= e) return bad("unterminated string");
    ++p;
    return true;
  }
  bool integer(int64_t* v)
  {
    ws();
    bool neg = false;
    if (p < e && *p == '-') {
      neg = true;
      ++p;
    }
    if (p >= e || *p < '0' || *p > '9') return bad("expected an integer");
    uint64_t x = 0;
    while (p < e && *p >= '0' && *p <= '9') {
      const uint64_t d = (uint64_t)(*p++ - '0');
      if (x > (UINT64_MAX - d) / 10) return bad("integer overflow");
      x = x * 10 + d;
    }
    if (p < e && (*p == '.' || *p == 'e' || *p == 'E')) return bad("expected an integer");
    if (x > (uint64_t)INT64_MAX) return bad("integer overflow");
    *v = neg ? -(int64_t)x : (int64_t)x;
    return true;
  }
  bool skip()
  {
    ws();
    if (p >= e) return bad("truncated value");
    if (++depth > 64) return bad("nesting too deep");
    bool ok = true;
    if (*p == '"') {
      std::string t;
      ok = str(&t);
    } else if (*p == '{') {
      ++p;
      if (!eat('}')) {
        do {
          std::string k;
          ok = str(&k) && (eat(':') || bad("expected ':'")) && skip();
        } while (ok && eat(','));
        ok = ok && (eat('}') || bad("expected '}'"));
      }
    } else if (*p == '[') {
      ++p;
      if (!eat(']')) {
        do {
          ok = skip();
        } while (ok && eat(','));
        ok = ok && (eat(']') || bad("expected ']'"));
      }
    } else {
      const char* s = p;
      while (p < e && (std::strchr("+-.0123456789eE", *p) != nullptr || (*p >= 'a' && *p <= 'z')))
        ++p;
      const std::string lit(s, p);
      if (lit.empty()) ok = bad("unexpected character");
      else if ((lit[0] >= 'a' && lit[0] <= 'z') && lit != "true" && lit != "false" && lit != "null")
        ok = bad("bad literal");
    }
    --depth;
    return ok;
  }
};

int dtype_of(const std::string& s)
{
  static const std::pair<const char*, int> k[] = {
      {"F32", ST_F32}, {"F16", ST_F16}, {"BF16", ST_BF16}, {"U32", ST_U32}, {"I32", ST_I32},
      {"U8", ST_U8}, {"I8", ST_I8}, {"F64", ST_F64}, {"I64", ST_I64}, {"U16", ST_U16},
      {"I16", ST_I16}, {"BOOL", ST_BOOL}};
  for (const auto& x : k)
    if (s == x.first) return x.second;
  return -1;
}

// IEEE 754 binary16 -> binary32 (exact).
float half_to_f32(uint16_t h)
{
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {   // subnormal: normalize
      int e = -1;
      do {
        ++e;
        man <<= 1;
      } while ((man & 0x400u) == 0);
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

uint16_t f32_to_bf16_rne(float f)
{
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu) != 0)
    return (uint16_t)((u >> 16) | 0x40u);   // quiet NaN
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

}  // namespace

SafeTensors::~SafeTensors()
{
  if (_map != nullptr) munmap(_map, _map_bytes);
}

size_t SafeTensors::elem_size(int dtype)
{
  switch (dtype) {
    case ST_F64: case ST_I64: return 8;
    case ST_F32: case ST_U32: case ST_I32: return 4;
    case ST_F16: case ST_BF16: case ST_U16: case ST_I16: return 2;
    case ST_U8: case ST_I8: case ST_BOOL: return 1;
    default: return 0;
  }
}

bool SafeTensors::open(const std::string& path, std::string* err)
{
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) return fail(err, "cannot open '" + path + "'");
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 8) {
    ::close(fd);
    return fail(err, "'" + path + "' is not a safetensors file (too short)");
  }
  void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (m == MAP_FAILED) return fail(err, "cannot map '" + path + "'");
  _map = m;
  _map_bytes = (size_t)st.st_size;
  return parse(static_cast<const uint8_t*>(m), _map_bytes, err);
}

bool SafeTensors::parse(const uint8_t* base, size_t size, std::string* err)
{
  _tensors.clear();
  _index.clear();
  _meta.clear();
  if (size < 8) return fail(err, "safetensors: shorter than its length word");
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | base[i];
  if (hlen > size - 8) return fail(err, "safetensors: header length past the end of the file");
  const uint8_t* data = base + 8 + hlen;
  const uint64_t dsize = size - 8 - hlen;
  Json j{reinterpret_cast<const char*>(base + 8), reinterpret_cast<const char*>(base + 8 + hlen)};
  if (!j.eat('{')) return fail(err, "safetensors: header is not a JSON object");
  if (!j.eat('}')) {
    do {
      std::string name;
      if (!j.str(&name) || !(j.eat(':') || j.bad("expected ':'"))) break;
      if (name == "__metadata__") {
        if (!j.eat('{')) {
          j.bad("__metadata__ is not an object");
          break;
        }
        if (!j.eat('}')) {
          bool ok = true;
          do {
            std::string k, v;
            ok = j.str(&k) && (j.eat(':') || j.bad("expected ':'"));
            if (!ok) break;
            j.ws();
            if (j.p < j.e && *j.p == '"') ok = j.str(&v);
            else ok = j.skip();   // a non-string value: not a key this reads
            if (ok) _meta[k] = v;
          } while (ok && j.eat(','));
          if (!ok || !(j.eat('}') || j.bad("expected '}'"))) break;
        }
        continue;
      }
      if (_index.count(name)) {
        j.bad("tensor '" + name + "' appears twice");
        break;
      }
      StTensor t;
      t.name = name;
      std::string dt;
      int64_t b0 = -1, b1 = -1;
      bool have_shape = false, have_dtype = false, have_offsets = false;
      bool ok = j.eat('{') || j.bad("expected '{'");
      if (ok && !j.eat('}')) {
        do {
          std::string k;
          ok = j.str(&k) && (j.eat(':') || j.bad("expected ':'"));
          if (!ok) break;
          // one of each key: a repeated one would silently replace (or, for
          // shape, extend) what the first said
          if ((k == "dtype" && have_dtype) || (k == "shape" && have_shape) ||
              (k == "data_offsets" && have_offsets)) {
            ok = j.bad("tensor '" + name + "' repeats its " + k);
            break;
          }
          if (k == "dtype") {
            ok = j.str(&dt);
            have_dtype = true;
          } else if (k == "shape") {
            ok = j.eat('[') || j.bad("shape is not an array");
            have_shape = true;
            if (ok && !j.eat(']')) {
              do {
                int64_t d = 0;
                ok = j.integer(&d) && (d >= 0 || j.bad("negative dimension")) &&
                     (t.shape.size() < (size_t)kStMaxDims ||
                      j.bad("tensor '" + name + "' has more than " +
                            std::to_string(kStMaxDims) + " dimensions"));
                if (ok) t.shape.push_back(d);
              } while (ok && j.eat(','));
              ok = ok && (j.eat(']') || j.bad("expected ']'"));
            }
          } else if (k == "data_offsets") {
            have_offsets = true;
            ok = (j.eat('[') || j.bad("data_offsets is not an array")) && j.integer(&b0) &&
                 (j.eat(',') || j.bad("data_offsets needs two entries")) && j.integer(&b1) &&
                 (j.eat(']') || j.bad("data_offsets has more than two entries"));
          } else {
            ok = j.skip();
          }
        } while (ok && j.eat(','));
        ok = ok && (j.eat('}') || j.bad("expected '}'"));
      }
      if (!ok) break;
      if (!have_dtype || !have_shape || b0 < 0 || b1 < 0) {
        j.bad("tensor '" + name + "' lacks dtype, shape or data_offsets");
        break;
      }
      t.dtype = dtype_of(dt);
      if (t.dtype < 0) {
        j.bad("tensor '" + name + "' has dtype '" + dt + "', which this reader does not know");
        break;
      }
      uint64_t n = 1;
      bool over = false;
      for (int64_t d : t.shape) {
        if (d != 0 && n > UINT64_MAX / (uint64_t)d) over = true;
        n *= (uint64_t)d;
      }
      const uint64_t es = elem_size(t.dtype);
      if (over || n > UINT64_MAX / es || b1 < b0 || (uint64_t)(b1 - b0) != n * es) {
        j.bad("tensor '" + name + "': data_offsets span " + std::to_string(b1 - b0) +
              " bytes, its shape and dtype " + std::to_string(n * es));
        break;
      }
      if ((uint64_t)b1 > dsize) {
        j.bad("tensor '" + name + "' ends past the end of the file");
        break;
      }
      t.data = data + b0;
      t.bytes = (uint64_t)(b1 - b0);
      _index[name] = (int)_tensors.size();
      _tensors.push_back(std::move(t));
    } while (j.eat(','));
    if (j.err.empty() && !j.eat('}')) j.bad("expected '}' or ','");
  }
  if (j.err.empty()) {
    j.ws();
    if (j.p != j.e) j.bad("trailing bytes after the header object");
  }
  if (!j.err.empty()) {
    _tensors.clear();
    _index.clear();
    _meta.clear();
    return fail(err, "safetensors header: " + j.err);
  }
  return true;
}

int SafeTensors::find(const std::string& name) const
{
  auto it = _index.find(name);
  return it == _index.end() ? -1 : it->second;
}

const std::string* SafeTensors::metadata(const std::string& key) const
{
  auto it = _meta.find(key);
  return it == _meta.end() ? nullptr : &it->second;
}

bool SafeTensors::to_f32(const StTensor& t, size_t off, size_t n, float* out)
{
  const size_t es = elem_size(t.dtype);
  if (es == 0 || (off + n) * es > t.bytes) return false;
  const uint8_t* p = t.data + off * es;
  switch (t.dtype) {
    case ST_F32:
      std::memcpy(out, p, n * 4);
      return true;
    case ST_F16:
      for (size_t i = 0; i < n; ++i) {
        uint16_t h;
        std::memcpy(&h, p + 2 * i, 2);
        out[i] = half_to_f32(h);
      }
      return true;
    case ST_BF16:
      for (size_t i = 0; i < n; ++i) {
        uint16_t h;
        std::memcpy(&h, p + 2 * i, 2);
        const uint32_t u = (uint32_t)h << 16;
        std::memcpy(out + i, &u, 4);
      }
      return true;
    default:
      return false;
  }
}

bool SafeTensors::to_bf16(const StTensor& t, size_t off, size_t n, uint16_t* out)
{
  if (t.dtype == ST_BF16) {
    if ((off + n) * 2 > t.bytes) return false;
    std::memcpy(out, t.data + off * 2, n * 2);
    return true;
  }
  std::vector<float> f(n);
  if (!to_f32(t, off, n, f.data())) return false;
  for (size_t i = 0; i < n; ++i) out[i] = f32_to_bf16_rne(f[i]);
  return true;
}

}  // namespace ltx25
