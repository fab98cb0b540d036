// safetensors reader and conv+BN folding for the PSA / C2PSA weights.
//
// The reference loads YOLO26 checkpoints from safetensors
// (examples/yolo26.rs:3403-3470): for every conv+BN pair it reads
// `{name}.conv.weight` and the four `{name}.bn.{weight,bias,running_mean,
// running_var}` tensors and folds them with eps = 1e-3 (the BatchNorm2d eps of
// conv.rs:39,64): scale = γ / √(var + eps), w' = w·scale, b' = β − mean·scale.
// This is the same loader for the weights this library's ops take, on the
// host: one read of the file, a parse of its JSON header (a map from tensor
// name to dtype, shape and byte range, plus an optional "__metadata__"
// entry), and f32/f16/bf16 tensors converted to f32.
//
// File layout (safetensors): u64 little-endian header size n, n bytes of
// UTF-8 JSON, then the tensor bytes; data_offsets are relative to the end of
// the header.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <map>
#include <string>
#include <vector>

#include "va_common.cuh"

namespace va {
namespace {

struct TensorEntry {
  int dtype = -1;  // VA_ST_F32 / F16 / BF16, -1 for other dtypes
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;
};

// A minimal JSON reader for the safetensors header: objects, arrays, strings
// and numbers (plus true/false/null, which only appear inside __metadata__).
struct Json {
  const char* p;
  const char* e;
  bool ok = true;

  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool eat(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool str(std::string& out) {
    ws();
    if (p >= e || *p != '"') return ok = false;
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      if (*p == '\\') {
        if (++p >= e) return ok = false;
        switch (*p) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u':  // keep the escape as text: tensor names of interest are plain ASCII
            out += "\\u";
            break;
          default: out += *p;
        }
        ++p;
      } else {
        out += *p++;
      }
    }
    if (p >= e) return ok = false;
    ++p;
    return true;
  }
  bool integer(int64_t& v) {
    ws();
    bool neg = false;
    if (p < e && *p == '-') {
      neg = true;
      ++p;
    }
    if (p >= e || *p < '0' || *p > '9') return ok = false;
    v = 0;
    while (p < e && *p >= '0' && *p <= '9') {
      if (v > (INT64_MAX - 9) / 10) return ok = false;
      v = v * 10 + (*p++ - '0');
    }
    if (neg) v = -v;
    return true;
  }
  // skip any value (for __metadata__ and unknown fields)
  bool skip(int depth = 0) {
    ws();
    if (p >= e || depth > 64) return ok = false;
    if (*p == '"') {
      std::string s;
      return str(s);
    }
    if (*p == '{' || *p == '[') {
      const char close = *p == '{' ? '}' : ']';
      const bool obj = *p == '{';
      ++p;
      if (eat(close)) return true;
      do {
        if (obj) {
          std::string k;
          if (!str(k) || !eat(':')) return ok = false;
        }
        if (!skip(depth + 1)) return false;
      } while (eat(','));
      if (eat(close)) return true;
      ok = false;
      return false;
    }
    while (p < e && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n') ++p;  // number/literal
    return true;
  }
};

}  // namespace
}  // namespace va

struct va_safetensors {
  std::vector<unsigned char> bytes;  // the whole file
  size_t data0 = 0;                  // start of the tensor bytes
  std::map<std::string, va::TensorEntry> tensors;
};

using namespace va;

namespace {

int parse_dtype(const std::string& s) {
  if (s == "F32") return VA_ST_F32;
  if (s == "F16") return VA_ST_F16;
  if (s == "BF16") return VA_ST_BF16;
  return -1;
}

int parse_header(va_safetensors* st, const char* path) {
  if (st->bytes.size() < 8) return set_error(VA_ERR_SHAPE, "safetensors %s: file shorter than its header size", path);
  uint64_t n = 0;
  for (int i = 7; i >= 0; --i) n = (n << 8) | st->bytes[i];
  if (n > st->bytes.size() - 8) return set_error(VA_ERR_SHAPE, "safetensors %s: header size %llu past the file end", path,
                                                 (unsigned long long)n);
  st->data0 = 8 + n;
  Json js{reinterpret_cast<const char*>(st->bytes.data()) + 8, reinterpret_cast<const char*>(st->bytes.data()) + 8 + n};
  if (!js.eat('{')) return set_error(VA_ERR_SHAPE, "safetensors %s: header is not a JSON object", path);
  const uint64_t data_len = st->bytes.size() - st->data0;
  if (!js.eat('}')) {
    do {
      std::string key;
      if (!js.str(key) || !js.eat(':')) return set_error(VA_ERR_SHAPE, "safetensors %s: malformed header", path);
      if (key == "__metadata__") {
        if (!js.skip()) return set_error(VA_ERR_SHAPE, "safetensors %s: malformed __metadata__", path);
        continue;
      }
      TensorEntry t;
      bool have_offsets = false, have_dtype = false, have_shape = false;
      if (!js.eat('{')) return set_error(VA_ERR_SHAPE, "safetensors %s: entry '%s' is not an object", path, key.c_str());
      if (!js.eat('}')) {
        do {
          std::string field;
          if (!js.str(field) || !js.eat(':')) return set_error(VA_ERR_SHAPE, "safetensors %s: malformed entry", path);
          if (field == "dtype") {
            std::string d;
            if (!js.str(d)) return set_error(VA_ERR_SHAPE, "safetensors %s: bad dtype", path);
            t.dtype = parse_dtype(d);
            have_dtype = true;
          } else if (field == "shape" || field == "data_offsets") {
            std::vector<int64_t> v;
            if (!js.eat('[')) return set_error(VA_ERR_SHAPE, "safetensors %s: %s is not an array", path, field.c_str());
            if (!js.eat(']')) {
              do {
                int64_t x;
                if (!js.integer(x) || x < 0) return set_error(VA_ERR_SHAPE, "safetensors %s: bad %s", path, field.c_str());
                v.push_back(x);
              } while (js.eat(','));
              if (!js.eat(']')) return set_error(VA_ERR_SHAPE, "safetensors %s: bad %s", path, field.c_str());
            }
            if (field == "shape") {
              if (v.size() > 8) return set_error(VA_ERR_SHAPE, "safetensors %s: rank > 8", path);
              t.shape = v;
              have_shape = true;
            } else {
              if (v.size() != 2 || v[0] > v[1] || (uint64_t)v[1] > data_len)
                return set_error(VA_ERR_SHAPE, "safetensors %s: data_offsets of '%s' out of the file", path,
                                 key.c_str());
              t.begin = (uint64_t)v[0];
              t.end = (uint64_t)v[1];
              have_offsets = true;
            }
          } else if (!js.skip()) {
            return set_error(VA_ERR_SHAPE, "safetensors %s: malformed entry", path);
          }
        } while (js.eat(','));
        if (!js.eat('}')) return set_error(VA_ERR_SHAPE, "safetensors %s: malformed entry", path);
      }
      if (!have_offsets || !have_dtype || !have_shape)
        return set_error(VA_ERR_SHAPE, "safetensors %s: entry '%s' lacks dtype, shape or data_offsets", path,
                         key.c_str());
      st->tensors[key] = t;
    } while (js.eat(','));
    if (!js.eat('}')) return set_error(VA_ERR_SHAPE, "safetensors %s: malformed header", path);
  }
  return VA_OK;
}

// element count, or -1 if it does not fit in 63 bits
int64_t numel(const TensorEntry& t) {
  int64_t n = 1;
  for (int64_t d : t.shape) {
    if (d != 0 && n > INT64_MAX / d) return -1;
    n *= d;
  }
  return n;
}

float half_bits_to_f32(uint16_t h) {
  const uint32_t s = (uint32_t)(h & 0x8000u) << 16, ex = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
  uint32_t bits;
  if (ex == 0) {
    if (m == 0) {
      bits = s;
    } else {  // subnormal: m · 2^-24
      const float f = (float)m * 5.9604644775390625e-8f;
      memcpy(&bits, &f, 4);
      bits |= s;
    }
  } else if (ex == 31) {
    bits = s | 0x7F800000u | (m << 13);
  } else {
    bits = s | ((ex + 112) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

const TensorEntry* find(va_safetensors* st, const char* key) {
  auto it = st->tensors.find(key);
  return it == st->tensors.end() ? nullptr : &it->second;
}

// the tensor as f32 values (host)
int read_f32(va_safetensors* st, const char* key, std::vector<float>& out) {
  const TensorEntry* t = find(st, key);
  if (!t) return set_error(VA_ERR_SHAPE, "safetensors: no tensor '%s'", key);
  const int64_t n = numel(*t);
  const int es = t->dtype == VA_ST_F32 ? 4 : (t->dtype == VA_ST_F16 || t->dtype == VA_ST_BF16) ? 2 : 0;
  if (!es) return set_error(VA_ERR_UNSUPPORTED, "safetensors: '%s' is not F32, F16 or BF16", key);
  if (n < 0 || (uint64_t)n > (t->end - t->begin) / (uint64_t)es || (uint64_t)n * es != t->end - t->begin)
    return set_error(VA_ERR_SHAPE, "safetensors: '%s' holds %llu bytes for %lld elements", key,
                     (unsigned long long)(t->end - t->begin), (long long)n);
  out.resize((size_t)n);
  const unsigned char* src = st->bytes.data() + st->data0 + t->begin;
  for (int64_t i = 0; i < n; ++i) {
    if (es == 4) {
      uint32_t u = (uint32_t)src[4 * i] | (uint32_t)src[4 * i + 1] << 8 | (uint32_t)src[4 * i + 2] << 16 |
                   (uint32_t)src[4 * i + 3] << 24;
      memcpy(&out[i], &u, 4);
    } else {
      const uint16_t h = (uint16_t)(src[2 * i] | src[2 * i + 1] << 8);
      if (t->dtype == VA_ST_BF16) {
        const uint32_t u = (uint32_t)h << 16;
        memcpy(&out[i], &u, 4);
      } else {
        out[i] = half_bits_to_f32(h);
      }
    }
  }
  return VA_OK;
}

}  // namespace

extern "C" {

int va_safetensors_open(const char* path, va_safetensors** out) {
  clear_error();
  VA_CHECK_ARG(path && out, "safetensors: null path or output");
  *out = nullptr;
  FILE* f = fopen(path, "rb");
  if (!f) return set_error(VA_ERR_SHAPE, "safetensors: cannot open %s", path);
  va_safetensors* st = new va_safetensors();
  int rc = VA_OK;
  if (fseek(f, 0, SEEK_END) != 0) rc = set_error(VA_ERR_SHAPE, "safetensors %s: cannot seek", path);
  long len = rc ? -1 : ftell(f);
  if (!rc && len < 0) rc = set_error(VA_ERR_SHAPE, "safetensors %s: cannot size", path);
  if (!rc && fseek(f, 0, SEEK_SET) != 0) rc = set_error(VA_ERR_SHAPE, "safetensors %s: cannot seek", path);
  if (!rc) {
    st->bytes.resize((size_t)len);
    if (len > 0 && fread(st->bytes.data(), 1, (size_t)len, f) != (size_t)len)
      rc = set_error(VA_ERR_SHAPE, "safetensors %s: short read", path);
  }
  fclose(f);
  if (!rc) rc = parse_header(st, path);
  if (rc) {
    delete st;
    return rc;
  }
  *out = st;
  return VA_OK;
}

void va_safetensors_close(va_safetensors* st) { delete st; }

int va_safetensors_tensor_info(va_safetensors* st, const char* key, int* dtype, int64_t* shape, int* rank) {
  clear_error();
  VA_CHECK_ARG(st && key && dtype && shape && rank, "safetensors info: null argument");
  const TensorEntry* t = find(st, key);
  if (!t) return set_error(VA_ERR_SHAPE, "safetensors: no tensor '%s'", key);
  *dtype = t->dtype;
  *rank = (int)t->shape.size();
  for (size_t i = 0; i < t->shape.size(); ++i) shape[i] = t->shape[i];
  return VA_OK;
}

int va_safetensors_read_f32(va_safetensors* st, const char* key, float* dst, size_t count) {
  clear_error();
  VA_CHECK_ARG(st && key && dst, "safetensors read: null argument");
  std::vector<float> v;
  if (int rc = read_f32(st, key, v)) return rc;
  if (v.size() != count)
    return set_error(VA_ERR_SHAPE, "safetensors: '%s' has %zu elements, %zu asked", key, v.size(), count);
  memcpy(dst, v.data(), count * sizeof(float));
  return VA_OK;
}

int va_safetensors_fold_conv_bn(va_safetensors* st, const char* prefix, float eps, float* w_out, float* b_out,
                                size_t w_count, int c_out) {
  clear_error();
  VA_CHECK_ARG(st && prefix && w_out && b_out && c_out > 0, "safetensors fold: null argument");
  VA_CHECK_ARG(eps > 0.f, "safetensors fold: eps %g", (double)eps);
  const std::string p(prefix);
  std::vector<float> w, g, b, m, v;
  if (int rc = read_f32(st, (p + ".conv.weight").c_str(), w)) return rc;
  if (int rc = read_f32(st, (p + ".bn.weight").c_str(), g)) return rc;
  if (int rc = read_f32(st, (p + ".bn.bias").c_str(), b)) return rc;
  if (int rc = read_f32(st, (p + ".bn.running_mean").c_str(), m)) return rc;
  if (int rc = read_f32(st, (p + ".bn.running_var").c_str(), v)) return rc;
  if (w.size() != w_count || w_count % (size_t)c_out)
    return set_error(VA_ERR_SHAPE, "safetensors fold: '%s.conv.weight' has %zu elements, %zu asked", prefix, w.size(),
                     w_count);
  if (g.size() != (size_t)c_out || b.size() != (size_t)c_out || m.size() != (size_t)c_out || v.size() != (size_t)c_out)
    return set_error(VA_ERR_SHAPE, "safetensors fold: '%s.bn.*' do not have %d channels", prefix, c_out);
  return va_fold_bn_f32(w.data(), g.data(), b.data(), m.data(), v.data(), eps, c_out, (int)(w_count / c_out), w_out,
                        b_out);
}

}  // extern "C"
