// safetensors.cpp -- the checkpoint format of ActorCritic::save / load
// (zealot-rl/src/ppo.rs:512-650): an 8-byte little-endian header length, a
// JSON header {"name": {"dtype": "F32", "shape": [...], "data_offsets":
// [begin, end]}, ...} padded with spaces to a multiple of 8, then the raw
// little-endian tensor bytes.  Tensors are laid out sorted by name (the
// order the safetensors writer uses for same-dtype tensors), so files are
// byte-comparable with the reference's.
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <string>
#include <vector>

namespace zrl {

struct StTensor {
  std::vector<int64_t> shape;
  std::vector<float> data;
};

std::vector<uint8_t> st_serialize(const std::map<std::string, StTensor> &ts) {
  std::vector<std::string> names;
  for (auto &kv : ts) names.push_back(kv.first);
  std::sort(names.begin(), names.end());
  std::string hdr = "{";
  int64_t off = 0;
  bool first = true;
  for (auto &n : names) {
    const StTensor &t = ts.at(n);
    const int64_t bytes = (int64_t)t.data.size() * 4;
    if (!first) hdr += ",";
    first = false;
    hdr += "\"" + n + "\":{\"dtype\":\"F32\",\"shape\":[";
    for (size_t i = 0; i < t.shape.size(); ++i) {
      if (i) hdr += ",";
      hdr += std::to_string(t.shape[i]);
    }
    hdr += "],\"data_offsets\":[" + std::to_string(off) + "," +
           std::to_string(off + bytes) + "]}";
    off += bytes;
  }
  hdr += "}";
  while (hdr.size() % 8) hdr += ' ';
  std::vector<uint8_t> out(8 + hdr.size() + (size_t)off);
  const uint64_t hl = hdr.size();
  for (int i = 0; i < 8; ++i) out[i] = (uint8_t)(hl >> (8 * i));
  memcpy(out.data() + 8, hdr.data(), hdr.size());
  uint8_t *p = out.data() + 8 + hdr.size();
  for (auto &n : names) {
    const StTensor &t = ts.at(n);
    memcpy(p, t.data.data(), t.data.size() * 4);
    p += t.data.size() * 4;
  }
  return out;
}

namespace {

struct Cursor {
  const char *p, *e;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\t' || *p == '\r')) ++p;
  }
  bool eat(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool str(std::string *s) {
    ws();
    if (p >= e || *p != '"') return false;
    ++p;
    s->clear();
    while (p < e && *p != '"') {
      if (*p == '\\' && p + 1 < e) ++p;
      s->push_back(*p++);
    }
    if (p >= e) return false;
    ++p;
    return true;
  }
  bool num(int64_t *v) {
    ws();
    bool neg = false;
    if (p < e && *p == '-') {
      neg = true;
      ++p;
    }
    if (p >= e || *p < '0' || *p > '9') return false;
    int64_t x = 0;
    while (p < e && *p >= '0' && *p <= '9') x = x * 10 + (*p++ - '0');
    *v = neg ? -x : x;
    return true;
  }
  bool int_list(std::vector<int64_t> *v) {
    v->clear();
    if (!eat('[')) return false;
    if (eat(']')) return true;
    for (;;) {
      int64_t x;
      if (!num(&x)) return false;
      v->push_back(x);
      if (eat(']')) return true;
      if (!eat(',')) return false;
    }
  }
  // skip any JSON value (used for __metadata__)
  bool skip() {
    ws();
    if (p >= e) return false;
    if (*p == '"') {
      std::string s;
      return str(&s);
    }
    if (*p == '{' || *p == '[') {
      const char open = *p, close = open == '{' ? '}' : ']';
      int depth = 0;
      bool in_str = false;
      for (; p < e; ++p) {
        if (in_str) {
          if (*p == '\\') ++p;
          else if (*p == '"') in_str = false;
          continue;
        }
        if (*p == '"') in_str = true;
        else if (*p == open) ++depth;
        else if (*p == close && --depth == 0) {
          ++p;
          return true;
        }
      }
      return false;
    }
    while (p < e && *p != ',' && *p != '}') ++p;
    return true;
  }
};

}  // namespace

bool st_parse(const uint8_t *buf, size_t len, std::map<std::string, StTensor> *out,
              std::string *err) {
  if (len < 8) {
    *err = "safetensors: file too short";
    return false;
  }
  uint64_t hl = 0;
  for (int i = 0; i < 8; ++i) hl |= (uint64_t)buf[i] << (8 * i);
  if (hl > len - 8) {
    *err = "safetensors: header length out of range";
    return false;
  }
  const uint8_t *data = buf + 8 + hl;
  const size_t dlen = len - 8 - hl;
  Cursor c{(const char *)buf + 8, (const char *)buf + 8 + hl};
  if (!c.eat('{')) {
    *err = "safetensors: header is not a JSON object";
    return false;
  }
  if (c.eat('}')) return true;
  for (;;) {
    std::string name;
    if (!c.str(&name) || !c.eat(':')) {
      *err = "safetensors: malformed header";
      return false;
    }
    if (name == "__metadata__") {
      if (!c.skip()) {
        *err = "safetensors: malformed metadata";
        return false;
      }
    } else {
      if (!c.eat('{')) {
        *err = "safetensors: malformed tensor entry " + name;
        return false;
      }
      std::string dtype;
      std::vector<int64_t> shape, offs;
      bool have_shape = false, have_offs = false;
      if (!c.eat('}')) {
        for (;;) {
          std::string key;
          if (!c.str(&key) || !c.eat(':')) {
            *err = "safetensors: malformed tensor entry " + name;
            return false;
          }
          bool ok = true;
          if (key == "dtype") ok = c.str(&dtype);
          else if (key == "shape") ok = have_shape = c.int_list(&shape);
          else if (key == "data_offsets") ok = have_offs = c.int_list(&offs);
          else ok = c.skip();
          if (!ok) {
            *err = "safetensors: bad field " + key + " of " + name;
            return false;
          }
          if (c.eat('}')) break;
          if (!c.eat(',')) {
            *err = "safetensors: malformed tensor entry " + name;
            return false;
          }
        }
      }
      if (dtype != "F32" || !have_shape || !have_offs || offs.size() != 2) {
        *err = "safetensors: tensor " + name + " is not an F32 tensor with offsets";
        return false;
      }
      int64_t numel = 1;
      for (int64_t s : shape) {
        if (s < 0) {
          *err = "safetensors: negative dim in " + name;
          return false;
        }
        numel *= s;
      }
      if (offs[0] < 0 || offs[1] < offs[0] || (size_t)offs[1] > dlen ||
          offs[1] - offs[0] != numel * 4) {
        *err = "safetensors: data offsets of " + name + " are inconsistent";
        return false;
      }
      StTensor t;
      t.shape = shape;
      t.data.resize((size_t)numel);
      memcpy(t.data.data(), data + offs[0], (size_t)numel * 4);
      (*out)[name] = std::move(t);
    }
    if (c.eat('}')) break;
    if (!c.eat(',')) {
      *err = "safetensors: malformed header";
      return false;
    }
  }
  return true;
}

}  // namespace zrl
