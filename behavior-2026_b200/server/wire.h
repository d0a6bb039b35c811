// wire.h — the policy server's wire formats, written for this server: SHA-1 and base64 (the RFC 6455
// opening handshake), WebSocket frames (RFC 6455 section 5), and MessagePack values (the msgpack
// specification) with openpi's numpy convention, an array packed as the map
// {"__ndarray__": true, "data": <bin>, "dtype": "<f4", "shape": [..]} (openpi msgpack_numpy).
// The reference server built the same pieces by hand (docs/archive/windows/π05_네이티브엔진.md:120-123).
#pragma once
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace wire {

// ---------------------------------------------------------------- SHA-1 (FIPS 180-4)
inline std::string sha1(const std::string& msg) {
  uint32_t h[5] = {0x67452301u, 0xEFCDAB89u, 0x98BADCFEu, 0x10325476u, 0xC3D2E1F0u};
  std::string m = msg;
  const uint64_t bits = (uint64_t)msg.size() * 8;
  m.push_back((char)0x80);
  while (m.size() % 64 != 56) m.push_back(0);
  for (int i = 7; i >= 0; --i) m.push_back((char)(bits >> (8 * i)));
  auto rol = [](uint32_t x, int n) { return (x << n) | (x >> (32 - n)); };
  for (size_t off = 0; off < m.size(); off += 64) {
    uint32_t w[80];
    for (int i = 0; i < 16; ++i)
      w[i] = (uint32_t)(uint8_t)m[off + 4 * i] << 24 | (uint32_t)(uint8_t)m[off + 4 * i + 1] << 16 |
             (uint32_t)(uint8_t)m[off + 4 * i + 2] << 8 | (uint32_t)(uint8_t)m[off + 4 * i + 3];
    for (int i = 16; i < 80; ++i) w[i] = rol(w[i - 3] ^ w[i - 8] ^ w[i - 14] ^ w[i - 16], 1);
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4];
    for (int i = 0; i < 80; ++i) {
      uint32_t f, k;
      if (i < 20) {
        f = (b & c) | (~b & d);
        k = 0x5A827999u;
      } else if (i < 40) {
        f = b ^ c ^ d;
        k = 0x6ED9EBA1u;
      } else if (i < 60) {
        f = (b & c) | (b & d) | (c & d);
        k = 0x8F1BBCDCu;
      } else {
        f = b ^ c ^ d;
        k = 0xCA62C1D6u;
      }
      const uint32_t t = rol(a, 5) + f + e + k + w[i];
      e = d;
      d = c;
      c = rol(b, 30);
      b = a;
      a = t;
    }
    h[0] += a, h[1] += b, h[2] += c, h[3] += d, h[4] += e;
  }
  std::string out;
  for (uint32_t v : h)
    for (int i = 3; i >= 0; --i) out.push_back((char)(v >> (8 * i)));
  return out;
}

inline std::string base64(const std::string& in) {
  static const char* T = "ABCDEFGHIJKLMNOPQRSTUVWXYZabcdefghijklmnopqrstuvwxyz0123456789+/";
  std::string out;
  size_t i = 0;
  for (; i + 2 < in.size(); i += 3) {
    const uint32_t v = (uint8_t)in[i] << 16 | (uint8_t)in[i + 1] << 8 | (uint8_t)in[i + 2];
    out += T[v >> 18], out += T[(v >> 12) & 63], out += T[(v >> 6) & 63], out += T[v & 63];
  }
  if (i + 1 == in.size()) {
    const uint32_t v = (uint8_t)in[i] << 16;
    out += T[v >> 18], out += T[(v >> 12) & 63], out += "==";
  } else if (i + 2 == in.size()) {
    const uint32_t v = (uint8_t)in[i] << 16 | (uint8_t)in[i + 1] << 8;
    out += T[v >> 18], out += T[(v >> 12) & 63], out += T[(v >> 6) & 63], out += '=';
  }
  return out;
}

// Sec-WebSocket-Accept for a client's Sec-WebSocket-Key (RFC 6455 section 4.2.2)
inline std::string ws_accept(const std::string& key) {
  return base64(sha1(key + "258EAFA5-E914-47DA-95CA-C5AB0DC85B11"));
}

// Server-to-client frame (unmasked, FIN set) around `payload`.
inline std::string ws_frame(int opcode, const std::string& payload) {
  std::string f;
  f.push_back((char)(0x80 | opcode));
  const uint64_t n = payload.size();
  if (n < 126) {
    f.push_back((char)n);
  } else if (n < 65536) {
    f.push_back(126);
    f.push_back((char)(n >> 8));
    f.push_back((char)n);
  } else {
    f.push_back(127);
    for (int i = 7; i >= 0; --i) f.push_back((char)(n >> (8 * i)));
  }
  return f + payload;
}

// ---------------------------------------------------------------- MessagePack values
struct Value;
using VPtr = std::shared_ptr<Value>;
struct Value {
  enum Kind { NIL, BOOL, INT, FLOAT, STR, BIN, ARRAY, MAP } kind = NIL;
  bool b = false;
  int64_t i = 0;
  double f = 0;
  std::string s;  // STR or BIN bytes
  std::vector<VPtr> arr;
  std::vector<std::pair<VPtr, VPtr>> map;

  const Value* get(const std::string& key) const {
    for (const auto& kv : map)
      if ((kv.first->kind == STR || kv.first->kind == BIN) && kv.first->s == key) return kv.second.get();
    return nullptr;
  }
};

inline VPtr v_nil() { return std::make_shared<Value>(); }
inline VPtr v_bool(bool x) {
  auto v = std::make_shared<Value>();
  v->kind = Value::BOOL;
  v->b = x;
  return v;
}
inline VPtr v_int(int64_t x) {
  auto v = std::make_shared<Value>();
  v->kind = Value::INT;
  v->i = x;
  return v;
}
inline VPtr v_float(double x) {
  auto v = std::make_shared<Value>();
  v->kind = Value::FLOAT;
  v->f = x;
  return v;
}
inline VPtr v_str(const std::string& x, bool bin = false) {
  auto v = std::make_shared<Value>();
  v->kind = bin ? Value::BIN : Value::STR;
  v->s = x;
  return v;
}
inline VPtr v_array() {
  auto v = std::make_shared<Value>();
  v->kind = Value::ARRAY;
  return v;
}
inline VPtr v_map() {
  auto v = std::make_shared<Value>();
  v->kind = Value::MAP;
  return v;
}
inline void put(const VPtr& m, const std::string& k, const VPtr& v) { m->map.push_back({v_str(k), v}); }

class Reader {
 public:
  Reader(const uint8_t* p, size_t n) : p_(p), n_(n) {}
  VPtr value(int depth = 0) {
    if (depth > 64) throw std::runtime_error("msgpack: nesting too deep");
    const uint8_t t = u8();
    if (t <= 0x7f) return v_int(t);
    if (t >= 0xe0) return v_int((int8_t)t);
    if ((t & 0xf0) == 0x80) return map(t & 0x0f, depth);
    if ((t & 0xf0) == 0x90) return array(t & 0x0f, depth);
    if ((t & 0xe0) == 0xa0) return v_str(bytes(t & 0x1f));
    switch (t) {
      case 0xc0: return v_nil();
      case 0xc2: return v_bool(false);
      case 0xc3: return v_bool(true);
      case 0xc4: return v_str(bytes(u8()), true);
      case 0xc5: return v_str(bytes(be(2)), true);
      case 0xc6: return v_str(bytes(be(4)), true);
      case 0xca: {
        const uint32_t u = (uint32_t)be(4);
        float x;
        memcpy(&x, &u, 4);
        return v_float(x);
      }
      case 0xcb: {
        const uint64_t u = be(8);
        double x;
        memcpy(&x, &u, 8);
        return v_float(x);
      }
      case 0xcc: return v_int((int64_t)be(1));
      case 0xcd: return v_int((int64_t)be(2));
      case 0xce: return v_int((int64_t)be(4));
      case 0xcf: return v_int((int64_t)be(8));
      case 0xd0: return v_int((int8_t)be(1));
      case 0xd1: return v_int((int16_t)be(2));
      case 0xd2: return v_int((int32_t)be(4));
      case 0xd3: return v_int((int64_t)be(8));
      case 0xd9: return v_str(bytes(u8()));
      case 0xda: return v_str(bytes(be(2)));
      case 0xdb: return v_str(bytes(be(4)));
      case 0xdc: return array(be(2), depth);
      case 0xdd: return array(be(4), depth);
      case 0xde: return map(be(2), depth);
      case 0xdf: return map(be(4), depth);
      default: throw std::runtime_error("msgpack: unsupported type byte");
    }
  }
  size_t used() const { return at_; }

 private:
  const uint8_t* p_;
  size_t n_, at_ = 0;
  uint8_t u8() {
    if (at_ >= n_) throw std::runtime_error("msgpack: truncated");
    return p_[at_++];
  }
  uint64_t be(int k) {
    uint64_t v = 0;
    for (int i = 0; i < k; ++i) v = v << 8 | u8();
    return v;
  }
  std::string bytes(uint64_t k) {
    if (k > n_ - at_) throw std::runtime_error("msgpack: truncated");
    std::string s((const char*)p_ + at_, (size_t)k);
    at_ += (size_t)k;
    return s;
  }
  VPtr array(uint64_t k, int depth) {
    if (k > n_ - at_) throw std::runtime_error("msgpack: truncated");
    auto v = v_array();
    for (uint64_t i = 0; i < k; ++i) v->arr.push_back(value(depth + 1));
    return v;
  }
  VPtr map(uint64_t k, int depth) {
    if (k > n_ - at_) throw std::runtime_error("msgpack: truncated");
    auto v = v_map();
    for (uint64_t i = 0; i < k; ++i) {
      VPtr key = value(depth + 1);
      v->map.push_back({key, value(depth + 1)});
    }
    return v;
  }
};

inline void w_be(std::string& o, uint64_t v, int k) {
  for (int i = k - 1; i >= 0; --i) o.push_back((char)(v >> (8 * i)));
}

inline void pack(std::string& o, const Value& v) {
  switch (v.kind) {
    case Value::NIL: o.push_back((char)0xc0); break;
    case Value::BOOL: o.push_back((char)(v.b ? 0xc3 : 0xc2)); break;
    case Value::INT:
      if (v.i >= 0 && v.i <= 0x7f) {
        o.push_back((char)v.i);
      } else if (v.i < 0 && v.i >= -32) {
        o.push_back((char)(int8_t)v.i);
      } else if (v.i >= 0) {
        o.push_back((char)0xcf);
        w_be(o, (uint64_t)v.i, 8);
      } else {
        o.push_back((char)0xd3);
        w_be(o, (uint64_t)v.i, 8);
      }
      break;
    case Value::FLOAT: {
      uint64_t u;
      memcpy(&u, &v.f, 8);
      o.push_back((char)0xcb);
      w_be(o, u, 8);
      break;
    }
    case Value::STR:
    case Value::BIN: {
      const uint64_t n = v.s.size();
      if (v.kind == Value::STR && n < 32) {
        o.push_back((char)(0xa0 | n));
      } else {
        o.push_back((char)(v.kind == Value::STR ? 0xdb : 0xc6));
        w_be(o, n, 4);
      }
      o += v.s;
      break;
    }
    case Value::ARRAY:
      o.push_back((char)0xdd);
      w_be(o, v.arr.size(), 4);
      for (const auto& e : v.arr) pack(o, *e);
      break;
    case Value::MAP:
      o.push_back((char)0xdf);
      w_be(o, v.map.size(), 4);
      for (const auto& kv : v.map) {
        pack(o, *kv.first);
        pack(o, *kv.second);
      }
      break;
  }
}

// ---------------------------------------------------------------- numpy arrays (openpi msgpack_numpy)
struct NdArray {
  std::string dtype;  // numpy dtype.str: "|u1", "<f4", "<i4", ...
  std::vector<int64_t> shape;
  std::string data;  // raw little-endian bytes, C order
  int64_t size() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
  }
};

inline bool as_ndarray(const Value* v, NdArray* out) {
  if (!v || v->kind != Value::MAP) return false;
  const Value* flag = v->get("__ndarray__");
  const Value* data = v->get("data");
  const Value* dt = v->get("dtype");
  const Value* sh = v->get("shape");
  if (!flag || !data || !dt || !sh || sh->kind != Value::ARRAY) return false;
  out->dtype = dt->s;
  out->data = data->s;
  out->shape.clear();
  for (const auto& e : sh->arr) {
    if (e->kind != Value::INT || e->i < 0) return false;
    out->shape.push_back(e->i);
  }
  return true;
}

// openpi packs the array's keys as bytes (msgpack bin), and its unpacker looks them up as bytes
inline VPtr v_ndarray(const std::string& dtype, const std::vector<int64_t>& shape, const void* data, size_t bytes) {
  auto m = v_map();
  auto key = [](const char* k) { return v_str(k, true); };
  m->map.push_back({key("__ndarray__"), v_bool(true)});
  m->map.push_back({key("data"), v_str(std::string((const char*)data, bytes), true)});
  m->map.push_back({key("dtype"), v_str(dtype)});
  auto s = v_array();
  for (int64_t d : shape) s->arr.push_back(v_int(d));
  m->map.push_back({key("shape"), s});
  return m;
}

}  // namespace wire
