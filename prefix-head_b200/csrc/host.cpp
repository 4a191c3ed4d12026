// GGUF reading and the host-side repacks of crates/gem/src/q8.rs (see host.hpp).
#include "host.hpp"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <limits>

#include "../../include/gem.h"

namespace gem {

namespace {

struct Cursor {
  const uint8_t* b;
  size_t n, p = 0;
  bool short_ = false;
  bool take(size_t k, const uint8_t** out) {
    if (short_ || p + k > n || p + k < p) {
      short_ = true;
      return false;
    }
    *out = b + p;
    p += k;
    return true;
  }
  template <typename T>
  T get() {
    const uint8_t* s;
    T v{};
    if (take(sizeof(T), &s)) std::memcpy(&v, s, sizeof(T));
    return v;
  }
  std::string str() {
    uint64_t k = get<uint64_t>();
    const uint8_t* s;
    if (k > (1ull << 32) || !take((size_t)k, &s)) {
      short_ = true;
      return std::string();
    }
    return std::string((const char*)s, (size_t)k);
  }
  // gguf.rs:59-88 value types 0..12
  GgufValue value(uint32_t ty, int depth = 0) {
    GgufValue v;
    switch (ty) {
      case 0: v.kind = GgufValue::U; v.u = get<uint8_t>(); break;
      case 1: v.kind = GgufValue::I; v.i = get<int8_t>(); break;
      case 2: v.kind = GgufValue::U; v.u = get<uint16_t>(); break;
      case 3: v.kind = GgufValue::I; v.i = get<int16_t>(); break;
      case 4: v.kind = GgufValue::U; v.u = get<uint32_t>(); break;
      case 5: v.kind = GgufValue::I; v.i = get<int32_t>(); break;
      case 6: v.kind = GgufValue::F; v.f = get<float>(); break;
      case 7: v.kind = GgufValue::B; v.b = get<uint8_t>() != 0; break;
      case 8: v.kind = GgufValue::S; v.s = str(); break;
      case 9: {
        if (depth > 4) throw Error(GEM_E_FORMAT, "GGUF: nested arrays too deep");
        uint32_t t = get<uint32_t>();
        uint64_t cnt = get<uint64_t>();
        for (uint64_t k = 0; k < cnt && !short_; ++k) (void)value(t, depth + 1);
        v.kind = GgufValue::ARR;
        break;
      }
      case 10: v.kind = GgufValue::U; v.u = get<uint64_t>(); break;
      case 11: v.kind = GgufValue::I; v.i = get<int64_t>(); break;
      case 12: v.kind = GgufValue::F; v.f = get<double>(); break;
      default:
        if (!short_) throw Error(GEM_E_FORMAT, "GGUF: unknown value type " + std::to_string(ty));
    }
    return v;
  }
};

}  // namespace

Gguf::Gguf(const std::string& path) : path_(path) {
  fd_ = ::open(path.c_str(), O_RDONLY);
  if (fd_ < 0) throw Error(GEM_E_IO, path + ": cannot open");
  struct stat st;
  if (fstat(fd_, &st) != 0) throw Error(GEM_E_IO, path + ": cannot stat");
  size_ = (uint64_t)st.st_size;
  // Read the header in growing chunks until it parses (gguf.rs:93-107).
  std::vector<uint8_t> data;
  size_t chunk = 1 << 22;
  for (;;) {
    size_t old = data.size();
    data.resize(old + chunk);
    ssize_t n = ::pread(fd_, data.data() + old, chunk, (off_t)old);
    if (n < 0) throw Error(GEM_E_IO, path + ": read error");
    data.resize(old + (size_t)n);
    if (parse(data)) break;
    if (n == 0) {
      ::close(fd_);
      fd_ = -1;
      throw Error(GEM_E_IO, path + ": truncated GGUF header");
    }
  }
}

Gguf::~Gguf() {
  if (fd_ >= 0) ::close(fd_);
}

bool Gguf::parse(const std::vector<uint8_t>& data) {  // gguf.rs:109-143
  Cursor r{data.data(), data.size()};
  const uint8_t* magic;
  if (!r.take(4, &magic)) return false;
  if (std::memcmp(magic, "GGUF", 4) != 0) throw Error(GEM_E_FORMAT, path_ + ": not a GGUF file");
  uint32_t version = r.get<uint32_t>();
  if (!r.short_ && (version < 2 || version > 3)) throw Error(GEM_E_FORMAT, path_ + ": unsupported GGUF version " + std::to_string(version));
  uint64_t nt = r.get<uint64_t>(), nkv = r.get<uint64_t>();
  if (r.short_) return false;
  if (nt > (1u << 24) || nkv > (1u << 24)) throw Error(GEM_E_FORMAT, path_ + ": implausible GGUF counts");
  std::map<std::string, GgufValue> meta;
  for (uint64_t k = 0; k < nkv; ++k) {
    std::string key = r.str();
    uint32_t ty = r.get<uint32_t>();
    GgufValue v = r.value(ty);
    if (r.short_) return false;
    meta[key] = v;
  }
  std::map<std::string, GgufTensor> ts;
  for (uint64_t k = 0; k < nt; ++k) {
    std::string name = r.str();
    uint32_t nd = r.get<uint32_t>();
    if (nd > 4) throw Error(GEM_E_FORMAT, name + ": too many dimensions");
    GgufTensor t;
    for (uint32_t d = 0; d < nd; ++d) t.dims.push_back(r.get<uint64_t>());
    t.type = r.get<uint32_t>();
    t.offset = r.get<uint64_t>();
    if (r.short_) return false;
    ts[name] = t;
  }
  uint64_t align = 32;
  auto it = meta.find("general.alignment");
  if (it != meta.end() && it->second.kind == GgufValue::U && it->second.u > 0) align = it->second.u;
  meta_ = std::move(meta);
  tensors_ = std::move(ts);
  base_ = (r.p + align - 1) / align * align;
  return true;
}

const GgufTensor& Gguf::info(const std::string& name) const {
  auto it = tensors_.find(name);
  if (it == tensors_.end()) throw Error(GEM_E_FORMAT, "missing tensor " + name);
  return it->second;
}

std::vector<uint8_t> Gguf::read(const std::string& name) const {  // gguf.rs:145-159
  const GgufTensor& t = info(name);
  // element count and byte size in checked arithmetic: a crafted header cannot wrap them around
  uint64_t n = 1;
  for (uint64_t d : t.dims)
    if (__builtin_mul_overflow(n, d, &n)) throw Error(GEM_E_FORMAT, name + ": dimensions overflow");
  uint64_t bytes;
  bool over = false;
  switch (t.type) {
    case GGUF_F32: over = __builtin_mul_overflow(n, (uint64_t)4, &bytes); break;
    case GGUF_F16: over = __builtin_mul_overflow(n, (uint64_t)2, &bytes); break;
    case GGUF_Q8_0: over = __builtin_mul_overflow(n / 32, (uint64_t)34, &bytes); break;
    case GGUF_Q4_0: over = __builtin_mul_overflow(n / 32, (uint64_t)18, &bytes); break;
    default: throw Error(GEM_E_FORMAT, name + ": unsupported tensor type " + std::to_string(t.type));
  }
  if (over) throw Error(GEM_E_FORMAT, name + ": tensor size overflows");
  if (base_ > size_ || t.offset > size_ - base_ || bytes > size_ - base_ - t.offset)
    throw Error(GEM_E_IO, name + ": tensor data past end of file");
  std::vector<uint8_t> buf(bytes);
  size_t got = 0;
  while (got < bytes) {
    ssize_t k = ::pread(fd_, buf.data() + got, bytes - got, (off_t)(base_ + t.offset + got));
    if (k <= 0) throw Error(GEM_E_IO, name + ": short read");
    got += (size_t)k;
  }
  return buf;
}

std::vector<float> Gguf::f32s(const std::string& name) const {
  if (info(name).type != GGUF_F32) throw Error(GEM_E_FORMAT, name + ": expected F32");
  auto b = read(name);
  std::vector<float> v(b.size() / 4);
  std::memcpy(v.data(), b.data(), b.size());
  return v;
}
std::vector<float> Gguf::f32s_or_empty(const std::string& name) const { return has(name) ? f32s(name) : std::vector<float>(); }
const std::string& Gguf::text(const std::string& key) const {
  auto it = meta_.find(key);
  if (it == meta_.end() || it->second.kind != GgufValue::S) throw Error(GEM_E_FORMAT, "missing string " + key);
  return it->second.s;
}
bool Gguf::flag(const std::string& key) const {
  auto it = meta_.find(key);
  return it != meta_.end() && it->second.kind == GgufValue::B && it->second.b;
}
uint64_t Gguf::u(const std::string& key) const {
  auto it = meta_.find(key);
  if (it != meta_.end() && it->second.kind == GgufValue::U) return it->second.u;
  if (it != meta_.end() && it->second.kind == GgufValue::I && it->second.i >= 0) return (uint64_t)it->second.i;
  throw Error(GEM_E_FORMAT, "missing integer " + key);
}
uint64_t Gguf::u_or(const std::string& key, uint64_t def) const { return meta_.count(key) ? u(key) : def; }
float Gguf::f(const std::string& key) const {
  auto it = meta_.find(key);
  if (it == meta_.end() || it->second.kind != GgufValue::F) throw Error(GEM_E_FORMAT, "missing float " + key);
  return (float)it->second.f;
}

// ---------------------------------------------------------------------------------------------
float f16_value(uint16_t x) {  // q8.rs:17-26 (exponent 31 decodes as +-inf, NaN included)
  float sign = (x & 0x8000) ? -1.0f : 1.0f;
  int e = (x >> 10) & 0x1f;
  float mant = (float)(x & 0x3ff);
  if (e == 0) return sign * mant * std::ldexp(1.0f, -24);
  if (e == 31) return sign * std::numeric_limits<float>::infinity();
  return sign * (1.0f + mant / 1024.0f) * std::ldexp(1.0f, e - 15);
}

float HostMat::scale(size_t i) const { return scale_f32() ? s32[i] : f16_value(s16[i]); }

HostMat load_mat(const Gguf& g, const std::string& name) {
  const GgufTensor& t = g.info(name);
  if (t.dims.size() < 2) throw Error(GEM_E_FORMAT, name + ": not a matrix");
  HostMat m;
  m.cols = (size_t)t.dims[0];
  m.rows = (size_t)t.dims[1];
  for (size_t k = 2; k < t.dims.size(); ++k) m.rows *= (size_t)t.dims[k];
  if (m.cols % 32 != 0) throw Error(GEM_E_FORMAT, name + ": columns not a multiple of 32");
  auto raw = g.read(name);
  size_t nb = m.rows * m.cols / 32;
  if (t.type == GGUF_Q8_0) {  // q8.rs:29-39
    m.bits = 8;
    m.q.resize(m.rows * m.cols);
    m.s16.resize(nb);
    for (size_t b = 0; b < nb; ++b) {
      const uint8_t* blk = raw.data() + b * 34;
      m.s16[b] = (uint16_t)(blk[0] | (blk[1] << 8));
      std::memcpy(&m.q[b * 32], blk + 2, 32);
    }
  } else if (t.type == GGUF_Q4_0) {  // q8.rs:42-52
    m.bits = 4;
    m.q.resize(m.rows * m.cols / 2);
    m.s16.resize(nb);
    for (size_t b = 0; b < nb; ++b) {
      const uint8_t* blk = raw.data() + b * 18;
      m.s16[b] = (uint16_t)(blk[0] | (blk[1] << 8));
      std::memcpy(&m.q[b * 16], blk + 2, 16);
    }
  } else if (t.type == GGUF_F16) {  // q8.rs:55-58
    m.bits = 16;
    m.q = std::move(raw);
  } else {
    throw Error(GEM_E_FORMAT, name + ": unsupported tensor type " + std::to_string(t.type));
  }
  return m;
}

static int8_t round_i8(float v) {  // Rust f32::round (half away) + saturating `as i8`
  float r = std::round(v);
  if (std::isnan(r)) return 0;
  if (r > 127.0f) return 127;
  if (r < -128.0f) return -128;
  return (int8_t)r;
}

HostMat to_q8(const HostMat& m) {  // q8.rs:129-145
  if (m.bits == 8) return m;
  if (m.bits != 16) throw Error(GEM_E_ARG, "requantize to 8 bits needs an F16 or Q8_0 matrix");
  HostMat o;
  o.bits = 8, o.rows = m.rows, o.cols = m.cols;
  size_t nb = m.rows * m.cols / 32;
  o.q.resize(m.rows * m.cols);
  o.s32.resize(nb);
  const uint16_t* src = (const uint16_t*)m.q.data();
  float w[32];
  for (size_t b = 0; b < nb; ++b) {
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) {
      w[j] = f16_value(src[b * 32 + j]);
      amax = std::fmax(amax, std::fabs(w[j]));
    }
    float d = amax / 127.0f;
    float inv = d > 0.0f ? 1.0f / d : 0.0f;
    for (int j = 0; j < 32; ++j) o.q[b * 32 + j] = (uint8_t)round_i8(w[j] * inv);
    o.s32[b] = d;
  }
  return o;
}

HostMat to_q4(const HostMat& m) {  // q8.rs:148-165
  if (m.bits == 16) return to_q4(to_q8(m));
  if (m.bits == 4) return m;
  HostMat o;
  o.bits = 4, o.rows = m.rows, o.cols = m.cols;
  size_t nb = m.rows * m.cols / 32;
  o.q.resize(m.rows * m.cols / 2);
  o.s32.resize(nb);
  float w[32];
  uint8_t n[32];
  for (size_t b = 0; b < nb; ++b) {
    float scale = m.scale(b), amax = 0.0f;
    for (int j = 0; j < 32; ++j) {
      w[j] = (float)(int8_t)m.q[b * 32 + j] * scale;
      amax = std::fmax(amax, std::fabs(w[j]));
    }
    float d = amax / 7.0f;
    float inv = d > 0.0f ? 1.0f / d : 0.0f;
    for (int j = 0; j < 32; ++j) {
      float r = std::round(w[j] * inv);
      r = r < -8.0f ? -8.0f : (r > 7.0f ? 7.0f : r);
      n[j] = (uint8_t)((int)r + 8);
    }
    for (int j = 0; j < 16; ++j) o.q[b * 16 + j] = (uint8_t)(n[j] | (n[j + 16] << 4));
    o.s32[b] = d;
  }
  return o;
}

HostMat concat_rows(const std::vector<const HostMat*>& parts) {
  HostMat o = *parts[0];
  for (size_t i = 1; i < parts.size(); ++i) {
    const HostMat& p = *parts[i];
    if (p.bits != o.bits || p.cols != o.cols || p.scale_f32() != o.scale_f32())
      throw Error(GEM_E_FORMAT, "projection matrices of one layer must share a type and width");
    o.rows += p.rows;
    o.q.insert(o.q.end(), p.q.begin(), p.q.end());
    o.s16.insert(o.s16.end(), p.s16.begin(), p.s16.end());
    o.s32.insert(o.s32.end(), p.s32.begin(), p.s32.end());
  }
  return o;
}

size_t canonical_bytes(const HostMat& m) { return m.q.size() + m.s16.size() * 2 + m.s32.size() * 4; }

}  // namespace gem
