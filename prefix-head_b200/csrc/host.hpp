// Host-side model loading: a GGUF reader and the weight repacks / requantizations of
// crates/gem/src/q8.rs, producing the planes the device kernels read.
#pragma once
#include <cstddef>
#include <cstdint>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace gem {

// Error carrying a gem_status code across the C++ layer; converted at the C ABI.
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

constexpr uint32_t GGUF_F32 = 0, GGUF_F16 = 1, GGUF_Q4_0 = 2, GGUF_Q8_0 = 8;  // gguf.rs:19-22

struct GgufValue {
  enum Kind { U, I, F, B, S, ARR } kind = U;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  bool b = false;
  std::string s;
};
struct GgufTensor {
  uint32_t type = 0;
  std::vector<uint64_t> dims;  // dims[0] = columns, dims[1] = rows (model.rs:74)
  uint64_t offset = 0;
};

// GGUF v2/v3 container (crates/gem/src/gguf.rs:93-203): header parsed once, tensors read on demand.
class Gguf {
 public:
  explicit Gguf(const std::string& path);
  ~Gguf();
  Gguf(const Gguf&) = delete;
  Gguf& operator=(const Gguf&) = delete;
  bool has(const std::string& name) const { return tensors_.count(name) > 0; }
  const GgufTensor& info(const std::string& name) const;
  std::vector<uint8_t> read(const std::string& name) const;
  std::vector<float> f32s(const std::string& name) const;
  std::vector<float> f32s_or_empty(const std::string& name) const;
  const std::string& text(const std::string& key) const;
  bool flag(const std::string& key) const;
  uint64_t u(const std::string& key) const;
  uint64_t u_or(const std::string& key, uint64_t def) const;
  float f(const std::string& key) const;

 private:
  bool parse(const std::vector<uint8_t>& data);
  int fd_ = -1;
  std::string path_;
  uint64_t size_ = 0, base_ = 0;
  std::map<std::string, GgufValue> meta_;
  std::map<std::string, GgufTensor> tensors_;
};

// Host copy of a matrix in device layout (q8.rs:9-15): q = int8 / nibble / f16 bytes; scales either
// f16 bits (as in the GGUF file) or f32 (after requantization).
struct HostMat {
  int bits = 8;
  size_t rows = 0, cols = 0;
  std::vector<uint8_t> q;
  std::vector<uint16_t> s16;
  std::vector<float> s32;
  bool scale_f32() const { return !s32.empty(); }
  size_t row_bytes() const { return cols * (size_t)bits / 8; }
  float scale(size_t i) const;
};

float f16_value(uint16_t x);                                   // q8.rs:17-26
HostMat load_mat(const Gguf& g, const std::string& name);      // model.rs:71-79 + q8.rs:29-58
HostMat to_q8(const HostMat& m);                               // q8.rs:129-145
HostMat to_q4(const HostMat& m);                               // q8.rs:148-165
HostMat concat_rows(const std::vector<const HostMat*>& parts); // stacks matrices of one type
size_t canonical_bytes(const HostMat& m);                      // bytes of the planes as stored

}  // namespace gem
