// TEST INFRASTRUCTURE ONLY — the oracle (see gem_oracle.h for what it is and what pins it).
// A CPU restatement of prefix-head's crates/gem scoring path. Each function cites the reference
// file:line it follows. Built with -ffp-contract=off and without -ffast-math: Rust neither fuses a*b+c
// nor reassociates sums, so neither may this file. SIMD paths use the same intrinsic sequences as the
// reference (GCC's _mm512_reduce_add_ps reduces in the same halving order as Rust's).
#include "gem_oracle.h"

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <functional>
#include <limits>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <unistd.h>
#include <vector>

namespace {

thread_local std::string g_err;
struct Fail : std::runtime_error {
  using std::runtime_error::runtime_error;
};
[[noreturn]] void fail(const std::string& m) { throw Fail(m); }

// ---------------------------------------------------------------------------------------------
// nn::fast (crates/nn/src/fast.rs:126-132, 78-81): the reference's own exp and tanh.
// ---------------------------------------------------------------------------------------------
float clampf(float x, float lo, float hi) {  // Rust f32::clamp: NaN passes through
  if (x < lo) x = lo;
  if (x > hi) x = hi;
  return x;
}
float exp_fast(float x) {  // fast.rs:126-132
  const float log2e = 1.44269504088896340736f;
  float t = clampf(x * log2e, -126.0f, 126.0f);
  float n = std::floor(t + 0.5f);
  float f = t - n;
  float p = 1.0f + f * (6.931471806e-01f + f * (2.402265070e-01f + f * (5.550410866e-02f +
            f * (9.618129108e-03f + f * (1.333355815e-03f + f * 1.540353039e-04f)))));
  uint32_t bits = (uint32_t)(((int32_t)n + 127) << 23);
  float s;
  std::memcpy(&s, &bits, 4);
  return p * s;
}
float tanh_fast(float x) {  // fast.rs:78-81
  float e = exp_fast(2.0f * clampf(x, -10.0f, 10.0f));
  return (e - 1.0f) / (e + 1.0f);
}

// lse (main.rs:118-121): fold max, then a sequential f32 sum of std exp, then ln.
float lse(const float* v, size_t n) {
  float mx = -std::numeric_limits<float>::infinity();
  for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, v[i]);
  float s = 0.0f;
  for (size_t i = 0; i < n; ++i) s += std::exp(v[i] - mx);
  return mx + std::log(s);
}
// argmax (lean.rs:36-38): the first index of the maximum.
size_t argmax(const float* v, size_t n) {
  size_t b = 0;
  for (size_t i = 0; i < n; ++i)
    if (v[i] > v[b]) b = i;
  return b;
}

// q8.rs:17-26 — f16 decoding as the reference writes it (exponent 31 is ±inf for NaN too).
float f16(uint16_t x) {
  float sign = (x & 0x8000) ? -1.0f : 1.0f;
  int exp = (x >> 10) & 0x1f;
  float mant = (float)(x & 0x3ff);
  if (exp == 0) return sign * mant * std::ldexp(1.0f, -24);
  if (exp == 31) return sign * std::numeric_limits<float>::infinity();
  return sign * (1.0f + mant / 1024.0f) * std::ldexp(1.0f, exp - 15);
}

// Rust `f32::round` (half away from zero) and the saturating `as i8` cast.
int8_t round_i8(float v) {
  float r = std::round(v);
  if (std::isnan(r)) return 0;
  if (r > 127.0f) return 127;
  if (r < -128.0f) return -128;
  return (int8_t)r;
}

// ---------------------------------------------------------------------------------------------
// Pool (pool.rs): persistent spinning workers; the caller runs t = 0. Workers spin 2^16 times, then
// yield, then sleep on a condition variable once idle for 50 ms.
// ---------------------------------------------------------------------------------------------
class Pool {
 public:
  explicit Pool(int n) : n_(n < 1 ? 1 : n) {  // pool.rs:35-73
    for (int t = 1; t < n_; ++t) th_.emplace_back([this, t] { worker(t); });
  }
  ~Pool() {  // pool.rs:102-109
    stop_.store(true, std::memory_order_release);
    advance();
    for (auto& t : th_) t.join();
  }
  int threads() const { return n_; }
  // pool.rs:80-89
  void run(const std::function<void(int)>& f) {
    job_ = &f;
    done_.store(0, std::memory_order_release);
    advance();
    f(0);
    while (done_.load(std::memory_order_acquire) < (size_t)(n_ - 1)) _mm_pause();
  }

 private:
  void advance() {  // pool.rs:93-99
    gen_.fetch_add(1, std::memory_order_seq_cst);
    if (asleep_.load(std::memory_order_seq_cst) > 0) {
      std::lock_guard<std::mutex> g(mu_);
      cv_.notify_all();
    }
  }
  void worker(int t) {
    size_t seen = 0;
    for (;;) {
      uint32_t spins = 0;
      bool have_since = false;
      auto since = std::chrono::steady_clock::now();
      while (gen_.load(std::memory_order_acquire) == seen) {
        _mm_pause();
        if (++spins > (1u << 16)) {
          std::this_thread::yield();
          if (!have_since) {
            since = std::chrono::steady_clock::now();
            have_since = true;
          }
          if (std::chrono::steady_clock::now() - since > std::chrono::milliseconds(50)) {
            asleep_.fetch_add(1, std::memory_order_seq_cst);
            std::unique_lock<std::mutex> g(mu_);
            while (gen_.load(std::memory_order_seq_cst) == seen) cv_.wait(g);
            g.unlock();
            asleep_.fetch_sub(1, std::memory_order_seq_cst);
          }
        }
      }
      seen = gen_.load(std::memory_order_acquire);
      if (stop_.load(std::memory_order_acquire)) return;
      (*job_)(t);
      done_.fetch_add(1, std::memory_order_acq_rel);
    }
  }
  int n_;
  std::vector<std::thread> th_;
  std::atomic<size_t> gen_{0}, done_{0}, asleep_{0};
  std::atomic<bool> stop_{false};
  std::mutex mu_;
  std::condition_variable cv_;
  const std::function<void(int)>* job_ = nullptr;
};

// ---------------------------------------------------------------------------------------------
// q8.rs — matrices, activation quantization, row dots, matvec.
// ---------------------------------------------------------------------------------------------
enum Isa { AVX512, AVX2, SCALAR };

Isa detect_isa() {  // q8.rs:395-408
  const char* e = std::getenv("GEM_ISA");
  if (e && std::string(e) == "avx2") return AVX2;
  if (e && std::string(e) == "scalar") return SCALAR;
  __builtin_cpu_init();
  if (__builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw")) return AVX512;
  if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) return AVX2;
  return SCALAR;
}
Isa parse_isa(const char* s) {
  if (!s || !*s) return detect_isa();
  std::string v(s);
  if (v == "avx512") return AVX512;
  if (v == "avx2") return AVX2;
  if (v == "scalar") return SCALAR;
  fail("unknown isa " + v);
}
const char* isa_name(Isa i) { return i == AVX512 ? "avx512" : i == AVX2 ? "avx2" : "scalar"; }

struct Mat {  // q8.rs:9-15
  std::vector<int8_t> q;
  std::vector<float> s;
  size_t rows = 0, cols = 0;
  int bits = 8;

  size_t row_bytes() const { return cols * (size_t)bits / 8; }  // q8.rs:108-110
  size_t bytes() const { return q.size() + s.size() * 4; }       // q8.rs:171-173

  static Mat from_q8_0(const uint8_t* raw, size_t len, size_t rows, size_t cols) {  // q8.rs:29-39
    size_t nb = rows * cols / 32;
    if (len != nb * 34) fail("Q8_0 size mismatch");
    Mat m;
    m.rows = rows, m.cols = cols, m.bits = 8;
    m.q.resize(rows * cols);
    m.s.resize(nb);
    for (size_t b = 0; b < nb; ++b) {
      const uint8_t* blk = raw + b * 34;
      m.s[b] = f16((uint16_t)(blk[0] | (blk[1] << 8)));
      std::memcpy(&m.q[b * 32], blk + 2, 32);
    }
    return m;
  }
  static Mat from_q4_0(const uint8_t* raw, size_t len, size_t rows, size_t cols) {  // q8.rs:42-52
    size_t nb = rows * cols / 32;
    if (len != nb * 18) fail("Q4_0 size mismatch");
    Mat m;
    m.rows = rows, m.cols = cols, m.bits = 4;
    m.q.resize(rows * cols / 2);
    m.s.resize(nb);
    for (size_t b = 0; b < nb; ++b) {
      const uint8_t* blk = raw + b * 18;
      m.s[b] = f16((uint16_t)(blk[0] | (blk[1] << 8)));
      std::memcpy(&m.q[b * 16], blk + 2, 16);
    }
    return m;
  }
  static Mat from_f16(const uint8_t* raw, size_t len, size_t rows, size_t cols) {  // q8.rs:55-58
    if (len != rows * cols * 2) fail("F16 size mismatch");
    Mat m;
    m.rows = rows, m.cols = cols, m.bits = 16;
    m.q.assign((const int8_t*)raw, (const int8_t*)raw + len);
    return m;
  }

  void permute_rows(const std::vector<uint32_t>& order) {  // q8.rs:65-91
    if (order.size() != rows) fail("permute_rows: order length");
    size_t c = row_bytes(), b = s.empty() ? 0 : cols / 32;
    std::vector<char> done(rows, 0);
    std::vector<int8_t> tq(c);
    std::vector<float> ts(b);
    for (size_t start = 0; start < rows; ++start) {
      if (done[start] || order[start] == start) {
        done[start] = 1;
        continue;
      }
      std::memcpy(tq.data(), &q[start * c], c);
      if (b) std::memcpy(ts.data(), &s[start * b], b * 4);
      size_t i = start;
      for (;;) {
        done[i] = 1;
        size_t src = order[i];
        if (src == start) {
          std::memcpy(&q[i * c], tq.data(), c);
          if (b) std::memcpy(&s[i * b], ts.data(), b * 4);
          break;
        }
        std::memmove(&q[i * c], &q[src * c], c);
        if (b) std::memmove(&s[i * b], &s[src * b], b * 4);
        i = src;
      }
    }
  }

  Mat gather(const uint32_t* ids, size_t n) const {  // q8.rs:94-106
    size_t c = row_bytes(), b = cols / 32;
    Mat m;
    m.rows = n, m.cols = cols, m.bits = bits;
    m.q.reserve(n * c);
    for (size_t k = 0; k < n; ++k) {
      size_t r = ids[k];
      m.q.insert(m.q.end(), q.begin() + r * c, q.begin() + (r + 1) * c);
      if (!s.empty()) m.s.insert(m.s.end(), s.begin() + r * b, s.begin() + (r + 1) * b);
    }
    return m;
  }

  float weight(size_t r, size_t j) const {  // q8.rs:112-126
    size_t c = cols;
    if (bits == 16) {
      size_t i = (r * c + j) * 2;
      return f16((uint16_t)((uint8_t)q[i] | ((uint8_t)q[i + 1] << 8)));
    }
    float scale = s[(r * c + j) / 32];
    if (bits == 8) return (float)q[r * c + j] * scale;
    size_t blk = j / 32, k = j % 32;
    uint8_t byte = (uint8_t)q[r * c / 2 + blk * 16 + k % 16];
    uint8_t nib = k < 16 ? (byte & 15) : (byte >> 4);
    return (float)((int)nib - 8) * scale;
  }

  Mat to_q8() const {  // q8.rs:129-145
    if (bits == 8) return *this;
    if (bits != 16) fail("to_q8 from bits " + std::to_string(bits));
    Mat m;
    m.rows = rows, m.cols = cols, m.bits = 8;
    m.q.reserve(rows * cols);
    m.s.reserve(rows * cols / 32);
    float w[32];
    for (size_t blk = 0; blk < q.size() / 64; ++blk) {
      const int8_t* p = &q[blk * 64];
      for (int j = 0; j < 32; ++j) w[j] = f16((uint16_t)((uint8_t)p[2 * j] | ((uint8_t)p[2 * j + 1] << 8)));
      float amax = 0.0f;
      for (int j = 0; j < 32; ++j) amax = std::fmax(amax, std::fabs(w[j]));
      float d = amax / 127.0f;
      float inv = d > 0.0f ? 1.0f / d : 0.0f;
      for (int j = 0; j < 32; ++j) m.q.push_back(round_i8(w[j] * inv));
      m.s.push_back(d);
    }
    return m;
  }

  Mat to_q4() const {  // q8.rs:148-165
    if (bits == 16) return to_q8().to_q4();
    if (bits != 8) fail("to_q4 from bits " + std::to_string(bits));
    Mat m;
    m.rows = rows, m.cols = cols, m.bits = 4;
    m.q.reserve(q.size() / 2);
    m.s.reserve(s.size());
    float w[32];
    uint8_t n[32];
    for (size_t blk = 0; blk < s.size(); ++blk) {
      float scale = s[blk];
      for (int j = 0; j < 32; ++j) w[j] = (float)q[blk * 32 + j] * scale;
      float amax = 0.0f;
      for (int j = 0; j < 32; ++j) amax = std::fmax(amax, std::fabs(w[j]));
      float d = amax / 7.0f;
      float inv = d > 0.0f ? 1.0f / d : 0.0f;
      for (int j = 0; j < 32; ++j) n[j] = (uint8_t)((int)clampf(std::round(w[j] * inv), -8.0f, 7.0f) + 8);
      for (int j = 0; j < 16; ++j) m.q.push_back((int8_t)(n[j] | (uint8_t)(n[j + 16] << 4)));
      m.s.push_back(d);
    }
    return m;
  }

  std::vector<float> row_f32(size_t r) const {  // q8.rs:167-169
    std::vector<float> v(cols);
    for (size_t j = 0; j < cols; ++j) v[j] = weight(r, j);
    return v;
  }
};

struct Act {  // q8.rs:176-246
  std::vector<int8_t> q;
  std::vector<float> s, x;
  explicit Act(size_t n = 0) : q(n), s(n / 32), x(n) {}

  void quantize(const float* in, size_t n, Isa isa) {  // q8.rs:187-203
    if (x.size() != n) fail("Act::quantize length");
    std::memcpy(x.data(), in, n * 4);
    if (isa == AVX512) return quantize_avx512(in, n);
    if (isa == AVX2) return quantize_avx2(in, n);
    for (size_t b = 0; b < n / 32; ++b) {
      const float* c = in + b * 32;
      float amax = 0.0f;
      for (int j = 0; j < 32; ++j) amax = std::fmax(amax, std::fabs(c[j]));
      float d = amax / 127.0f;
      float inv = d > 0.0f ? 1.0f / d : 0.0f;
      s[b] = d;
      for (int j = 0; j < 32; ++j) q[b * 32 + j] = round_i8(c[j] * inv);
    }
  }

  __attribute__((target("avx512f,avx512bw"))) void quantize_avx512(const float* in, size_t n) {  // q8.rs:207-222
    for (size_t b = 0; b < n / 32; ++b) {
      __m512 lo = _mm512_loadu_ps(in + b * 32);
      __m512 hi = _mm512_loadu_ps(in + b * 32 + 16);
      float amax = _mm512_reduce_max_ps(_mm512_max_ps(_mm512_abs_ps(lo), _mm512_abs_ps(hi)));
      float d = amax / 127.0f;
      __m512 inv = _mm512_set1_ps(d > 0.0f ? 1.0f / d : 0.0f);
      s[b] = d;
      __m128i* out = (__m128i*)(q.data() + b * 32);
      _mm_storeu_si128(out, _mm512_cvtepi32_epi8(_mm512_cvtps_epi32(_mm512_mul_ps(lo, inv))));
      _mm_storeu_si128(out + 1, _mm512_cvtepi32_epi8(_mm512_cvtps_epi32(_mm512_mul_ps(hi, inv))));
    }
  }

  __attribute__((target("avx2"))) void quantize_avx2(const float* in, size_t n) {  // q8.rs:224-245
    __m256 sign = _mm256_set1_ps(-0.0f);
    for (size_t b = 0; b < n / 32; ++b) {
      __m256 v[4];
      for (int i = 0; i < 4; ++i) v[i] = _mm256_loadu_ps(in + b * 32 + i * 8);
      __m256 m = _mm256_setzero_ps();
      for (int i = 0; i < 4; ++i) m = _mm256_max_ps(m, _mm256_andnot_ps(sign, v[i]));
      float lanes[8];
      _mm256_storeu_ps(lanes, m);
      float a = 0.0f;
      for (int i = 0; i < 8; ++i) a = std::fmax(a, lanes[i]);
      float d = a / 127.0f;
      __m256 inv = _mm256_set1_ps(d > 0.0f ? 1.0f / d : 0.0f);
      s[b] = d;
      int32_t ints[32];
      for (int i = 0; i < 4; ++i) _mm256_storeu_si256((__m256i*)(ints + i * 8), _mm256_cvtps_epi32(_mm256_mul_ps(v[i], inv)));
      for (int j = 0; j < 32; ++j) q[b * 32 + j] = (int8_t)ints[j];
    }
  }
};

float dot_scalar(const int8_t* wq, const float* ws, const Act& a, size_t cols) {  // q8.rs:248-255
  float acc = 0.0f;
  for (size_t b = 0; b < cols / 32; ++b) {
    int32_t s = 0;
    for (int j = 0; j < 32; ++j) s += (int32_t)wq[b * 32 + j] * (int32_t)a.q[b * 32 + j];
    acc += (float)s * ws[b] * a.s[b];
  }
  return acc;
}
__attribute__((target("avx512f,avx512bw"))) float dot_avx512(const int8_t* wq, const float* ws, const Act& a, size_t cols) {  // q8.rs:257-270
  __m512 acc = _mm512_setzero_ps();
  for (size_t b = 0; b < cols / 32; ++b) {
    __m512i w = _mm512_cvtepi8_epi16(_mm256_loadu_si256((const __m256i*)(wq + b * 32)));
    __m512i x = _mm512_cvtepi8_epi16(_mm256_loadu_si256((const __m256i*)(a.q.data() + b * 32)));
    __m512 p = _mm512_cvtepi32_ps(_mm512_madd_epi16(w, x));
    acc = _mm512_fmadd_ps(p, _mm512_set1_ps(ws[b] * a.s[b]), acc);
  }
  return _mm512_reduce_add_ps(acc);
}
__attribute__((target("avx2,fma"))) float hsum256(__m256 acc) {  // q8.rs:286-290
  __m128 lo = _mm256_castps256_ps128(acc);
  __m128 hi = _mm256_extractf128_ps(acc, 1);
  __m128 s = _mm_add_ps(lo, hi);
  s = _mm_hadd_ps(s, s);
  return _mm_cvtss_f32(_mm_hadd_ps(s, s));
}
__attribute__((target("avx2,fma"))) float dot_avx2(const int8_t* wq, const float* ws, const Act& a, size_t cols) {  // q8.rs:272-292
  __m256 acc = _mm256_setzero_ps();
  for (size_t b = 0; b < cols / 32; ++b)
    for (int h = 0; h < 2; ++h) {
      size_t o = b * 32 + h * 16;
      __m256i w = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(wq + o)));
      __m256i x = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(a.q.data() + o)));
      __m256 p = _mm256_cvtepi32_ps(_mm256_madd_epi16(w, x));
      acc = _mm256_fmadd_ps(p, _mm256_set1_ps(ws[b] * a.s[b]), acc);
    }
  return hsum256(acc);
}
float dot4_scalar(const int8_t* wq, const float* ws, const Act& a, size_t cols) {  // q8.rs:294-305
  float acc = 0.0f;
  for (size_t b = 0; b < cols / 32; ++b) {
    int32_t s = 0;
    for (int j = 0; j < 16; ++j) {
      uint8_t byte = (uint8_t)wq[b * 16 + j];
      s += ((int32_t)(byte & 15) - 8) * (int32_t)a.q[b * 32 + j] + ((int32_t)(byte >> 4) - 8) * (int32_t)a.q[b * 32 + j + 16];
    }
    acc += (float)s * ws[b] * a.s[b];
  }
  return acc;
}
__attribute__((target("avx512f,avx512bw,avx2"))) float dot4_avx512(const int8_t* wq, const float* ws, const Act& a, size_t cols) {  // q8.rs:307-326
  __m512 acc = _mm512_setzero_ps();
  __m128i mask = _mm_set1_epi8(15);
  __m256i eight = _mm256_set1_epi8(8);
  for (size_t b = 0; b < cols / 32; ++b) {
    __m128i raw = _mm_loadu_si128((const __m128i*)(wq + b * 16));
    __m128i lo = _mm_and_si128(raw, mask);
    __m128i hi = _mm_and_si128(_mm_srli_epi16(raw, 4), mask);
    __m256i w8 = _mm256_sub_epi8(_mm256_set_m128i(hi, lo), eight);
    __m512i w = _mm512_cvtepi8_epi16(w8);
    __m512i x = _mm512_cvtepi8_epi16(_mm256_loadu_si256((const __m256i*)(a.q.data() + b * 32)));
    __m512 p = _mm512_cvtepi32_ps(_mm512_madd_epi16(w, x));
    acc = _mm512_fmadd_ps(p, _mm512_set1_ps(ws[b] * a.s[b]), acc);
  }
  return _mm512_reduce_add_ps(acc);
}
__attribute__((target("avx2,fma"))) float dot4_avx2(const int8_t* wq, const float* ws, const Act& a, size_t cols) {  // q8.rs:328-352
  __m256 acc = _mm256_setzero_ps();
  __m128i mask = _mm_set1_epi8(15);
  __m128i eight = _mm_set1_epi8(8);
  for (size_t b = 0; b < cols / 32; ++b) {
    __m128i raw = _mm_loadu_si128((const __m128i*)(wq + b * 16));
    __m128i lo = _mm_sub_epi8(_mm_and_si128(raw, mask), eight);
    __m128i hi = _mm_sub_epi8(_mm_and_si128(_mm_srli_epi16(raw, 4), mask), eight);
    __m256 scale = _mm256_set1_ps(ws[b] * a.s[b]);
    __m128i halves[2] = {lo, hi};
    for (int h = 0; h < 2; ++h) {
      __m256i w = _mm256_cvtepi8_epi16(halves[h]);
      __m256i x = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(a.q.data() + b * 32 + h * 16)));
      acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(_mm256_madd_epi16(w, x)), scale, acc);
    }
  }
  return hsum256(acc);
}
float dot16_scalar(const int8_t* wq, const Act& a, size_t cols) {  // q8.rs:354-356
  float acc = 0.0f;
  for (size_t j = 0; j < cols; ++j) acc += f16((uint16_t)((uint8_t)wq[2 * j] | ((uint8_t)wq[2 * j + 1] << 8))) * a.x[j];
  return acc;
}
__attribute__((target("avx512f,f16c"))) float dot16_avx512(const int8_t* wq, const Act& a, size_t cols) {  // q8.rs:358-369
  __m512 acc = _mm512_setzero_ps();
  for (size_t i = 0; i < cols / 16; ++i) {
    __m512 w = _mm512_cvtph_ps(_mm256_loadu_si256((const __m256i*)(wq + i * 32)));
    acc = _mm512_fmadd_ps(w, _mm512_loadu_ps(a.x.data() + i * 16), acc);
  }
  return _mm512_reduce_add_ps(acc);
}
__attribute__((target("avx2,fma,f16c"))) float dot16_avx2(const int8_t* wq, const Act& a, size_t cols) {  // q8.rs:371-386
  __m256 acc = _mm256_setzero_ps();
  for (size_t i = 0; i < cols / 8; ++i) {
    __m256 w = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(wq + i * 16)));
    acc = _mm256_fmadd_ps(w, _mm256_loadu_ps(a.x.data() + i * 8), acc);
  }
  return hsum256(acc);
}

void rows(const Mat& m, const Act& a, Isa isa, size_t r0, float* out, size_t count) {  // q8.rs:410-433
  size_t c = m.row_bytes(), b = m.cols / 32;
  for (size_t i = 0; i < count; ++i) {
    size_t r = r0 + i;
    const int8_t* wq = &m.q[r * c];
    if (m.bits == 16) {
      out[i] = isa == AVX512 ? dot16_avx512(wq, a, m.cols) : isa == AVX2 ? dot16_avx2(wq, a, m.cols) : dot16_scalar(wq, a, m.cols);
      continue;
    }
    const float* ws = &m.s[r * b];
    if (m.bits == 8)
      out[i] = isa == AVX512 ? dot_avx512(wq, ws, a, m.cols) : isa == AVX2 ? dot_avx2(wq, ws, a, m.cols) : dot_scalar(wq, ws, a, m.cols);
    else
      out[i] = isa == AVX512 ? dot4_avx512(wq, ws, a, m.cols) : isa == AVX2 ? dot4_avx2(wq, ws, a, m.cols) : dot4_scalar(wq, ws, a, m.cols);
  }
}

// q8.rs:445-461: rows split into one contiguous range per thread; inline when n == 1 or count < 64.
void matvec_rows(Pool& pool, Isa isa, const Mat& m, size_t first, const Act& a, float* y, size_t count) {
  size_t n = (size_t)pool.threads();
  if (first + count > m.rows) fail("matvec_rows out of range");
  if (n == 1 || count < 64) return rows(m, a, isa, first, y, count);
  size_t per = (count + n - 1) / n;
  pool.run([&](int t) {
    size_t r0 = std::min((size_t)t * per, count), r1 = std::min(((size_t)t + 1) * per, count);
    rows(m, a, isa, first + r0, y + r0, r1 - r0);
  });
}
void matvec(Pool& pool, Isa isa, const Mat& m, const Act& a, float* y) { matvec_rows(pool, isa, m, 0, a, y, m.rows); }  // q8.rs:439-442

// ---------------------------------------------------------------------------------------------
// gguf.rs — header parse (with the short-read retry) and on-demand tensor reads.
// ---------------------------------------------------------------------------------------------
struct Val {
  enum K { U, I, F, B, S, ARR } k = U;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  bool b = false;
  std::string s;
};
struct TensorInfo {
  uint32_t kind = 0;
  std::vector<size_t> dims;
  size_t off = 0;
};
constexpr uint32_t T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8;  // gguf.rs:19-22

struct Reader {  // gguf.rs:31-89
  const uint8_t* b;
  size_t n, p = 0;
  bool short_ = false;
  const uint8_t* take(size_t k) {
    static const uint8_t zeros[16] = {0};
    if (short_ || p + k > n) {
      short_ = true;
      return zeros;
    }
    const uint8_t* s = b + p;
    p += k;
    return s;
  }
  uint32_t u32() { uint32_t v; std::memcpy(&v, take(4), 4); return v; }
  uint64_t u64() { uint64_t v; std::memcpy(&v, take(8), 8); return v; }
  std::string str() {
    uint64_t k = u64();
    if (short_ || p + k > n) { short_ = true; return std::string(); }
    return std::string((const char*)take(k), k);
  }
  Val val(uint32_t ty) {
    Val v;
    switch (ty) {
      case 0: v.k = Val::U; v.u = take(1)[0]; break;
      case 1: v.k = Val::I; v.i = (int8_t)take(1)[0]; break;
      case 2: { uint16_t x; std::memcpy(&x, take(2), 2); v.k = Val::U; v.u = x; break; }
      case 3: { int16_t x; std::memcpy(&x, take(2), 2); v.k = Val::I; v.i = x; break; }
      case 4: v.k = Val::U; v.u = u32(); break;
      case 5: v.k = Val::I; v.i = (int32_t)u32(); break;
      case 6: { float x; std::memcpy(&x, take(4), 4); v.k = Val::F; v.f = x; break; }
      case 7: v.k = Val::B; v.b = take(1)[0] != 0; break;
      case 8: v.k = Val::S; v.s = str(); break;
      case 9: {
        uint32_t t = u32();
        uint64_t cnt = u64();
        for (uint64_t k = 0; k < cnt && !short_; ++k) (void)val(t);
        v.k = Val::ARR;
        break;
      }
      case 10: v.k = Val::U; v.u = u64(); break;
      case 11: v.k = Val::I; v.i = (int64_t)u64(); break;
      case 12: { double x; std::memcpy(&x, take(8), 8); v.k = Val::F; v.f = x; break; }
      default:
        if (short_) break;
        fail("gguf value type " + std::to_string(ty));
    }
    return v;
  }
};

struct Gguf {
  int fd = -1;
  std::map<std::string, Val> meta;
  std::map<std::string, TensorInfo> tensors;
  size_t base = 0;

  explicit Gguf(const std::string& path) {  // gguf.rs:93-107
    fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) fail(path + ": cannot open");
    std::vector<uint8_t> data;
    std::vector<uint8_t> chunk(1 << 22);
    for (;;) {
      ssize_t n = ::read(fd, chunk.data(), chunk.size());
      if (n < 0) fail(path + ": read error");
      data.insert(data.end(), chunk.begin(), chunk.begin() + n);
      if (header(data)) break;
      if (n == 0) fail("truncated GGUF header");
    }
  }
  ~Gguf() { if (fd >= 0) ::close(fd); }

  bool header(const std::vector<uint8_t>& data) {  // gguf.rs:109-143
    Reader r{data.data(), data.size()};
    const uint8_t* magic = r.take(4);
    if (!r.short_ && std::memcmp(magic, "GGUF", 4) != 0) fail("not a GGUF file");
    (void)r.u32();
    uint64_t nt = r.u64(), nkv = r.u64();
    std::map<std::string, Val> m;
    for (uint64_t k = 0; k < nkv; ++k) {
      std::string key = r.str();
      uint32_t ty = r.u32();
      Val v = r.val(ty);
      if (r.short_) return false;
      m[key] = v;
    }
    std::map<std::string, TensorInfo> ts;
    for (uint64_t k = 0; k < nt; ++k) {
      std::string name = r.str();
      uint32_t nd = r.u32();
      TensorInfo t;
      for (uint32_t d = 0; d < nd && !r.short_; ++d) t.dims.push_back((size_t)r.u64());
      t.kind = r.u32();
      t.off = (size_t)r.u64();
      if (r.short_) return false;
      ts[name] = t;
    }
    size_t align = 32;
    auto it = m.find("general.alignment");
    if (it != m.end() && it->second.k == Val::U) align = (size_t)it->second.u;
    meta = std::move(m);
    tensors = std::move(ts);
    base = (r.p + align - 1) / align * align;
    return true;
  }

  bool has(const std::string& name) const { return tensors.count(name) > 0; }
  std::vector<uint8_t> tensor(const std::string& name, TensorInfo* info) const {  // gguf.rs:145-159
    auto it = tensors.find(name);
    if (it == tensors.end()) fail("missing tensor " + name);
    const TensorInfo& t = it->second;
    size_t n = 1;
    for (size_t d : t.dims) n *= d;
    size_t bytes;
    switch (t.kind) {
      case T_F32: bytes = n * 4; break;
      case T_F16: bytes = n * 2; break;
      case T_Q8_0: bytes = n / 32 * 34; break;
      case T_Q4_0: bytes = n / 32 * 18; break;
      default: fail("tensor type " + std::to_string(t.kind));
    }
    std::vector<uint8_t> buf(bytes);
    size_t got = 0;
    while (got < bytes) {
      ssize_t k = ::pread(fd, buf.data() + got, bytes - got, (off_t)(base + t.off + got));
      if (k <= 0) fail("short read of tensor " + name);
      got += (size_t)k;
    }
    if (info) *info = t;
    return buf;
  }
  std::vector<float> f32s(const std::string& name) const {  // gguf.rs:161-165
    TensorInfo t;
    auto b = tensor(name, &t);
    if (t.kind != T_F32) fail(name + ": not F32");
    std::vector<float> v(b.size() / 4);
    std::memcpy(v.data(), b.data(), b.size());
    return v;
  }
  std::vector<float> f32s_or_empty(const std::string& name) const { return has(name) ? f32s(name) : std::vector<float>(); }  // gguf.rs:171-173
  const std::string& text(const std::string& key) const {  // gguf.rs:175-180
    auto it = meta.find(key);
    if (it == meta.end() || it->second.k != Val::S) fail("missing string " + key);
    return it->second.s;
  }
  bool flag(const std::string& key) const {  // gguf.rs:182-184
    auto it = meta.find(key);
    return it != meta.end() && it->second.k == Val::B && it->second.b;
  }
  size_t u(const std::string& key) const {  // gguf.rs:190-196
    auto it = meta.find(key);
    if (it != meta.end() && it->second.k == Val::U) return (size_t)it->second.u;
    if (it != meta.end() && it->second.k == Val::I) return (size_t)it->second.i;
    fail("missing integer " + key);
  }
  size_t u_or(const std::string& key, size_t def) const { return meta.count(key) ? u(key) : def; }  // gguf.rs:186-188
  float f(const std::string& key) const {  // gguf.rs:198-203
    auto it = meta.find(key);
    if (it == meta.end() || it->second.k != Val::F) fail("missing float " + key);
    return (float)it->second.f;
  }
};

Mat load_mat(const Gguf& g, const std::string& name) {  // model.rs:71-79 (dims[0] = cols, dims[1] = rows)
  TensorInfo t;
  auto b = g.tensor(name, &t);
  if (t.dims.size() < 2) fail(name + ": not a matrix");
  size_t cols = t.dims[0], rows = t.dims[1];
  switch (t.kind) {
    case T_Q8_0: return Mat::from_q8_0(b.data(), b.size(), rows, cols);
    case T_Q4_0: return Mat::from_q4_0(b.data(), b.size(), rows, cols);
    case T_F16: return Mat::from_f16(b.data(), b.size(), rows, cols);
    default: fail(name + ": unsupported tensor type " + std::to_string(t.kind));
  }
}

// ---------------------------------------------------------------------------------------------
// model.rs — the decoder.
// ---------------------------------------------------------------------------------------------
void rmsnorm(const float* x, const float* w, float eps, float* out, size_t n) {  // model.rs:81-87
  float ss = 0.0f;
  for (size_t i = 0; i < n; ++i) ss += x[i] * x[i];
  float ms = ss / (float)n;
  float r = 1.0f / std::sqrt(ms + eps);
  for (size_t i = 0; i < n; ++i) out[i] = x[i] * r * w[i];
}
void rmsnorm_inplace(float* x, const float* w, float eps, size_t n) {  // model.rs:89-95
  float ss = 0.0f;
  for (size_t i = 0; i < n; ++i) ss += x[i] * x[i];
  float ms = ss / (float)n;
  float r = 1.0f / std::sqrt(ms + eps);
  for (size_t i = 0; i < n; ++i) x[i] *= r * w[i];
}
void rope(float* x, const float* sn, const float* cs, size_t half) {  // model.rs:97-104
  for (size_t i = 0; i < half; ++i) {
    float a = x[i], b = x[i + half];
    x[i] = a * cs[i] - b * sn[i];
    x[i + half] = a * sn[i] + b * cs[i];
  }
}
__attribute__((target("avx512f"))) float dot512(const float* a, const float* b, size_t n) {  // model.rs:106-120
  __m512 acc = _mm512_setzero_ps();
  size_t k = n / 16;
  for (size_t i = 0; i < k; ++i) acc = _mm512_fmadd_ps(_mm512_loadu_ps(a + i * 16), _mm512_loadu_ps(b + i * 16), acc);
  float s = _mm512_reduce_add_ps(acc);
  for (size_t i = k * 16; i < n; ++i) s += a[i] * b[i];
  return s;
}
__attribute__((target("avx512f"))) void axpy512(float p, const float* x, float* y, size_t n) {  // model.rs:122-135
  __m512 pv = _mm512_set1_ps(p);
  size_t k = n / 16;
  for (size_t i = 0; i < k; ++i) _mm512_storeu_ps(y + i * 16, _mm512_fmadd_ps(pv, _mm512_loadu_ps(x + i * 16), _mm512_loadu_ps(y + i * 16)));
  for (size_t i = k * 16; i < n; ++i) y[i] += p * x[i];
}
void axpy(float p, const float* x, float* y, size_t n, Isa isa) {  // model.rs:137-145
  if (isa == AVX512) return axpy512(p, x, y, n);
  for (size_t i = 0; i < n; ++i) y[i] += p * x[i];
}
float dotf(const float* a, const float* b, size_t n, Isa isa) {  // model.rs:147-149
  if (isa == AVX512) return dot512(a, b, n);
  float s = 0.0f;
  for (size_t i = 0; i < n; ++i) s += a[i] * b[i];
  return s;
}

struct Layer {  // model.rs:12-30
  Mat q, k, v, o, gate, up, down;
  std::vector<float> attn_norm, q_norm, k_norm, post_attn, ffn_norm, post_ffw, bq, bk, bv;
  bool swa = false;
};

struct Gemma {  // model.rs:32-69
  size_t d = 0, vocab = 0, nh = 0, nkv = 0, hd = 0, ff = 0, window = 0, ctx = 0;
  float eps = 0, embed_scale = 1;
  bool silu = false, has_emb = true, has_out = false;
  std::vector<Layer> layers;
  Mat emb, out;
  std::vector<uint32_t> row_of;
  int64_t bos = -1;
  std::vector<float> out_norm;
  std::vector<std::vector<float>> kc, vc;
  std::vector<float> x, xn, q, k, v, att, tmp, g, u, scores, gt, acc;
  Act ad, aq, aff;
  std::vector<float> inv_freq[2], rot_s[2], rot_c[2];

  const Mat& head() const { return has_out ? out : emb; }  // model.rs:236-238
  Mat& head_mut() { return has_out ? out : emb; }

  void load(const Gguf& g, size_t ctx_, bool tie) {  // model.rs:154-233
    has_out = g.has("output.weight");
    if (has_out) out = load_mat(g, "output.weight");
    bool tied = tie && has_out;
    has_emb = !tied;
    if (has_emb) emb = load_mat(g, "token_embd.weight");
    vocab = has_out ? out.rows : emb.rows;
    std::string a = g.text("general.architecture");
    bool gemma = a == "gemma3";
    if (!gemma && a != "qwen2") fail("unsupported architecture " + a);
    d = g.u(a + ".embedding_length");
    size_t nl = g.u(a + ".block_count");
    nh = g.u(a + ".attention.head_count");
    nkv = g.u(a + ".attention.head_count_kv");
    hd = g.u_or(a + ".attention.key_length", d / nh);
    ff = g.u(a + ".feed_forward_length");
    eps = g.f(a + ".attention.layer_norm_rms_epsilon");
    window = g.u_or(a + ".attention.sliding_window", 0);
    float base = g.f(a + ".rope.freq_base");
    layers.resize(nl);
    for (size_t l = 0; l < nl; ++l) {
      auto p = [&](const char* s) { return "blk." + std::to_string(l) + "." + s; };
      Layer& L = layers[l];
      L.q = load_mat(g, p("attn_q.weight"));
      L.k = load_mat(g, p("attn_k.weight"));
      L.v = load_mat(g, p("attn_v.weight"));
      L.o = load_mat(g, p("attn_output.weight"));
      L.gate = load_mat(g, p("ffn_gate.weight"));
      L.up = load_mat(g, p("ffn_up.weight"));
      L.down = load_mat(g, p("ffn_down.weight"));
      L.attn_norm = g.f32s(p("attn_norm.weight"));
      L.q_norm = g.f32s_or_empty(p("attn_q_norm.weight"));
      L.k_norm = g.f32s_or_empty(p("attn_k_norm.weight"));
      L.post_attn = g.f32s_or_empty(p("post_attention_norm.weight"));
      L.ffn_norm = g.f32s(p("ffn_norm.weight"));
      L.post_ffw = g.f32s_or_empty(p("post_ffw_norm.weight"));
      L.bq = g.f32s_or_empty(p("attn_q.bias"));
      L.bk = g.f32s_or_empty(p("attn_k.bias"));
      L.bv = g.f32s_or_empty(p("attn_v.bias"));
      L.swa = gemma && l % 6 < 5;
    }
    bos = g.flag("tokenizer.ggml.add_bos_token") ? (int64_t)g.u("tokenizer.ggml.bos_token_id") : -1;
    embed_scale = gemma ? std::sqrt((float)d) : 1.0f;
    silu = !gemma;
    out_norm = g.f32s("output_norm.weight");
    ctx = ctx_;
    kc.assign(nl, std::vector<float>(ctx * nkv * hd, 0.0f));
    vc.assign(nl, std::vector<float>(ctx * nkv * hd, 0.0f));
    x.assign(d, 0), xn.assign(d, 0), q.assign(nh * hd, 0), k.assign(nkv * hd, 0), v.assign(nkv * hd, 0);
    att.assign(nh * hd, 0), tmp.assign(d, 0);
    this->g.assign(ff, 0), u.assign(ff, 0), scores.assign(nh * ctx, 0), gt.assign(ff, 0);
    ad = Act(d), aq = Act(nh * hd), aff = Act(ff);
    float bases[2] = {10000.0f, base};
    for (int i = 0; i < 2; ++i) {
      inv_freq[i].resize(hd / 2);
      for (size_t j = 0; j < hd / 2; ++j) inv_freq[i][j] = std::pow(bases[i], -2.0f * (float)j / (float)hd);
      rot_s[i].assign(hd / 2, 0.0f);
      rot_c[i].assign(hd / 2, 1.0f);
    }
  }

  size_t row_index(uint32_t tok) const { return row_of.empty() ? tok : row_of[tok]; }  // model.rs:251-253
  std::vector<float> embedding(uint32_t tok) const {  // model.rs:255-257
    if (!has_emb) return head().row_f32(row_index(tok));
    if (!has_out) return emb.row_f32(row_index(tok));
    return emb.row_f32(tok);
  }
  void requantize_head(int bits) {  // model.rs:259-266
    if (bits == 8) head_mut() = head().to_q8();
    else if (bits == 4) head_mut() = head().to_q4();
  }
  void requantize(bool body4, bool head4) {  // model.rs:268-279
    if (body4)
      for (auto& L : layers)
        for (Mat* m : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down}) *m = m->to_q4();
    if (head4) emb = emb.to_q4();
  }

  // model.rs:286-430
  const float* forward(uint32_t tok, size_t pos, Pool& pool, Isa isa) {
    if (pos >= ctx) fail("pos >= ctx");
    if (tok >= vocab) fail("token id out of range");
    float scale = embed_scale;
    std::vector<float> row = embedding(tok);
    for (size_t i = 0; i < d; ++i) x[i] = row[i] * scale;
    size_t threads = (size_t)pool.threads();
    if (acc.size() != threads * nh * hd) acc.assign(threads * nh * hd, 0.0f);
    for (int i = 0; i < 2; ++i)
      for (size_t j = 0; j < hd / 2; ++j) {
        float ang = (float)pos * inv_freq[i][j];
        rot_s[i][j] = std::sin(ang);
        rot_c[i][j] = std::cos(ang);
      }
    for (size_t l = 0; l < layers.size(); ++l) {
      const Layer& L = layers[l];
      rmsnorm(x.data(), L.attn_norm.data(), eps, xn.data(), d);
      ad.quantize(xn.data(), d, isa);
      matvec(pool, isa, L.q, ad, q.data());
      matvec(pool, isa, L.k, ad, k.data());
      matvec(pool, isa, L.v, ad, v.data());
      for (size_t i = 0; i < L.bq.size() && i < q.size(); ++i) q[i] += L.bq[i];
      for (size_t i = 0; i < L.bk.size() && i < k.size(); ++i) k[i] += L.bk[i];
      for (size_t i = 0; i < L.bv.size() && i < v.size(); ++i) v[i] += L.bv[i];
      int tb = L.swa ? 0 : 1;
      float qs = 1.0f / std::sqrt((float)hd);
      for (size_t h = 0; h < nh; ++h) {
        float* qh = &q[h * hd];
        if (!L.q_norm.empty()) rmsnorm_inplace(qh, L.q_norm.data(), eps, hd);
        rope(qh, rot_s[tb].data(), rot_c[tb].data(), hd / 2);
        for (size_t i = 0; i < hd; ++i) qh[i] *= qs;
      }
      for (size_t h = 0; h < nkv; ++h) {
        float* kh = &k[h * hd];
        if (!L.k_norm.empty()) rmsnorm_inplace(kh, L.k_norm.data(), eps, hd);
        rope(kh, rot_s[tb].data(), rot_c[tb].data(), hd / 2);
      }
      size_t rw = nkv * hd;
      std::memcpy(&kc[l][pos * rw], k.data(), rw * 4);
      std::memcpy(&vc[l][pos * rw], v.data(), rw * 4);
      size_t lo = L.swa ? ((pos + 1 > window) ? pos + 1 - window : 0) : 0;
      size_t n_pos = pos + 1 - lo;
      size_t per = (n_pos + threads - 1) / threads;
      size_t group = nh / nkv;
      const float* kcl = kc[l].data();
      const float* vcl = vc[l].data();
      pool.run([&](int t) {
        for (size_t i = std::min((size_t)t * per, n_pos); i < std::min(((size_t)t + 1) * per, n_pos); ++i) {
          const float* krow = kcl + (lo + i) * rw;
          for (size_t h = 0; h < nh; ++h) {
            size_t kvh = h / group;
            scores[h * ctx + i] = dotf(&q[h * hd], krow + kvh * hd, hd, isa);
          }
        }
      });
      for (size_t h = 0; h < nh; ++h) {
        float* s = &scores[h * ctx];
        float mx = -std::numeric_limits<float>::infinity();
        for (size_t i = 0; i < n_pos; ++i) mx = std::fmax(mx, s[i]);
        for (size_t i = 0; i < n_pos; ++i) s[i] -= mx;
        for (size_t i = 0; i < n_pos; ++i) s[i] = exp_fast(s[i]);
        float sum = 0.0f;
        for (size_t i = 0; i < n_pos; ++i) sum += s[i];
        float inv = 1.0f / sum;
        for (size_t i = 0; i < n_pos; ++i) s[i] *= inv;
      }
      size_t width = nh * hd;
      std::fill(acc.begin(), acc.end(), 0.0f);
      pool.run([&](int t) {
        float* outp = &acc[(size_t)t * width];
        for (size_t i = std::min((size_t)t * per, n_pos); i < std::min(((size_t)t + 1) * per, n_pos); ++i) {
          const float* vrow = vcl + (lo + i) * rw;
          for (size_t h = 0; h < nh; ++h) {
            size_t kvh = h / group;
            axpy(scores[h * ctx + i], vrow + kvh * hd, outp + h * hd, hd, isa);
          }
        }
      });
      std::fill(att.begin(), att.end(), 0.0f);
      for (size_t t = 0; t < threads; ++t)
        for (size_t i = 0; i < width; ++i) att[i] += acc[t * width + i];
      aq.quantize(att.data(), width, isa);
      matvec(pool, isa, L.o, aq, tmp.data());
      if (!L.post_attn.empty()) rmsnorm_inplace(tmp.data(), L.post_attn.data(), eps, d);
      for (size_t i = 0; i < d; ++i) x[i] += tmp[i];
      rmsnorm(x.data(), L.ffn_norm.data(), eps, xn.data(), d);
      ad.quantize(xn.data(), d, isa);
      matvec(pool, isa, L.gate, ad, g.data());
      matvec(pool, isa, L.up, ad, u.data());
      if (silu) {
        for (size_t i = 0; i < ff; ++i) gt[i] = -g[i];
        for (size_t i = 0; i < ff; ++i) gt[i] = exp_fast(gt[i]);
        for (size_t i = 0; i < ff; ++i) g[i] = g[i] / (1.0f + gt[i]) * u[i];
      } else {
        for (size_t i = 0; i < ff; ++i) {
          float gv = g[i];
          gt[i] = 0.7978846f * (gv + 0.044715f * gv * gv * gv);
        }
        for (size_t i = 0; i < ff; ++i) gt[i] = tanh_fast(gt[i]);
        for (size_t i = 0; i < ff; ++i) g[i] = 0.5f * g[i] * (1.0f + gt[i]) * u[i];
      }
      aff.quantize(g.data(), ff, isa);
      matvec(pool, isa, L.down, aff, tmp.data());
      if (!L.post_ffw.empty()) rmsnorm_inplace(tmp.data(), L.post_ffw.data(), eps, d);
      for (size_t i = 0; i < d; ++i) x[i] += tmp[i];
    }
    rmsnorm(x.data(), out_norm.data(), eps, xn.data(), d);
    return xn.data();
  }
};

// ---------------------------------------------------------------------------------------------
// main.rs heads
// ---------------------------------------------------------------------------------------------
struct TwoLevel {  // main.rs:40-76
  std::vector<float> a, b;
  std::vector<Mat> blocks;
  std::vector<std::vector<uint32_t>> members;
  std::vector<uint32_t> cls_of, pos_of;
  Act act;
  std::vector<float> cl, inner;
  size_t d = 0;
};

std::vector<uint8_t> read_file(const std::string& p) {
  FILE* f = std::fopen(p.c_str(), "rb");
  if (!f) fail(p + ": cannot open");
  std::vector<uint8_t> v;
  uint8_t buf[1 << 16];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) v.insert(v.end(), buf, buf + n);
  std::fclose(f);
  return v;
}

}  // namespace

struct orc_model {
  Gemma m;
  std::unique_ptr<Pool> pool;
  Isa isa = SCALAR;
  Act full_act;
  std::vector<float> logits;
  std::unique_ptr<TwoLevel> two;
};
struct orc_mat {
  Mat m;
};

#define GUARD_BEGIN try {
#define GUARD_END                 \
  }                               \
  catch (const std::exception& e) { \
    g_err = e.what();             \
    return -1;                    \
  }

extern "C" {

const char* orc_last_error(void) { return g_err.c_str(); }
const char* orc_detect_isa(void) { return isa_name(detect_isa()); }

orc_model* orc_open(const char* path, int ctx, int body_bits, int head_bits, int threads, const char* isa) {
  try {
    auto om = std::make_unique<orc_model>();
    om->isa = parse_isa(isa);
    Gguf g(path);
    om->m.load(g, (size_t)ctx, false);
    om->m.requantize(body_bits == 4, false);  // main.rs:209
    om->m.requantize_head(head_bits);          // main.rs:210
    om->pool = std::make_unique<Pool>(threads);
    om->full_act = Act(om->m.d);              // main.rs:26-28
    om->logits.assign(om->m.vocab, 0.0f);
    return om.release();
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}
void orc_close(orc_model* m) { delete m; }
int orc_info(const orc_model* om, int64_t* o) {
  const Gemma& m = om->m;
  o[0] = (int64_t)m.d, o[1] = (int64_t)m.vocab, o[2] = (int64_t)m.layers.size(), o[3] = (int64_t)m.ctx, o[4] = m.bos;
  return 0;
}
const char* orc_isa(const orc_model* m) { return isa_name(m->isa); }

int orc_forward(orc_model* om, uint32_t tok, uint32_t pos, float* h) {
  GUARD_BEGIN
  const float* r = om->m.forward(tok, pos, *om->pool, om->isa);
  if (h) std::memcpy(h, r, om->m.d * 4);
  return 0;
  GUARD_END
}

int orc_full(orc_model* om, const float* h, uint32_t target, float* lp, uint32_t* am, float* logits_out) {
  GUARD_BEGIN
  Gemma& m = om->m;
  if (target >= m.vocab) fail("target out of range");
  om->full_act.quantize(h, m.d, om->isa);  // main.rs:30-33
  matvec(*om->pool, om->isa, m.head(), om->full_act, om->logits.data());
  // main.rs:35-37 (logits are indexed by token: the head is unpermuted here)
  if (lp) *lp = om->logits[target] - lse(om->logits.data(), m.vocab);
  if (am) *am = (uint32_t)argmax(om->logits.data(), m.vocab);
  if (logits_out) std::memcpy(logits_out, om->logits.data(), m.vocab * 4);
  return 0;
  GUARD_END
}

int orc_twolevel_load(orc_model* om, const char* prefix) {  // main.rs:57-76
  GUARD_BEGIN
  Gemma& m = om->m;
  std::string p(prefix);
  auto ob = read_file(p + ".order"), ab = read_file(p + ".A"), bb = read_file(p + ".b");
  std::vector<uint32_t> order(ob.size() / 4);
  std::memcpy(order.data(), ob.data(), order.size() * 4);
  auto t = std::make_unique<TwoLevel>();
  t->a.resize(ab.size() / 4);
  std::memcpy(t->a.data(), ab.data(), t->a.size() * 4);
  t->b.resize(bb.size() / 4);
  std::memcpy(t->b.data(), bb.data(), t->b.size() * 4);
  size_t k = t->b.size();
  if (k == 0) fail("empty .b");
  size_t per = (order.size() + k - 1) / k;
  for (size_t c = 0; c * per < order.size(); ++c)
    t->members.emplace_back(order.begin() + c * per, order.begin() + std::min(order.size(), (c + 1) * per));
  if (t->members.size() != k) fail("class count mismatch: .order chunks vs .b length");
  t->cls_of.assign(m.vocab, 0);
  t->pos_of.assign(m.vocab, 0);
  for (size_t c = 0; c < k; ++c)
    for (size_t j = 0; j < t->members[c].size(); ++j) {
      uint32_t tok = t->members[c][j];
      if (tok >= m.vocab) fail(".order token out of range");
      t->cls_of[tok] = (uint32_t)c;
      t->pos_of[tok] = (uint32_t)j;
    }
  for (size_t c = 0; c < k; ++c) t->blocks.push_back(m.head().gather(t->members[c].data(), t->members[c].size()));
  t->act = Act(m.d);
  t->cl.assign(k, 0.0f);
  t->inner.assign(per, 0.0f);
  t->d = m.d;
  if (t->a.size() != k * m.d) fail(".A size does not match k * d");
  om->two = std::move(t);
  return 0;
  GUARD_END
}

int orc_twolevel(orc_model* om, const float* h, uint32_t target, float* lp, uint32_t* am, float* cl_out, float* inner_out) {
  GUARD_BEGIN
  if (!om->two) fail("two-level head not loaded");
  TwoLevel& t = *om->two;
  Pool& pool = *om->pool;
  Isa isa = om->isa;
  size_t k = t.cl.size(), d = t.d;
  if (target >= t.cls_of.size()) fail("target out of range");
  // classes (main.rs:82-93)
  size_t per = (k + (size_t)pool.threads() - 1) / (size_t)pool.threads();
  pool.run([&](int th) {
    for (size_t c = std::min((size_t)th * per, k); c < std::min(((size_t)th + 1) * per, k); ++c)
      t.cl[c] = dotf(&t.a[c * d], h, d, isa) + t.b[c];
  });
  // logprob (main.rs:101-107); within (main.rs:95-99)
  size_t c = t.cls_of[target];
  t.act.quantize(h, d, isa);
  size_t n = t.blocks[c].rows;
  matvec(pool, isa, t.blocks[c], t.act, t.inner.data());
  float lse_cl = lse(t.cl.data(), k);
  if (lp) *lp = t.cl[c] - lse_cl + t.inner[t.pos_of[target]] - lse(t.inner.data(), n);
  if (inner_out) std::memcpy(inner_out, t.inner.data(), n * 4);
  if (cl_out) std::memcpy(cl_out, t.cl.data(), k * 4);
  if (am) {  // lean.rs:46-76 with top = 1: best raw logit inside the most likely class
    size_t top = argmax(t.cl.data(), k);
    std::vector<float> in2(t.blocks[top].rows);
    matvec(pool, isa, t.blocks[top], t.act, in2.data());
    *am = t.members[top][argmax(in2.data(), in2.size())];
  }
  return 0;
  GUARD_END
}

// lean.rs:46-76 (Classes::next) and lean.rs:93-107 (next_token): the greedy token for hidden state h
// by screening the `top` most likely classes and the always-on rows (indices into the class-ordered
// rows of the permuted head), highest raw logit wins; when the most likely class's probability is
// below min_confidence, the full head's argmax over the class-ordered rows instead (*fell_back = 1).
int orc_greedy(orc_model* om, const float* h, int top, float min_confidence, const uint32_t* always, int n_always,
               uint32_t* tok, int* fell_back) {
  GUARD_BEGIN
  if (!om->two) fail("two-level head not loaded");
  TwoLevel& t = *om->two;
  Pool& pool = *om->pool;
  Isa isa = om->isa;
  const size_t k = t.cl.size(), d = t.d, per = t.inner.size();
  for (size_t c = 0; c < k; ++c) t.cl[c] = dotf(&t.a[c * d], h, d, isa) + t.b[c];
  const float norm = lse(t.cl.data(), k);
  t.act.quantize(h, d, isa);
  std::vector<size_t> ranked(k);
  for (size_t c = 0; c < k; ++c) ranked[c] = c;
  std::stable_sort(ranked.begin(), ranked.end(), [&](size_t x, size_t y) { return t.cl[y] < t.cl[x]; });
  if (fell_back) *fell_back = 0;
  if (std::exp(t.cl[ranked[0]] - norm) < min_confidence) {
    std::vector<float> z;  // the permuted head: class blocks in order
    float best = -std::numeric_limits<float>::infinity();
    size_t brow = 0, row = 0;
    for (size_t c = 0; c < k; ++c) {
      z.assign(t.blocks[c].rows, 0.0f);
      matvec(pool, isa, t.blocks[c], t.act, z.data());
      for (size_t j = 0; j < z.size(); ++j, ++row)
        if (z[j] > best || row == 0) best = z[j], brow = row;
    }
    if (fell_back) *fell_back = 1;
    *tok = t.members[brow / per][brow % per];
    return 0;
  }
  float best = -std::numeric_limits<float>::infinity();
  size_t brow = 0;
  for (int i = 0; i < top && (size_t)i < k; ++i) {
    const size_t c = ranked[(size_t)i];
    std::vector<float> z(t.blocks[c].rows);
    matvec(pool, isa, t.blocks[c], t.act, z.data());
    const size_t j = argmax(z.data(), z.size());
    if (z[j] > best) best = z[j], brow = c * per + j;
  }
  for (int i = 0; i < n_always; ++i) {
    const size_t row = always[i], c = row / per;
    if (c >= k || row % per >= t.blocks[c].rows) fail("always-on row out of range");
    std::vector<float> z(t.blocks[c].rows);
    matvec(pool, isa, t.blocks[c], t.act, z.data());
    if (z[row % per] > best) best = z[row % per], brow = row;
  }
  *tok = t.members[brow / per][brow % per];
  return 0;
  GUARD_END
}

// main.rs:123-141: uniform (xorshift64, 24 bits) and draw (softmax at temperature, sequential scan).
static float uniform01(uint64_t* rng) {
  uint64_t x = *rng;
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  *rng = x;
  return (float)(x >> 40) / (float)(1ull << 24);
}
static size_t draw(const float* l, size_t n, float temp, uint64_t* rng) {
  float mx = -std::numeric_limits<float>::infinity();
  for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, l[i]);
  std::vector<float> w(n);
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) w[i] = std::exp((l[i] - mx) / temp);
  for (size_t i = 0; i < n; ++i) sum += w[i];
  float r = uniform01(rng) * sum;
  for (size_t i = 0; i < n; ++i) {
    r -= w[i];
    if (r <= 0.0f) return i;
  }
  return n - 1;
}

// TwoLevel::sample (main.rs:109-116): a class drawn from the class logits, then a member of it.
int orc_twolevel_sample(orc_model* om, const float* h, float temp, uint64_t* rng, uint32_t* tok) {
  GUARD_BEGIN
  if (!om->two) fail("two-level head not loaded");
  TwoLevel& t = *om->two;
  Pool& pool = *om->pool;
  const size_t k = t.cl.size(), d = t.d;
  for (size_t c = 0; c < k; ++c) t.cl[c] = dotf(&t.a[c * d], h, d, om->isa) + t.b[c];
  const size_t c = draw(t.cl.data(), k, temp, rng);
  t.act.quantize(h, d, om->isa);
  const size_t n = t.blocks[c].rows;
  matvec(pool, om->isa, t.blocks[c], t.act, t.inner.data());
  *tok = t.members[c][draw(t.inner.data(), n, temp, rng)];
  return 0;
  GUARD_END
}

int orc_score(orc_model* om, const uint32_t* toks, size_t n, int head, float* lp, uint32_t* am, double* body_s, double* head_s) {
  GUARD_BEGIN
  Gemma& m = om->m;
  size_t off = m.bos >= 0 ? 1 : 0;
  if (m.bos >= 0) m.forward((uint32_t)m.bos, 0, *om->pool, om->isa);  // main.rs:270-272
  std::vector<float> h(m.d);
  double tb = 0, th = 0;
  for (size_t i = 0; i < n; ++i) {  // main.rs:275-289
    auto a = std::chrono::steady_clock::now();
    std::memcpy(h.data(), m.forward(toks[i], i + off, *om->pool, om->isa), m.d * 4);
    auto b = std::chrono::steady_clock::now();
    int rc = head == 0 ? orc_full(om, h.data(), toks[i + 1], &lp[i], am ? &am[i] : nullptr, nullptr)
                       : orc_twolevel(om, h.data(), toks[i + 1], &lp[i], am ? &am[i] : nullptr, nullptr, nullptr);
    if (rc) return rc;
    auto c = std::chrono::steady_clock::now();
    tb += std::chrono::duration<double>(b - a).count();
    th += std::chrono::duration<double>(c - b).count();
  }
  if (body_s) *body_s = tb;
  if (head_s) *head_s = th;
  return 0;
  GUARD_END
}

orc_mat* orc_mat_from_gguf(int kind, const uint8_t* raw, size_t rows, size_t cols) {
  try {
    auto w = std::make_unique<orc_mat>();
    if (kind == 8) w->m = Mat::from_q8_0(raw, rows * cols / 32 * 34, rows, cols);
    else if (kind == 2) w->m = Mat::from_q4_0(raw, rows * cols / 32 * 18, rows, cols);
    else if (kind == 1) w->m = Mat::from_f16(raw, rows * cols * 2, rows, cols);
    else fail("unknown kind");
    return w.release();
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}
void orc_mat_free(orc_mat* w) { delete w; }
orc_mat* orc_mat_requant(const orc_mat* w, int bits) {
  try {
    auto o = std::make_unique<orc_mat>();
    o->m = bits == 8 ? w->m.to_q8() : w->m.to_q4();
    return o.release();
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}
int orc_mat_info(const orc_mat* w, int64_t* o) {
  o[0] = w->m.bits, o[1] = (int64_t)w->m.rows, o[2] = (int64_t)w->m.cols, o[3] = (int64_t)w->m.q.size(), o[4] = (int64_t)w->m.s.size();
  return 0;
}
int orc_mat_planes(const orc_mat* w, int8_t* q, float* s) {
  if (q) std::memcpy(q, w->m.q.data(), w->m.q.size());
  if (s) std::memcpy(s, w->m.s.data(), w->m.s.size() * 4);
  return 0;
}
int orc_mat_dequant(const orc_mat* w, float* out) {
  for (size_t r = 0; r < w->m.rows; ++r)
    for (size_t j = 0; j < w->m.cols; ++j) out[r * w->m.cols + j] = w->m.weight(r, j);
  return 0;
}
int orc_matvec(const orc_mat* w, const float* x, const char* isa, int threads, float* y) {
  GUARD_BEGIN
  Isa i = parse_isa(isa);
  Pool pool(threads);
  Act a(w->m.cols);
  a.quantize(x, w->m.cols, i);
  matvec(pool, i, w->m, a, y);
  return 0;
  GUARD_END
}
int orc_quantize(const float* x, size_t n, const char* isa, int8_t* q, float* s) {
  GUARD_BEGIN
  Act a(n);
  a.quantize(x, n, parse_isa(isa));
  std::memcpy(q, a.q.data(), n);
  std::memcpy(s, a.s.data(), n / 32 * 4);
  return 0;
  GUARD_END
}
float orc_exp_fast(float x) { return exp_fast(x); }
float orc_tanh_fast(float x) { return tanh_fast(x); }
float orc_lse(const float* v, size_t n) { return lse(v, n); }
float orc_f16(uint16_t h) { return f16(h); }

}  // extern "C"
