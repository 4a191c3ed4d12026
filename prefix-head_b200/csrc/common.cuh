// Device helpers shared by the kernels: IEEE-rounded arithmetic where the reference's rounding must
// be reproduced, the reference's exp/tanh, warp reductions and the Q8_0/Q4_0 block dot.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

namespace gem {

// ----- exact single-rounding float ops (no contraction into FMA: Rust never fuses a*b+c) -----
__device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float div(float a, float b) { return __fdiv_rn(a, b); }

// crates/nn/src/fast.rs:126-132: e^x = 2^n * p(f), n = floor(x*log2e + 0.5), degree-6 Taylor p.
__device__ __forceinline__ float exp_fast(float x) {
  float t = mul(x, 1.44269504088896340736f);
  t = fminf(fmaxf(t, -126.0f), 126.0f);
  float n = floorf(add(t, 0.5f));
  float f = sub(t, n);
  float p = add(1.333355815e-03f, mul(f, 1.540353039e-04f));
  p = add(9.618129108e-03f, mul(f, p));
  p = add(5.550410866e-02f, mul(f, p));
  p = add(2.402265070e-01f, mul(f, p));
  p = add(6.931471806e-01f, mul(f, p));
  p = add(1.0f, mul(f, p));
  return mul(p, __int_as_float(((int)n + 127) << 23));
}
// crates/nn/src/fast.rs:78-81
__device__ __forceinline__ float tanh_fast(float x) {
  float e = exp_fast(mul(2.0f, fminf(fmaxf(x, -10.0f), 10.0f)));
  return div(sub(e, 1.0f), add(e, 1.0f));
}

// ----- reductions -----
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Block-wide sum over all threads; `red` holds >= 32 floats of shared memory. All threads get the sum.
__device__ __forceinline__ float block_sum(float v, float* red) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.0f;
  t = warp_sum(t);
  return t;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : -INFINITY;
  return warp_max(t);
}

// ----- online log-sum-exp state: value m, sum s of e^(z - m); merge is associative -----
struct Lse {
  float m, s;
};
__device__ __forceinline__ Lse lse_merge(Lse a, Lse b) {
  if (a.m < b.m) { Lse t = a; a = b; b = t; }
  if (b.m == -INFINITY) return a;
  return Lse{a.m, a.s + b.s * expf(b.m - a.m)};
}
__device__ __forceinline__ Lse lse_add(Lse a, float z) {
  if (z > a.m) return Lse{z, a.s * expf(a.m - z) + 1.0f};
  return Lse{a.m, a.s + expf(z - a.m)};
}
// argmax candidate: larger value wins, ties go to the smaller token id (the reference's first index).
struct Best {
  float v;
  uint32_t tok;
};
__device__ __forceinline__ Best best_merge(Best a, Best b) {
  if (b.v > a.v || (b.v == a.v && b.tok < a.tok)) return b;
  return a;
}

// Argmax over the rows of an output matrix held in class order: a thread keeps its best row and reads
// row_tok (row -> token; null: rows are tokens) only to break an exact tie by the lower token id, then
// turns the row into its token before candidates of several threads merge by best_merge.
__device__ __forceinline__ void best_row_add(Best& B, float v, uint32_t r, const uint32_t* row_tok) {
  if (v > B.v || (v == B.v && (B.tok == 0xffffffffu || (row_tok ? row_tok[r] < row_tok[B.tok] : r < B.tok))))
    B = Best{v, r};
}
__device__ __forceinline__ void best_row_to_token(Best& B, const uint32_t* row_tok) {
  if (row_tok && B.tok != 0xffffffffu) B.tok = row_tok[B.tok];
}

// Warp-wide merge of log-sum-exp states and argmax candidates: the maximum first, then the sums
// rescaled to it (one exp per lane instead of one per merge step); every lane gets the result.
__device__ __forceinline__ void warp_lse_best(Lse& L, Best& B) {
  float m = L.m;
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = L.m == -INFINITY ? 0.0f : L.s * expf(L.m - m);
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    B = best_merge(B, Best{__shfl_xor_sync(0xffffffffu, B.v, o), __shfl_xor_sync(0xffffffffu, B.tok, o)});
  }
  L = Lse{m, s};
}
// The same over the block (every thread calls it; blockDim a multiple of 32): the result in every lane
// of warp 0. red_* hold one entry per warp and are free when it is called.
__device__ __forceinline__ void block_lse_best(Lse& L, Best& B, float* red_m, float* red_s, float* red_v,
                                               uint32_t* red_t) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  warp_lse_best(L, B);
  if (lane == 0) red_m[warp] = L.m, red_s[warp] = L.s, red_v[warp] = B.v, red_t[warp] = B.tok;
  __syncthreads();
  if (warp == 0) {
    L = lane < nw ? Lse{red_m[lane], red_s[lane]} : Lse{-INFINITY, 0.0f};
    B = lane < nw ? Best{red_v[lane], red_t[lane]} : Best{-INFINITY, 0xffffffffu};
    warp_lse_best(L, B);
  }
}

// ----- scale loads -----
__device__ __forceinline__ float ld_scale(const __half* s, size_t i) { return __half2float(s[i]); }
__device__ __forceinline__ float ld_scale(const float* s, size_t i) { return s[i]; }

// Programmatic dependent launch: a kernel launched with launch_k may be scheduled while its
// predecessor drains; its first action waits for the predecessor's completion and memory (a no-op when
// launched without the attribute), so nothing reads a predecessor's output early.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ----- int8 block dot: 32 weights (two 16-byte words) against 32 activation bytes -----
__device__ __forceinline__ int dot32_i8(int4 w0, int4 w1, const int4 a0, const int4 a1) {
  int s = 0;
  s = __dp4a(w0.x, a0.x, s); s = __dp4a(w0.y, a0.y, s); s = __dp4a(w0.z, a0.z, s); s = __dp4a(w0.w, a0.w, s);
  s = __dp4a(w1.x, a1.x, s); s = __dp4a(w1.y, a1.y, s); s = __dp4a(w1.z, a1.z, s); s = __dp4a(w1.w, a1.w, s);
  return s;
}
// Q4_0 block (16 bytes: byte j = (w[j]+8) | (w[j+16]+8) << 4) against 32 activation bytes.
__device__ __forceinline__ int dot32_q4(int4 w, const int4 a0, const int4 a1) {
  const unsigned m = 0x0f0f0f0fu, e = 0x08080808u;
  auto lo = [&](int v) { return (int)__vsub4((unsigned)v & m, e); };
  auto hi = [&](int v) { return (int)__vsub4(((unsigned)v >> 4) & m, e); };
  int s = 0;
  s = __dp4a(lo(w.x), a0.x, s); s = __dp4a(lo(w.y), a0.y, s); s = __dp4a(lo(w.z), a0.z, s); s = __dp4a(lo(w.w), a0.w, s);
  s = __dp4a(hi(w.x), a1.x, s); s = __dp4a(hi(w.y), a1.y, s); s = __dp4a(hi(w.z), a1.z, s); s = __dp4a(hi(w.w), a1.w, s);
  return s;
}

__device__ __forceinline__ int4 ldg_stream(const int4* p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

}  // namespace gem
