// Exact-numerics device helpers (see kernels_exact.cu): the reference's AVX-512 lane structure and
// sequential sums, shared by the per-kernel exact path and the layer-pipelined scoring kernel.
#pragma once
#include "common.cuh"
#include "kernels.cuh"

namespace gem {

// _mm512_reduce_add_ps over 16 lanes held as 8 + 8 by the two threads of a lane pair (lane ^ 1).
__device__ __forceinline__ float reduce16_pair(const float (&a)[8]) {
  float b[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) b[i] = add(a[i], __shfl_xor_sync(0xffffffffu, a[i], 1));  // a_i + a_(i+8)
  float c0 = add(b[0], b[4]), c1 = add(b[1], b[5]), c2 = add(b[2], b[6]), c3 = add(b[3], b[7]);
  return add(add(c0, c2), add(c1, c3));
}

// Low / high int16 pair of a packed word as one madd_epi16 lane: w0*a0 + w1*a1 (exact).
__device__ __forceinline__ float madd_lo(int w, int a) { return (float)__dp4a(w & 0x0000ffff, a, 0); }
__device__ __forceinline__ float madd_hi(int w, int a) { return (float)__dp4a(w & (int)0xffff0000, a, 0); }

// One row's dot with the reference's lane structure. `half` selects lanes 8*half .. 8*half + 7.
// Returns the reduced value in both threads of the pair. Weight and scale loads for U blocks are
// issued before the FMA chain consumes them, so each thread keeps U 16-byte loads in flight.
template <int BITS>
__device__ __forceinline__ int4 load_block(const MatView& w, size_t r, int b, int half) {
  if constexpr (BITS == 8) {
    return ldg_stream((const int4*)((const int8_t*)w.q + r * w.cols) + 2 * b + half);
  } else {  // dot4_avx512 (q8.rs:307-326): bytes 0..15 low nibbles, 16..31 high nibbles, minus 8
    int4 raw = ldg_stream((const int4*)((const uint8_t*)w.q + r * (w.cols / 2)) + b);
    const unsigned m = 0x0f0f0f0fu, e = 0x08080808u;
    int sh = half * 4;
    int4 wv;
    wv.x = (int)__vsub4(((unsigned)raw.x >> sh) & m, e);
    wv.y = (int)__vsub4(((unsigned)raw.y >> sh) & m, e);
    wv.z = (int)__vsub4(((unsigned)raw.z >> sh) & m, e);
    wv.w = (int)__vsub4(((unsigned)raw.w >> sh) & m, e);
    return wv;
  }
}

__device__ __forceinline__ void block_fma(float (&acc)[8], int4 wv, const int4 av, float s) {
  acc[0] = fmaf(madd_lo(wv.x, av.x), s, acc[0]);
  acc[1] = fmaf(madd_hi(wv.x, av.x), s, acc[1]);
  acc[2] = fmaf(madd_lo(wv.y, av.y), s, acc[2]);
  acc[3] = fmaf(madd_hi(wv.y, av.y), s, acc[3]);
  acc[4] = fmaf(madd_lo(wv.z, av.z), s, acc[4]);
  acc[5] = fmaf(madd_hi(wv.z, av.z), s, acc[5]);
  acc[6] = fmaf(madd_lo(wv.w, av.w), s, acc[6]);
  acc[7] = fmaf(madd_hi(wv.w, av.w), s, acc[7]);
}

template <int BITS, typename ST>
__device__ __forceinline__ float row_dot_exact(const MatView& w, size_t r, int half, const int8_t* saq, const float* sas,
                                               const float* sx) {
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  constexpr int U = 8;
  if constexpr (BITS == 16) {  // dot16_avx512 (q8.rs:358-369): lane i sums w[16c+i]*x[16c+i]
    const int4* row = (const int4*)((const __half*)w.q + r * w.cols);
    const int nc = w.cols / 16;
    int c = 0;
    for (; c < nc; c += U) {
      int4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = c + u < nc ? ldg_stream(row + 2 * (c + u) + half) : make_int4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (c + u >= nc) break;
        const __half2* h2 = (const __half2*)&v[u];
        const float* xv = sx + (c + u) * 16 + half * 8;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float2 f = __half22float2(h2[k]);
          acc[2 * k] = fmaf(f.x, xv[2 * k], acc[2 * k]);
          acc[2 * k + 1] = fmaf(f.y, xv[2 * k + 1], acc[2 * k + 1]);
        }
      }
    }
  } else {
    const int nb = w.cols / 32;
    const ST* srow = (const ST*)w.s + r * nb;
    int b = 0;
    for (; b + U <= nb; b += U) {
      int4 wv[U];
      float sc[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        wv[u] = load_block<BITS>(w, r, b + u, half);
        sc[u] = ld_scale(srow, b + u);
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
        block_fma(acc, wv[u], *(const int4*)(saq + (b + u) * 32 + half * 16), mul(sc[u], sas[b + u]));
    }
    for (; b < nb; ++b)
      block_fma(acc, load_block<BITS>(w, r, b, half), *(const int4*)(saq + b * 32 + half * 16), mul(ld_scale(srow, b), sas[b]));
  }
  return reduce16_pair(acc);
}

// dot512 (model.rs:106-120) of two fp32 vectors of length n (a multiple of 16): lane i sums
// a[16c+i]*b[16c+i] with FMA, then the halving reduction. Lane pair as above.
__device__ __forceinline__ float dot512_pair(const float* a, const float* b, int n, int half) {
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll 8
  for (int c = 0; c < n / 16; ++c) {
    const float4 a0 = *(const float4*)(a + c * 16 + half * 8), a1 = *(const float4*)(a + c * 16 + half * 8 + 4);
    const float4 b0 = *(const float4*)(b + c * 16 + half * 8), b1 = *(const float4*)(b + c * 16 + half * 8 + 4);
    acc[0] = fmaf(a0.x, b0.x, acc[0]); acc[1] = fmaf(a0.y, b0.y, acc[1]);
    acc[2] = fmaf(a0.z, b0.z, acc[2]); acc[3] = fmaf(a0.w, b0.w, acc[3]);
    acc[4] = fmaf(a1.x, b1.x, acc[4]); acc[5] = fmaf(a1.y, b1.y, acc[5]);
    acc[6] = fmaf(a1.z, b1.z, acc[6]); acc[7] = fmaf(a1.w, b1.w, acc[7]);
  }
  return reduce16_pair(acc);
}

// Rust `iter().map(|v| v * v).sum::<f32>()`: one thread, in order.
__device__ __forceinline__ float seq_sumsq(const float* v, int n) {
  float s = 0.0f;
#pragma unroll 4
  for (int i = 0; i < n; i += 4) {
    float4 t = *(const float4*)(v + i);
    s = add(s, mul(t.x, t.x));
    s = add(s, mul(t.y, t.y));
    s = add(s, mul(t.z, t.z));
    s = add(s, mul(t.w, t.w));
  }
  return s;
}
__device__ __forceinline__ float rms_r_exact(float ss, int n, float eps) {
  return div(1.0f, __fsqrt_rn(add(div(ss, (float)n), eps)));
}

__device__ __forceinline__ void quant_block_warp_x(float v, int lane, int8_t* q, float* s) {
  float amax = warp_max(fabsf(v));
  float d = div(amax, 127.0f);
  float inv = d > 0.0f ? div(1.0f, d) : 0.0f;
  q[lane] = (int8_t)__float2int_rn(mul(v, inv));
  if (lane == 0) *s = d;
}

// QK-norm, RoPE, q scale, KV append for one token and kv group `g` (the body of the per-token
// kernel below and of the sequence-parallel one): raw projections `qkv`, position `pos`, normalised
// queries to `qn` ([nh][hd] of this token). `smp` holds (G + 2) * hd floats, `s_r` G + 1.
__device__ inline void attn_prep_token(const AttnArgs& A, const float* qkv, uint32_t pos, int g, float* qn, float* smp,
                                float* s_r) {
  const int hd = A.hd, G = A.nh / A.nkv;
  float* sq = smp;           // G*hd
  float* sk = sq + G * hd;   // hd
  float* sv = sk + hd;       // hd
  const int rw = A.nkv * hd;
  const float* bq = A.bqkv;
#pragma unroll 4
  for (int j = threadIdx.x; j < G * hd; j += blockDim.x) {
    size_t i = (size_t)g * G * hd + j;
    sq[j] = bq ? add(qkv[i], bq[i]) : qkv[i];
  }
#pragma unroll 2
  for (int j = threadIdx.x; j < hd; j += blockDim.x) {
    size_t ik = (size_t)A.nh * hd + g * hd + j, iv = (size_t)A.nh * hd + rw + g * hd + j;
    sk[j] = bq ? add(qkv[ik], bq[ik]) : qkv[ik];
    sv[j] = bq ? add(qkv[iv], bq[iv]) : qkv[iv];
  }
  __syncthreads();
  // per-head sequential sums of squares, one thread per head (+1 for k)
  if ((int)threadIdx.x <= G) {
    const float* v = threadIdx.x < (unsigned)G ? sq + threadIdx.x * hd : sk;
    const float* nw = threadIdx.x < (unsigned)G ? A.q_norm : A.k_norm;
    s_r[threadIdx.x] = nw ? rms_r_exact(seq_sumsq(v, hd), hd, A.eps) : 1.0f;
  }
  __syncthreads();
  const float* sn = A.rope_sin + (size_t)pos * (hd / 2);
  const float* cs = A.rope_cos + (size_t)pos * (hd / 2);
  const int half = hd / 2;
  for (int t = threadIdx.x; t < (G + 1) * half; t += blockDim.x) {
    int h = t / half, i = t % half;
    float* v = h < G ? sq + h * hd : sk;
    const float* nw = h < G ? A.q_norm : A.k_norm;
    float r = s_r[h];
    float a = v[i], b = v[i + half];
    if (nw) {  // rmsnorm_inplace: v *= r * w
      a = mul(a, mul(r, nw[i]));
      b = mul(b, mul(r, nw[i + half]));
    }
    float na = sub(mul(a, cs[i]), mul(b, sn[i]));  // rope (model.rs:97-104)
    float nb = add(mul(a, sn[i]), mul(b, cs[i]));
    if (h < G) {  // q * 1/sqrt(hd) (model.rs:317-324)
      na = mul(na, A.qscale);
      nb = mul(nb, A.qscale);
      qn[(size_t)(g * G + h) * hd + i] = na;
      qn[(size_t)(g * G + h) * hd + i + half] = nb;
    } else {
      A.kcache[(size_t)pos * rw + g * hd + i] = na;  // KV append (model.rs:333-335)
      A.kcache[(size_t)pos * rw + g * hd + i + half] = nb;
    }
  }
  for (int j = threadIdx.x; j < hd; j += blockDim.x) A.vcache[(size_t)pos * rw + g * hd + j] = sv[j];
}

}  // namespace gem
