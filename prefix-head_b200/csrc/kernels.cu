// sm_100a kernels of the scoring path: embedding, RMSNorm + activation quantization, block-dequant
// GEMV (Q8_0 / Q4_0 / F16), split-KV GQA attention with QK-norm and RoPE, GELU-tanh gating, the full
// head with fused online log-sum-exp / argmax, and the fused two-level head.
//
// Numerics follow the reference (crates/gem): element-wise steps round exactly as the Rust code does
// (explicit _rn intrinsics, no FMA contraction); sums use tree orders, which differ from the
// reference's sequential sums only in the last bits.
#include "kernels.cuh"

namespace gem {

// ------------------------------------------------------------------------------------------------
// Embedding (model.rs:255-257, 290-293): x = dequantized head row * sqrt(d). `row` is the token's row
// in the (possibly class-permuted) output matrix.
// ------------------------------------------------------------------------------------------------
template <int BITS, typename ST>
__global__ void k_embed(MatView head, const uint32_t* row_of, const StepCur* cur, float scale, float* x) {
  pdl_wait();
  uint32_t tok = cur->tok;
  size_t row = row_of ? row_of[tok] : tok;
  for (int j = threadIdx.x; j < head.cols; j += blockDim.x) x[j] = mul(weight_at<BITS, ST>(head, row, j), scale);
}

// Output-matrix rows gathered into another matrix of the same shape: dst row i = src row src_row[i]
// (weights as 16-byte pieces, a row being a multiple of 16 bytes; scales as 2-byte pieces).
__global__ void k_gather_rows(MatView src, const uint32_t* src_row, MatView dst) {
  const size_t rb = (size_t)src.cols * src.bits / 8;
  const size_t sb = src.bits == 16 ? 0 : (size_t)(src.cols / 32) * (src.scale_f32 ? 4 : 2);
  for (int i = blockIdx.x; i < dst.rows; i += gridDim.x) {
    const size_t r = src_row[i];
    const int4* a = (const int4*)((const unsigned char*)src.q + r * rb);
    int4* b = (int4*)((unsigned char*)dst.q + (size_t)i * rb);
    for (size_t j = threadIdx.x; j < rb / 16; j += blockDim.x) b[j] = a[j];
    const uint16_t* c = (const uint16_t*)((const unsigned char*)src.s + r * sb);
    uint16_t* e = (uint16_t*)((unsigned char*)dst.s + (size_t)i * sb);
    for (size_t j = threadIdx.x; j < sb / 2; j += blockDim.x) e[j] = c[j];
  }
}
__global__ void k_gather_f32(const float* x, const uint32_t* idx, int n, float* y) {
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) y[i] = x[idx[i]];
}

// Dequantized rows (Mat::row_f32) for tests of the bit-exact dequant definition.
template <int BITS, typename ST>
__global__ void k_dequant_rows(MatView w, size_t r0, int nrows, float* out) {
  for (int i = blockIdx.x; i < nrows; i += gridDim.x)
    for (int j = threadIdx.x; j < w.cols; j += blockDim.x) out[(size_t)i * w.cols + j] = weight_at<BITS, ST>(w, r0 + i, j);
}

// ------------------------------------------------------------------------------------------------
// Act::quantize (q8.rs:207-222, the AVX-512 path): per 32 values d = amax/127, inv = 1/d (0 if d = 0),
// q = round-to-nearest-even(x * inv). One warp per block of 32.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void quant_block_warp(float v, int lane, int8_t* q, float* s) {
  float amax = warp_max(fabsf(v));
  float d = div(amax, 127.0f);
  float inv = d > 0.0f ? div(1.0f, d) : 0.0f;
  q[lane] = (int8_t)__float2int_rn(mul(v, inv));
  if (lane == 0) *s = d;
}

// rmsnorm (model.rs:81-87): out = x * r * w with r = 1/sqrt(sum(x^2)/n + eps).
__device__ __forceinline__ float rms_r(float ss, int n, float eps) {
  return div(1.0f, __fsqrt_rn(add(div(ss, (float)n), eps)));
}

// Residual + post-norm, then pre-norm + quantize for the next projection (model.rs:386-395,
// 419-426 and 302-305). One CTA. If delta != nullptr: x += rmsnorm_inplace(delta, w_post) (or delta
// itself when w_post is null). Then xn = rmsnorm(x, w_pre) and (aq, as) = quantize(xn); xn_out (fp32)
// is written when not null (the final-norm hidden state of model.rs:428).
__global__ void k_residual_norm_quant(float* x, const float* delta, const float* w_post, const float* w_pre,
                                      float eps, int d, int8_t* aq, float* as, float* xn_out) {
  pdl_wait();
  extern __shared__ float sm[];
  float* xs = sm;            // d
  float* red = sm + d;       // 32
  int tid = threadIdx.x;
  if (delta) {
    float r = 1.0f;
    if (w_post) {
      float ss = 0.0f;
      for (int j = tid; j < d; j += blockDim.x) { float t = delta[j]; ss += mul(t, t); }
      r = rms_r(block_sum(ss, red), d, eps);
    }
    for (int j = tid; j < d; j += blockDim.x) {
      float t = delta[j];
      if (w_post) t = mul(t, mul(r, w_post[j]));  // rmsnorm_inplace: v *= r * w
      xs[j] = add(x[j], t);
    }
  } else {
    for (int j = tid; j < d; j += blockDim.x) xs[j] = x[j];
  }
  __syncthreads();
  float ss = 0.0f;
  for (int j = tid; j < d; j += blockDim.x) ss += mul(xs[j], xs[j]);
  float r = rms_r(block_sum(ss, red), d, eps);
  __syncthreads();
  if (delta)
    for (int j = tid; j < d; j += blockDim.x) x[j] = xs[j];
  for (int j = tid; j < d; j += blockDim.x) xs[j] = mul(mul(xs[j], r), w_pre[j]);  // rmsnorm: v * r * w
  __syncthreads();
  if (xn_out)
    for (int j = tid; j < d; j += blockDim.x) xn_out[j] = xs[j];
  if (aq) {
    int lane = tid & 31;
    for (int b = tid >> 5; b < d / 32; b += blockDim.x >> 5) quant_block_warp(xs[b * 32 + lane], lane, aq + b * 32, as + b);
  }
}

// Quantize an fp32 vector (Act::quantize) for the kernel-level entry points.
__global__ void k_quantize(const float* x, int n, int8_t* aq, float* as) {
  pdl_wait();
  int lane = threadIdx.x & 31;
  int warps = (blockDim.x >> 5) * gridDim.x;
  for (int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n / 32; b += warps)
    quant_block_warp(x[b * 32 + lane], lane, aq + b * 32, as + b);
}

// ------------------------------------------------------------------------------------------------
// Block-dequant GEMV (q8.rs:248-386, 410-461): y[r] = sum_b (sum_j wq*aq) * (ws[b] * as[b]) for 8/4-bit
// weights; y[r] = sum_j f16(w) * x[j] for F16 weights. One warp per row, each lane one 32-block at a
// time; 128-bit streaming loads; activation staged in shared memory.
// ------------------------------------------------------------------------------------------------
template <int BITS, typename ST>
__device__ __forceinline__ float row_dot(const MatView& w, size_t r, const int8_t* saq, const float* sas,
                                         const float* sx, int lane) {
  const int nb = w.cols / 32;
  float acc = 0.0f;
  if constexpr (BITS == 16) {
    const int4* row = (const int4*)((const __half*)w.q + r * w.cols);
    for (int c = lane; c < w.cols / 8; c += 32) {
      int4 v = ldg_stream(row + c);
      const __half2* h = (const __half2*)&v;
      const float* xv = sx + c * 8;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float2 f = __half22float2(h[k]);
        acc = fmaf(f.x, xv[2 * k], acc);
        acc = fmaf(f.y, xv[2 * k + 1], acc);
      }
    }
  } else if constexpr (BITS == 8) {
    const int4* row = (const int4*)((const int8_t*)w.q + r * w.cols);
    const ST* srow = (const ST*)w.s + r * nb;
    for (int b = lane; b < nb; b += 32) {
      int4 w0 = ldg_stream(row + 2 * b), w1 = ldg_stream(row + 2 * b + 1);
      const int4* a = (const int4*)(saq + b * 32);
      int is = dot32_i8(w0, w1, a[0], a[1]);
      acc = fmaf((float)is, mul(ld_scale(srow, b), sas[b]), acc);
    }
  } else {
    const int4* row = (const int4*)((const uint8_t*)w.q + r * (w.cols / 2));
    const ST* srow = (const ST*)w.s + r * nb;
    for (int b = lane; b < nb; b += 32) {
      int4 wv = ldg_stream(row + b);
      const int4* a = (const int4*)(saq + b * 32);
      int is = dot32_q4(wv, a[0], a[1]);
      acc = fmaf((float)is, mul(ld_scale(srow, b), sas[b]), acc);
    }
  }
  return warp_sum(acc);
}

__device__ __forceinline__ void stage_act(int cols, const int8_t* aq, const float* as, const float* x, int8_t* saq,
                                          float* sas, float* sx, bool f16w) {
  if (f16w) {
    for (int j = threadIdx.x; j < cols; j += blockDim.x) sx[j] = x[j];
  } else {
    for (int j = threadIdx.x; j < cols / 16; j += blockDim.x) ((int4*)saq)[j] = ((const int4*)aq)[j];
    for (int j = threadIdx.x; j < cols / 32; j += blockDim.x) sas[j] = as[j];
  }
  __syncthreads();
}

template <int BITS, typename ST>
__global__ void k_gemv(MatView w, const int8_t* aq, const float* as, const float* x, float* y) {
  pdl_wait();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int8_t* saq = (int8_t*)smem_raw;
  float* sas = (float*)(smem_raw + w.cols);
  float* sx = (float*)smem_raw;
  stage_act(w.cols, aq, as, x, saq, sas, sx, BITS == 16);
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int r = blockIdx.x * nw + warp; r < w.rows; r += gridDim.x * nw) {
    float v = row_dot<BITS, ST>(w, r, saq, sas, sx, lane);
    if (lane == 0) y[r] = v;
  }
}

// ------------------------------------------------------------------------------------------------
// Attention (model.rs:316-383): QK-norm (rmsnorm_inplace), NeoX RoPE with host-computed sin/cos,
// q * 1/sqrt(hd), KV append, scores over the window, softmax with exp_fast, P.V. Split-KV: CTA (s, g)
// handles positions [lo + s*chunk, lo + (s+1)*chunk) for the q heads of kv group g and writes a
// partial (max, sum, unnormalised output); k_attn_merge combines them.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void rmsnorm_inplace_block(float* v, const float* w, int n, float eps, float* red) {
  float ss = 0.0f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) ss += mul(v[j], v[j]);
  float r = rms_r(block_sum(ss, red), n, eps);
  __syncthreads();
  for (int j = threadIdx.x; j < n; j += blockDim.x) v[j] = mul(v[j], mul(r, w[j]));
  __syncthreads();
}
__device__ __forceinline__ void rope_block(float* v, const float* sn, const float* cs, int half) {
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float a = v[i], b = v[i + half];
    v[i] = sub(mul(a, cs[i]), mul(b, sn[i]));
    v[i + half] = add(mul(a, sn[i]), mul(b, cs[i]));
  }
  __syncthreads();
}

__global__ void k_attn_partial(AttnArgs A) {
  pdl_wait();
  extern __shared__ __align__(16) float asm_[];
  const int hd = A.hd, G = A.nh / A.nkv, g = blockIdx.y, s = blockIdx.x;
  float* sq = asm_;                   // G * hd
  float* sk = sq + G * hd;            // hd
  float* sv = sk + hd;                // hd
  float* sc = sv + hd;                // G * chunk scores
  float* red = sc + G * A.chunk;      // 32
  float* stat = red + 32;             // 2 * G
  const uint32_t pos = A.cur->pos;
  const int seq = 0;
  (void)seq;
  const uint32_t lo = (A.window > 0 && pos + 1 > (uint32_t)A.window) ? pos + 1 - A.window : 0;
  const uint32_t n_pos = pos + 1 - lo;
  const uint32_t p0 = lo + (uint32_t)s * A.chunk;
  const uint32_t p1 = min(pos + 1, p0 + (uint32_t)A.chunk);
  const float* sn = A.rope_sin + (size_t)pos * (hd / 2);
  const float* cs = A.rope_cos + (size_t)pos * (hd / 2);
  float* part = A.part + ((size_t)g * A.nsplit + s) * G * (hd + 2);
  (void)n_pos;
  if (p0 > pos) {  // empty split
    for (int j = threadIdx.x; j < G * (hd + 2); j += blockDim.x) part[j] = 0.0f;
    if (threadIdx.x < G) part[threadIdx.x * (hd + 2)] = -INFINITY;
    return;
  }
  const int rw = A.nkv * hd;
  const float* qkv = A.qkv;
  // raw projections plus biases (model.rs:311-315)
  const float* bq = A.bqkv;
  for (int j = threadIdx.x; j < G * hd; j += blockDim.x) {
    size_t i = (size_t)g * G * hd + j;
    sq[j] = bq ? add(qkv[i], bq[i]) : qkv[i];
  }
  for (int j = threadIdx.x; j < hd; j += blockDim.x) {
    size_t ik = (size_t)A.nh * hd + g * hd + j, iv = (size_t)A.nh * hd + rw + g * hd + j;
    sk[j] = bq ? add(qkv[ik], bq[ik]) : qkv[ik];
    sv[j] = bq ? add(qkv[iv], bq[iv]) : qkv[iv];
  }
  __syncthreads();
  for (int h = 0; h < G; ++h) {
    if (A.q_norm) rmsnorm_inplace_block(sq + h * hd, A.q_norm, hd, A.eps, red);
    rope_block(sq + h * hd, sn, cs, hd / 2);
  }
  for (int j = threadIdx.x; j < G * hd; j += blockDim.x) sq[j] = mul(sq[j], A.qscale);
  if (A.k_norm) rmsnorm_inplace_block(sk, A.k_norm, hd, A.eps, red);
  rope_block(sk, sn, cs, hd / 2);
  // KV append (model.rs:333-335): the split that owns `pos` writes the new row.
  float* kc = A.kcache;
  float* vc = A.vcache;
  if (p1 == pos + 1) {
    for (int j = threadIdx.x; j < hd; j += blockDim.x) {
      kc[(size_t)pos * rw + g * hd + j] = sk[j];
      vc[(size_t)pos * rw + g * hd + j] = sv[j];
    }
  }
  // scores: one warp per position
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (uint32_t p = p0 + warp; p < p1; p += nw) {
    const float* krow = (p == pos) ? sk : kc + (size_t)p * rw + g * hd;
    float kreg[8];
    const int per = hd / 32;
    for (int t = 0; t < per; ++t) kreg[t] = krow[lane + 32 * t];
    for (int h = 0; h < G; ++h) {
      float acc = 0.0f;
      for (int t = 0; t < per; ++t) acc = fmaf(sq[h * hd + lane + 32 * t], kreg[t], acc);
      acc = warp_sum(acc);
      if (lane == 0) sc[h * A.chunk + (p - p0)] = acc;
    }
  }
  __syncthreads();
  const int np = (int)(p1 - p0);
  // partial softmax per head: m = max, e = exp_fast(score - m), l = sum e
  for (int h = warp; h < G; h += nw) {
    float m = -INFINITY;
    for (int i = lane; i < np; i += 32) m = fmaxf(m, sc[h * A.chunk + i]);
    m = warp_max(m);
    float l = 0.0f;
    for (int i = lane; i < np; i += 32) {
      float e = exp_fast(sub(sc[h * A.chunk + i], m));
      sc[h * A.chunk + i] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) { stat[2 * h] = m; stat[2 * h + 1] = l; }
  }
  __syncthreads();
  // unnormalised output o[h][j] = sum_i e[h][i] * v_i[j]
  for (int j = threadIdx.x; j < hd; j += blockDim.x) {
    float o[8];
    for (int h = 0; h < G; ++h) o[h] = 0.0f;
    for (int i = 0; i < np; ++i) {
      uint32_t p = p0 + i;
      float vv = (p == pos) ? sv[j] : vc[(size_t)p * rw + g * hd + j];
      for (int h = 0; h < G; ++h) o[h] = fmaf(sc[h * A.chunk + i], vv, o[h]);
    }
    for (int h = 0; h < G; ++h) part[h * (hd + 2) + 2 + j] = o[h];
  }
  if (threadIdx.x < G) {
    part[threadIdx.x * (hd + 2)] = stat[2 * threadIdx.x];
    part[threadIdx.x * (hd + 2) + 1] = stat[2 * threadIdx.x + 1];
  }
}

// Merge the split partials of head h, normalise, and quantize the head's output blocks (the
// Act::quantize of model.rs:384). One CTA per q head, hd threads.
__global__ void k_attn_merge(AttnArgs A, int8_t* aq, float* as) {
  pdl_wait();
  __shared__ float wsm[64];
  __shared__ float tot;
  const int hd = A.hd, G = A.nh / A.nkv, h = blockIdx.x, g = h / G, hh = h % G;
  const float* base = A.part + (size_t)g * A.nsplit * G * (hd + 2) + hh * (hd + 2);
  const size_t stride = (size_t)G * (hd + 2);
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int s = 0; s < A.nsplit; ++s) M = fmaxf(M, base[s * stride]);
    float L = 0.0f;
    for (int s = 0; s < A.nsplit; ++s) {
      float m = base[s * stride], l = base[s * stride + 1];
      float w = (l > 0.0f) ? exp_fast(sub(m, M)) : 0.0f;
      wsm[s] = w;
      L = fmaf(l, w, L);
    }
    tot = div(1.0f, L);
  }
  __syncthreads();
  for (int j = threadIdx.x; j < hd; j += blockDim.x) {
    float o = 0.0f;
    for (int s = 0; s < A.nsplit; ++s)
      if (wsm[s] != 0.0f) o = fmaf(base[s * stride + 2 + j], wsm[s], o);
    float v = mul(o, tot);
    if (A.att_out) A.att_out[h * hd + j] = v;
    // quantize: blocks of 32 never straddle heads (hd is a multiple of 32)
    quant_block_warp(v, threadIdx.x & 31, aq + h * hd + (j & ~31), as + (h * hd + j) / 32);
  }
}

// ------------------------------------------------------------------------------------------------
// GELU-tanh gate (model.rs:408-416): g = 0.5*g*(1 + tanh_fast(0.7978846*(g + 0.044715*g^3)))*u, then
// Act::quantize (model.rs:417). SiLU for qwen2 (model.rs:400-407). gu holds [gate | up].
// ------------------------------------------------------------------------------------------------
__global__ void k_glu_quant(const float* gu, int ff, int silu, int8_t* aq, float* as, float* gout) {
  pdl_wait();
  int lane = threadIdx.x & 31;
  int warps = (blockDim.x >> 5) * gridDim.x;
  for (int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < ff / 32; b += warps) {
    int i = b * 32 + lane;
    float g = gu[i], u = gu[ff + i], v;
    if (silu) {
      float t = exp_fast(-g);
      v = mul(div(g, add(1.0f, t)), u);
    } else {
      float t = mul(0.7978846f, add(g, mul(mul(mul(0.044715f, g), g), g)));
      t = tanh_fast(t);
      v = mul(mul(mul(0.5f, g), add(1.0f, t)), u);
    }
    if (gout) gout[i] = v;
    quant_block_warp(v, lane, aq + b * 32, as + b);
  }
}

// Step bookkeeping for the scoring loop: token, position and target of step `step`.
// Token ids come from caller memory: ids >= vocab are recorded in *err and replaced by 0.
__global__ void k_begin_step(const uint32_t* toks, uint32_t* step, uint32_t base_pos, uint32_t vocab, StepCur* cur, int* err) {
  pdl_wait();
  uint32_t i = *step;
  uint32_t t = toks[i], u = toks[i + 1];
  if (t >= vocab || u >= vocab) {
    atomicExch(err, ERR_RANGE);
    t = t >= vocab ? 0 : t;
    u = u >= vocab ? 0 : u;
  }
  cur->tok = t;
  cur->target = u;
  cur->pos = base_pos + i;
  cur->slot = i;
}
__global__ void k_end_step(uint32_t* step) { pdl_wait(); *step += 1; }

// ------------------------------------------------------------------------------------------------
// Full head (main.rs:20-38): logits = head . quantize(h); online (max, sum e^(z-max)), argmax and the
// target's logit, per CTA; k_head_full_merge finishes lse and logprob = logit[t] - lse. `row_tok` maps
// a row of a class-permuted head back to its token (null = identity). blockIdx.y = batch item.
// ------------------------------------------------------------------------------------------------
template <int BITS, typename ST>
__global__ void k_head_full(HeadArgs H) {
  pdl_wait();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red_m[32], red_s[32], red_v[32];
  __shared__ uint32_t red_t[32];
  const int bi = blockIdx.y;
  const MatView& w = H.w;
  int8_t* saq = (int8_t*)smem_raw;
  float* sas = (float*)(smem_raw + w.cols);
  float* sx = (float*)smem_raw;
  stage_act(w.cols, H.aq + (size_t)bi * w.cols, H.as + (size_t)bi * (w.cols / 32), H.h + (size_t)bi * w.cols, saq, sas,
            sx, BITS == 16);
  uint32_t target = H.targets ? H.targets[bi] : H.cur->target;
  if (target >= (uint32_t)w.rows) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(H.err, ERR_RANGE);
    target = 0;
  }
  const uint32_t trow = H.row_of ? H.row_of[target] : target;
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  Lse L{-INFINITY, 0.0f};
  Best B{-INFINITY, 0xffffffffu};
  for (int r = blockIdx.x * nw + warp; r < w.rows; r += gridDim.x * nw) {
    float z = row_dot<BITS, ST>(w, r, saq, sas, sx, lane);
    L = lse_add(L, z);
    best_row_add(B, z, (uint32_t)r, H.row_tok);
    if ((uint32_t)r == trow && lane == 0) H.tlogit[bi] = z;
  }
  best_row_to_token(B, H.row_tok);
  if (lane == 0) { red_m[warp] = L.m; red_s[warp] = L.s; red_v[warp] = B.v; red_t[warp] = B.tok; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < nw; ++i) {
      L = lse_merge(L, Lse{red_m[i], red_s[i]});
      B = best_merge(B, Best{red_v[i], red_t[i]});
    }
    float4* p = (float4*)(H.part + ((size_t)bi * gridDim.x + blockIdx.x) * 4);
    *p = make_float4(L.m, L.s, B.v, __uint_as_float(B.tok));
  }
}

__global__ void k_head_full_merge(HeadArgs H, int nparts) {
  pdl_wait();
  head_merge(H, blockIdx.x, nparts);
}

// ------------------------------------------------------------------------------------------------
// Two-level head (main.rs:82-107, lean.rs:46-76). Stage 1: class logits cl[c] = A[c].h + b[c] (fp32,
// unquantized h) on the first `class_ctas` CTAs, and the target class's block of rows on the rest.
// Stage 2 (one CTA): lse over classes, the target's logprob, the most likely class, and the best raw
// logit inside it (re-using the target block when the classes coincide).
// ------------------------------------------------------------------------------------------------
template <int BITS, typename ST>
__global__ void k_tl_stage1(TwoLevelArgs T) {
  pdl_wait();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int bi = blockIdx.y;
  const int d = T.w.cols;
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const float* h = T.h + (size_t)bi * d;
  if ((int)blockIdx.x < T.class_ctas) {
    float* sh = (float*)smem_raw;
    for (int j = threadIdx.x; j < d; j += blockDim.x) sh[j] = h[j];
    __syncthreads();
    for (int c = blockIdx.x * nw + warp; c < T.k; c += T.class_ctas * nw) {
      const float4* a = (const float4*)(T.A + (size_t)c * d);
      float acc = 0.0f;
      for (int j = lane; j < d / 4; j += 32) {
        float4 v = a[j];
        acc = fmaf(v.x, sh[4 * j], acc);
        acc = fmaf(v.y, sh[4 * j + 1], acc);
        acc = fmaf(v.z, sh[4 * j + 2], acc);
        acc = fmaf(v.w, sh[4 * j + 3], acc);
      }
      acc = warp_sum(acc);
      if (lane == 0) T.cl[(size_t)bi * T.k + c] = add(acc, T.b[c]);
    }
    return;
  }
  int8_t* saq = (int8_t*)smem_raw;
  float* sas = (float*)(smem_raw + d);
  float* sx = (float*)smem_raw;
  stage_act(d, T.aq + (size_t)bi * d, T.as + (size_t)bi * (d / 32), h, saq, sas, sx, BITS == 16);
  uint32_t target = T.targets ? T.targets[bi] : T.cur->target;
  if (target >= (uint32_t)T.vocab) target = 0;  // recorded by stage 2
  const uint32_t c = T.cls_of[target];
  const uint32_t first = c * T.per;
  const uint32_t n = min((uint32_t)T.per, (uint32_t)T.w.rows - first);
  const int bctas = gridDim.x - T.class_ctas;
  for (uint32_t j = (blockIdx.x - T.class_ctas) * nw + warp; j < n; j += bctas * nw) {
    float z = row_dot<BITS, ST>(T.w, first + j, saq, sas, sx, lane);
    if (lane == 0) T.inner[(size_t)bi * T.per + j] = z;
  }
}

template <int BITS, typename ST>
__global__ void k_tl_stage2(TwoLevelArgs T) {
  pdl_wait();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[32];
  __shared__ float red2[32];
  __shared__ uint32_t redi[32];
  __shared__ uint32_t s_top;
  const int bi = blockIdx.x;
  const int d = T.w.cols;
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const float* cl = T.cl + (size_t)bi * T.k;
  const float* inner = T.inner + (size_t)bi * T.per;
  uint32_t target = T.targets ? T.targets[bi] : T.cur->target;
  if (target >= (uint32_t)T.vocab) {
    if (threadIdx.x == 0) atomicExch(T.err, ERR_RANGE);
    target = 0;
  }
  const uint32_t ct = T.cls_of[target];
  const uint32_t nt = min((uint32_t)T.per, (uint32_t)T.w.rows - ct * T.per);
  // class lse + first argmax
  Lse L{-INFINITY, 0.0f};
  float bv = -INFINITY;
  uint32_t bc = 0xffffffffu;
  for (int c = threadIdx.x; c < T.k; c += blockDim.x) {
    float z = cl[c];
    L = lse_add(L, z);
    if (z > bv || (z == bv && (uint32_t)c < bc)) { bv = z; bc = c; }
  }
  for (int o = 16; o > 0; o >>= 1) {
    Lse l2{__shfl_xor_sync(0xffffffffu, L.m, o), __shfl_xor_sync(0xffffffffu, L.s, o)};
    L = lse_merge(L, l2);
    float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
    uint32_t c2 = __shfl_xor_sync(0xffffffffu, bc, o);
    if (v2 > bv || (v2 == bv && c2 < bc)) { bv = v2; bc = c2; }
  }
  if (lane == 0) { red[warp] = L.m; red2[warp] = L.s; }
  __syncthreads();
  __shared__ float s_bv[32];
  if (lane == 0) { s_bv[warp] = bv; redi[warp] = bc; }
  __syncthreads();
  __shared__ float s_lse_cl;
  if (threadIdx.x == 0) {
    for (int i = 1; i < nw; ++i) {
      L = lse_merge(L, Lse{red[i], red2[i]});
      if (s_bv[i] > bv || (s_bv[i] == bv && redi[i] < bc)) { bv = s_bv[i]; bc = redi[i]; }
    }
    s_lse_cl = L.m + logf(L.s);
    s_top = bc < (uint32_t)T.k ? bc : 0;  // only NaN logits leave no candidate
  }
  __syncthreads();
  // inner lse over the target block
  Lse Li{-INFINITY, 0.0f};
  for (uint32_t j = threadIdx.x; j < nt; j += blockDim.x) Li = lse_add(Li, inner[j]);
  for (int o = 16; o > 0; o >>= 1) {
    Lse l2{__shfl_xor_sync(0xffffffffu, Li.m, o), __shfl_xor_sync(0xffffffffu, Li.s, o)};
    Li = lse_merge(Li, l2);
  }
  __syncthreads();
  if (lane == 0) { red[warp] = Li.m; red2[warp] = Li.s; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < nw; ++i) Li = lse_merge(Li, Lse{red[i], red2[i]});
    float lse_in = Li.m + logf(Li.s);
    uint32_t slot = T.targets ? (uint32_t)bi : T.cur->slot;
    if (T.lp_out) T.lp_out[slot] = cl[ct] - s_lse_cl + inner[T.pos_of[target]] - lse_in;
  }
  if (!T.am_out) return;
  // greedy token inside the most likely class
  const uint32_t top = s_top;
  const uint32_t first = top * T.per;
  const uint32_t n = min((uint32_t)T.per, (uint32_t)T.w.rows - first);
  float* sco = (float*)(smem_raw + ((d * 5 + 15) / 16) * 16 * (BITS == 16 ? 1 : 1));
  if (top == ct) {
    for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) sco[j] = inner[j];
  } else {
    int8_t* saq = (int8_t*)smem_raw;
    float* sas = (float*)(smem_raw + d);
    float* sx = (float*)smem_raw;
    const float* h = T.h + (size_t)bi * d;
    stage_act(d, T.aq + (size_t)bi * d, T.as + (size_t)bi * (d / 32), h, saq, sas, sx, BITS == 16);
    for (uint32_t j = warp; j < n; j += nw) {
      float z = row_dot<BITS, ST>(T.w, first + j, saq, sas, sx, lane);
      if (lane == 0) sco[j] = z;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t bj = 0;
    for (uint32_t j = 1; j < n; ++j)
      if (sco[j] > sco[bj]) bj = j;
    uint32_t slot = T.targets ? (uint32_t)bi : T.cur->slot;
    T.am_out[slot] = T.order[first + bj];
  }
}

// Two-level head, split form used by the exact path: select = class lse, most likely class (first
// maximum), target logprob (main.rs:101-107); argmax = best raw logit inside the top class block
// (lean.rs:46-76 with top = 1), whose logits another kernel wrote to top_inner.
__global__ void k_tl_select(TwoLevelArgs T, uint32_t* top_of) {
  pdl_wait();
  __shared__ float rm[32], rs[32], rv[32];
  __shared__ uint32_t rc[32];
  __shared__ float s_lse_cl;
  const int bi = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const float* cl = T.cl + (size_t)bi * T.k;
  const float* inner = T.inner + (size_t)bi * T.per;
  uint32_t target = T.targets ? T.targets[bi] : T.cur->target;
  if (target >= (uint32_t)T.vocab) {
    if (threadIdx.x == 0) atomicExch(T.err, ERR_RANGE);
    target = 0;
  }
  const uint32_t ct = T.cls_of[target];
  const uint32_t nt = min((uint32_t)T.per, (uint32_t)T.w.rows - ct * T.per);
  Lse L{-INFINITY, 0.0f};
  Best B{-INFINITY, 0xffffffffu};
  for (int c = threadIdx.x; c < T.k; c += blockDim.x) {
    L = lse_add(L, cl[c]);
    B = best_merge(B, Best{cl[c], (uint32_t)c});
  }
  for (int o = 16; o > 0; o >>= 1) {
    L = lse_merge(L, Lse{__shfl_xor_sync(0xffffffffu, L.m, o), __shfl_xor_sync(0xffffffffu, L.s, o)});
    B = best_merge(B, Best{__shfl_xor_sync(0xffffffffu, B.v, o), __shfl_xor_sync(0xffffffffu, B.tok, o)});
  }
  if (lane == 0) { rm[warp] = L.m; rs[warp] = L.s; rv[warp] = B.v; rc[warp] = B.tok; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < nw; ++i) {
      L = lse_merge(L, Lse{rm[i], rs[i]});
      B = best_merge(B, Best{rv[i], rc[i]});
    }
    s_lse_cl = L.m + logf(L.s);
    top_of[bi] = B.tok < (uint32_t)T.k ? B.tok : 0;  // only NaN logits leave no candidate
  }
  __syncthreads();
  Lse Li{-INFINITY, 0.0f};
  for (uint32_t j = threadIdx.x; j < nt; j += blockDim.x) Li = lse_add(Li, inner[j]);
  for (int o = 16; o > 0; o >>= 1)
    Li = lse_merge(Li, Lse{__shfl_xor_sync(0xffffffffu, Li.m, o), __shfl_xor_sync(0xffffffffu, Li.s, o)});
  if (lane == 0) { rm[warp] = Li.m; rs[warp] = Li.s; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < nw; ++i) Li = lse_merge(Li, Lse{rm[i], rs[i]});
    uint32_t slot = T.targets ? (uint32_t)bi : T.cur->slot;
    if (T.lp_out) T.lp_out[slot] = cl[ct] - s_lse_cl + inner[T.pos_of[target]] - (Li.m + logf(Li.s));
  }
}

__global__ void k_tl_argmax(TwoLevelArgs T, const uint32_t* top_of, const float* top_inner) {
  pdl_wait();
  __shared__ float rv[32];
  __shared__ uint32_t rj[32];
  const int bi = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const uint32_t top = top_of[bi], first = top * T.per;
  const uint32_t n = min((uint32_t)T.per, (uint32_t)T.w.rows - first);
  const float* z = top_inner + (size_t)bi * T.per;
  Best B{-INFINITY, 0xffffffffu};
  for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) B = best_merge(B, Best{z[j], j});
  for (int o = 16; o > 0; o >>= 1)
    B = best_merge(B, Best{__shfl_xor_sync(0xffffffffu, B.v, o), __shfl_xor_sync(0xffffffffu, B.tok, o)});
  if (lane == 0) { rv[warp] = B.v; rj[warp] = B.tok; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < nw; ++i) B = best_merge(B, Best{rv[i], rj[i]});
    uint32_t slot = T.targets ? (uint32_t)bi : T.cur->slot;
    if (T.am_out) T.am_out[slot] = T.order[first + (B.tok < n ? B.tok : 0)];
  }
}

// ------------------------------------------------------------------------------------------------
// Explicit instantiations and launchers
// ------------------------------------------------------------------------------------------------
#define GEM_DISPATCH(bits, scale_f32, F)                      \
  do {                                                        \
    if ((bits) == 8 && !(scale_f32)) { F(8, __half); }        \
    else if ((bits) == 8) { F(8, float); }                    \
    else if ((bits) == 4 && !(scale_f32)) { F(4, __half); }   \
    else if ((bits) == 4) { F(4, float); }                    \
    else { F(16, __half); }                                   \
  } while (0)

static size_t act_smem(int cols, int bits) {
  return bits == 16 ? (size_t)cols * 4 : (size_t)cols + (size_t)cols / 32 * 4;
}

void launch_embed(const MatView& head, const uint32_t* row_of, const StepCur* cur, float scale, float* x, cudaStream_t st) {
#define F(B, S) launch_k(k_embed<B, S>, dim3(1), dim3(256), 0, st, head, row_of, cur, scale, x)
  GEM_DISPATCH(head.bits, head.scale_f32, F);
#undef F
}
void launch_gather_rows(const MatView& src, const uint32_t* src_row, const MatView& dst, cudaStream_t st) {
  k_gather_rows<<<min(dst.rows, 4 * 1184), 128, 0, st>>>(src, src_row, dst);
}
void launch_gather_f32(const float* x, const uint32_t* idx, int n, float* y, cudaStream_t st) {
  launch_k(k_gather_f32, dim3(min((n + 255) / 256, 4096)), dim3(256), 0, st, x, idx, n, y);
}
void launch_dequant_rows(const MatView& w, size_t r0, int nrows, float* out, cudaStream_t st) {
#define F(B, S) k_dequant_rows<B, S><<<min(nrows, 1024), 256, 0, st>>>(w, r0, nrows, out)
  GEM_DISPATCH(w.bits, w.scale_f32, F);
#undef F
}
void launch_residual_norm_quant(float* x, const float* delta, const float* w_post, const float* w_pre, float eps, int d,
                                int8_t* aq, float* as, float* xn_out, cudaStream_t st) {
  launch_k(k_residual_norm_quant, dim3(1), dim3(1024), (size_t)(d + 32) * 4, st, x, delta, w_post, w_pre, eps, d, aq, as, xn_out);
}
void launch_quantize(const float* x, int n, int8_t* aq, float* as, cudaStream_t st) {
  int blocks = (n / 32 + 7) / 8;
  launch_k(k_quantize, dim3(blocks), dim3(256), 0, st, x, n, aq, as);
}
void launch_gemv(const MatView& w, const int8_t* aq, const float* as, const float* x, float* y, int sms, cudaStream_t st) {
  const int threads = 256, nw = threads / 32;
  int blocks = (w.rows + nw - 1) / nw;
  blocks = min(blocks, sms * 8);
  size_t sm = act_smem(w.cols, w.bits);
#define F(B, S)                                                                                     \
  do {                                                                                              \
    static bool init = false;                                                                       \
    if (!init) { cudaFuncSetAttribute(k_gemv<B, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); init = true; } \
    launch_k(k_gemv<B, S>, dim3(blocks), dim3(threads), sm, st, w, aq, as, x, y);                   \
  } while (0)
  GEM_DISPATCH(w.bits, w.scale_f32, F);
#undef F
}
void launch_attn(const AttnArgs& A, int8_t* aq, float* as, cudaStream_t st) {
  dim3 grid(A.nsplit, A.nkv);
  int G = A.nh / A.nkv;
  size_t sm = (size_t)(G * A.hd + 2 * A.hd + G * A.chunk + 32 + 2 * G) * 4;
  launch_k(k_attn_partial, grid, dim3(256), sm, st, A);
  launch_k(k_attn_merge, dim3(A.nh), dim3(A.hd), 0, st, A, aq, as);
}
void launch_glu_quant(const float* gu, int ff, int silu, int8_t* aq, float* as, float* gout, cudaStream_t st) {
  int blocks = (ff / 32 + 7) / 8;
  launch_k(k_glu_quant, dim3(blocks), dim3(256), 0, st, gu, ff, silu, aq, as, gout);
}
void launch_begin_step(const uint32_t* toks, uint32_t* step, uint32_t base_pos, uint32_t vocab, StepCur* cur, int* err,
                       cudaStream_t st) {
  launch_k(k_begin_step, dim3(1), dim3(1), 0, st, toks, step, base_pos, vocab, cur, err);
}
void launch_end_step(uint32_t* step, cudaStream_t st) { launch_k(k_end_step, dim3(1), dim3(1), 0, st, step); }

int head_full_parts(int sms) { return sms * 2; }

void launch_head_full(const HeadArgs& H, int batch, int sms, cudaStream_t st) {
  int parts = head_full_parts(sms);
  dim3 grid(parts, batch);
  size_t sm = act_smem(H.w.cols, H.w.bits);
#define F(B, S)                                                                                     \
  do {                                                                                              \
    static bool init = false;                                                                       \
    if (!init) { cudaFuncSetAttribute(k_head_full<B, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); init = true; } \
    launch_k(k_head_full<B, S>, grid, dim3(512), sm, st, H);                                          \
  } while (0)
  GEM_DISPATCH(H.w.bits, H.w.scale_f32, F);
#undef F
  launch_head_full_merge(H, batch, parts, st);
}

void launch_head_full_merge(const HeadArgs& H, int batch, int parts, cudaStream_t st) {
  launch_k(k_head_full_merge, dim3(batch), dim3(256), 0, st, H, parts);
}

void launch_tl_select(const TwoLevelArgs& T, int batch, uint32_t* top_of, cudaStream_t st) {
  launch_k(k_tl_select, dim3(batch), dim3(256), 0, st, T, top_of);
}
void launch_tl_argmax(const TwoLevelArgs& T, int batch, const uint32_t* top_of, const float* top_inner, cudaStream_t st) {
  launch_k(k_tl_argmax, dim3(batch), dim3(256), 0, st, T, top_of, top_inner);
}

void launch_head_twolevel(const TwoLevelArgs& T, int batch, int sms, cudaStream_t st) {
  int block_ctas = max(1, min(8, (T.per + 15) / 16));
  int class_ctas = max(1, min(sms - block_ctas, (T.k + 7) / 8));
  TwoLevelArgs t2 = T;
  t2.class_ctas = class_ctas;
  dim3 grid(class_ctas + block_ctas, batch);
  size_t sm1 = max(act_smem(T.w.cols, T.w.bits), (size_t)T.w.cols * 4);
  size_t sm2 = ((size_t)(T.w.cols * 5 + 15) / 16) * 16 + (size_t)T.per * 4;
  sm2 = max(sm2, act_smem(T.w.cols, T.w.bits) + (size_t)T.per * 4 + 64);
#define F(B, S)                                                                                     \
  do {                                                                                              \
    static bool init = false;                                                                       \
    if (!init) {                                                                                    \
      cudaFuncSetAttribute(k_tl_stage1<B, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); \
      cudaFuncSetAttribute(k_tl_stage2<B, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); \
      init = true;                                                                                  \
    }                                                                                               \
    launch_k(k_tl_stage1<B, S>, grid, dim3(256), sm1, st, t2);                                        \
    launch_k(k_tl_stage2<B, S>, dim3(batch), dim3(256), sm2, st, t2);                                 \
  } while (0)
  GEM_DISPATCH(T.w.bits, T.w.scale_f32, F);
#undef F
}

}  // namespace gem
