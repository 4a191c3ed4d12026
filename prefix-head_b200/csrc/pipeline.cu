// Layer-pipelined scoring: one persistent kernel scores a whole sequence with exact numerics.
//
// In scoring mode every input token is known up front, and token t+1 at layer l needs only its own
// residual from layer l-1 and the KV rows that tokens <= t wrote at layer l. So the grid is split into
// stages - G CTAs per decoder layer plus GH CTAs for the output head - and tokens flow through the
// stages as a wavefront: while layer l works on token t, layer l+1 works on token t-1. Each token's
// arithmetic is exactly the per-token forward's (model.rs:286-430, bit-identical to the reference's
// AVX-512 path, see exact.cuh) and each token still reads every weight once, so the bytes per token
// are unchanged; what changes is that HBM streaming of all layers overlaps instead of waiting on the
// per-token dependency chain (norm -> GEMV -> attention -> GEMV ...), whose latency bounds a
// token-at-a-time forward.
//
// Synchronisation: inside a stage, a counter barrier among its CTAs; between stages, a ring of R
// residual slots with ready / consumed counters. Every wait is bounded by a clock deadline; on
// timeout the kernel records ERR_TIMEOUT and every CTA returns. All CTAs are co-resident (cooperative
// launch, one CTA per SM), so waits between CTAs of one grid always make progress.
#include "exact.cuh"
#include "kernels.cuh"
#include "pipeline.cuh"

namespace gem {

namespace {


__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_err(const int* p) { return *(const volatile int*)p; }

// One thread: wait until *p >= target. False on timeout or when another CTA has failed.
__device__ bool wait_geq(const unsigned* p, unsigned target, int* err, unsigned long long limit_ns) {
  if (ld_acquire(p) >= target) return true;
  const unsigned long long t0 = now_ns();
  for (unsigned it = 0;; ++it) {
    if (ld_acquire(p) >= target) return true;
    if ((it & 63) == 0) {
      if (ld_err(err) != 0) return false;
      if (now_ns() - t0 > limit_ns) {
        atomicCAS(err, 0, ERR_TIMEOUT);
        return false;
      }
    }
  }
}

// Barrier among the `n` CTAs of a stage. `epoch` counts this CTA's barriers (same sequence in every
// CTA of the stage). Returns false (in every thread) when the kernel must stop.
__device__ bool stage_barrier(unsigned* ctr, unsigned& epoch, unsigned n, int* err, int* s_ok, unsigned long long limit_ns) {
  __syncthreads();
  if (threadIdx.x == 0) {
    epoch += 1;
    __threadfence();
    atomicAdd(ctr, 1u);
    *s_ok = wait_geq(ctr, epoch * n, err, limit_ns);
    __threadfence();
  }
  __syncthreads();
  return *s_ok;
}

__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }

// dot512 (model.rs:106-120) where `b` lives in global memory written by another CTA (L2 loads).
__device__ __forceinline__ float dot512_pair_cg(const float* a, const float* b, int n, int half) {
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  for (int c = 0; c < n / 16; ++c) {
    const float4 a0 = *(const float4*)(a + c * 16 + half * 8), a1 = *(const float4*)(a + c * 16 + half * 8 + 4);
    const float4 b0 = __ldcg((const float4*)(b + c * 16 + half * 8)), b1 = __ldcg((const float4*)(b + c * 16 + half * 8 + 4));
    acc[0] = fmaf(a0.x, b0.x, acc[0]); acc[1] = fmaf(a0.y, b0.y, acc[1]);
    acc[2] = fmaf(a0.z, b0.z, acc[2]); acc[3] = fmaf(a0.w, b0.w, acc[3]);
    acc[4] = fmaf(a1.x, b1.x, acc[4]); acc[5] = fmaf(a1.y, b1.y, acc[5]);
    acc[6] = fmaf(a1.z, b1.z, acc[6]); acc[7] = fmaf(a1.w, b1.w, acc[7]);
  }
  return reduce16_pair(acc);
}

// Rows [r0, r1) of w against the staged activation; lane pairs per row, 16 rows per warp step.
template <int BITS, typename ST, typename F>
__device__ __forceinline__ void rows_exact(const MatView& w, int r0, int r1, const int8_t* saq, const float* sas,
                                           const float* sx, F&& out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, half = lane & 1;
  for (int base = r0 + warp * 16; base < r1; base += nw * 16) {
    int r = base + (lane >> 1);
    bool ok = r < r1;
    float v = row_dot_exact<BITS, ST>(w, ok ? r : r1 - 1, half, saq, sas, sx);
    if (ok && half == 0) out(r, v);
  }
}

template <int BITS, typename ST>
__device__ __forceinline__ float emb_weight(const MatView& w, size_t r, int j) {
  if constexpr (BITS == 16) {
    return __half2float(((const __half*)w.q)[r * w.cols + j]);
  } else if constexpr (BITS == 8) {
    return mul((float)((const int8_t*)w.q)[r * w.cols + j], ld_scale((const ST*)w.s, (r * w.cols + j) / 32));
  } else {
    int blk = j / 32, k = j % 32;
    uint8_t byte = ((const uint8_t*)w.q)[r * w.cols / 2 + blk * 16 + (k % 16)];
    return mul((float)((k < 16 ? (byte & 15) : (byte >> 4)) - 8), ld_scale((const ST*)w.s, (r * w.cols + j) / 32));
  }
}

// Quantize `n` floats of smem `v` into smem (q, s): Act::quantize, one warp per 32-block.
__device__ __forceinline__ void quantize_smem(const float* v, int n, int8_t* q, float* s) {
  const int lane = threadIdx.x & 31;
  for (int b = threadIdx.x >> 5; b < n / 32; b += blockDim.x >> 5) quant_block_warp_x(v[b * 32 + lane], lane, q + b * 32, s + b);
}

// Floats of the scores / class-logit / FFN-slice buffer.
__host__ __device__ inline size_t pipe_p_floats(const PipeArgs& P) {
  size_t a = (size_t)P.nh * P.max_npos, b = (size_t)P.k, c = 2 * ((size_t)(P.ff + P.G - 1) / P.G + 32);
  return a > b ? (a > c ? a : c) : (b > c ? b : c);
}

struct Smem {
  float* x;      // d: residual
  float* xn;     // max(d, ff): normalised / staged fp32 activation
  int8_t* aq;    // max(d, nh*hd, ff): quantized activation
  float* as;     // max(..)/32
  float* q;      // nh*hd
  float* k;      // nkv*hd
  float* v;      // nkv*hd
  float* p;      // nh * max_npos: scores, then probabilities
  float* r;      // 32 scalars
  int* ok;
};

__device__ Smem carve(unsigned char* base, const PipeArgs& P) {
  Smem S;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    unsigned char* p = base + off;
    off += (bytes + 15) / 16 * 16;
    return p;
  };
  int wide = max(max(P.d, P.nh * P.hd), P.ff);
  S.x = (float*)take((size_t)P.d * 4);
  S.xn = (float*)take((size_t)wide * 4);
  S.aq = (int8_t*)take((size_t)wide);
  S.as = (float*)take((size_t)wide / 32 * 4);
  S.q = (float*)take((size_t)P.nh * P.hd * 4);
  S.k = (float*)take((size_t)P.nkv * P.hd * 4);
  S.v = (float*)take((size_t)P.nkv * P.hd * 4);
  S.p = (float*)take(pipe_p_floats(P) * 4);
  S.r = (float*)take(32 * 4);
  S.ok = (int*)take(16);
  return S;
}

// ------------------------------------------------------------------------------------------------
// A decoder layer stage.
// ------------------------------------------------------------------------------------------------
template <int BITS, typename ST, int BH, typename SH>
__device__ void layer_stage(const PipeArgs& P, int l, int c, const Smem& S) {
  const PipeLayer& L = P.layers[l];
  const int d = P.d, hd = P.hd, nh = P.nh, nkv = P.nkv, ff = P.ff, G = P.G, T = P.ref_threads;
  const int grp = nh / nkv, rw = nkv * hd, qkv_rows = (nh + 2 * nkv) * hd;
  const int tid = threadIdx.x, nt = blockDim.x;
  float* scr = P.scratch + (size_t)l * P.scratch_stride;  // layout of pipe_scratch_floats
  auto r16 = [](size_t f) { return (f + 15) / 16 * 16; };
  float* qkv_g = scr;                                     // qkv_rows
  float* sc_g = qkv_g + r16(qkv_rows);                    // nh * max_npos
  float* pv_g = sc_g + r16((size_t)nh * P.max_npos);      // T * nh*hd
  float* o_g = pv_g + r16((size_t)T * nh * hd);           // d
  float* dn_g = o_g + r16(d);                             // d
  float* gs_g = dn_g + r16(d);                            // ff/32
  int8_t* gq_g = (int8_t*)(gs_g + r16(ff / 32));          // ff bytes
  unsigned* bar = P.bar + l * 32;
  unsigned epoch = 0;
  const float* nw = L.attn_norm;
  auto span = [&](int total, int align) {  // this CTA's share of [0, total), in multiples of align
    int per = ((total + G - 1) / G + align - 1) / align * align;
    int a = min(total, c * per), b = min(total, a + per);
    return make_int2(a, b);
  };

  for (int t = 0; t < P.n; ++t) {
    const uint32_t pos = P.base_pos + t;
    const int slot = t % PIPE_RING;
    // ---- input residual ----
    if (l == 0) {
      uint32_t tok = P.toks[t];
      if (tok >= (uint32_t)P.vocab) {
        if (tid == 0) atomicCAS(P.err, 0, ERR_RANGE);
        tok = 0;
      }
      for (int j = tid; j < d; j += nt) S.x[j] = mul(emb_weight<BH, SH>(P.emb, tok, j), P.embed_scale);
    } else {
      if (tid == 0) *S.ok = wait_geq(P.ready + l * PIPE_RING + slot, (unsigned)t + 1, P.err, P.wait_ns);
      __syncthreads();
      if (!*S.ok) return;
      const float* src = P.ring + ((size_t)l * PIPE_RING + slot) * d;
      for (int j = tid; j < d; j += nt) S.x[j] = ldcg(src + j);
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        atomicAdd(P.consumed + l, 1u);
      }
    }
    __syncthreads();
    // ---- attn_norm + quantize (model.rs:304-305) ----
    if (tid == 0) S.r[0] = rms_r_exact(seq_sumsq(S.x, d), d, P.eps);
    __syncthreads();
    for (int j = tid; j < d; j += nt) S.xn[j] = mul(mul(S.x[j], S.r[0]), nw[j]);
    __syncthreads();
    quantize_smem(S.xn, d, S.aq, S.as);
    __syncthreads();
    // ---- q/k/v projections, this CTA's rows (model.rs:307-309) ----
    {
      int2 rr = span(qkv_rows, 16);
      rows_exact<BITS, ST>(L.qkv, rr.x, rr.y, S.aq, S.as, S.xn, [&](int r, float v) { qkv_g[r] = v; });
    }
    if (!stage_barrier(bar, epoch, G, P.err, S.ok, P.wait_ns)) return;
    // ---- QK-norm, RoPE, q scale (model.rs:311-332), redundant in every CTA ----
    for (int j = tid; j < qkv_rows; j += nt) {
      float v = ldcg(qkv_g + j);
      if (L.bqkv) v = add(v, L.bqkv[j]);
      if (j < nh * hd) S.q[j] = v;
      else if (j < (nh + nkv) * hd) S.k[j - nh * hd] = v;
      else S.v[j - (nh + nkv) * hd] = v;
    }
    __syncthreads();
    if (tid < nh + nkv) {
      const float* vv = tid < nh ? S.q + tid * hd : S.k + (tid - nh) * hd;
      const float* w = tid < nh ? L.q_norm : L.k_norm;
      S.r[1 + tid] = w ? rms_r_exact(seq_sumsq(vv, hd), hd, P.eps) : 1.0f;
    }
    __syncthreads();
    {
      const int half = hd / 2;
      const float* sn = L.rope_sin + (size_t)pos * half;
      const float* cs = L.rope_cos + (size_t)pos * half;
      for (int u = tid; u < (nh + nkv) * half; u += nt) {
        int h = u / half, i = u % half;
        float* vv = h < nh ? S.q + h * hd : S.k + (h - nh) * hd;
        const float* w = h < nh ? L.q_norm : L.k_norm;
        float r = S.r[1 + h], a = vv[i], b = vv[i + half];
        if (w) {
          a = mul(a, mul(r, w[i]));
          b = mul(b, mul(r, w[i + half]));
        }
        float na = sub(mul(a, cs[i]), mul(b, sn[i])), nb = add(mul(a, sn[i]), mul(b, cs[i]));
        if (h < nh) {
          na = mul(na, P.qscale);
          nb = mul(nb, P.qscale);
        }
        vv[i] = na;
        vv[i + half] = nb;
      }
    }
    __syncthreads();
    if (c == 0)  // KV append (model.rs:333-335)
      for (int j = tid; j < rw; j += nt) {
        L.kcache[(size_t)pos * rw + j] = S.k[j];
        L.vcache[(size_t)pos * rw + j] = S.v[j];
      }
    // ---- scores for this CTA's positions (model.rs:344-353) ----
    const uint32_t lo = (L.window > 0 && pos + 1 > (uint32_t)L.window) ? pos + 1 - L.window : 0;
    const int n_pos = (int)(pos + 1 - lo);
    {
      int2 pr = span(n_pos, 1);
      const int lane = tid & 31, warp = tid >> 5, nw2 = nt >> 5, half = lane & 1;
      const int total = (pr.y - pr.x) * nh;
      for (int base = warp * 16; base < total; base += nw2 * 16) {
        int u = base + (lane >> 1);
        bool okk = u < total;
        int uu = okk ? u : 0;
        int i = pr.x + uu / nh, h = uu % nh;
        const int g = h / grp;
        float s;
        if (lo + i == pos) s = dot512_pair(S.q + h * hd, S.k + g * hd, hd, half);
        else s = dot512_pair_cg(S.q + h * hd, L.kcache + (size_t)(lo + i) * rw + g * hd, hd, half);
        if (okk && half == 0) sc_g[(size_t)h * P.max_npos + i] = s;
      }
    }
    if (!stage_barrier(bar, epoch, G, P.err, S.ok, P.wait_ns)) return;
    // ---- softmax per head, reference order (model.rs:354-361), redundant in every CTA ----
    for (int u = tid; u < nh * n_pos; u += nt) {
      int h = u / n_pos, i = u % n_pos;
      S.p[h * P.max_npos + i] = ldcg(sc_g + (size_t)h * P.max_npos + i);
    }
    __syncthreads();
    {
      const int lane = tid & 31, warp = tid >> 5;
      if (warp < nh) {  // one warp per head: max, then exp_fast(s - max)
        float* ph = S.p + warp * P.max_npos;
        float m = -INFINITY;
        for (int i = lane; i < n_pos; i += 32) m = fmaxf(m, ph[i]);
        m = warp_max(m);
        for (int i = lane; i < n_pos; i += 32) ph[i] = exp_fast(sub(ph[i], m));
        __syncwarp();
        if (lane == 0) {
          float sum = 0.0f;
          for (int i = 0; i < n_pos; ++i) sum = add(sum, ph[i]);
          S.r[16 + warp] = div(1.0f, sum);
        }
      }
    }
    __syncthreads();
    for (int u = tid; u < nh * n_pos; u += nt) {
      int h = u / n_pos, i = u % n_pos;
      S.p[h * P.max_npos + i] = mul(S.p[h * P.max_npos + i], S.r[16 + h]);
    }
    __syncthreads();
    // ---- P.V over the pool's position ranges (model.rs:362-376), this CTA's ranges ----
    {
      const int per = (n_pos + T - 1) / T;
      for (int tt = c; tt < T; tt += G) {
        const int i0 = min(tt * per, n_pos), i1 = min((tt + 1) * per, n_pos);
        for (int u = tid; u < nh * hd; u += nt) {
          const int h = u / hd, j = u % hd, g = h / grp;
          float acc = 0.0f;
          for (int i = i0; i < i1; ++i) {
            float vv = (lo + i == pos) ? S.v[g * hd + j] : ldcg(L.vcache + (size_t)(lo + i) * rw + g * hd + j);
            acc = fmaf(S.p[h * P.max_npos + i], vv, acc);
          }
          pv_g[(size_t)tt * nh * hd + u] = acc;
        }
      }
    }
    if (!stage_barrier(bar, epoch, G, P.err, S.ok, P.wait_ns)) return;
    // ---- partials summed in thread order (model.rs:377-382), quantize (model.rs:384) ----
    for (int u = tid; u < nh * hd; u += nt) {
      float a = 0.0f;
      for (int tt = 0; tt < T; ++tt) a = add(a, ldcg(pv_g + (size_t)tt * nh * hd + u));
      S.xn[u] = a;
    }
    __syncthreads();
    quantize_smem(S.xn, nh * hd, S.aq, S.as);
    __syncthreads();
    // ---- O projection, this CTA's rows (model.rs:386) ----
    {
      int2 rr = span(d, 16);
      rows_exact<BITS, ST>(L.o, rr.x, rr.y, S.aq, S.as, S.xn, [&](int r, float v) { o_g[r] = v; });
    }
    if (!stage_barrier(bar, epoch, G, P.err, S.ok, P.wait_ns)) return;
    // ---- post-attention norm, residual, ffn norm, quantize (model.rs:388-395) ----
    for (int j = tid; j < d; j += nt) S.xn[j] = ldcg(o_g + j);
    __syncthreads();
    if (tid == 0) S.r[0] = L.post_attn ? rms_r_exact(seq_sumsq(S.xn, d), d, P.eps) : 1.0f;
    __syncthreads();
    for (int j = tid; j < d; j += nt) {
      float t2 = S.xn[j];
      if (L.post_attn) t2 = mul(t2, mul(S.r[0], L.post_attn[j]));
      S.x[j] = add(S.x[j], t2);
    }
    __syncthreads();
    if (tid == 0) S.r[0] = rms_r_exact(seq_sumsq(S.x, d), d, P.eps);
    __syncthreads();
    for (int j = tid; j < d; j += nt) S.xn[j] = mul(mul(S.x[j], S.r[0]), L.ffn_norm[j]);
    __syncthreads();
    quantize_smem(S.xn, d, S.aq, S.as);
    __syncthreads();
    // ---- gate/up for this CTA's FFN slice, GELU / SiLU, quantize (model.rs:397-417) ----
    {
      int2 fr = span(ff, 32);
      float* gbuf = S.p;  // reuse: 2 * slice floats
      const int n = fr.y - fr.x;
      rows_exact<BITS, ST>(L.gu, fr.x, fr.y, S.aq, S.as, S.xn, [&](int r, float v) { gbuf[r - fr.x] = v; });
      rows_exact<BITS, ST>(L.gu, ff + fr.x, ff + fr.y, S.aq, S.as, S.xn, [&](int r, float v) { gbuf[n + r - ff - fr.x] = v; });
      __syncthreads();
      for (int i = tid; i < n; i += nt) {
        float g = gbuf[i], u = gbuf[n + i], vv;
        if (P.silu) {
          vv = mul(div(g, add(1.0f, exp_fast(-g))), u);
        } else {
          float tt = mul(0.7978846f, add(g, mul(mul(mul(0.044715f, g), g), g)));
          vv = mul(mul(mul(0.5f, g), add(1.0f, tanh_fast(tt))), u);
        }
        gbuf[i] = vv;
      }
      __syncthreads();
      const int lane = tid & 31;
      for (int b = tid >> 5; b < n / 32; b += nt >> 5)
        quant_block_warp_x(gbuf[b * 32 + lane], lane, gq_g + fr.x + b * 32, gs_g + fr.x / 32 + b);
    }
    if (!stage_barrier(bar, epoch, G, P.err, S.ok, P.wait_ns)) return;
    // ---- down projection, this CTA's rows (model.rs:419) ----
    for (int j = tid; j < ff / 16; j += nt) ((int4*)S.aq)[j] = __ldcg((const int4*)gq_g + j);
    for (int j = tid; j < ff / 32; j += nt) S.as[j] = ldcg(gs_g + j);
    __syncthreads();
    {
      int2 rr = span(d, 16);
      rows_exact<BITS, ST>(L.down, rr.x, rr.y, S.aq, S.as, S.xn, [&](int r, float v) { dn_g[r] = v; });
    }
    if (!stage_barrier(bar, epoch, G, P.err, S.ok, P.wait_ns)) return;
    // ---- post-FFN norm and residual (model.rs:421-426); CTA 0 hands the residual on ----
    if (c == 0) {
      for (int j = tid; j < d; j += nt) S.xn[j] = ldcg(dn_g + j);
      __syncthreads();
      if (tid == 0) S.r[0] = L.post_ffw ? rms_r_exact(seq_sumsq(S.xn, d), d, P.eps) : 1.0f;
      __syncthreads();
      for (int j = tid; j < d; j += nt) {
        float t2 = S.xn[j];
        if (L.post_ffw) t2 = mul(t2, mul(S.r[0], L.post_ffw[j]));
        S.x[j] = add(S.x[j], t2);
      }
      if (l == P.withhold_stage) {  // test hook: nothing downstream will ever see this token
        __syncthreads();
        continue;
      }
      const int nxt = l + 1, gnext = nxt < P.nl ? G : P.GH;
      if (tid == 0) *S.ok = t < PIPE_RING ? 1 : wait_geq(P.consumed + nxt, (unsigned)(t - PIPE_RING + 1) * gnext, P.err, P.wait_ns);
      __syncthreads();
      if (!*S.ok) return;
      float* dst = P.ring + ((size_t)nxt * PIPE_RING + slot) * d;
      for (int j = tid; j < d; j += nt) dst[j] = S.x[j];
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        st_release(P.ready + nxt * PIPE_RING + slot, (unsigned)t + 1);
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------
// The two-level head stage (main.rs:82-107; greedy token as lean.rs:46-76 with top = 1).
// ------------------------------------------------------------------------------------------------
template <int BITS, typename ST>
__device__ void head_stage(const PipeArgs& P, int c, const Smem& S) {
  const int d = P.d, GH = P.GH, tid = threadIdx.x, nt = blockDim.x;
  float* cl_g = P.head_scratch;            // k
  float* in_g = cl_g + P.k;                // per
  float* top_g = in_g + P.per;             // per
  unsigned* bar = P.bar + P.nl * 32;
  unsigned epoch = 0;
  const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  auto span = [&](int total, int align) {
    int per = ((total + GH - 1) / GH + align - 1) / align * align;
    int a = min(total, c * per), b = min(total, a + per);
    return make_int2(a, b);
  };
  for (int t = 0; t < P.n; ++t) {
    const int slot = t % PIPE_RING;
    uint32_t target = P.toks[t + 1];
    if (target >= (uint32_t)P.vocab) {
      if (tid == 0 && c == 0) atomicCAS(P.err, 0, ERR_RANGE);
      target = 0;
    }
    if (tid == 0) *S.ok = wait_geq(P.ready + P.nl * PIPE_RING + slot, (unsigned)t + 1, P.err, P.wait_ns);
    __syncthreads();
    if (!*S.ok) return;
    const float* src = P.ring + ((size_t)P.nl * PIPE_RING + slot) * d;
    for (int j = tid; j < d; j += nt) S.x[j] = ldcg(src + j);
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      atomicAdd(P.consumed + P.nl, 1u);
    }
    // final norm (model.rs:428) and Act::quantize of h (main.rs:96)
    if (tid == 0) S.r[0] = rms_r_exact(seq_sumsq(S.x, d), d, P.eps);
    __syncthreads();
    for (int j = tid; j < d; j += nt) S.xn[j] = mul(mul(S.x[j], S.r[0]), P.out_norm[j]);
    __syncthreads();
    quantize_smem(S.xn, d, S.aq, S.as);
    __syncthreads();
    if (t == P.n - 1 && c == 0 && P.h_last)
      for (int j = tid; j < d; j += nt) P.h_last[j] = S.xn[j];
    // class logits, this CTA's classes: dot512(A[c], h) + b[c] (main.rs:82-93)
    {
      int2 cr = span(P.k, 16);
      const int half = lane & 1;
      for (int base = cr.x + warp * 16; base < cr.y; base += nw * 16) {
        int cc = base + (lane >> 1);
        bool ok = cc < cr.y;
        float z = dot512_pair(P.A + (size_t)(ok ? cc : cr.x) * d, S.xn, d, half);
        if (ok && half == 0) cl_g[cc] = add(z, P.b[cc]);
      }
    }
    // the target class's block (main.rs:95-99)
    const uint32_t ct = P.cls_of[target];
    const int first = (int)ct * P.per;
    const int nrow = min(P.per, P.blocks.rows - first);
    {
      int2 rr = span(nrow, 16);
      rows_exact<BITS, ST>(P.blocks, first + rr.x, first + rr.y, S.aq, S.as, S.xn, [&](int r, float v) { in_g[r - first] = v; });
    }
    if (!stage_barrier(bar, epoch, GH, P.err, S.ok, P.wait_ns)) return;
    // most likely class: first maximum (every CTA, same result); lse over classes
    float* cl = S.p;  // k floats
    for (int i = tid; i < P.k; i += nt) cl[i] = ldcg(cl_g + i);
    __syncthreads();
    {
      Lse Lc{-INFINITY, 0.0f};
      Best B{-INFINITY, 0xffffffffu};
      for (int i = tid; i < P.k; i += nt) {
        Lc = lse_add(Lc, cl[i]);
        B = best_merge(B, Best{cl[i], (uint32_t)i});
      }
      for (int o = 16; o > 0; o >>= 1) {
        Lc = lse_merge(Lc, Lse{__shfl_xor_sync(0xffffffffu, Lc.m, o), __shfl_xor_sync(0xffffffffu, Lc.s, o)});
        B = best_merge(B, Best{__shfl_xor_sync(0xffffffffu, B.v, o), __shfl_xor_sync(0xffffffffu, B.tok, o)});
      }
      __shared__ float sm_m[32], sm_s[32], sm_v[32];
      __shared__ uint32_t sm_t[32];
      if (lane == 0) { sm_m[warp] = Lc.m; sm_s[warp] = Lc.s; sm_v[warp] = B.v; sm_t[warp] = B.tok; }
      __syncthreads();
      if (tid == 0) {
        for (int i = 1; i < nw; ++i) {
          Lc = lse_merge(Lc, Lse{sm_m[i], sm_s[i]});
          B = best_merge(B, Best{sm_v[i], sm_t[i]});
        }
        S.r[2] = Lc.m + logf(Lc.s);
        ((uint32_t*)S.r)[3] = B.tok < (uint32_t)P.k ? B.tok : 0;
      }
      __syncthreads();
    }
    const uint32_t top = ((uint32_t*)S.r)[3];
    if (c == 0 && tid < 32) {  // target log-prob (main.rs:101-107)
      Lse Li{-INFINITY, 0.0f};
      for (int j = lane; j < nrow; j += 32) Li = lse_add(Li, ldcg(in_g + j));
      for (int o = 16; o > 0; o >>= 1)
        Li = lse_merge(Li, Lse{__shfl_xor_sync(0xffffffffu, Li.m, o), __shfl_xor_sync(0xffffffffu, Li.s, o)});
      if (lane == 0)
        P.lp_out[t] = cl[ct] - S.r[2] + ldcg(in_g + P.pos_of[target]) - (Li.m + logf(Li.s));
    }
    // the top class's block
    const int tfirst = (int)top * P.per;
    const int tn = min(P.per, P.blocks.rows - tfirst);
    {
      int2 rr = span(tn, 16);
      rows_exact<BITS, ST>(P.blocks, tfirst + rr.x, tfirst + rr.y, S.aq, S.as, S.xn, [&](int r, float v) { top_g[r - tfirst] = v; });
    }
    if (!stage_barrier(bar, epoch, GH, P.err, S.ok, P.wait_ns)) return;
    if (c == 0 && tid < 32) {
      Best B{-INFINITY, 0xffffffffu};
      for (int j = lane; j < tn; j += 32) B = best_merge(B, Best{ldcg(top_g + j), (uint32_t)j});
      for (int o = 16; o > 0; o >>= 1)
        B = best_merge(B, Best{__shfl_xor_sync(0xffffffffu, B.v, o), __shfl_xor_sync(0xffffffffu, B.tok, o)});
      if (lane == 0 && P.am_out) P.am_out[t] = P.order[tfirst + (B.tok < (uint32_t)tn ? B.tok : 0)];
    }
    __syncthreads();
  }
}

// BL/SL: body weight format; BH/SH: output matrix format (also the tied embedding).
template <int BL, typename SL, int BH, typename SH>
__global__ void __launch_bounds__(512, 1) k_pipe_score(PipeArgs P) {
  extern __shared__ __align__(16) unsigned char smem_pipe[];
  Smem S = carve(smem_pipe, P);
  if ((int)blockIdx.x < P.nl * P.G) layer_stage<BL, SL, BH, SH>(P, blockIdx.x / P.G, blockIdx.x % P.G, S);
  else if ((int)blockIdx.x < P.nl * P.G + P.GH) head_stage<BH, SH>(P, blockIdx.x - P.nl * P.G, S);
}

}  // namespace

size_t pipe_scratch_floats(int nh, int nkv, int hd, int d, int ff, int max_npos, int ref_threads) {
  auto r16 = [](size_t f) { return (f + 15) / 16 * 16; };
  size_t f = r16((size_t)(nh + 2 * nkv) * hd) + r16((size_t)nh * max_npos) + r16((size_t)ref_threads * nh * hd) +
             2 * r16(d) + r16(ff / 32) + r16(((size_t)ff + 3) / 4);
  return (f + 63) / 64 * 64;
}

size_t pipe_smem_bytes(const PipeArgs& P) {
  auto r16 = [](size_t b) { return (b + 15) / 16 * 16; };
  size_t wide = std::max(std::max(P.d, P.nh * P.hd), P.ff);
  size_t p = pipe_p_floats(P);
  return r16(P.d * 4) + r16(wide * 4) + r16(wide) + r16(wide / 32 * 4) + r16((size_t)P.nh * P.hd * 4) +
         2 * r16((size_t)P.nkv * P.hd * 4) + r16(p * 4) + r16(128) + 16;
}

int launch_pipe_score(const PipeArgs& P, size_t smem, cudaStream_t st) {
  if (P.emb.bits != P.blocks.bits || P.emb.scale_f32 != P.blocks.scale_f32) return -1;
  void* args[] = {(void*)&P};
  dim3 grid(P.nl * P.G + P.GH), block(512);
  cudaError_t e = cudaErrorInvalidValue;
  auto fmt = [](int bits, int f32) { return bits * 2 + (f32 ? 1 : 0); };
  const int body = fmt(P.layers_bits, P.layers_scale_f32), head = fmt(P.blocks.bits, P.blocks.scale_f32);
  bool found = false;
#define L(BL, SL, BH, SH)                                                                                  \
  if (!found && body == fmt(BL, sizeof(SL) == 4) && head == fmt(BH, sizeof(SH) == 4 && BH != 16)) {        \
    found = true;                                                                                          \
    cudaFuncSetAttribute(k_pipe_score<BL, SL, BH, SH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    e = cudaLaunchCooperativeKernel((void*)k_pipe_score<BL, SL, BH, SH>, grid, block, args, smem, st);    \
  }
  L(8, __half, 8, __half)    // Q8_0 GGUF: body and head as stored
  L(8, __half, 8, float)     // Q8_0 body, head requantized to 8 bits from F16
  L(8, __half, 4, float)     // Q8_0 body, head requantized to 4 bits
  L(4, __half, 16, __half)   // Q4_0 body, F16 head (4-bit QAT files)
  L(4, __half, 8, float)     // Q4_0 body, F16 head requantized to Q8
  L(4, float, 8, __half)     // Q8_0 body requantized to 4 bits
  L(4, float, 8, float)
  L(16, __half, 16, __half)  // F16 files
#undef L
  if (!found) return -1;
  return e == cudaSuccess ? 0 : (int)e;
}

}  // namespace gem
