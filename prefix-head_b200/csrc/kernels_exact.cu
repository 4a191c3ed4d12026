// Exact-numerics kernels: bit-identical to the reference's AVX-512 path (crates/gem/src/q8.rs,
// model.rs with Isa::Avx512) for a given CPU thread-pool size.
//
// Int8 activation quantization makes the forward chaotic: a last-bit difference in any value that is
// quantized later can flip an int8 code and grow to ~1e-2 nats per token, which is also how far the
// reference's own AVX2 and AVX-512 paths disagree. So these kernels reproduce the reference's
// summation orders exactly:
//   - row dots (dot_avx512, dot4_avx512, dot16_avx512): 16 fp32 lanes, lane i holds
//     w[2i]*a[2i] + w[2i+1]*a[2i+1] per 32-block, accumulated with one FMA per block, then reduced in
//     _mm512_reduce_add_ps's halving order (i + 8, i + 4, i + 2, i + 1). Two threads hold a row's 16
//     lanes, 8 each.
//   - dot512 (attention scores, class logits): 16 lanes over 16-float chunks, same reduction.
//   - rmsnorm / softmax sums: sequential fp32 additions (Rust's Iterator::sum), one thread.
//   - P.V: the pool's per-thread position ranges, FMA per element (axpy512), partials summed in
//     thread order.
#include <algorithm>
#include "kernels.cuh"
#include "exact.cuh"

namespace gem {


// ------------------------------------------------------------------------------------------------
// GEMV, exact, for one activation vector: a row's 16 lanes (lane i = pair i of every 32-block, one
// FMA per block with scale ws*as, q8.rs:248-292; for F16 lane i = element i of every 16-chunk,
// q8.rs:358-369) go to 8 threads with 2 lanes each, thread o holding lanes 2o and 2o + 1 (one
// 4-byte word of weights per block), so that even 640-row matrices spread over the SMs. Each thread
// issues kGemvU weight loads before its FMA chain consumes them. The halving reduction runs over the
// 8 threads: lane i + lane i + 8 is partner o ^ 4, + 4 is o ^ 2, + 2 is o ^ 1, then the thread's own
// two lanes.
// ------------------------------------------------------------------------------------------------
constexpr int kGemvThreads = 64, kGemvU = 32;

template <int BITS>
__device__ __forceinline__ int load_word(const MatView& w, size_t r, int b, int o) {
  if constexpr (BITS == 8) {
    return __ldg((const int*)((const int8_t*)w.q + r * w.cols + (size_t)b * 32) + o);
  } else {  // dot4_avx512 (q8.rs:307-326): bytes 0..15 low nibbles (weights 0..15), high nibbles 16..31
    const unsigned raw = (unsigned)__ldg((const int*)((const uint8_t*)w.q + r * (w.cols / 2) + (size_t)b * 16) + (o & 3));
    return (int)__vsub4((raw >> (4 * (o >> 2))) & 0x0f0f0f0fu, 0x08080808u);
  }
}

template <int BITS, typename ST>
__global__ void __launch_bounds__(kGemvThreads) k_gemv_exact(MatView w, const int8_t* aq, const float* as, const float* x,
                                                             float* y) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int8_t* saq = (int8_t*)smem_raw;
  float* sas = (float*)(smem_raw + w.cols);
  float* sx = (float*)smem_raw;
  const int o = threadIdx.x & 7;
  const int r = blockIdx.x * (kGemvThreads / 8) + (threadIdx.x >> 3);
  const bool ok = r < w.rows;  // a row's 8 threads are consecutive lanes: the shuffles stay inside them
  const size_t rr = ok ? r : w.rows - 1;
  // The weights depend on no earlier kernel: the first kGemvU blocks are requested before the wait for
  // the previous kernel (programmatic dependent launch), so their latency passes while it finishes.
  // The activation vector is its output, staged after the wait.
  auto stage_act = [&]() {
    pdl_wait();
    if (BITS == 16) {
      for (int j = threadIdx.x; j < w.cols; j += blockDim.x) sx[j] = x[j];
    } else {
      for (int j = threadIdx.x; j < w.cols / 16; j += blockDim.x) ((int4*)saq)[j] = ((const int4*)aq)[j];
      for (int j = threadIdx.x; j < w.cols / 32; j += blockDim.x) sas[j] = as[j];
    }
    __syncthreads();
  };
  float a0 = 0.0f, a1 = 0.0f;  // lanes 2o, 2o + 1
  if constexpr (BITS == 16) {
    const __half2* row = (const __half2*)((const __half*)w.q + rr * w.cols);
    const int nc = w.cols / 16;
    __half2 v[kGemvU];
    for (int c0 = 0; c0 < nc; c0 += kGemvU) {
#pragma unroll
      for (int u = 0; u < kGemvU; ++u)
        if (c0 + u < nc) v[u] = __ldg(row + (size_t)(c0 + u) * 8 + o);
      if (c0 == 0) stage_act();
#pragma unroll
      for (int u = 0; u < kGemvU; ++u) {
        if (c0 + u >= nc) break;
        const float2 f = __half22float2(v[u]);
        const float* xv = sx + (c0 + u) * 16 + 2 * o;
        a0 = fmaf(f.x, xv[0], a0);
        a1 = fmaf(f.y, xv[1], a1);
      }
    }
  } else {
    const int nb = w.cols / 32;
    const ST* srow = (const ST*)w.s + rr * nb;
    int wv[kGemvU];
    float sc[kGemvU];
    for (int b0 = 0; b0 < nb; b0 += kGemvU) {
#pragma unroll
      for (int u = 0; u < kGemvU; ++u)
        if (b0 + u < nb) {
          wv[u] = load_word<BITS>(w, rr, b0 + u, o);
          sc[u] = ld_scale(srow, b0 + u);
        }
      if (b0 == 0) stage_act();
#pragma unroll
      for (int u = 0; u < kGemvU; ++u) {
        if (b0 + u >= nb) break;
        const int av = ((const int*)saq)[(b0 + u) * 8 + o];
        const float s = mul(sc[u], sas[b0 + u]);
        a0 = fmaf(madd_lo(wv[u], av), s, a0);
        a1 = fmaf(madd_hi(wv[u], av), s, a1);
      }
    }
  }
  a0 = add(a0, __shfl_xor_sync(0xffffffffu, a0, 4));
  a1 = add(a1, __shfl_xor_sync(0xffffffffu, a1, 4));
  a0 = add(a0, __shfl_xor_sync(0xffffffffu, a0, 2));
  a1 = add(a1, __shfl_xor_sync(0xffffffffu, a1, 2));
  a0 = add(a0, __shfl_xor_sync(0xffffffffu, a0, 1));
  a1 = add(a1, __shfl_xor_sync(0xffffffffu, a1, 1));
  if (ok && o == 0) y[r] = add(a0, a1);
}

// ------------------------------------------------------------------------------------------------
// Residual + norms + quantize with sequential sums (see k_residual_norm_quant).
// ------------------------------------------------------------------------------------------------
__global__ void k_residual_norm_quant_exact(float* x, const float* delta, const float* w_post, const float* w_pre,
                                            float eps, int d, int8_t* aq, float* as, float* xn_out) {
  pdl_wait();
  extern __shared__ __align__(16) float smx[];
  float* xs = smx;       // d
  float* tv = smx + d;   // d
  __shared__ float s_r;
  int tid = threadIdx.x;
  if (delta) {
    for (int j = tid; j < d; j += blockDim.x) tv[j] = delta[j];
    __syncthreads();
    if (w_post) {
      if (tid == 0) s_r = rms_r_exact(seq_sumsq(tv, d), d, eps);
      __syncthreads();
    }
    float r = s_r;
    for (int j = tid; j < d; j += blockDim.x) {
      float t = tv[j];
      if (w_post) t = mul(t, mul(r, w_post[j]));  // rmsnorm_inplace (model.rs:89-95): v *= r * w
      xs[j] = add(x[j], t);
    }
  } else {
    for (int j = tid; j < d; j += blockDim.x) xs[j] = x[j];
  }
  __syncthreads();
  if (tid == 0) s_r = rms_r_exact(seq_sumsq(xs, d), d, eps);
  __syncthreads();
  float r = s_r;
  if (delta)
    for (int j = tid; j < d; j += blockDim.x) x[j] = xs[j];
  for (int j = tid; j < d; j += blockDim.x) xs[j] = mul(mul(xs[j], r), w_pre[j]);  // rmsnorm (model.rs:81-87)
  __syncthreads();
  if (xn_out)
    for (int j = tid; j < d; j += blockDim.x) xn_out[j] = xs[j];
  if (aq) {
    int lane = tid & 31;
    for (int b = tid >> 5; b < d / 32; b += blockDim.x >> 5) quant_block_warp_x(xs[b * 32 + lane], lane, aq + b * 32, as + b);
  }
}

// ------------------------------------------------------------------------------------------------
// Attention, exact (model.rs:316-383).
// ------------------------------------------------------------------------------------------------
// One CTA per kv group; writes normalised q to qn.
__global__ void k_attn_prep_exact(AttnArgs A, float* qn) {
  // the norm weights, this position's RoPE rows and the biases depend on no earlier kernel: their
  // lines come into L1 while the previous kernel (the q/k/v GEMV) finishes
  {
    const int hd = A.hd, G = A.nh / A.nkv, g = blockIdx.x;
    const uint32_t pos = A.cur->pos;  // set when the token began, several kernels back
    auto pf = [](const float* p, int n) {
      if (p)
        for (int j = threadIdx.x * 32; j < n; j += blockDim.x * 32) asm volatile("prefetch.global.L1 [%0];" ::"l"(p + j));
    };
    pf(A.q_norm, hd);
    pf(A.k_norm, hd);
    pf(A.rope_sin + (size_t)pos * (hd / 2), hd / 2);
    pf(A.rope_cos + (size_t)pos * (hd / 2), hd / 2);
    if (A.bqkv) {
      pf(A.bqkv + (size_t)g * G * hd, G * hd);
      pf(A.bqkv + (size_t)A.nh * hd + g * hd, hd);
      pf(A.bqkv + (size_t)A.nh * hd + A.nkv * hd + g * hd, hd);
    }
  }
  pdl_wait();
  extern __shared__ __align__(16) float smp[];
  __shared__ float s_r[17];
  attn_prep_token(A, A.qkv, A.cur->pos, blockIdx.x, qn, smp, s_r);
}

// scores[h][i] = dot512(q_h, k_(lo+i)) for every head and position (model.rs:344-353).
__global__ void k_attn_scores_exact(AttnArgs A, const float* qn, float* scores, int sstride) {
  const int hd = A.hd, G = A.nh / A.nkv;
  const uint32_t pos = A.cur->pos;  // set when the token began, several kernels back
  const uint32_t lo = (A.window > 0 && pos + 1 > (uint32_t)A.window) ? pos + 1 - A.window : 0;
  const uint32_t n_pos = pos + 1 - lo;
  const int rw = A.nkv * hd;
  const int lane = threadIdx.x & 31, half = lane & 1;
  const int pairs = (blockDim.x * gridDim.x) / 2;
  const uint32_t total = n_pos * A.nh;
  // The K rows of earlier positions were written by earlier tokens' kernels: their lines come into L1
  // while the previous kernel (which writes this position's row and the queries) finishes.
  for (uint32_t t = (blockIdx.x * blockDim.x + threadIdx.x) / 2; t < total; t += pairs) {
    const uint32_t i = t / A.nh, h = t % A.nh;
    if (lo + i < pos) {
      const float* k = A.kcache + (size_t)(lo + i) * rw + (h / G) * hd;
      for (int c = half; c < hd / 32; c += 2) asm volatile("prefetch.global.L1 [%0];" ::"l"(k + 32 * c));
    }
  }
  pdl_wait();
  for (uint32_t t = (blockIdx.x * blockDim.x + threadIdx.x) / 2; t < ((total + 15) / 16) * 16; t += pairs) {
    bool ok = t < total;
    uint32_t tt = ok ? t : 0;
    uint32_t i = tt / A.nh, h = tt % A.nh;
    const float* k = A.kcache + (size_t)(lo + i) * rw + (h / G) * hd;
    float s = dot512_pair(qn + (size_t)h * hd, k, hd, half);
    if (ok && half == 0) scores[(size_t)h * sstride + i] = s;
  }
}

// Softmax per head with the reference's order (model.rs:354-361): max, subtract, exp_fast,
// sequential sum, multiply by 1/sum. One CTA per head.
__global__ void k_attn_softmax_exact(AttnArgs A, float* scores, int sstride) {
  pdl_wait();
  __shared__ float red[32];
  __shared__ float s_inv;
  const uint32_t pos = A.cur->pos;
  const uint32_t lo = (A.window > 0 && pos + 1 > (uint32_t)A.window) ? pos + 1 - A.window : 0;
  const int n_pos = (int)(pos + 1 - lo);
  float* s = scores + (size_t)blockIdx.x * sstride;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n_pos; i += blockDim.x) m = fmaxf(m, s[i]);
  m = block_max(m, red);
  for (int i = threadIdx.x; i < n_pos; i += blockDim.x) s[i] = exp_fast(sub(s[i], m));
  __syncthreads();
  if (threadIdx.x == 0) {
    float sum = 0.0f;
    for (int i = 0; i < n_pos; ++i) sum = add(sum, s[i]);
    s_inv = div(1.0f, sum);
  }
  __syncthreads();
  float inv = s_inv;
  for (int i = threadIdx.x; i < n_pos; i += blockDim.x) s[i] = mul(s[i], inv);
}

// P.V with the pool's partition (model.rs:362-382): positions split into `threads` ranges of
// per = ceil(n_pos / threads); each range accumulates acc = fma(p, v, acc) in order; att = partials
// summed in thread order. Then Act::quantize of the head's blocks. Grid (nh, hd / 32), block 32 * T.
__global__ void k_attn_pv_exact(AttnArgs A, const float* scores, int sstride, int threads, int8_t* aq, float* as) {
  extern __shared__ float part[];  // [threads][32]
  const int hd = A.hd, G = A.nh / A.nkv, h = blockIdx.x, j0 = blockIdx.y * 32;
  const uint32_t pos = A.cur->pos;  // set when the token began, several kernels back
  const uint32_t lo = (A.window > 0 && pos + 1 > (uint32_t)A.window) ? pos + 1 - A.window : 0;
  const int n_pos = (int)(pos + 1 - lo);
  const int per = (n_pos + threads - 1) / threads;
  const int rw = A.nkv * hd;
  const int lane = threadIdx.x & 31, t = threadIdx.x >> 5;
  const float* p = scores + (size_t)h * sstride;
  const float* vc = A.vcache + (h / G) * hd + j0 + lane;
  // The V rows were all written by kernels that finished before the previous one (the softmax)
  // started: this warp's rows come into L1 (one 128-byte line per row) while the softmax runs.
  for (int tt = t; tt < threads; tt += blockDim.x >> 5) {
    const int i0 = min(tt * per, n_pos), i1 = min((tt + 1) * per, n_pos);
    for (int i = i0 + lane; i < i1; i += 32)
      asm volatile("prefetch.global.L1 [%0];" ::"l"(A.vcache + (size_t)(lo + i) * rw + (h / G) * hd + j0));
  }
  pdl_wait();
  for (int tt = t; tt < threads; tt += blockDim.x >> 5) {
    float acc = 0.0f;
    int i0 = min(tt * per, n_pos), i1 = min((tt + 1) * per, n_pos);
    for (int i = i0; i < i1; ++i) acc = fmaf(p[i], vc[(size_t)(lo + i) * rw], acc);
    part[tt * 32 + lane] = acc;
  }
  __syncthreads();
  if (t == 0) {
    float a = 0.0f;
    for (int tt = 0; tt < threads; ++tt) a = add(a, part[tt * 32 + lane]);
    if (A.att_out) A.att_out[h * hd + j0 + lane] = a;
    quant_block_warp_x(a, lane, aq + h * hd + j0, as + (h * hd + j0) / 32);
  }
}

// ------------------------------------------------------------------------------------------------
// Heads, exact logits.
// ------------------------------------------------------------------------------------------------
template <int BITS, typename ST>
__global__ void k_head_full_exact(HeadArgs H) {
  pdl_wait();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red_m[32], red_s[32], red_v[32];
  __shared__ uint32_t red_t[32];
  const int bi = blockIdx.y;
  const MatView& w = H.w;
  int8_t* saq = (int8_t*)smem_raw;
  float* sas = (float*)(smem_raw + w.cols);
  float* sx = (float*)smem_raw;
  if (BITS == 16) {
    for (int j = threadIdx.x; j < w.cols; j += blockDim.x) sx[j] = H.h[(size_t)bi * w.cols + j];
  } else {
    for (int j = threadIdx.x; j < w.cols / 16; j += blockDim.x) ((int4*)saq)[j] = ((const int4*)(H.aq + (size_t)bi * w.cols))[j];
    for (int j = threadIdx.x; j < w.cols / 32; j += blockDim.x) sas[j] = H.as[(size_t)bi * (w.cols / 32) + j];
  }
  __syncthreads();
  uint32_t target = H.targets ? H.targets[bi] : H.cur->target;
  if (target >= (uint32_t)w.rows) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(H.err, ERR_RANGE);
    target = 0;
  }
  const uint32_t trow = H.row_of ? H.row_of[target] : target;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, half = lane & 1;
  Lse L{-INFINITY, 0.0f};
  Best B{-INFINITY, 0xffffffffu};
  for (int base = (blockIdx.x * nw + warp) * 16; base < w.rows; base += gridDim.x * nw * 16) {
    int r = base + (lane >> 1);
    bool ok = r < w.rows;
    float z = row_dot_exact<BITS, ST>(w, ok ? r : w.rows - 1, half, saq, sas, sx);
    if (ok && half == 0) {
      L = lse_add(L, z);
      best_row_add(B, z, (uint32_t)r, H.row_tok);
      if ((uint32_t)r == trow) H.tlogit[bi] = z;
    }
  }
  best_row_to_token(B, H.row_tok);
  for (int o = 16; o > 0; o >>= 1) {
    Lse l2{__shfl_xor_sync(0xffffffffu, L.m, o), __shfl_xor_sync(0xffffffffu, L.s, o)};
    Best b2{__shfl_xor_sync(0xffffffffu, B.v, o), __shfl_xor_sync(0xffffffffu, B.tok, o)};
    L = lse_merge(L, l2);
    B = best_merge(B, b2);
  }
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

// ------------------------------------------------------------------------------------------------
// Full head streamed through shared memory (Q8_0 output matrix with f16 scales, a few hidden states).
// The matrix's GEMV copy is laid out [16-row group][block][row][32 bytes], its scales [group][block][16
// rows], so G consecutive groups (a stage) are two contiguous bulk copies, and a warp reads one block
// of its 16 rows as 512 contiguous bytes. NS stages per CTA: the next lands while one is used. A
// thread pair takes a row, lanes 0-7 / 8-15, with row_dot_exact's additions in row_dot_exact's order.
// ------------------------------------------------------------------------------------------------
namespace {
__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ bool hb_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  unsigned long long t0 = 0;
  for (int i = 0;; ++i) {
    uint32_t done;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(done) : "r"(a), "r"(parity) : "memory");
    if (done) return true;
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    if (i == 0) t0 = t;
    else if (t - t0 > 1000000000ull) return false;  // 1 s: the copy never landed
  }
}
__device__ __forceinline__ void hb_issue(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
}  // namespace

__global__ void k_head_bulk_layout(MatView w, unsigned char* wq, __half* ws) {
  const int nb = w.cols / 32, ng = (w.rows + 15) / 16;
  const size_t n = (size_t)ng * nb * 16 * 2;  // 16-byte pieces: (group, block, row, half)
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int h = (int)(i & 1), row = (int)((i >> 1) & 15);
    const size_t gb = i >> 5;
    const int b = (int)(gb % nb), g = (int)(gb / nb), r = g * 16 + row;
    int4 v = make_int4(0, 0, 0, 0);
    if (r < w.rows) v = *(const int4*)((const int8_t*)w.q + (size_t)r * w.cols + b * 32 + h * 16);
    *(int4*)(wq + i * 16) = v;
    if (h == 0) ws[gb * 16 + row] = r < w.rows ? ((const __half*)w.s)[(size_t)r * nb + b] : __float2half(0.0f);
  }
}

template <int G, int NS>
__global__ void __launch_bounds__(G * 32) k_head_full_bulk(HeadArgs H, const unsigned char* __restrict__ wq,
                                                          const __half* __restrict__ wsc, int ng) {
  extern __shared__ __align__(128) unsigned char sm[];
  __shared__ __align__(8) uint64_t full[NS];
  __shared__ float red_m[32], red_s[32], red_v[32];
  __shared__ uint32_t red_t[32];
  const MatView& w = H.w;
  const int bi = blockIdx.y, nb = w.cols / 32;
  const size_t qst = (size_t)G * nb * 512, sst = (size_t)G * nb * 32;  // one stage's quants and scales
  int8_t* saq = (int8_t*)sm;
  float* sas = (float*)(sm + w.cols);
  unsigned char* buf = sm + ((w.cols + nb * 4 + 127) & ~127);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, half = lane & 1;
  const int nst = (ng + G - 1) / G;
  auto issue = [&](int s, int k) {  // stage s into buffer k
    const int gc = min(G, ng - s * G);
    unsigned char* q = buf + (size_t)k * (qst + sst);
    const uint32_t qb = (uint32_t)gc * nb * 512, sb = (uint32_t)gc * nb * 32;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&full[k])), "r"(qb + sb) : "memory");
    hb_issue(q, wq + (size_t)s * qst, qb, &full[k]);
    hb_issue(q + qst, wsc + (size_t)s * G * nb * 16, sb, &full[k]);
  };
  if (threadIdx.x == 0) {
    for (int k = 0; k < NS; ++k) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&full[k])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0)  // the output matrix depends on no earlier kernel: its first stages load during the wait
    for (int k = 0; k < NS; ++k)
      if ((int)(blockIdx.x + k * gridDim.x) < nst) issue(blockIdx.x + k * gridDim.x, k);
  pdl_wait();
  if (H.aq) {
    for (int j = threadIdx.x; j < w.cols / 16; j += blockDim.x) ((int4*)saq)[j] = ((const int4*)(H.aq + (size_t)bi * w.cols))[j];
    for (int j = threadIdx.x; j < nb; j += blockDim.x) sas[j] = H.as[(size_t)bi * nb + j];
  } else {  // Act::quantize of the fp32 hidden state here (q8.rs:187-246), a warp per 32-block
    for (int b = warp; b < nb; b += G)
      quant_block_warp_x(H.h[(size_t)bi * w.cols + b * 32 + lane], lane, saq + b * 32, sas + b);
  }
  __syncthreads();
  uint32_t target = H.targets ? H.targets[bi] : H.cur->target;
  if (target >= (uint32_t)w.rows) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(H.err, ERR_RANGE);
    target = 0;
  }
  const uint32_t trow = H.row_of ? H.row_of[target] : target;
  Lse L{-INFINITY, 0.0f};
  Best B{-INFINITY, 0xffffffffu};
  bool ok = true;
  int i = 0;
  for (int s = blockIdx.x; s < nst && ok; s += gridDim.x, ++i) {
    const int k = i % NS;
    ok = hb_wait(&full[k], (uint32_t)((i / NS) & 1));
    if (!ok) {
      if (lane == 0) atomicExch(H.err, ERR_TIMEOUT);
      break;
    }
    const int g = s * G + warp;
    if (g < ng) {
      const unsigned char* q = buf + (size_t)k * (qst + sst) + (size_t)warp * nb * 512 + (lane >> 1) * 32 + half * 16;
      const __half* sc = (const __half*)(buf + (size_t)k * (qst + sst) + qst) + (size_t)warp * nb * 16 + (lane >> 1);
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
#pragma unroll 4
      for (int b = 0; b < nb; ++b)
        block_fma(acc, *(const int4*)(q + (size_t)b * 512), *(const int4*)(saq + b * 32 + half * 16),
                  mul(__half2float(sc[b * 16]), sas[b]));
      const float z = reduce16_pair(acc);
      const int r = g * 16 + (lane >> 1);
      if (r < w.rows && half == 0) {
        L = lse_add(L, z);
        best_row_add(B, z, (uint32_t)r, H.row_tok);
        if ((uint32_t)r == trow) H.tlogit[bi] = z;
      }
    }
    __syncthreads();  // every warp is done with buffer k
    if (threadIdx.x == 0 && s + NS * (int)gridDim.x < nst) issue(s + NS * gridDim.x, k);
  }
  best_row_to_token(B, H.row_tok);
  for (int o = 16; o > 0; o >>= 1) {
    Lse l2{__shfl_xor_sync(0xffffffffu, L.m, o), __shfl_xor_sync(0xffffffffu, L.s, o)};
    Best b2{__shfl_xor_sync(0xffffffffu, B.v, o), __shfl_xor_sync(0xffffffffu, B.tok, o)};
    L = lse_merge(L, l2);
    B = best_merge(B, b2);
  }
  if (lane == 0) { red_m[warp] = L.m; red_s[warp] = L.s; red_v[warp] = B.v; red_t[warp] = B.tok; }
  if (H.cnt) __threadfence();  // this thread's target-logit store is visible before the CTA counts itself
  __syncthreads();
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    for (int j = 1; j < G; ++j) {
      L = lse_merge(L, Lse{red_m[j], red_s[j]});
      B = best_merge(B, Best{red_v[j], red_t[j]});
    }
    float4* p = (float4*)(H.part + ((size_t)bi * gridDim.x + blockIdx.x) * 4);
    *p = make_float4(L.m, L.s, B.v, __uint_as_float(B.tok));
    s_last = 0;
    if (H.cnt) {  // the partial before the count
      __threadfence();
      s_last = atomicAdd(H.cnt + bi, 1) == (int)gridDim.x - 1;
    }
  }
  __syncthreads();
  if (s_last) {  // every CTA's partial is written: merge them here instead of in a separate kernel
    __threadfence();
    head_merge(H, bi, gridDim.x);
    if (threadIdx.x == 0) H.cnt[bi] = 0;  // ready for the next launch
  }
}

// rows of a stage in 16-row groups (one warp each), two stages: G * 2 * nb * 544 bytes <= ~200 KB
static int head_bulk_groups(int nb) { return nb * 544 * 8 * 2 <= 196 * 1024 ? 8 : 4; }

size_t head_bulk_bytes(const MatView& w) {
  const size_t ng = ((size_t)w.rows + 15) / 16, nb = w.cols / 32;
  return ng * nb * 512 + ng * nb * 32;
}
bool head_bulk_supported(const MatView& w) {
  const int nb = w.cols / 32;
  return w.bits == 8 && !w.scale_f32 && w.cols % 32 == 0 && (size_t)head_bulk_groups(nb) * nb * 544 * 2 + w.cols * 2 + 256 <= 200 * 1024;
}
void launch_head_bulk_layout(const MatView& w, unsigned char* wq, __half* ws, cudaStream_t st) {
  k_head_bulk_layout<<<1184, 256, 0, st>>>(w, wq, ws);
}
void launch_head_full_bulk(const HeadArgs& H, const unsigned char* wq, const __half* ws, int batch, int sms, cudaStream_t st) {
  const int nb = H.w.cols / 32, ng = (H.w.rows + 15) / 16, G = head_bulk_groups(nb);
  const int nst = (ng + G - 1) / G, ctas = std::min(nst, std::min(sms, head_full_parts(sms)));
  const size_t sm = (size_t)((H.w.cols + nb * 4 + 127) & ~127) + (size_t)2 * G * nb * 544;
  dim3 grid(ctas, batch);
  if (G == 8) {
    static bool init = false;
    if (!init) { cudaFuncSetAttribute(k_head_full_bulk<8, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 210 * 1024); init = true; }
    launch_k(k_head_full_bulk<8, 2>, grid, dim3(256), sm, st, H, wq, ws, ng);
  } else {
    static bool init = false;
    if (!init) { cudaFuncSetAttribute(k_head_full_bulk<4, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 210 * 1024); init = true; }
    launch_k(k_head_full_bulk<4, 2>, grid, dim3(128), sm, st, H, wq, ws, ng);
  }
  if (!H.cnt) launch_head_full_merge(H, batch, ctas, st);
}

// Two-level stage 1, exact: class logits dot512(A[c], h) + b[c] (main.rs:82-93) and the target
// class's block rows.
template <int BITS, typename ST>
__global__ void k_tl_stage1_exact(TwoLevelArgs T) {
  pdl_wait();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int bi = blockIdx.y;
  const int d = T.w.cols;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, half = lane & 1;
  const float* h = T.h + (size_t)bi * d;
  if ((int)blockIdx.x < T.class_ctas) {
    float* sh = (float*)smem_raw;
    for (int j = threadIdx.x; j < d; j += blockDim.x) sh[j] = h[j];
    __syncthreads();
    // task (warp w, CTA x) = w * class_ctas + x: the first class_ctas tasks land on distinct SMs
    for (int base = (warp * T.class_ctas + (int)blockIdx.x) * 16; base < T.k; base += T.class_ctas * nw * 16) {
      int c = base + (lane >> 1);
      bool ok = c < T.k;
      float z = dot512_pair(T.A + (size_t)(ok ? c : 0) * d, sh, d, half);
      if (ok && half == 0) T.cl[(size_t)bi * T.k + c] = add(z, T.b[c]);
    }
    return;
  }
  int8_t* saq = (int8_t*)smem_raw;
  float* sas = (float*)(smem_raw + d);
  float* sx = (float*)smem_raw;
  if (BITS == 16) {
    for (int j = threadIdx.x; j < d; j += blockDim.x) sx[j] = h[j];
  } else {
    for (int j = threadIdx.x; j < d / 16; j += blockDim.x) ((int4*)saq)[j] = ((const int4*)(T.aq + (size_t)bi * d))[j];
    for (int j = threadIdx.x; j < d / 32; j += blockDim.x) sas[j] = T.as[(size_t)bi * (d / 32) + j];
  }
  __syncthreads();
  uint32_t target = T.targets ? T.targets[bi] : T.cur->target;
  if (target >= (uint32_t)T.vocab) target = 0;
  const uint32_t c = T.cls_of[target];
  const uint32_t first = c * T.per;
  const int n = (int)min((uint32_t)T.per, (uint32_t)T.w.rows - first);
  const int bctas = gridDim.x - T.class_ctas;
  for (int base = ((blockIdx.x - T.class_ctas) * nw + warp) * 16; base < n; base += bctas * nw * 16) {
    int j = base + (lane >> 1);
    bool ok = j < n;
    float z = row_dot_exact<BITS, ST>(T.w, first + (ok ? j : 0), half, saq, sas, sx);
    if (ok && half == 0) T.inner[(size_t)bi * T.per + j] = z;
  }
}

// Stage 2 reuses the fast kernel's logic but recomputes the top class block with exact rows.
template <int BITS, typename ST>
__global__ void k_tl_top_exact(TwoLevelArgs T, const uint32_t* top_of, float* top_inner) {
  pdl_wait();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int bi = blockIdx.y;
  const int d = T.w.cols;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, half = lane & 1;
  int8_t* saq = (int8_t*)smem_raw;
  float* sas = (float*)(smem_raw + d);
  float* sx = (float*)smem_raw;
  if (BITS == 16) {
    for (int j = threadIdx.x; j < d; j += blockDim.x) sx[j] = T.h[(size_t)bi * d + j];
  } else {
    for (int j = threadIdx.x; j < d / 16; j += blockDim.x) ((int4*)saq)[j] = ((const int4*)(T.aq + (size_t)bi * d))[j];
    for (int j = threadIdx.x; j < d / 32; j += blockDim.x) sas[j] = T.as[(size_t)bi * (d / 32) + j];
  }
  __syncthreads();
  const uint32_t c = top_of[bi];
  const uint32_t first = c * T.per;
  const int n = (int)min((uint32_t)T.per, (uint32_t)T.w.rows - first);
  for (int base = (blockIdx.x * nw + warp) * 16; base < n; base += gridDim.x * nw * 16) {
    int j = base + (lane >> 1);
    bool ok = j < n;
    float z = row_dot_exact<BITS, ST>(T.w, first + (ok ? j : 0), half, saq, sas, sx);
    if (ok && half == 0) top_inner[(size_t)bi * T.per + j] = z;
  }
}

// ------------------------------------------------------------------------------------------------
// The two-level head in one launch (TwoLevel::logprob, main.rs:82-107, and the greedy token of
// lean.rs:46-76 with top = 1). The tasks of one hidden state are its k class logits dot512(A[c], h) +
// b[c] on the fp32 hidden state and the rows of the target class's block: the row dot on the
// quantized hidden state (dot_avx512 / dot4_avx512) or on the fp32 one (dot16_avx512 for an F16
// matrix). They spread over P CTAs in contiguous ranges; a CTA takes its range in rounds of 32 tasks,
// one 16-thread group per task and one of the dot's 16 lanes per thread, in the reference's order.
// A round's class rows and block rows are each one contiguous range of memory: one bulk copy each
// into shared memory (the class rows of the first round are requested before the wait on the previous
// kernel: they depend on nothing it writes), the block rows' scales by plain loads. Each CTA leaves its
// partial class log-sum-exp and most likely class, and the target block's log-sum-exp; the last CTA
// of a hidden state (a per-item counter, zero between launches) merges them, stages the most likely
// class's block in one copy (unless it is the target's, whose logits are already written) and takes
// its first maximum: the greedy token.
// With the class logits given (T.cl_in, [batch][k], from the tile product over many hidden states),
// the tasks are the target block's rows alone, 32 a CTA, and each CTA also folds its slice of the
// given logits (classes [k * x / P, k * (x + 1) / P) for CTA x) into its class partial.
// ------------------------------------------------------------------------------------------------
constexpr int kTlThreads = 512, kTlGroups = kTlThreads / 16, kTlPart = 12;
static_assert(kTlGroups == 32, "k_tl_fused merges its groups' partials with one warp: one group per lane");

// Lane i of dot512 (model.rs:106-120) on a row in shared memory: the sum over chunks c of
// a[16c + i] * x[16c + i], fused, in order.
__device__ __forceinline__ float lane512_s(const float* a, const float* sx, int nc, int i) {
  float acc = 0.0f;
#pragma unroll 8
  for (int c = 0; c < nc; ++c) acc = fmaf(a[16 * c + i], sx[16 * c + i], acc);
  return acc;
}

// Lane i of the reference's row dot on a row in shared memory: Q8_0 / Q4_0 rows against the quantized
// hidden state (lane i is the madd pair 2i, 2i + 1 of every 32-block, one FMA per block with scale
// ws * as; sc holds the row's scales as fp32), F16 rows against the fp32 one (lane i sums w[16c + i] *
// x[16c + i]).
template <int BITS>
__device__ __forceinline__ float lane_row_s(const unsigned char* q, const float* sc, int d, int i, const int8_t* saq,
                                            const float* sas, const float* sx) {
  float acc = 0.0f;
  if constexpr (BITS == 16) {
    const __half* row = (const __half*)q;
#pragma unroll 8
    for (int c = 0; c < d / 16; ++c) acc = fmaf(__half2float(row[16 * c + i]), sx[16 * c + i], acc);
  } else {
#pragma unroll 4
    for (int b = 0; b < d / 32; ++b) {
      int w0, w1;
      if constexpr (BITS == 8) {
        const uint16_t wp = *((const uint16_t*)(q + 32 * b) + i);
        w0 = (int)(int8_t)(wp & 0xffu), w1 = (int)(int8_t)(wp >> 8);
      } else {  // q8.rs:42-52: byte j holds weight j (low nibble) and j + 16 (high nibble), each + 8
        const uint16_t wp = *((const uint16_t*)(q + 16 * b) + (i & 7));
        const int sh = i < 8 ? 0 : 4;
        w0 = (int)((wp >> sh) & 15u) - 8, w1 = (int)((wp >> (8 + sh)) & 15u) - 8;
      }
      const int p = w0 * (int)saq[32 * b + 2 * i] + w1 * (int)saq[32 * b + 2 * i + 1];
      acc = fmaf((float)p, mul(sc[b], sas[b]), acc);
    }
  }
  return acc;
}

// The halving reduction of the 16 lanes held by 16 consecutive threads of a half-warp (lane i in its
// thread i): lanes i + 8 onto i, then 4, 2, 1 apart (_mm512_reduce_add_ps). The group's first thread
// gets the result. The shuffles name only the group's 16 threads: the two halves of a warp run
// separate tasks and may leave their loops at different times.
__device__ __forceinline__ float reduce16_group(float v) {
  const unsigned m = 0xffffu << (threadIdx.x & 16);
  v = add(v, __shfl_down_sync(m, v, 8, 16));
  v = add(v, __shfl_down_sync(m, v, 4, 16));
  v = add(v, __shfl_down_sync(m, v, 2, 16));
  return add(v, __shfl_down_sync(m, v, 1, 16));
}

// Bytes of one output-matrix row's weights (Q8_0: d, Q4_0: d / 2, F16: 2d).
__host__ __device__ constexpr size_t tl_row_bytes(int bits, int d) {
  return bits == 16 ? (size_t)d * 2 : bits == 8 ? (size_t)d : (size_t)d / 2;
}
// Shared memory of k_tl_fused: the hidden state (fp32, int8, block scales), then the staging area:
// weights of max(32 class rows, rows_b block rows), the block rows' scales as fp32, the top block's
// token ids.
__host__ __device__ constexpr size_t tl_head_off(int d) { return ((size_t)d * 5 + (size_t)d / 8 + 127) & ~(size_t)127; }
__host__ __device__ constexpr size_t tl_stage_q(int bits, int d, int rows_b) {
  return (size_t)kTlGroups * 4 * d > (size_t)rows_b * tl_row_bytes(bits, d) ? (size_t)kTlGroups * 4 * d
                                                                              : (size_t)rows_b * tl_row_bytes(bits, d);
}
__host__ __device__ constexpr size_t tl_smem(int bits, int d, int rows_b) {
  return tl_head_off(d) + tl_stage_q(bits, d, rows_b) + (size_t)(rows_b > kTlGroups ? rows_b : kTlGroups) * (d / 32) * 4 +
         (size_t)rows_b * 4;
}

__device__ __forceinline__ int lds_u16(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return (int)v;
}
__device__ __forceinline__ float lds_f32(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}

// Lanes i of four rows of the reference's row dot (the 16-lane order of lane_row_s), rows at shared
// addresses q[u]: four independent FMA chains, each in order. For Q8_0 / Q4_0 rows the fp32 at sc[u] +
// 4b holds block b's scale product RN(ws * as); the pair sum w0 a0 + w1 a1 is one dp4a (exact in int32;
// Q4_0's nibbles carry +8, taken off as 8 (a0 + a1)).
template <int BITS>
__device__ __forceinline__ void lane_rows4_s(const uint32_t (&q)[4], const uint32_t (&sc)[4], int d, int i,
                                             const int8_t* saq, const float* sx, float (&acc)[4]) {
#pragma unroll
  for (int u = 0; u < 4; ++u) acc[u] = 0.0f;
  if constexpr (BITS == 16) {
#pragma unroll 4
    for (int c = 0; c < d / 16; ++c) {
      const float x = sx[16 * c + i];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        acc[u] = fmaf(__half2float(__ushort_as_half((unsigned short)lds_u16(q[u] + 2 * (16 * c + i)))), x, acc[u]);
    }
  } else {
    const int sh = i < 8 ? 0 : 4;
    const uint32_t qa = (uint32_t)__cvta_generic_to_shared(saq) + 2 * i;
#pragma unroll 2
    for (int b = 0; b < d / 32; ++b) {
      const int ap = lds_u16(qa + 32 * b);  // a0, a1 as signed bytes, upper bytes zero
      const int off8 = BITS == 4 ? 8 * ((int)(int8_t)(ap & 0xff) + (int)(int8_t)(ap >> 8)) : 0;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        int p;
        if constexpr (BITS == 8) {
          p = __dp4a(lds_u16(q[u] + 32 * b + 2 * i), ap, 0);
        } else {  // q8.rs:42-52: byte j holds weight j (low nibble) and j + 16 (high nibble), each + 8
          p = __dp4a((lds_u16(q[u] + 16 * b + 2 * (i & 7)) >> sh) & 0x0f0f, ap, 0) - off8;
        }
        acc[u] = fmaf((float)p, lds_f32(sc[u] + 4 * b), acc[u]);
      }
    }
  }
}

// Per-CTA partial of the two-level head: class log-sum-exp and most likely class, the target block's
// log-sum-exp and first maximum, and the target's class logit and row logit where this CTA computed them.
struct TlAcc {
  Lse c;
  Best bc;
  Lse t;
  Best bt;
};
__device__ __forceinline__ TlAcc tl_acc0() {
  return TlAcc{Lse{-INFINITY, 0.0f}, Best{-INFINITY, 0xffffffffu}, Lse{-INFINITY, 0.0f}, Best{-INFINITY, 0xffffffffu}};
}
__device__ __forceinline__ TlAcc tl_merge(TlAcc a, TlAcc b) {
  return TlAcc{lse_merge(a.c, b.c), best_merge(a.bc, b.bc), lse_merge(a.t, b.t), best_merge(a.bt, b.bt)};
}
// Merges 32 lanes' partials: maxima first, then the sums rescaled to them (one exp per lane).
__device__ __forceinline__ TlAcc tl_warp_merge(TlAcc v) {
  float mc = v.c.m, mt = v.t.m;
  for (int o = 16; o > 0; o >>= 1) {
    mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
  }
  float sc = v.c.m == -INFINITY ? 0.0f : v.c.s * expf(v.c.m - mc);
  float st = v.t.m == -INFINITY ? 0.0f : v.t.s * expf(v.t.m - mt);
  for (int o = 16; o > 0; o >>= 1) {
    sc += __shfl_xor_sync(0xffffffffu, sc, o);
    st += __shfl_xor_sync(0xffffffffu, st, o);
    v.bc = best_merge(v.bc, Best{__shfl_xor_sync(0xffffffffu, v.bc.v, o), __shfl_xor_sync(0xffffffffu, v.bc.tok, o)});
    v.bt = best_merge(v.bt, Best{__shfl_xor_sync(0xffffffffu, v.bt.v, o), __shfl_xor_sync(0xffffffffu, v.bt.tok, o)});
  }
  return TlAcc{Lse{mc, sc}, v.bc, Lse{mt, st}, v.bt};
}

// The target of hidden state bi (an id >= vocab is replaced by 0; the last CTA reports it), its class,
// its place in the class and that class's rows [first, first + n) of the class-ordered matrix.
struct TlTarget {
  uint32_t tok, ct, pos, first;
  int n;
  bool bad;
};
__device__ __forceinline__ TlTarget tl_target(const TwoLevelArgs& T, int bi) {
  uint32_t t = T.targets ? T.targets[bi] : T.cur->target;
  const bool bad = t >= (uint32_t)T.vocab;
  if (bad) t = 0;
  const uint32_t c = T.cls_of[t], f = c * T.per;
  return TlTarget{t, c, T.pos_of[t], f, (int)min((uint32_t)T.per, (uint32_t)T.w.rows - f), bad};
}

// n scales of whole rows' blocks (nb a row) as fp32 in shared memory, times the hidden state's block
// scale (RN(ws * as), the factor of the row dot's FMA) when sas is given: eight independent loads in
// flight per thread.
template <typename ST>
__device__ __forceinline__ void tl_stage_scales(float* dst, const ST* src, int n, int nb, const float* sas) {
  for (int e0 = threadIdx.x; e0 < n; e0 += 8 * kTlThreads) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = e0 + u * kTlThreads;
      v[u] = e < n ? ld_scale(src, e) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = e0 + u * kTlThreads;
      if (e < n) dst[e] = sas ? mul(v[u], sas[e % nb]) : v[u];
    }
  }
}

template <int BITS, typename ST>
__global__ void __launch_bounds__(kTlThreads) k_tl_fused(TwoLevelArgs T, int P, int rows_b, int* cnt, float* part) {
  extern __shared__ __align__(16) unsigned char smem_raw[];  // bulk copies land on 16-byte boundaries
  __shared__ __align__(8) uint64_t bar;
  __shared__ TlAcc red[kTlGroups];  // one partial per 16-thread group
  __shared__ int s_last;
  __shared__ float s_zcl, s_zin, s_lse_cl, s_lse_t;
  __shared__ uint32_t s_top, s_jt;
  const int bi = blockIdx.y, d = T.w.cols, nb = d / 32, nc = d / 16;
  const int g = threadIdx.x >> 4, i = threadIdx.x & 15, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const size_t RB = tl_row_bytes(BITS, d);
  float* sx = (float*)smem_raw;     // the fp32 hidden state [d]
  int8_t* saq = (int8_t*)(sx + d);  // quantized [d]
  float* sas = (float*)(saq + d);   // its block scales [d / 32]
  unsigned char* stage = smem_raw + tl_head_off(d);
  float* ssc = (float*)(stage + tl_stage_q(BITS, d, rows_b));                   // staged rows' scales
  uint32_t* sorder = (uint32_t*)(ssc + (size_t)max(rows_b, kTlGroups) * nb);  // the top block's token ids
  // Tasks: the k class logits, then the target block's rows. With the class logits given (computed
  // for many hidden states at once by a product), a CTA reads its slice [c_lo, c_hi) of them and takes
  // only block rows as tasks.
  const bool given = T.cl_in != nullptr;
  const int tasks_max = T.k + T.per, tpc = given ? (T.per + P - 1) / P : (tasks_max + P - 1) / P;
  const int t_begin = given ? T.k + blockIdx.x * tpc : blockIdx.x * tpc;
  int t_end = min(tasks_max, t_begin + tpc);
  const int c_lo = given ? (int)((long long)T.k * blockIdx.x / P) : 0;
  const int c_hi = given ? (int)((long long)T.k * (blockIdx.x + 1) / P) : 0;
  const uint32_t abar = smem_u32(&bar);
  // the first round's class rows: A depends on no earlier kernel, so its copy starts before the wait
  const int c0_end = min(min(t_begin + kTlGroups, t_end), T.k);
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(abar));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (c0_end > t_begin) {
      const uint32_t bytes = (uint32_t)(c0_end - t_begin) * 4u * d;
      asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(abar), "r"(bytes) : "memory");
      hb_issue(stage, T.A + (size_t)t_begin * d, bytes, &bar);
    }
    s_zcl = NAN, s_zin = NAN;
  }
  pdl_wait();
  // the hidden state: fp32 (its first 1536 values requested before the target lookup's dependent loads),
  // and Act::quantize, a warp per 32-block (q8.rs:187-246)
  const float* hrow = T.h + (size_t)bi * d;
  float hv[3];
#pragma unroll
  for (int u = 0; u < 3; ++u) hv[u] = threadIdx.x + u * kTlThreads < d ? hrow[threadIdx.x + u * kTlThreads] : 0.0f;
  const TlTarget tg = tl_target(T, bi);
#pragma unroll
  for (int u = 0; u < 3; ++u)
    if (threadIdx.x + u * kTlThreads < d) sx[threadIdx.x + u * kTlThreads] = hv[u];
  for (int j = threadIdx.x + 3 * kTlThreads; j < d; j += kTlThreads) sx[j] = hrow[j];
  __syncthreads();
  for (int b = warp; b < nb; b += kTlThreads / 32) {
    const float v = sx[32 * b + lane];
    const float amax = warp_max(fabsf(v));
    const float dd = div(amax, 127.0f);
    const float inv = dd > 0.0f ? div(1.0f, dd) : 0.0f;
    saq[32 * b + lane] = (int8_t)__float2int_rn(mul(v, inv));
    if (lane == 0) sas[b] = dd;
  }
  t_end = min(t_end, T.k + tg.n);
  TlAcc v = tl_acc0();
  bool ok = true;
  uint32_t parity = 0;
  for (int t0 = t_begin, r = 0; t0 < t_end && ok; t0 += kTlGroups, ++r) {
    const int n = min(kTlGroups, t_end - t0);
    const int nca = max(0, min(t0 + n, T.k) - t0);         // the round's class rows [t0, t0 + nca)
    const int ja = max(t0, T.k) - T.k, jb = t0 + n - T.k;  // and block rows [ja, jb) of the target class
    const int t = t0 + g;
    const float bias = g < nca && i == 0 ? T.b[t] : 0.0f;  // loads while the rows land
    if (r > 0) __syncthreads();  // every group is done with the previous round's rows
    if (threadIdx.x == 0) {      // round 0's class rows are on their way already
      const uint32_t cbytes = r == 0 ? 0u : (uint32_t)nca * 4u * d;
      const uint32_t bbytes = jb > ja ? (uint32_t)((jb - ja) * RB) : 0u;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(abar), "r"(cbytes + bbytes) : "memory");
      if (cbytes) hb_issue(stage, T.A + (size_t)t0 * d, cbytes, &bar);
      if (bbytes) hb_issue(stage + (size_t)nca * 4 * d, (const unsigned char*)T.w.q + (tg.first + ja) * RB, bbytes, &bar);
    }
    if constexpr (BITS != 16)
      if (jb > ja) tl_stage_scales(ssc, (const ST*)T.w.s + (size_t)(tg.first + ja) * nb, (jb - ja) * nb, nb, (const float*)nullptr);
    __syncthreads();  // the scales (and, in round 0, the hidden state) are in place
    ok = __syncthreads_and(hb_wait(&bar, parity));  // one answer for the whole CTA
    parity ^= 1u;
    if (!ok) {
      if (threadIdx.x == 0) atomicExch(T.err, ERR_TIMEOUT);
      break;
    }
    if (g < n) {
      if (t < T.k) {
        const float z = reduce16_group(lane512_s((const float*)stage + (size_t)g * d, sx, nc, i));
        if (i == 0) {
          const float zc = add(z, bias);
          v.c = lse_add(v.c, zc);
          v.bc = best_merge(v.bc, Best{zc, (uint32_t)t});
          if ((uint32_t)t == tg.ct) s_zcl = zc;
        }
      } else {
        const int jr = g - nca;  // this row's place among the round's block rows
        const float z = reduce16_group(
            lane_row_s<BITS>(stage + (size_t)nca * 4 * d + jr * RB, ssc + (size_t)jr * nb, d, i, saq, sas, sx));
        if (i == 0) {
          const uint32_t j = (uint32_t)(t - T.k);
          v.t = lse_add(v.t, z);
          v.bt = best_merge(v.bt, Best{z, j});
          if (j == tg.pos) s_zin = z;
        }
      }
    }
  }
  if (given) {  // this CTA's slice of the given class logits: a thread each, merged into group leaders
    TlAcc vc = tl_acc0();
    for (int c = c_lo + threadIdx.x; c < c_hi; c += kTlThreads) {
      const float zc = T.cl_in[(size_t)bi * T.k + c];
      vc.c = lse_add(vc.c, zc);
      vc.bc = best_merge(vc.bc, Best{zc, (uint32_t)c});
      if ((uint32_t)c == tg.ct) s_zcl = zc;
    }
    vc = tl_warp_merge(vc);
    if (lane == 0) v = tl_merge(v, vc);  // lane 0 leads group 2 * warp
  }
  if (i == 0) red[g] = v;  // a group's partials sit in its first thread
  __syncthreads();
  if (warp == 0) v = tl_warp_merge(red[lane]);
  if (threadIdx.x == 0) {
    float4* p = (float4*)(part + ((size_t)bi * P + blockIdx.x) * kTlPart);
    p[0] = make_float4(v.c.m, v.c.s, v.bc.v, __uint_as_float(v.bc.tok));
    p[1] = make_float4(v.t.m, v.t.s, v.bt.v, __uint_as_float(v.bt.tok));
    p[2] = make_float4(s_zcl, s_zin, 0.0f, 0.0f);
    __threadfence();  // the partial before the count
    s_last = atomicAdd(cnt + bi, 1) == P - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // ---- the last CTA: merge the partials (a thread each, then the warps' merges) ----
  v = tl_acc0();
  for (int j = threadIdx.x; j < P; j += kTlThreads) {
    const float4* p = (const float4*)(part + ((size_t)bi * P + j) * kTlPart);
    const float4 a = __ldcg(p), b = __ldcg(p + 1), c = __ldcg(p + 2);
    v = tl_merge(v, TlAcc{Lse{a.x, a.y}, Best{a.z, __float_as_uint(a.w)}, Lse{b.x, b.y}, Best{b.z, __float_as_uint(b.w)}});
    if (!isnan(c.x)) s_zcl = c.x;  // exactly one CTA computed each
    if (!isnan(c.y)) s_zin = c.y;
  }
  v = tl_warp_merge(v);
  __syncthreads();  // red is free
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = tl_warp_merge(lane < kTlThreads / 32 ? red[lane] : tl_acc0());
    if (lane == 0) {
      if (tg.bad) atomicExch(T.err, ERR_RANGE);
      s_lse_cl = v.c.m + logf(v.c.s);
      s_lse_t = v.t.m + logf(v.t.s);
      s_top = v.bc.tok < (uint32_t)T.k ? v.bc.tok : 0;  // only NaN logits leave no candidate
      s_jt = v.bt.tok;
    }
  }
  __syncthreads();
  const uint32_t top = s_top, first = top * T.per;
  const int n = (int)min((uint32_t)T.per, (uint32_t)T.w.rows - first);
  // the most likely class's block: its first maximum (the target block's, already merged, when they are
  // the same class); its token ids load while its logits are computed
  const bool ids_staged = n <= rows_b;
  if (ids_staged)
    for (int j = threadIdx.x; j < n; j += kTlThreads) sorder[j] = T.order[first + j];
  Best bt{-INFINITY, 0xffffffffu};
  if (top == tg.ct) {
    if (threadIdx.x == 0) bt = Best{0.0f, s_jt};
  } else if (ok) {
    for (int j0 = 0; j0 < n && ok; j0 += rows_b) {
      const int m = min(rows_b, n - j0);
      __syncthreads();  // every group is done with the staging area
      if (threadIdx.x == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(abar), "r"((uint32_t)(m * RB)) : "memory");
        hb_issue(stage, (const unsigned char*)T.w.q + (first + j0) * RB, (uint32_t)(m * RB), &bar);
      }
      if constexpr (BITS != 16) tl_stage_scales(ssc, (const ST*)T.w.s + (size_t)(first + j0) * nb, m * nb, nb, sas);
      __syncthreads();
      ok = __syncthreads_and(hb_wait(&bar, parity));
      parity ^= 1u;
      if (!ok) {
        if (threadIdx.x == 0) atomicExch(T.err, ERR_TIMEOUT);
        break;
      }
      // four rows per group at once: j, j + 32, j + 64, j + 96 (a row past the end repeats row j)
      const uint32_t stage_a = (uint32_t)__cvta_generic_to_shared(stage), ssc_a = (uint32_t)__cvta_generic_to_shared(ssc);
      for (int j = g; j < m; j += 4 * kTlGroups) {
        uint32_t q4[4], s4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int ju = j + u * kTlGroups < m ? j + u * kTlGroups : j;
          q4[u] = stage_a + (uint32_t)(ju * RB);
          s4[u] = ssc_a + (uint32_t)(ju * nb * 4);
        }
        float acc[4];
        lane_rows4_s<BITS>(q4, s4, d, i, saq, sx, acc);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float z = reduce16_group(acc[u]);
          if (i == 0 && j + u * kTlGroups < m) bt = best_merge(bt, Best{z, (uint32_t)(j0 + j + u * kTlGroups)});
        }
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1)
    bt = best_merge(bt, Best{__shfl_xor_sync(0xffffffffu, bt.v, o), __shfl_xor_sync(0xffffffffu, bt.tok, o)});
  __syncthreads();
  if (lane == 0) red[warp].bt = bt;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kTlThreads / 32; ++w) bt = best_merge(bt, red[w].bt);
    const uint32_t slot = T.targets ? (uint32_t)bi : T.cur->slot;
    const uint32_t jbest = bt.tok < (uint32_t)n ? bt.tok : 0;
    if (T.lp_out) T.lp_out[slot] = s_zcl - s_lse_cl + s_zin - s_lse_t;
    if (T.am_out) T.am_out[slot] = ids_staged ? sorder[jbest] : T.order[first + jbest];
    cnt[bi] = 0;  // zero for the next launch
  }
}

// ------------------------------------------------------------------------------------------------
#define GEM_DISPATCH_X(bits, scale_f32, F)                    \
  do {                                                        \
    if ((bits) == 8 && !(scale_f32)) { F(8, __half); }        \
    else if ((bits) == 8) { F(8, float); }                    \
    else if ((bits) == 4 && !(scale_f32)) { F(4, __half); }   \
    else if ((bits) == 4) { F(4, float); }                    \
    else { F(16, __half); }                                   \
  } while (0)

static size_t act_smem_x(int cols, int bits) {
  return bits == 16 ? (size_t)cols * 4 : (size_t)cols + (size_t)cols / 32 * 4;
}

void launch_gemv_exact(const MatView& w, const int8_t* aq, const float* as, const float* x, float* y, int sms,
                       cudaStream_t st) {
  const int blocks = (w.rows + kGemvThreads / 8 - 1) / (kGemvThreads / 8);  // 8 rows per CTA
  size_t sm = act_smem_x(w.cols, w.bits);
#define F(B, S)                                                                                     \
  do {                                                                                              \
    static bool init = false;                                                                       \
    if (!init) { cudaFuncSetAttribute(k_gemv_exact<B, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); init = true; } \
    launch_k(k_gemv_exact<B, S>, dim3(blocks), dim3(kGemvThreads), sm, st, w, aq, as, x, y);        \
  } while (0)
  GEM_DISPATCH_X(w.bits, w.scale_f32, F);
#undef F
}

void launch_residual_norm_quant_exact(float* x, const float* delta, const float* w_post, const float* w_pre, float eps,
                                      int d, int8_t* aq, float* as, float* xn_out, cudaStream_t st) {
  launch_k(k_residual_norm_quant_exact, dim3(1), dim3(1024), (size_t)2 * d * 4, st, x, delta, w_post, w_pre, eps, d, aq, as, xn_out);
}

void launch_attn_exact(const AttnArgs& A, float* qn, float* scores, int sstride, int threads, int8_t* aq, float* as,
                       int sms, cudaStream_t st) {
  int G = A.nh / A.nkv;
  launch_k(k_attn_prep_exact, dim3(A.nkv), dim3(256), (size_t)(G * A.hd + 2 * A.hd) * 4, st, A, qn);
  int max_npos = A.window > 0 ? A.window : A.chunk * A.nsplit;
  int pairs = max_npos * A.nh;
  int blocks = min(sms * 4, max(1, (pairs * 2 + 255) / 256));
  launch_k(k_attn_scores_exact, dim3(blocks), dim3(256), 0, st, A, (const float*)qn, scores, sstride);
  launch_k(k_attn_softmax_exact, dim3(A.nh), dim3(256), 0, st, A, scores, sstride);
  int tb = min(threads, 32) * 32;
  launch_k(k_attn_pv_exact, dim3(A.nh, A.hd / 32), dim3(tb), (size_t)threads * 32 * 4, st, A, (const float*)scores, sstride, threads, aq, as);
}

void launch_head_full_exact(const HeadArgs& H, int batch, int sms, cudaStream_t st) {
  int parts = head_full_parts(sms);
  dim3 grid(parts, batch);
  size_t sm = act_smem_x(H.w.cols, H.w.bits);
#define F(B, S)                                                                                     \
  do {                                                                                              \
    static bool init = false;                                                                       \
    if (!init) { cudaFuncSetAttribute(k_head_full_exact<B, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); init = true; } \
    launch_k(k_head_full_exact<B, S>, grid, dim3(512), sm, st, H);                                    \
  } while (0)
  GEM_DISPATCH_X(H.w.bits, H.w.scale_f32, F);
#undef F
  launch_head_full_merge(H, batch, parts, st);
}

void launch_tl_stage1_exact(const TwoLevelArgs& T, int batch, int class_ctas, int block_ctas, cudaStream_t st) {
  dim3 grid(class_ctas + block_ctas, batch);
  size_t sm = max(act_smem_x(T.w.cols, T.w.bits), (size_t)T.w.cols * 4);
#define F(B, S)                                                                                     \
  do {                                                                                              \
    static bool init = false;                                                                       \
    if (!init) { cudaFuncSetAttribute(k_tl_stage1_exact<B, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); init = true; } \
    launch_k(k_tl_stage1_exact<B, S>, grid, dim3(256), sm, st, T);                                  \
  } while (0)
  GEM_DISPATCH_X(T.w.bits, T.w.scale_f32, F);
#undef F
}

int tl_parts(int k, int per, int batch, int sms) {
  const int most = (k + per + 15) / 16;  // at least 16 tasks per CTA
  return std::max(1, std::min(most, batch <= 1 ? sms : 2 * sms / batch));
}
int tl_part_floats(int k, int per) { return (k + per + 15) / 16 * kTlPart; }

bool launch_tl_fused(const TwoLevelArgs& T, int batch, int sms, int* cnt, float* part, cudaStream_t st) {
  // with the class logits given, one round of block rows per CTA: ceil(per / 32) CTAs a hidden state
  constexpr size_t kMax = 200 * 1024;
  const int d = T.w.cols;
  int rows_b = T.per;  // the most likely class's block in one copy where it fits
  while (rows_b > 16 && tl_smem(T.w.bits, d, rows_b) > kMax) rows_b -= 16;
  if (d % 32 || tl_smem(T.w.bits, d, rows_b) > kMax) return false;
  const int P = T.cl_in ? std::max(1, (T.per + kTlGroups - 1) / kTlGroups) : tl_parts(T.k, T.per, batch, sms);
  const size_t sm = tl_smem(T.w.bits, d, rows_b);
#define F(B, S)                                                                                     \
  do {                                                                                              \
    static bool init = false;                                                                       \
    if (!init) { cudaFuncSetAttribute(k_tl_fused<B, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMax); init = true; } \
    launch_k(k_tl_fused<B, S>, dim3(P, batch), dim3(kTlThreads), sm, st, T, P, rows_b, cnt, part);   \
  } while (0)
  GEM_DISPATCH_X(T.w.bits, T.w.scale_f32, F);
#undef F
  return true;
}

void launch_tl_top_exact(const TwoLevelArgs& T, int batch, const uint32_t* top_of, float* top_inner, cudaStream_t st) {
  int ctas = max(1, min(8, (T.per + 63) / 64));
  dim3 grid(ctas, batch);
  size_t sm = act_smem_x(T.w.cols, T.w.bits);
#define F(B, S)                                                                                     \
  do {                                                                                              \
    static bool init = false;                                                                       \
    if (!init) { cudaFuncSetAttribute(k_tl_top_exact<B, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); init = true; } \
    launch_k(k_tl_top_exact<B, S>, grid, dim3(128), sm, st, T, top_of, top_inner);                  \
  } while (0)
  GEM_DISPATCH_X(T.w.bits, T.w.scale_f32, F);
#undef F
}

}  // namespace gem
