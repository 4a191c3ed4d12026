// Sequence-parallel scoring: all positions of a known token sequence go through each layer together.
//
// The reference scores a text one token at a time (crates/gem/src/main.rs:270-289): forward(tok, pos)
// then the head. The tokens are all known in advance, and position i depends on earlier positions
// only through the KV cache of each layer, so a layer can run for every position of a chunk at once,
// provided the chunk's K/V rows are written before its attention reads them. Each position's
// arithmetic is unchanged: every kernel here reproduces the exact-numerics orders of
// kernels_exact.cu (the reference's AVX-512 path), so the results are bit-identical to scoring one
// token after another. What changes is the shape of the work: the projections become matrix products
// (weights read once per chunk instead of once per token), bound by CUDA-core arithmetic rather than
// by HBM bandwidth.
//
// Kernels (T = positions in the chunk):
//   k_seq_embed        x[t] = dequantized row of tok[t] * sqrt(d)                 (model.rs:290-293)
//   k_seq_norm         residual + post-norm, pre-norm, Act::quantize; warp per position
//   k_seq_gemm         Y[t][r] = row r . act[t] with the reference's 16-lane order (q8.rs:248-292)
//   k_seq_attn_prep    QK-norm, RoPE, q scale, K/V append                           (model.rs:316-335)
//   k_seq_scores       dot512(q[t][h], K[p]) for p in the window of t             (model.rs:344-353)
//   k_seq_softmax      max, exp_fast, sequential sum, 1/sum                         (model.rs:354-361)
//   k_seq_pv           P.V in the pool's position ranges, then Act::quantize        (model.rs:362-382)
//   k_seq_glu_quant    GELU-tanh (or SiLU) gate * up, Act::quantize                 (model.rs:408-416)
//   k_seq_class_logits two-level class logits dot512(A[c], h[t]) + b[c]            (main.rs:82-93)
//   k_seq_logit_reduce full-head log-sum-exp, argmax and target logit per position  (main.rs:30-37)
#include <algorithm>

#include "kernels.cuh"
#include "exact.cuh"

namespace gem {

namespace {

__device__ __forceinline__ unsigned smem_addr(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
// cp.async with zero fill when `ok` is false (nothing is read from `src` then).
__device__ __forceinline__ void cp16(void* dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(ok ? 16 : 0));
}
__device__ __forceinline__ void cp4(void* dst, const void* src, bool ok) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(ok ? 4 : 0));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// One madd_epi16 lane as an exact float: the int32 pair sum p (|p| <= 2 * 128 * 127) is added to the
// bit pattern of 1.5 * 2^23 by the dot instruction itself, which gives the float 1.5 * 2^23 + p
// exactly; subtracting 1.5 * 2^23 leaves p. Two full-rate instructions instead of a conversion.
constexpr int kMagicI = 0x4B400000;
constexpr float kMagicF = 12582912.0f;
__device__ __forceinline__ float madd_lo_f(int w, int a) { return sub(__int_as_float(__dp4a(w & 0x0000ffff, a, kMagicI)), kMagicF); }
__device__ __forceinline__ float madd_hi_f(int w, int a) { return sub(__int_as_float(__dp4a(w & (int)0xffff0000, a, kMagicI)), kMagicF); }

__device__ __forceinline__ uint32_t window_lo(uint32_t pos, int window) {
  return (window > 0 && pos + 1 > (uint32_t)window) ? pos + 1 - window : 0;
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// Embedding: one CTA per position. Ids >= vocab are recorded in *err and replaced by 0.
// ------------------------------------------------------------------------------------------------
template <int BITS, typename ST>
__global__ void k_seq_embed(MatView E, const uint32_t* toks, int vocab, float scale, float* x, int* err) {
  const int t = blockIdx.x;
  uint32_t tok = toks[t];
  if (tok >= (uint32_t)vocab) {
    if (threadIdx.x == 0) atomicExch(err, ERR_RANGE);
    tok = 0;
  }
  for (int j = threadIdx.x; j < E.cols; j += blockDim.x) x[(size_t)t * E.cols + j] = mul(weight_at<BITS, ST>(E, tok, j), scale);
}

// ------------------------------------------------------------------------------------------------
// Residual + post-norm, then pre-norm + quantize (k_residual_norm_quant_exact per position). One warp
// per position: squares in parallel, lane 0 adds them in order (Rust's sequential f32 sum).
// ------------------------------------------------------------------------------------------------
constexpr int kNormWarps = 8;

__device__ __forceinline__ float warp_seq_sum(const float* sq, int n, int lane) {
  float s = 0.0f;
  if (lane == 0)
    for (int j = 0; j < n; j += 4) {
      float4 v = *(const float4*)(sq + j);
      s = add(s, v.x);
      s = add(s, v.y);
      s = add(s, v.z);
      s = add(s, v.w);
    }
  return __shfl_sync(0xffffffffu, s, 0);
}

__global__ void __launch_bounds__(kNormWarps * 32) k_seq_norm(float* x, const float* delta, const float* w_post,
                                                              const float* w_pre, float eps, int d, int T, int8_t* aq,
                                                              float* as, float* xn_out) {
  extern __shared__ __align__(16) float sn[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x * kNormWarps + warp;
  if (t >= T) return;
  float* xs = sn + (size_t)warp * 2 * d;
  float* sq = xs + d;
  float* xt = x + (size_t)t * d;
  if (delta) {
    const float* dt = delta + (size_t)t * d;
    float r = 1.0f;
    if (w_post) {
      for (int j = lane; j < d; j += 32) {
        float v = dt[j];
        sq[j] = mul(v, v);
      }
      __syncwarp();
      r = rms_r_exact(warp_seq_sum(sq, d, lane), d, eps);
    }
    for (int j = lane; j < d; j += 32) {
      float v = dt[j];
      if (w_post) v = mul(v, mul(r, w_post[j]));  // rmsnorm_inplace (model.rs:89-95)
      float s = add(xt[j], v);
      xs[j] = s;
      xt[j] = s;
      sq[j] = mul(s, s);
    }
  } else {
    for (int j = lane; j < d; j += 32) {
      float s = xt[j];
      xs[j] = s;
      sq[j] = mul(s, s);
    }
  }
  __syncwarp();
  const float r = rms_r_exact(warp_seq_sum(sq, d, lane), d, eps);
  const int nb = d / 32;
  for (int b = 0; b < nb; ++b) {
    const int j = b * 32 + lane;
    float v = mul(mul(xs[j], r), w_pre[j]);  // rmsnorm (model.rs:81-87)
    if (xn_out) xn_out[(size_t)t * d + j] = v;
    if (aq) quant_block_warp_x(v, lane, aq + (size_t)t * d + b * 32, as + (size_t)t * nb + b);
  }
}

// ------------------------------------------------------------------------------------------------
// Exact int8 matrix product: Y[t][r] = row_dot(W[r], act[t]) for Q8 / Q4 weights, with the lane
// structure of dot_avx512 / dot4_avx512 (lane i = w[2i]a[2i] + w[2i+1]a[2i+1] per 32-block, one FMA
// per block with scale ws*as, halving reduction). A thread pair holds the 16 lanes of one row for 8
// positions (8 + 8 lanes, as in row_dot_exact). CTA tile: 32 rows x 32 positions, 8 warps
// (warp w: rows 16*(w&1) .. +15, positions 8*(w>>1) .. +7), K staged through shared memory in
// chunks of 8 blocks (256 columns) by cp.async, three stages deep.
// ------------------------------------------------------------------------------------------------
constexpr int kGemmBM = 32, kGemmBN = 32, kGemmKB = 8, kGemmStages = 3, kGemmThreads = 256;

template <int BITS, typename ST>
struct GemmTile {
  static constexpr int WB = BITS == 8 ? 32 : 16;       // weight bytes per 32-block of a row
  static constexpr int WROW = kGemmKB * WB + 16;       // padded row: 16-row reads hit distinct banks
  static constexpr int SB = (int)sizeof(ST);
  static constexpr int A_OFF = kGemmBM * WROW;                        // activations [BN][KB*32]
  static constexpr int SW_OFF = A_OFF + kGemmBN * kGemmKB * 32;       // weight scales [BM][KB]
  static constexpr int SA_OFF = SW_OFF + kGemmBM * kGemmKB * SB;      // activation scales [KB][BN]
  static constexpr int STAGE = (SA_OFF + kGemmKB * kGemmBN * 4 + 127) / 128 * 128;
  static constexpr int SMEM = kGemmStages * STAGE;
};

template <int BITS, typename ST>
__device__ __forceinline__ void gemm_issue(unsigned char* stage, const MatView& w, const int8_t* aq, const float* as,
                                           int T, int row0, int tok0, int b0, int kb) {
  using G = GemmTile<BITS, ST>;
  const int tid = threadIdx.x, nb = w.cols / 32;
  const size_t rowbytes = (size_t)nb * G::WB;
  constexpr int WP = kGemmKB * G::WB / 16;  // 16-byte pieces per weight row
  for (int i = tid; i < kGemmBM * WP; i += kGemmThreads) {
    const int r = i / WP, p = i % WP;
    const bool ok = p * 16 < kb * G::WB && row0 + r < w.rows;
    const unsigned char* src = (const unsigned char*)w.q + (ok ? (size_t)(row0 + r) * rowbytes + (size_t)b0 * G::WB + p * 16 : 0);
    cp16(stage + r * G::WROW + p * 16, src, ok);
  }
  constexpr int AP = kGemmKB * 2;
  for (int i = tid; i < kGemmBN * AP; i += kGemmThreads) {
    const int t = i / AP, p = i % AP;
    const bool ok = p < 2 * kb && tok0 + t < T;
    const int8_t* src = aq + (ok ? (size_t)(tok0 + t) * w.cols + (size_t)b0 * 32 + p * 16 : 0);
    cp16(stage + G::A_OFF + t * (kGemmKB * 32) + p * 16, src, ok);
  }
  constexpr int SP = kGemmKB * G::SB / 4;  // 4-byte pieces of one row's scales
  for (int i = tid; i < kGemmBM * SP; i += kGemmThreads) {
    const int r = i / SP, p = i % SP;
    const bool ok = p * 4 < kb * G::SB && row0 + r < w.rows;
    const unsigned char* src = (const unsigned char*)w.s + (ok ? ((size_t)(row0 + r) * nb + b0) * G::SB + p * 4 : 0);
    cp4(stage + G::SW_OFF + r * kGemmKB * G::SB + p * 4, src, ok);
  }
  for (int i = tid; i < kGemmKB * kGemmBN; i += kGemmThreads) {
    const int b = i / kGemmBN, t = i % kGemmBN;
    const bool ok = b < kb && tok0 + t < T;
    const float* src = as + (ok ? (size_t)(tok0 + t) * nb + b0 + b : 0);
    cp4(stage + G::SA_OFF + (b * kGemmBN + t) * 4, src, ok);
  }
}

template <int BITS, typename ST>
__global__ void __launch_bounds__(kGemmThreads, 2) k_seq_gemm(MatView w, const int8_t* aq, const float* as, int T,
                                                               float* y, int ldy) {
  using G = GemmTile<BITS, ST>;
  extern __shared__ __align__(128) unsigned char sg[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, half = lane & 1;
  const int tok0 = blockIdx.x * kGemmBN, row0 = blockIdx.y * kGemmBM;
  const int rl = (warp & 1) * 16 + (lane >> 1);  // row inside the tile
  const int tl = (warp >> 1) * 8;                // first of this thread's 8 positions
  const int nb = w.cols / 32;
  const int nchunks = (nb + kGemmKB - 1) / kGemmKB;

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[i][k] = 0.0f;

#pragma unroll
  for (int s = 0; s < kGemmStages - 1; ++s) {
    if (s < nchunks) gemm_issue<BITS, ST>(sg + s * G::STAGE, w, aq, as, T, row0, tok0, s * kGemmKB, min(kGemmKB, nb - s * kGemmKB));
    cp_commit();
  }
  for (int c = 0; c < nchunks; ++c) {
    cp_wait<kGemmStages - 2>();
    __syncthreads();
    {
      const int cn = c + kGemmStages - 1;
      if (cn < nchunks)
        gemm_issue<BITS, ST>(sg + (cn % kGemmStages) * G::STAGE, w, aq, as, T, row0, tok0, cn * kGemmKB,
                             min(kGemmKB, nb - cn * kGemmKB));
      cp_commit();
    }
    const unsigned char* S = sg + (c % kGemmStages) * G::STAGE;
    const int kb = min(kGemmKB, nb - c * kGemmKB);
    const unsigned char* wrow = S + rl * G::WROW;
    const ST* wsc = (const ST*)(S + G::SW_OFF + rl * kGemmKB * G::SB);
    const float* asc = (const float*)(S + G::SA_OFF) + tl;
    const unsigned char* arow = S + G::A_OFF + tl * (kGemmKB * 32) + half * 16;
    for (int b = 0; b < kb; ++b) {
      int4 wv;
      if constexpr (BITS == 8) {
        wv = *(const int4*)(wrow + b * 32 + half * 16);
      } else {  // dot4_avx512 (q8.rs:307-326): low nibbles are weights 0..15, high nibbles 16..31
        const int4 raw = *(const int4*)(wrow + b * 16);
        const unsigned m = 0x0f0f0f0fu, e = 0x08080808u;
        const int sh = half * 4;
        wv.x = (int)__vsub4(((unsigned)raw.x >> sh) & m, e);
        wv.y = (int)__vsub4(((unsigned)raw.y >> sh) & m, e);
        wv.z = (int)__vsub4(((unsigned)raw.z >> sh) & m, e);
        wv.w = (int)__vsub4(((unsigned)raw.w >> sh) & m, e);
      }
      const float swb = ld_scale(wsc, b);
      const float4 sa0 = *(const float4*)(asc + b * kGemmBN), sa1 = *(const float4*)(asc + b * kGemmBN + 4);
      const float sa[8] = {sa0.x, sa0.y, sa0.z, sa0.w, sa1.x, sa1.y, sa1.z, sa1.w};
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int4 av = *(const int4*)(arow + k * (kGemmKB * 32) + b * 32);
        const float s = mul(swb, sa[k]);
        acc[k][0] = fmaf(madd_lo_f(wv.x, av.x), s, acc[k][0]);
        acc[k][1] = fmaf(madd_hi_f(wv.x, av.x), s, acc[k][1]);
        acc[k][2] = fmaf(madd_lo_f(wv.y, av.y), s, acc[k][2]);
        acc[k][3] = fmaf(madd_hi_f(wv.y, av.y), s, acc[k][3]);
        acc[k][4] = fmaf(madd_lo_f(wv.z, av.z), s, acc[k][4]);
        acc[k][5] = fmaf(madd_hi_f(wv.z, av.z), s, acc[k][5]);
        acc[k][6] = fmaf(madd_lo_f(wv.w, av.w), s, acc[k][6]);
        acc[k][7] = fmaf(madd_hi_f(wv.w, av.w), s, acc[k][7]);
      }
    }
  }
  cp_wait<0>();
  const int r = row0 + rl;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float v = reduce16_pair(acc[k]);
    const int t = tok0 + tl + k;
    if (half == 0 && r < w.rows && t < T) y[(size_t)t * ldy + r] = v;
  }
}

// ------------------------------------------------------------------------------------------------
// Attention, exact, for positions pos0 .. pos0 + T - 1 of one sequence.
// ------------------------------------------------------------------------------------------------
// QK-norm, RoPE, scale, K/V append: one CTA per (position, kv group).
__global__ void k_seq_attn_prep(AttnArgs A, const float* qkv, int qkv_ld, uint32_t pos0, float* qn) {
  extern __shared__ __align__(16) float smp[];
  __shared__ float s_r[17];
  const int t = blockIdx.x;
  attn_prep_token(A, qkv + (size_t)t * qkv_ld, pos0 + t, blockIdx.y, qn + (size_t)t * A.nh * A.hd, smp, s_r);
}

// scores[t][h][i] = dot512(q[t][h], K[lo_t + i]) (model.rs:344-353). One CTA per position; a thread
// pair takes one key position and the G query heads that share its kv group (dot512_pair lanes).
template <int G>
__global__ void k_seq_scores(AttnArgs A, const float* qn, uint32_t pos0, float* scores, int sstride) {
  extern __shared__ __align__(16) float sq[];  // this position's queries [nh][hd]
  const int t = blockIdx.x, hd = A.hd;
  const uint32_t pos = pos0 + t, lo = window_lo(pos, A.window);
  const int n_pos = (int)(pos + 1 - lo);
  const int rw = A.nkv * hd;
  for (int j = threadIdx.x; j < A.nh * hd / 4; j += blockDim.x)
    ((float4*)sq)[j] = ((const float4*)(qn + (size_t)t * A.nh * hd))[j];
  __syncthreads();
  const int half = threadIdx.x & 1, pairs = blockDim.x / 2;
  const int tasks = n_pos * A.nkv;
  for (int base = 0; base < tasks; base += pairs) {
    const int task = base + (int)threadIdx.x / 2;
    const bool ok = task < tasks;
    const int i = ok ? task / A.nkv : 0, g = ok ? task % A.nkv : 0;
    const float* k = A.kcache + (size_t)(lo + i) * rw + g * hd + half * 8;
    float acc[G][8];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[h][e] = 0.0f;
    for (int c = 0; c < hd / 16; ++c) {
      const float4 k0 = __ldcg((const float4*)(k + c * 16)), k1 = __ldcg((const float4*)(k + c * 16 + 4));
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float* q = sq + (size_t)(g * G + h) * hd + c * 16 + half * 8;
        const float4 q0 = *(const float4*)q, q1 = *(const float4*)(q + 4);
        acc[h][0] = fmaf(q0.x, k0.x, acc[h][0]); acc[h][1] = fmaf(q0.y, k0.y, acc[h][1]);
        acc[h][2] = fmaf(q0.z, k0.z, acc[h][2]); acc[h][3] = fmaf(q0.w, k0.w, acc[h][3]);
        acc[h][4] = fmaf(q1.x, k1.x, acc[h][4]); acc[h][5] = fmaf(q1.y, k1.y, acc[h][5]);
        acc[h][6] = fmaf(q1.z, k1.z, acc[h][6]); acc[h][7] = fmaf(q1.w, k1.w, acc[h][7]);
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float s = reduce16_pair(acc[h]);
      if (ok && half == 0) scores[((size_t)t * A.nh + g * G + h) * sstride + i] = s;
    }
  }
}

// Softmax per (position, head) with the reference's order: max, exp_fast(s - max), sequential sum,
// multiply by 1/sum. One warp per (position, head).
__global__ void k_seq_softmax(AttnArgs A, int T, uint32_t pos0, float* scores, int sstride) {
  extern __shared__ __align__(16) float ss[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int task = blockIdx.x * nw + warp;
  if (task >= T * A.nh) return;
  const int t = task / A.nh;
  const uint32_t pos = pos0 + t, lo = window_lo(pos, A.window);
  const int n = (int)(pos + 1 - lo);
  float* s = scores + (size_t)task * sstride;
  float* e = ss + (size_t)warp * sstride;
  float m = -INFINITY;
  for (int i = lane; i < n; i += 32) m = fmaxf(m, s[i]);
  m = warp_max(m);
  for (int i = lane; i < n; i += 32) e[i] = exp_fast(sub(s[i], m));
  __syncwarp();
  float sum = 0.0f;
  if (lane == 0)
    for (int i = 0; i < n; ++i) sum = add(sum, e[i]);
  const float inv = div(1.0f, __shfl_sync(0xffffffffu, sum, 0));
  for (int i = lane; i < n; i += 32) s[i] = mul(e[i], inv);
}

// P.V with the pool's partition (model.rs:362-382): positions split into `threads` ranges of
// per = ceil(n / threads); range r accumulates fma(p, v, acc) in order; att = partials summed in
// range order. Then Act::quantize of att. One CTA per position, thread j = output element of every
// head; ranges are processed 8 at a time so their FMA chains overlap.
__global__ void k_seq_pv(AttnArgs A, uint32_t pos0, const float* scores, int sstride, int threads, int8_t* aq,
                         float* as) {
  const int t = blockIdx.x, hd = A.hd, G = A.nh / A.nkv, j = threadIdx.x;
  const uint32_t pos = pos0 + t, lo = window_lo(pos, A.window);
  const int n = (int)(pos + 1 - lo);
  const int per = (n + threads - 1) / threads;
  const int rw = A.nkv * hd;
  const int lane = j & 31;
  const int nbh = A.nh * hd / 32;
  for (int h = 0; h < A.nh; ++h) {
    const float* p = scores + ((size_t)t * A.nh + h) * sstride;
    const float* vc = A.vcache + (size_t)lo * rw + (h / G) * hd + j;
    float a = 0.0f;
    for (int r0 = 0; r0 < threads; r0 += 8) {
      float acc[8];
      int i0[8], i1[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        acc[u] = 0.0f;
        i0[u] = min((r0 + u) * per, n);
        i1[u] = r0 + u < threads ? min((r0 + u + 1) * per, n) : i0[u];
      }
      for (int k = 0; k < per; ++k) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = i0[u] + k;
          if (i < i1[u]) acc[u] = fmaf(p[i], vc[(size_t)i * rw], acc[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (r0 + u < threads) a = add(a, acc[u]);
    }
    const int b = (h * hd + j) / 32;
    quant_block_warp_x(a, lane, aq + (size_t)t * A.nh * hd + b * 32, as + (size_t)t * nbh + b);
  }
}

// ------------------------------------------------------------------------------------------------
// Gate (k_glu_quant per position): v = gelu_tanh(g) * u (or silu(g) * u), then Act::quantize.
// ------------------------------------------------------------------------------------------------
__global__ void k_seq_glu_quant(const float* gu, int ff, int T, int silu, int8_t* aq, float* as) {
  const int lane = threadIdx.x & 31;
  const int nbk = ff / 32;
  const long long warps = (long long)(blockDim.x >> 5) * gridDim.x;
  for (long long task = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < (long long)T * nbk;
       task += warps) {
    const int t = (int)(task / nbk), b = (int)(task % nbk);
    const int i = b * 32 + lane;
    const float* row = gu + (size_t)t * 2 * ff;
    const float g = row[i], u = row[ff + i];
    float v;
    if (silu) {
      const float e = exp_fast(-g);
      v = mul(div(g, add(1.0f, e)), u);
    } else {
      float k = mul(0.7978846f, add(g, mul(mul(mul(0.044715f, g), g), g)));
      k = tanh_fast(k);
      v = mul(mul(mul(0.5f, g), add(1.0f, k)), u);
    }
    quant_block_warp_x(v, lane, aq + (size_t)t * ff + b * 32, as + (size_t)t * nbk + b);
  }
}

// ------------------------------------------------------------------------------------------------
// Two-level class logits for every position: cl[t][c] = dot512(A[c], h[t]) + b[c]. A thread pair
// holds one class's 16 lanes for 8 positions; CTA tile 32 classes x 32 positions, the positions'
// hidden states staged in shared memory, class rows read from L2.
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256, 2) k_seq_class_logits(const float* A, const float* bias, int k, const float* h,
                                                             int d, int T, float* cl) {
  extern __shared__ __align__(16) float sh[];  // [32][d]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, half = lane & 1;
  const int tok0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  for (int i = threadIdx.x; i < 32 * d / 4; i += blockDim.x) {
    const int t = i / (d / 4), j = i % (d / 4);
    ((float4*)sh)[i] = tok0 + t < T ? ((const float4*)(h + (size_t)(tok0 + t) * d))[j] : make_float4(0, 0, 0, 0);
  }
  __syncthreads();
  const int c = c0 + (warp & 1) * 16 + (lane >> 1);
  const int tl = (warp >> 1) * 8;
  const float* arow = A + (size_t)min(c, k - 1) * d + half * 8;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[i][e] = 0.0f;
  for (int ch = 0; ch < d / 16; ++ch) {
    const float4 a0 = __ldg((const float4*)(arow + ch * 16)), a1 = __ldg((const float4*)(arow + ch * 16 + 4));
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float* hv = sh + (size_t)(tl + u) * d + ch * 16 + half * 8;
      const float4 b0 = *(const float4*)hv, b1 = *(const float4*)(hv + 4);
      acc[u][0] = fmaf(a0.x, b0.x, acc[u][0]); acc[u][1] = fmaf(a0.y, b0.y, acc[u][1]);
      acc[u][2] = fmaf(a0.z, b0.z, acc[u][2]); acc[u][3] = fmaf(a0.w, b0.w, acc[u][3]);
      acc[u][4] = fmaf(a1.x, b1.x, acc[u][4]); acc[u][5] = fmaf(a1.y, b1.y, acc[u][5]);
      acc[u][6] = fmaf(a1.z, b1.z, acc[u][6]); acc[u][7] = fmaf(a1.w, b1.w, acc[u][7]);
    }
  }
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const float z = reduce16_pair(acc[u]);
    const int t = tok0 + tl + u;
    if (half == 0 && c < k && t < T) cl[(size_t)t * k + c] = add(z, bias[c]);
  }
}

// ------------------------------------------------------------------------------------------------
// Full head from a logits matrix [T][V]: online log-sum-exp, argmax (first maximum) and the target's
// logit per position; logprob = logit[target] - lse. One CTA per position.
// ------------------------------------------------------------------------------------------------
__global__ void k_seq_logit_reduce(const float* logits, int V, const uint32_t* targets, float* lp, uint32_t* am,
                                   int* err) {
  __shared__ float red_m[32], red_s[32], red_v[32];
  __shared__ uint32_t red_t[32];
  const int t = blockIdx.x;
  const float* z = logits + (size_t)t * V;
  Lse L{-INFINITY, 0.0f};
  Best B{-INFINITY, 0xffffffffu};
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = z[i];
    L = lse_add(L, v);
    B = best_merge(B, Best{v, (uint32_t)i});
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int o = 16; o > 0; o >>= 1) {
    L = lse_merge(L, Lse{__shfl_xor_sync(0xffffffffu, L.m, o), __shfl_xor_sync(0xffffffffu, L.s, o)});
    B = best_merge(B, Best{__shfl_xor_sync(0xffffffffu, B.v, o), __shfl_xor_sync(0xffffffffu, B.tok, o)});
  }
  if (lane == 0) { red_m[warp] = L.m; red_s[warp] = L.s; red_v[warp] = B.v; red_t[warp] = B.tok; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < nw; ++i) {
      L = lse_merge(L, Lse{red_m[i], red_s[i]});
      B = best_merge(B, Best{red_v[i], red_t[i]});
    }
    uint32_t tg = targets[t];
    if (tg >= (uint32_t)V) {
      atomicExch(err, ERR_RANGE);
      tg = 0;
    }
    lp[t] = z[tg] - (L.m + logf(L.s));
    if (am) am[t] = B.tok;
  }
}

// ------------------------------------------------------------------------------------------------
// Launchers
// ------------------------------------------------------------------------------------------------
#define GEM_DISPATCH_Q(bits, scale_f32, F)                    \
  do {                                                        \
    if ((bits) == 8 && !(scale_f32)) { F(8, __half); }        \
    else if ((bits) == 8) { F(8, float); }                    \
    else if ((bits) == 4 && !(scale_f32)) { F(4, __half); }   \
    else { F(4, float); }                                     \
  } while (0)

void launch_seq_embed(const MatView& E, const uint32_t* toks, int T, int vocab, float scale, float* x, int* err,
                      cudaStream_t st) {
#define F(B, S) k_seq_embed<B, S><<<T, 256, 0, st>>>(E, toks, vocab, scale, x, err)
  if (E.bits == 16) F(16, __half);
  else GEM_DISPATCH_Q(E.bits, E.scale_f32, F);
#undef F
}

void launch_seq_norm(float* x, const float* delta, const float* w_post, const float* w_pre, float eps, int d, int T,
                     int8_t* aq, float* as, float* xn_out, cudaStream_t st) {
  size_t sm = (size_t)kNormWarps * 2 * d * 4;
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(k_seq_norm, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    init = true;
  }
  k_seq_norm<<<(T + kNormWarps - 1) / kNormWarps, kNormWarps * 32, sm, st>>>(x, delta, w_post, w_pre, eps, d, T, aq, as,
                                                                              xn_out);
}

bool seq_gemm_supported(const MatView& w) {
  if (w.bits != 8 && w.bits != 4) return false;
  if (w.cols % 32) return false;
  if (!w.scale_f32 && (w.cols / 32) % 2) return false;  // f16 scales are staged in 4-byte pieces
  return true;
}

void launch_seq_gemm(const MatView& w, const int8_t* aq, const float* as, int T, float* y, int ldy, cudaStream_t st) {
  dim3 grid((T + kGemmBN - 1) / kGemmBN, (w.rows + kGemmBM - 1) / kGemmBM);
#define F(B, S)                                                                                              \
  do {                                                                                                       \
    static bool init = false;                                                                                \
    if (!init) {                                                                                             \
      cudaFuncSetAttribute(k_seq_gemm<B, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmTile<B, S>::SMEM); \
      init = true;                                                                                           \
    }                                                                                                        \
    k_seq_gemm<B, S><<<grid, kGemmThreads, GemmTile<B, S>::SMEM, st>>>(w, aq, as, T, y, ldy);                \
  } while (0)
  GEM_DISPATCH_Q(w.bits, w.scale_f32, F);
#undef F
}

void launch_seq_attn(const AttnArgs& A, const float* qkv, int qkv_ld, int T, uint32_t pos0, float* qn, float* scores,
                     int sstride, int threads, int8_t* aq, float* as, cudaStream_t st) {
  const int G = A.nh / A.nkv;
  k_seq_attn_prep<<<dim3(T, A.nkv), 256, (size_t)(G + 2) * A.hd * 4, st>>>(A, qkv, qkv_ld, pos0, qn);
  const size_t qsm = (size_t)A.nh * A.hd * 4;
#define F(GG) k_seq_scores<GG><<<T, 256, qsm, st>>>(A, qn, pos0, scores, sstride)
  if (G == 1) F(1);
  else if (G == 2) F(2);
  else if (G == 4) F(4);
  else if (G == 8) F(8);
  else return;  // other group sizes are rejected by the caller before any launch
#undef F
  {
    static bool init = false;
    if (!init) {
      cudaFuncSetAttribute(k_seq_softmax, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      init = true;
    }
    const int nw = (int)std::max<size_t>(1, std::min<size_t>(8, (size_t)(200 * 1024) / ((size_t)sstride * 4)));
    k_seq_softmax<<<(T * A.nh + nw - 1) / nw, nw * 32, (size_t)nw * sstride * 4, st>>>(A, T, pos0, scores, sstride);
  }
  k_seq_pv<<<T, A.hd, 0, st>>>(A, pos0, scores, sstride, threads, aq, as);
}

void launch_seq_glu_quant(const float* gu, int ff, int T, int silu, int8_t* aq, float* as, int sms, cudaStream_t st) {
  const long long tasks = (long long)T * (ff / 32);
  const int blocks = (int)std::min<long long>((tasks + 7) / 8, (long long)sms * 16);
  k_seq_glu_quant<<<blocks, 256, 0, st>>>(gu, ff, T, silu, aq, as);
}

void launch_seq_class_logits(const float* A, const float* b, int k, const float* h, int d, int T, float* cl,
                             cudaStream_t st) {
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(k_seq_class_logits, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    init = true;
  }
  dim3 grid((T + 31) / 32, (k + 31) / 32);
  k_seq_class_logits<<<grid, 256, (size_t)32 * d * 4, st>>>(A, b, k, h, d, T, cl);
}

void launch_seq_logit_reduce(const float* logits, int V, int T, const uint32_t* targets, float* lp, uint32_t* am, int* err,
                             cudaStream_t st) {
  k_seq_logit_reduce<<<T, 1024, 0, st>>>(logits, V, targets, lp, am, err);
}

}  // namespace gem
