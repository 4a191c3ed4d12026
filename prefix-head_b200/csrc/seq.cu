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
//   k_seq_scores_tile8 dot512(q[t][h], K[p]) for p in the window of t             (model.rs:344-353)
//   k_seq_softmax      max, exp_fast, sequential sum, 1/sum                         (model.rs:354-361)
//   k_seq_pv_tile8     P.V partial sums over the pool's position ranges             (model.rs:362-382)
//                      (k_seq_pv_tile for head dims other than 256)
//   k_seq_pv_combine   partials added in range order, then Act::quantize
//   k_seq_glu_quant    GELU-tanh (or SiLU) gate * up, Act::quantize                 (model.rs:408-416)
//   k_seq_dot16_gemm   two-level class logits dot512(A[c], h[t]) + b[c]            (main.rs:82-93)
//                      and the full head of an F16 output matrix, dot16           (q8.rs:358-369)
//   k_seq_logit_reduce full-head log-sum-exp, argmax and target logit per position  (main.rs:30-37)
#include <algorithm>
#include <cstdlib>
#include <type_traits>

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


__host__ __device__ __forceinline__ uint32_t window_lo(uint32_t pos, int window) {
  return (window > 0 && pos + 1 > (uint32_t)window) ? pos + 1 - window : 0;
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// Embedding: one CTA per position. Ids >= vocab are recorded in *err and replaced by 0. row_of maps a
// token to its row when the matrix is held in class order (null: token order).
// ------------------------------------------------------------------------------------------------
template <int BITS, typename ST>
__global__ void k_seq_embed(MatView E, const uint32_t* row_of, const uint32_t* toks, int vocab, float scale, float* x,
                            int* err) {
  pdl_wait();
  const int t = blockIdx.x;
  uint32_t tok = toks[t];
  if (tok >= (uint32_t)vocab) {
    if (threadIdx.x == 0) atomicExch(err, ERR_RANGE);
    tok = 0;
  }
  const size_t row = row_of ? row_of[tok] : tok;
  for (int j = threadIdx.x; j < E.cols; j += blockDim.x) x[(size_t)t * E.cols + j] = mul(weight_at<BITS, ST>(E, row, j), scale);
}

// ------------------------------------------------------------------------------------------------
// Residual + post-norm, then pre-norm + quantize (k_residual_norm_quant_exact per position). One warp
// per position: squares in parallel, lane 0 adds them in order (Rust's sequential f32 sum).
// ------------------------------------------------------------------------------------------------
constexpr int kNormWarps = 4;

// n a multiple of 32. The next 16 values are loaded while the current 16 are added, so the chain of
// dependent adds is the only latency left.
__device__ __forceinline__ float warp_seq_sum(const float* sq, int n, int lane) {
  float s = 0.0f;
  if (lane == 0) {
    const float4* p = (const float4*)sq;
    const int n4 = n / 4;
    float4 a[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) a[u] = p[u];
    for (int j = 4; j <= n4; j += 4) {
      float4 nx[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) nx[u] = j < n4 ? p[j + u] : a[u];
#pragma unroll
      for (int u = 0; u < 4; ++u) s = add(add(add(add(s, a[u].x), a[u].y), a[u].z), a[u].w);
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = nx[u];
    }
  }
  return __shfl_sync(0xffffffffu, s, 0);
}

constexpr int kNormMaxV = 9;  // float4 per lane: d <= 1152

__global__ void __launch_bounds__(kNormWarps * 32) k_seq_norm(float* x, const float* delta, const float* w_post,
                                                              const float* w_pre, float eps, int d, int T, int8_t* aq,
                                                              float* as, float* xn_out) {
  extern __shared__ __align__(16) float sn[];  // w_post [d], w_pre [d], then per warp [2 d] (sq in the second half)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, n4 = d / 4;
  float* swpost = sn;
  float* swpre = sn + d;
  // the norm weights depend on no earlier kernel: they load while the previous kernel drains
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    ((float4*)swpre)[i] = ((const float4*)w_pre)[i];
    if (w_post) ((float4*)swpost)[i] = ((const float4*)w_post)[i];
  }
  const int t = blockIdx.x * kNormWarps + warp;
  float4* xt = (float4*)(x + (size_t)t * d);
  float4 xv[kNormMaxV], dv[kNormMaxV];
  // With a delta the residual stream x was last written by a norm at least three kernels back (the
  // previous kernel writes only delta), so it loads before the wait too; without one (the first norm,
  // right after the embedding) it loads after.
  if (delta && t < T)
#pragma unroll
    for (int k = 0; k < kNormMaxV; ++k)
      if (lane + 32 * k < n4) xv[k] = xt[lane + 32 * k];
  pdl_wait();
  __syncthreads();
  if (t >= T) return;
  float* sq = sn + 2 * d + (size_t)warp * 2 * d + d;
#pragma unroll
  for (int k = 0; k < kNormMaxV; ++k) {  // every load of this position issued before any is used
    const int i = lane + 32 * k;
    if (i < n4) {
      if (delta) dv[k] = ((const float4*)(delta + (size_t)t * d))[i];
      else xv[k] = xt[i];
    }
  }
  auto sq4 = [](float4 v) { return make_float4(mul(v.x, v.x), mul(v.y, v.y), mul(v.z, v.z), mul(v.w, v.w)); };
  if (delta) {
    float r = 1.0f;
    if (w_post) {
#pragma unroll
      for (int k = 0; k < kNormMaxV; ++k)
        if (lane + 32 * k < n4) ((float4*)sq)[lane + 32 * k] = sq4(dv[k]);
      __syncwarp();
      r = rms_r_exact(warp_seq_sum(sq, d, lane), d, eps);
    }
#pragma unroll
    for (int k = 0; k < kNormMaxV; ++k) {
      const int i = lane + 32 * k;
      if (i >= n4) continue;
      float4 v = dv[k];
      if (w_post) {  // rmsnorm_inplace (model.rs:89-95): v *= r * w
        const float4 w = ((const float4*)swpost)[i];
        v = make_float4(mul(v.x, mul(r, w.x)), mul(v.y, mul(r, w.y)), mul(v.z, mul(r, w.z)), mul(v.w, mul(r, w.w)));
      }
      const float4 o = xv[k];
      xv[k] = make_float4(add(o.x, v.x), add(o.y, v.y), add(o.z, v.z), add(o.w, v.w));
      xt[i] = xv[k];
    }
  }
#pragma unroll
  for (int k = 0; k < kNormMaxV; ++k) {
    const int i = lane + 32 * k;
    if (i < n4) ((float4*)sq)[i] = sq4(xv[k]);
  }
  __syncwarp();
  const float r = rms_r_exact(warp_seq_sum(sq, d, lane), d, eps);
  // rmsnorm (model.rs:81-87), then Act::quantize from registers: the 32-block b is float4s 8b .. 8b + 7,
  // held by 8 consecutive lanes, so a warp quantizes four blocks at once (block max over 8 lanes; a
  // max is exact in any order). d is a multiple of 32, so a group of 8 lanes is wholly in or out.
  const int nb = d / 32;
#pragma unroll
  for (int k = 0; k < kNormMaxV; ++k) {
    if (32 * k >= n4) break;
    const int i = lane + 32 * k;
    const bool in = i < n4;
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (in) {
      const float4 w = ((const float4*)swpre)[i];
      v = make_float4(mul(mul(xv[k].x, r), w.x), mul(mul(xv[k].y, r), w.y), mul(mul(xv[k].z, r), w.z),
                      mul(mul(xv[k].w, r), w.w));
      if (xn_out) ((float4*)(xn_out + (size_t)t * d))[i] = v;
    }
    if (aq) {
      float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
      if (in) {  // quant_block_warp_x's arithmetic: d = amax / 127, q = rn(v * (1 / d))
        const float dd = div(m, 127.0f);
        const float inv = dd > 0.0f ? div(1.0f, dd) : 0.0f;
        const uint32_t q0 = (uint32_t)__float2int_rn(mul(v.x, inv)) & 0xffu, q1 = (uint32_t)__float2int_rn(mul(v.y, inv)) & 0xffu,
                       q2 = (uint32_t)__float2int_rn(mul(v.z, inv)) & 0xffu, q3 = (uint32_t)__float2int_rn(mul(v.w, inv)) & 0xffu;
        ((uint32_t*)(aq + (size_t)t * d))[i] = q0 | (q1 << 8) | (q2 << 16) | (q3 << 24);
        if ((lane & 7) == 0) as[(size_t)t * nb + (i >> 3)] = dd;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Exact int8 matrix product: Y[t][r] = row_dot(W[r], act[t]) for Q8 / Q4 weights, with the lane
// structure of dot_avx512 / dot4_avx512 (lane i = w[2i]a[2i] + w[2i+1]a[2i+1] per 32-block, one FMA
// per block with scale ws*as, halving reduction). A thread pair holds the 16 lanes of one row for RN
// positions (8 + 8 lanes, as in row_dot_exact). CTA tile: 32 rows x 4*RN positions, 8 warps
// (warp w: rows 16*(w&1) .. +15, positions RN*(w>>1) .. +RN-1), K staged through shared memory in
// chunks of 8 blocks (256 columns) by cp.async, three stages deep. RN = 8 for large matrices, 4 where
// the smaller tile fills the SMs more evenly (640-row projections at 512 positions).
// ------------------------------------------------------------------------------------------------
constexpr int kGemmBM = 32, kGemmKB = 8, kGemmStages = 3, kGemmThreads = 256;

template <int BITS, typename ST, int RN>
struct GemmTile {
  static constexpr int BN = 4 * RN;                    // positions per CTA
  static constexpr int WB = BITS == 8 ? 32 : 16;       // weight bytes per 32-block of a row
  static constexpr int WROW = kGemmKB * WB + 16;       // padded row: 16-row reads hit distinct banks
  static constexpr int SB = (int)sizeof(ST);
  static constexpr int A_OFF = kGemmBM * WROW;                        // activations [BN][KB*32]
  static constexpr int SW_OFF = A_OFF + BN * kGemmKB * 32;            // weight scales [BM][KB]
  static constexpr int SA_OFF = SW_OFF + kGemmBM * kGemmKB * SB;      // activation scales [KB][BN]
  static constexpr int STAGE = (SA_OFF + kGemmKB * BN * 4 + 127) / 128 * 128;
  static constexpr int SMEM = kGemmStages * STAGE;
};

template <int BITS, typename ST, int RN>
__device__ __forceinline__ void gemm_issue(unsigned char* stage, const MatView& w, const int8_t* aq, const float* as,
                                           int T, int row0, int tok0, int b0, int kb) {
  using G = GemmTile<BITS, ST, RN>;
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
  for (int i = tid; i < G::BN * AP; i += kGemmThreads) {
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
  for (int i = tid; i < kGemmKB * G::BN; i += kGemmThreads) {
    const int b = i / G::BN, t = i % G::BN;
    const bool ok = b < kb && tok0 + t < T;
    const float* src = as + (ok ? (size_t)(tok0 + t) * nb + b0 + b : 0);
    cp4(stage + G::SA_OFF + (b * G::BN + t) * 4, src, ok);
  }
}

template <int BITS, typename ST, int RN>
__global__ void __launch_bounds__(kGemmThreads, RN == 8 ? 2 : 3) k_seq_gemm(MatView w, const int8_t* aq,
                                                                             const float* as, int T, float* y, int ldy) {
  pdl_wait();
  using G = GemmTile<BITS, ST, RN>;
  extern __shared__ __align__(128) unsigned char sg[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, half = lane & 1;
  const int tok0 = blockIdx.x * G::BN, row0 = blockIdx.y * kGemmBM;
  const int rl = (warp & 1) * 16 + (lane >> 1);  // row inside the tile
  const int tl = (warp >> 1) * RN;               // first of this thread's RN positions
  const int nb = w.cols / 32;
  const int nchunks = (nb + kGemmKB - 1) / kGemmKB;

  float2 acc[RN][4];  // lanes (2q, 2q + 1) of this thread's half, per position
#pragma unroll
  for (int i = 0; i < RN; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[i][k] = make_float2(0.0f, 0.0f);

#pragma unroll
  for (int s = 0; s < kGemmStages - 1; ++s) {
    if (s < nchunks)
      gemm_issue<BITS, ST, RN>(sg + s * G::STAGE, w, aq, as, T, row0, tok0, s * kGemmKB, min(kGemmKB, nb - s * kGemmKB));
    cp_commit();
  }
  for (int c = 0; c < nchunks; ++c) {
    cp_wait<kGemmStages - 2>();
    __syncthreads();
    {
      const int cn = c + kGemmStages - 1;
      if (cn < nchunks)
        gemm_issue<BITS, ST, RN>(sg + (cn % kGemmStages) * G::STAGE, w, aq, as, T, row0, tok0, cn * kGemmKB,
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
      // the low / high int16 pair of each weight word, masked once for all RN positions
      const int wl[4] = {wv.x & 0x0000ffff, wv.y & 0x0000ffff, wv.z & 0x0000ffff, wv.w & 0x0000ffff};
      const int wh[4] = {wv.x & (int)0xffff0000, wv.y & (int)0xffff0000, wv.z & (int)0xffff0000, wv.w & (int)0xffff0000};
      const float swb = ld_scale(wsc, b);
      float sa[RN];
#pragma unroll
      for (int k = 0; k < RN; k += (RN % 4 == 0 ? 4 : 2)) {  // this thread's RN scales start at a multiple of RN
        if constexpr (RN % 4 == 0) {
          const float4 v = *(const float4*)(asc + b * G::BN + k);
          sa[k] = v.x, sa[k + 1] = v.y, sa[k + 2] = v.z, sa[k + 3] = v.w;
        } else {
          const float2 v = *(const float2*)(asc + b * G::BN + k);
          sa[k] = v.x, sa[k + 1] = v.y;
        }
      }
#pragma unroll
      for (int k = 0; k < RN; ++k) {
        const int4 av = *(const int4*)(arow + k * (kGemmKB * 32) + b * 32);
        const float s = mul(swb, sa[k]);
        const float2 s2 = make_float2(s, s);
        const int a4[4] = {av.x, av.y, av.z, av.w};
        // two madd_epi16 lanes per step: exact int32 pair sums converted to fp32 (exact: |p| < 2^24),
        // then one packed FMA, which rounds each lane as fmaf does
#pragma unroll
        for (int q = 0; q < 4; ++q)
          acc[k][q] = __ffma2_rn(make_float2((float)__dp4a(wl[q], a4[q], 0), (float)__dp4a(wh[q], a4[q], 0)), s2, acc[k][q]);
      }
    }
  }
  cp_wait<0>();
  const int r = row0 + rl;
#pragma unroll
  for (int k = 0; k < RN; ++k) {
    const float a8[8] = {acc[k][0].x, acc[k][0].y, acc[k][1].x, acc[k][1].y, acc[k][2].x, acc[k][2].y, acc[k][3].x, acc[k][3].y};
    const float v = reduce16_pair(a8);
    const int t = tok0 + tl + k;
    if (half == 0 && r < w.rows && t < T) y[(size_t)t * ldy + r] = v;
  }
}

// ------------------------------------------------------------------------------------------------
// Attention, exact. The chunk holds `nseq` sequences of L positions each, rows ordered [seq][pos]:
// row t is position pos0 + t % L of sequence t / L, whose K/V cache starts kv_stride floats after the
// previous sequence's.
// ------------------------------------------------------------------------------------------------
// QK-norm, RoPE, scale, K/V append: one CTA per (position, kv group).
__device__ __forceinline__ AttnArgs seq_kv(const AttnArgs& A, int s, size_t kv_stride) {
  AttnArgs a = A;
  a.kcache += (size_t)s * kv_stride;
  a.vcache += (size_t)s * kv_stride;
  return a;
}

__global__ void k_seq_attn_prep(AttnArgs A, const float* qkv, int qkv_ld, int L, uint32_t pos0, size_t kv_stride,
                                float* qn) {
  pdl_wait();
  extern __shared__ __align__(16) float smp[];
  __shared__ float s_r[17];
  const int t = blockIdx.x, s = t / L;
  attn_prep_token(seq_kv(A, s, kv_stride), qkv + (size_t)t * qkv_ld, pos0 + t % L, blockIdx.y,
                  qn + (size_t)t * A.nh * A.hd, smp, s_r);
}

// Score tiles: a CTA takes kAttnTQ consecutive positions x the G query heads of kv group blockIdx.z
// (R rows) against kScKC key positions from pbase + blockIdx.y * kScKC (k_seq_scores_tile8 below).
constexpr int kAttnTQ = 8, kScKC = 32;

// Softmax per (position, head) with the reference's order: max, exp_fast(s - max), sequential sum,
// multiply by 1/sum. One warp per (position, head).
__global__ void k_seq_softmax(AttnArgs A, int T, int L, uint32_t pos0, float* scores, int sstride) {
  pdl_wait();
  extern __shared__ __align__(16) float ss[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int task = blockIdx.x * nw + warp;
  if (task >= T * A.nh) return;
  const int t = task / A.nh;
  const uint32_t pos = pos0 + t % L, lo = window_lo(pos, A.window);
  const int n = (int)(pos + 1 - lo);
  float* s = scores + (size_t)task * sstride;
  float* e = ss + (size_t)warp * (((sstride + 3) & ~3) + 16);  // 16-byte aligned rows, 16 floats of slack for the prefetch
  for (int i = lane; i < n; i += 32) cp4(e + i, s + i, true);
  cp_commit();
  cp_wait<0>();
  __syncwarp();
  float m = -INFINITY;
  for (int i = lane; i < n; i += 32) m = fmaxf(m, e[i]);
  m = warp_max(m);
  for (int i = lane; i < n; i += 32) e[i] = exp_fast(sub(e[i], m));
  __syncwarp();
  float sum = 0.0f;
  if (lane == 0) {  // in order; the next 16 values load while the current 16 are added
    const int n16 = n & ~15;
    const float4* p = (const float4*)e;
    float4 a[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) a[u] = p[u];  // a row has 16 floats of slack: loads past n are never added
    for (int j = 0; j < n16; j += 16) {
      float4 nx[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) nx[u] = p[j / 4 + 4 + u];
#pragma unroll
      for (int u = 0; u < 4; ++u) sum = add(add(add(add(sum, a[u].x), a[u].y), a[u].z), a[u].w);
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = nx[u];
    }
    for (int i = n16; i < n; ++i) sum = add(sum, e[i]);
  }
  const float inv = div(1.0f, __shfl_sync(0xffffffffu, sum, 0));
  for (int i = lane; i < n; i += 32) s[i] = mul(e[i], inv);
}

// P.V by range: the pool's partition (model.rs:362-382) makes each of the `threads` position ranges
// of a row an independent partial sum, so a CTA takes one range r of every row of a tile of
// kAttnTQ positions (all heads), stages the V rows of the tile's ranges in chunks of kPvRows, and
// writes the partials; k_seq_pv_combine adds them in range order. Thread j = output element.
constexpr int kPvRows = 32;

template <int G>
__global__ void __launch_bounds__(128) k_seq_pv_tile(AttnArgs A0, int L, uint32_t pos0, size_t kv_stride,
                                                     const float* scores, int sstride, int threads, float* part) {
  pdl_wait();
  constexpr int R = kAttnTQ * G;               // rows of the tile: position x head of the group
  extern __shared__ __align__(16) float sv[];  // V [kPvRows][hd], then probabilities P [kPvRows][R] (rows adjacent)
  __shared__ uint32_t s_lo[kAttnTQ], s_a[kAttnTQ], s_b[kAttnTQ];
  const int tps = (L + kAttnTQ - 1) / kAttnTQ, sq_i = blockIdx.x / tps;
  const AttnArgs A = seq_kv(A0, sq_i, kv_stride);
  scores += (size_t)sq_i * L * A.nh * sstride;
  part += (size_t)sq_i * L * A.nh * threads * A.hd;
  const int hd = A.hd, h4 = hd / 4, t0 = (blockIdx.x % tps) * kAttnTQ, tn = min(kAttnTQ, L - t0), r = blockIdx.y;
  const int j2 = threadIdx.x * 2;  // this thread's two output columns
  const int ve = (int)threadIdx.x % h4, vr0 = (int)threadIdx.x / h4;  // V staging: column, first row
  const int rw = A.nkv * hd;
  float* sp = sv + kPvRows * hd;
  if (threadIdx.x < kAttnTQ) {
    const int tt = threadIdx.x;
    uint32_t lo = 0, a = 0, b = 0;
    if (tt < tn) {
      const uint32_t pos = pos0 + t0 + tt;
      lo = window_lo(pos, A.window);
      const int n = (int)(pos + 1 - lo), per = (n + threads - 1) / threads;
      a = lo + min(r * per, n);
      b = lo + min((r + 1) * per, n);
    }
    s_lo[tt] = lo, s_a[tt] = a, s_b[tt] = b;
  }
  __syncthreads();
  uint32_t ua = 0xffffffffu, ub = 0;
  for (int tt = 0; tt < tn; ++tt)
    if (s_a[tt] < s_b[tt]) ua = min(ua, s_a[tt]), ub = max(ub, s_b[tt]);
  for (int g = 0; g < A.nkv; ++g) {
    float2 ac0[R / 2], ac1[R / 2];  // columns j2, j2 + 1: rows (2i, 2i + 1)
#pragma unroll
    for (int i = 0; i < R / 2; ++i) ac0[i] = ac1[i] = make_float2(0.0f, 0.0f);
    for (uint32_t c0 = ua; c0 < ub; c0 += kPvRows) {
      const int rows = (int)min((uint32_t)kPvRows, ub - c0), rows4 = (rows + 3) & ~3;
      __syncthreads();
      for (int pr = vr0; pr < rows4; pr += 2) {  // blockDim.x = 2 h4: a thread keeps its 16-byte column
        const bool ok = pr < rows;                // rows past `rows` are zero
        cp16(sv + pr * hd + ve * 4, A.vcache + (ok ? (size_t)(c0 + pr) * rw + g * hd + ve * 4 : 0), ok);
      }
      // a row's probabilities are zero outside its range, which makes its FMAs there exact no-ops
      // (a range's sum starts at +0 and never becomes -0, so adding 0 * v changes nothing)
      for (int i = threadIdx.x; i < R * kPvRows; i += blockDim.x) {
        const int row = i / kPvRows, pi = i % kPvRows, tt = row / G, h = row % G;
        const uint32_t p = c0 + pi;
        const bool ok = tt < tn && pi < rows && p >= s_a[tt] && p < s_b[tt];
        cp4(sp + pi * R + row, scores + (ok ? ((size_t)(t0 + tt) * A.nh + g * G + h) * sstride + (p - s_lo[tt]) : 0), ok);
      }
      cp_commit();
      cp_wait<0>();
      __syncthreads();
      // per position: V's two columns duplicated once, then every pair of adjacent rows in one FMA each
      for (int p = 0; p < rows; ++p) {
        const float2 v = *(const float2*)(sv + p * hd + j2);
        const float2 v0 = make_float2(v.x, v.x), v1 = make_float2(v.y, v.y);
        const float* pp = sp + p * R;
#pragma unroll
        for (int i = 0; i < R; i += 4) {
          const float4 q = *(const float4*)(pp + i);
          ac0[i / 2] = __ffma2_rn(make_float2(q.x, q.y), v0, ac0[i / 2]);
          ac0[i / 2 + 1] = __ffma2_rn(make_float2(q.z, q.w), v0, ac0[i / 2 + 1]);
          ac1[i / 2] = __ffma2_rn(make_float2(q.x, q.y), v1, ac1[i / 2]);
          ac1[i / 2 + 1] = __ffma2_rn(make_float2(q.z, q.w), v1, ac1[i / 2 + 1]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int tt = i / G, h = i % G;
      const float2 o = (i & 1) ? make_float2(ac0[i / 2].y, ac1[i / 2].y) : make_float2(ac0[i / 2].x, ac1[i / 2].x);
      if (tt < tn)
        *(float2*)(part + (((size_t)(t0 + tt) * A.nh + g * G + h) * threads + r) * hd + j2) = o;
    }
  }
}

// P.V by range for head_dim 256, with a register tile that feeds the FMA pipe: as k_seq_pv_tile (a
// CTA takes range r of every row of a tile of kAttnTQ positions x G heads, stages the range's V rows
// and probabilities in chunks of kPvRows, writes the partial sums), but warp w holds rows 8w .. + 8 and
// lane l columns 4l .. + 4 and 128 + 4l .. + 4, so per key 16 loaded values feed 64 FMAs (a row's
// probabilities are a broadcast, a lane's V columns 16-byte pieces of one contiguous row).
template <int G>
__global__ void __launch_bounds__(32 * G, G <= 4 ? 3 : 2) k_seq_pv_tile8(AttnArgs A0, int L, uint32_t pos0, size_t kv_stride,
                                                        const float* scores, int sstride, int threads, float* part) {
  pdl_wait();
  constexpr int R = kAttnTQ * G, HD = 256;
  extern __shared__ __align__(16) float sv[];  // V [kPvRows][HD], then probabilities P [kPvRows][R]
  __shared__ uint32_t s_lo[kAttnTQ], s_a[kAttnTQ], s_b[kAttnTQ];
  const int tps = (L + kAttnTQ - 1) / kAttnTQ, sq_i = blockIdx.x / tps;
  const AttnArgs A = seq_kv(A0, sq_i, kv_stride);
  scores += (size_t)sq_i * L * A.nh * sstride;
  part += (size_t)sq_i * L * A.nh * threads * HD;
  const int t0 = (blockIdx.x % tps) * kAttnTQ, tn = min(kAttnTQ, L - t0), r = blockIdx.y;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, rw = A.nkv * HD;
  float* sp = sv + kPvRows * HD;
  if (threadIdx.x < kAttnTQ) {
    const int tt = threadIdx.x;
    uint32_t lo = 0, a = 0, b = 0;
    if (tt < tn) {
      const uint32_t pos = pos0 + t0 + tt;
      lo = window_lo(pos, A.window);
      const int n = (int)(pos + 1 - lo), per = (n + threads - 1) / threads;
      a = lo + min(r * per, n);
      b = lo + min((r + 1) * per, n);
    }
    s_lo[tt] = lo, s_a[tt] = a, s_b[tt] = b;
  }
  __syncthreads();
  uint32_t ua = 0xffffffffu, ub = 0;
  for (int tt = 0; tt < tn; ++tt)
    if (s_a[tt] < s_b[tt]) ua = min(ua, s_a[tt]), ub = max(ub, s_b[tt]);
  for (int g = 0; g < A.nkv; ++g) {
    float2 acc[8][4];  // [row][(4l, 4l+1), (4l+2, 4l+3), (128+4l, +1), (128+4l+2, +3)]
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = make_float2(0.0f, 0.0f);
    for (uint32_t c0 = ua; c0 < ub; c0 += kPvRows) {
      const int rows = (int)min((uint32_t)kPvRows, ub - c0);
      __syncthreads();  // the previous chunk's reads are done
      for (int e = threadIdx.x; e < rows * (HD / 4); e += blockDim.x) {  // V: 64 pieces of 16 bytes per key
        const int pi = e / (HD / 4), c4 = e % (HD / 4);
        cp16(sv + pi * HD + c4 * 4, A.vcache + (size_t)(c0 + pi) * rw + g * HD + c4 * 4, true);
      }
      // a row's probabilities are zero outside its range, which makes its FMAs there exact no-ops
      // (a range's sum starts at +0 and never becomes -0, so adding 0 * v changes nothing)
      for (int i = threadIdx.x; i < R * kPvRows; i += blockDim.x) {
        const int row = i / kPvRows, pi = i % kPvRows, tt = row / G, h = row % G;
        const uint32_t p = c0 + pi;
        const bool ok = tt < tn && pi < rows && p >= s_a[tt] && p < s_b[tt];
        cp4(sp + pi * R + row, scores + (ok ? ((size_t)(t0 + tt) * A.nh + g * G + h) * sstride + (p - s_lo[tt]) : 0), ok);
      }
      cp_commit();
      cp_wait<0>();
      __syncthreads();
      const float* pp = sp + 8 * w;
      const float* vp = sv + 4 * lane;
#pragma unroll 1
      for (int k = 0; k < rows; ++k) {
        const float4 pa = *(const float4*)(pp + k * R), pb = *(const float4*)(pp + k * R + 4);
        const float4 va = *(const float4*)(vp + k * HD), vb = *(const float4*)(vp + k * HD + 128);
        const float pr[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 q = make_float2(pr[i], pr[i]);
          acc[i][0] = __ffma2_rn(q, make_float2(va.x, va.y), acc[i][0]);
          acc[i][1] = __ffma2_rn(q, make_float2(va.z, va.w), acc[i][1]);
          acc[i][2] = __ffma2_rn(q, make_float2(vb.x, vb.y), acc[i][2]);
          acc[i][3] = __ffma2_rn(q, make_float2(vb.z, vb.w), acc[i][3]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = 8 * w + i, tt = row / G, h = row % G;
      if (tt < tn) {
        float* o = part + (((size_t)(t0 + tt) * A.nh + g * G + h) * threads + r) * HD + 4 * lane;
        *(float4*)o = make_float4(acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y);
        *(float4*)(o + 128) = make_float4(acc[i][2].x, acc[i][2].y, acc[i][3].x, acc[i][3].y);
      }
    }
  }
}

// att[t][h][j] = partials summed in range order (from 0), then Act::quantize. One CTA per
// (position, head), all partial loads in flight before the ordered adds.
__global__ void k_seq_pv_combine(AttnArgs A, const float* part, int threads, int8_t* aq, float* as) {
  pdl_wait();
  const int t = blockIdx.x, h = blockIdx.y, hd = A.hd, j = threadIdx.x, lane = j & 31;
  const int nbh = A.nh * hd / 32;
  const float* pp = part + ((size_t)t * A.nh + h) * threads * hd + j;
  float a = 0.0f;
  for (int r0 = 0; r0 < threads; r0 += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = r0 + u < threads ? pp[(size_t)(r0 + u) * hd] : 0.0f;
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (r0 + u < threads) a = add(a, v[u]);
  }
  const int b = (h * hd + j) / 32;
  quant_block_warp_x(a, lane, aq + (size_t)t * A.nh * hd + b * 32, as + (size_t)t * nbh + b);
}

// ------------------------------------------------------------------------------------------------
// Gate (k_glu_quant per position): v = gelu_tanh(g) * u (or silu(g) * u), then Act::quantize.
// ------------------------------------------------------------------------------------------------
__global__ void k_seq_glu_quant(const float* gu, int ff, int T, int silu, int8_t* aq, float* as) {
  pdl_wait();
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
// Full head from a logits matrix [T][V]: online log-sum-exp, argmax (first maximum) and the target's
// logit per position; logprob = logit[target] - lse. One CTA per position. With the matrix in class
// order, row_tok maps a row to its token and row_of a token to its row (both null: token order); a
// thread keeps its best row (best_row_add), reading tokens only to break exact ties.
// ------------------------------------------------------------------------------------------------
__global__ void k_seq_logit_reduce(const float* logits, int V, const uint32_t* targets, const uint32_t* row_of,
                                   const uint32_t* row_tok, float* lp, uint32_t* am, int* err) {
  pdl_wait();
  __shared__ float red_m[32], red_s[32], red_v[32];
  __shared__ uint32_t red_t[32];
  const int t = blockIdx.x;
  const float* z = logits + (size_t)t * V;
  Lse L{-INFINITY, 0.0f};
  Best B{-INFINITY, 0xffffffffu};
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = z[i];
    L = lse_add(L, v);
    best_row_add(B, v, (uint32_t)i, row_tok);
  }
  best_row_to_token(B, row_tok);
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
    lp[t] = z[row_of ? row_of[tg] : tg] - (L.m + logf(L.s));
    if (am) am[t] = B.tok;
  }
}

// Vocab-sharded full head: this rank's rows [row0, row0 + V) of the output matrix give, per position,
// the partial log-sum-exp state, the best logit with its token id and the target's logit (NaN when
// the target is another rank's). out[t] = {m, s, best, best id bits, target logit}.
__global__ void k_seq_logit_partials(const float* logits, int V, uint32_t row0, const uint32_t* targets, uint32_t vocab,
                                     const uint32_t* row_of, const uint32_t* row_tok, float* out, int* err) {
  pdl_wait();
  __shared__ float red_m[32], red_s[32], red_v[32];
  __shared__ uint32_t red_t[32];
  const int t = blockIdx.x;
  const float* z = logits + (size_t)t * V;
  Lse L{-INFINITY, 0.0f};
  Best B{-INFINITY, 0xffffffffu};
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = z[i];
    L = lse_add(L, v);
    best_row_add(B, v, row0 + (uint32_t)i, row_tok);
  }
  best_row_to_token(B, row_tok);
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
    if (tg >= vocab) {
      atomicExch(err, ERR_RANGE);
      tg = 0;
    }
    const uint32_t tr = row_of ? row_of[tg] : tg;
    const float tl = tr >= row0 && tr < row0 + (uint32_t)V ? z[tr - row0] : __int_as_float(0x7fffffff);
    float* o = out + (size_t)t * 5;
    o[0] = L.m, o[1] = L.s, o[2] = B.v, o[3] = __uint_as_float(B.tok), o[4] = tl;
  }
}

// Merges the ranks' partials (gathered [nranks][T][5]) into logprob and argmax (ties: lowest id).
__global__ void k_seq_logit_combine(const float* parts, int nranks, int T, float* lp, uint32_t* am) {
  pdl_wait();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  Lse L{-INFINITY, 0.0f};
  Best B{-INFINITY, 0xffffffffu};
  float tl = __int_as_float(0x7fffffff);
  for (int r = 0; r < nranks; ++r) {
    const float* o = parts + ((size_t)r * T + t) * 5;
    L = lse_merge(L, Lse{o[0], o[1]});
    B = best_merge(B, Best{o[2], __float_as_uint(o[3])});
    if (!isnan(o[4])) tl = o[4];
  }
  lp[t] = tl - (L.m + logf(L.s));
  if (am) am[t] = B.tok;
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


bool pdl_on() {
  static const bool on = [] {
    const char* e = std::getenv("GEM_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

void launch_seq_embed(const MatView& E, const uint32_t* row_of, const uint32_t* toks, int T, int vocab, float scale,
                      float* x, int* err, cudaStream_t st) {
#define F(B, S) launch_k(k_seq_embed<B, S>, dim3(T), dim3(256), 0, st, E, row_of, toks, vocab, scale, x, err)
  if (E.bits == 16) F(16, __half);
  else GEM_DISPATCH_Q(E.bits, E.scale_f32, F);
#undef F
}

void launch_seq_norm(float* x, const float* delta, const float* w_post, const float* w_pre, float eps, int d, int T,
                     int8_t* aq, float* as, float* xn_out, cudaStream_t st) {
  size_t sm = (size_t)(kNormWarps + 1) * 2 * d * 4;
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(k_seq_norm, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    init = true;
  }
  launch_k(k_seq_norm, dim3((T + kNormWarps - 1) / kNormWarps), dim3(kNormWarps * 32), sm, st, x, delta, w_post, w_pre, eps, d, T, aq, as,
                                                                              xn_out);
}

// The halving reduction of dot512/dot16 over the 16 threads of a half-warp, as a reduce-scatter: thread
// l of the half holds lane l of 64 sums v[0..64); each round (partner l ^ 8, ^ 4, ^ 2, ^ 1) adds the
// partner's lane to the half of the sums this thread keeps, so the pairs are lane i + lane i + 8, then
// + 4, + 2, + 1 as in the reference. Thread l ends with sums 4l .. 4l + 3 in v[0..4).
__device__ __forceinline__ void half_reduce16(float (&v)[64], int l) {
#pragma unroll
  for (int m = 8, n = 32; m >= 1; m >>= 1, n >>= 1) {
    const bool up = (l & m) != 0;  // keep the upper n sums, send the lower ones
#pragma unroll
    for (int i = 0; i < n; ++i) {
      const float keep = up ? v[i + n] : v[i], send = up ? v[i] : v[i + n];
      v[i] = add(keep, __shfl_xor_sync(0xffffffffu, send, m));
    }
  }
}

// Exact products of 16-lane dots for T positions: y[p][r] = dot16 (q8.rs:358-369) of row r of an F16
// matrix (each weight converted to fp32) or dot512 (model.rs:106-120) of row r of an fp32 matrix, with
// the fp32 hidden state of position p, plus bias[r] when given (the two-level class logits,
// main.rs:101-107) -- lane i sums w[16c+i] * x[16c+i] by FMA in order of c, then the halving
// reduction, then the bias. A CTA takes kH16Rows rows x
// kH16Pos positions in stages of kH16Kc columns, double-buffered: the weights pass through registers
// (converted once per CTA and stored as fp32 rows), the hidden states arrive by asynchronous copies.
// Thread l of half h of warp w holds lane l of 8 rows (8 (w % 8) + r) x 8 positions
// (16 (w / 8) + 2p + h): 16 loaded values per 64 FMAs, the ratio at which loads into registers and
// the FMA pipe run at the same rate. Rows are padded to kH16Kc + 16 floats, so the two halves' position
// rows (adjacent) fall in opposite halves of the banks and the shared row loads broadcast.
constexpr int kH16Rows = 64, kH16Pos = 32, kH16Kc = 128, kH16Stride = kH16Kc + 16, kH16Threads = 512;
constexpr size_t kH16Smem = (size_t)2 * (kH16Rows + kH16Pos) * kH16Stride * 4;

template <typename WT>
__global__ void __launch_bounds__(kH16Threads, 1) k_seq_dot16_gemm(const WT* w, const float* bias, int rows, int d,
                                                                    const float* x, int T, float* y, int ldy) {
  pdl_wait();
  extern __shared__ __align__(16) float sm[];
  float* sw = sm;                                // [2][kH16Rows][kH16Stride]
  float* sx = sm + 2 * kH16Rows * kH16Stride;    // [2][kH16Pos][kH16Stride]
  const int tid = threadIdx.x, r0 = blockIdx.y * kH16Rows, p0 = blockIdx.x * kH16Pos;
  const int nk = (d + kH16Kc - 1) / kH16Kc;
  // staging: thread t copies halves 8 (t % 16) .. + 8 of rows t / 16 and t / 16 + 32, and floats
  // 4 (t % 16) .. + 4 and + 64 .. of position t / 16, of each stage
  const int sr = tid >> 4, sc = (tid & 15) * 8, xc = (tid & 15) * 4;
  const bool ok0 = r0 + sr < rows, ok1 = r0 + sr + 32 < rows, okx = p0 + sr < T;
  const WT* w0 = w + (size_t)(ok0 ? r0 + sr : 0) * d;
  const WT* w1 = w + (size_t)(ok1 ? r0 + sr + 32 : 0) * d;
  const float* xs = x + (size_t)(okx ? p0 + sr : 0) * d;
  int4 wv[2];
  auto load_w = [&](int kc, int buf) {
    const int c = kc * kH16Kc + sc;  // d is a multiple of 16: an 8-weight piece is whole or outside
    if constexpr (std::is_same<WT, float>::value) {  // fp32 rows: straight into the stage
      float* dst = sw + (buf * kH16Rows + sr) * kH16Stride + sc;
      const float* src0 = (const float*)w0 + c, *src1 = (const float*)w1 + c;
      cp16(dst, ok0 && c < d ? src0 : (const float*)w, ok0 && c < d);
      cp16(dst + 4, ok0 && c < d ? src0 + 4 : (const float*)w, ok0 && c < d);
      cp16(dst + 32 * kH16Stride, ok1 && c < d ? src1 : (const float*)w, ok1 && c < d);
      cp16(dst + 32 * kH16Stride + 4, ok1 && c < d ? src1 + 4 : (const float*)w, ok1 && c < d);
    } else {  // f16 rows: through registers, converted by store_w
      wv[0] = ok0 && c < d ? ldg_stream((const int4*)w0 + c / 8) : make_int4(0, 0, 0, 0);
      wv[1] = ok1 && c < d ? ldg_stream((const int4*)w1 + c / 8) : make_int4(0, 0, 0, 0);
    }
  };
  auto store_w = [&](int buf) {
    if constexpr (!std::is_same<WT, float>::value) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const __half2* h2 = (const __half2*)&wv[h];
        const float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]), f2 = __half22float2(h2[2]),
                     f3 = __half22float2(h2[3]);
        float* dst = sw + (buf * kH16Rows + sr + 32 * h) * kH16Stride + sc;
        *(float4*)dst = make_float4(f0.x, f0.y, f1.x, f1.y);
        *(float4*)(dst + 4) = make_float4(f2.x, f2.y, f3.x, f3.y);
      }
    }
  };
  auto load_x = [&](int kc, int buf) {
    float* dst = sx + (buf * kH16Pos + sr) * kH16Stride + xc;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = kc * kH16Kc + xc + 64 * h;
      const bool ok = okx && c < d;
      cp16(dst + 64 * h, xs + (ok ? c : 0), ok);
    }
  };
  load_w(0, 0);
  load_x(0, 0);
  cp_commit();
  store_w(0);
  const int lane = tid & 31, warp = tid >> 5, l = lane & 15, hh = lane >> 4;
  const int tr = (warp & 7) * 8, tp = (warp >> 3) * 16 + hh;
  float2 acc[8][4];  // [row][position pair (2j, 2j + 1)], lane l
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[r][j] = make_float2(0.0f, 0.0f);
  for (int kc = 0; kc < nk; ++kc) {
    const int buf = kc & 1;
    cp_wait<0>();
    __syncthreads();  // stage kc is in place; every warp is done with stage kc - 1's buffers
    if (kc + 1 < nk) {
      load_w(kc + 1, buf ^ 1);
      load_x(kc + 1, buf ^ 1);
      cp_commit();
    }
    const float* qp = sw + (buf * kH16Rows + tr) * kH16Stride + l;
    const float* kp = sx + (buf * kH16Pos + tp) * kH16Stride + l;
    const int nc = min(kH16Kc, d - kc * kH16Kc) / 16;
#pragma unroll 2
    for (int c = 0; c < nc; ++c) {
      float wr[8], xp[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) wr[r] = qp[r * kH16Stride + 16 * c];
#pragma unroll
      for (int p = 0; p < 8; ++p) xp[p] = kp[2 * p * kH16Stride + 16 * c];
#pragma unroll
      for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          acc[r][j] = __ffma2_rn(make_float2(wr[r], wr[r]), make_float2(xp[2 * j], xp[2 * j + 1]), acc[r][j]);
    }
    if (kc + 1 < nk) store_w(buf ^ 1);
  }
  float v[64];  // sum o = 8 row + position
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int j = 0; j < 4; ++j) v[8 * r + 2 * j] = acc[r][j].x, v[8 * r + 2 * j + 1] = acc[r][j].y;
  half_reduce16(v, l);
  const int row = r0 + tr + (l >> 1);  // sums 4l .. 4l + 3: row l / 2, positions 4 (l % 2) + i
  if (row < rows) {
    const float b = bias ? bias[row] : 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int p = p0 + tp + 2 * (4 * (l & 1) + i);
      if (p < T) y[(size_t)p * ldy + row] = bias ? add(v[i], b) : v[i];
    }
  }
}

// Tiled scores, dot512 (model.rs:344-353) of each query row with each key of the tile: kAttnTQ
// positions x G heads of kv group blockIdx.z against kScKC keys, both staged in shared memory, each
// key row read once per tile. Thread l of half h of a warp holds dot512's lane l of 8 rows x 8 keys
// (keys 16 kb + 2k + h), so 16 loaded values feed 64 FMAs; the halving reduction is the half-warp
// reduce-scatter. Only keys in a row's window [lo, pos] are written. Rows are padded to hd + 16 floats: the
// two halves' key rows (adjacent) fall in opposite halves of the banks and the query rows broadcast.
template <int G>
__global__ void __launch_bounds__(256, 2) k_seq_scores_tile8(AttnArgs A0, const float* qn, int L, uint32_t pos0,
                                                             size_t kv_stride, uint32_t pbase, float* scores,
                                                             int sstride) {
  pdl_wait();
  extern __shared__ __align__(16) float sm[];
  constexpr int R = kAttnTQ * G;  // a multiple of 8
  const int tps = (L + kAttnTQ - 1) / kAttnTQ, sq_i = blockIdx.x / tps;
  const AttnArgs A = seq_kv(A0, sq_i, kv_stride);
  const int hd = A.hd, g = blockIdx.z, rs = hd + 16;
  const int t0 = (blockIdx.x % tps) * kAttnTQ, tn = min(kAttnTQ, L - t0);  // positions inside the sequence
  qn += (size_t)sq_i * L * A.nh * hd;                                        // this sequence's rows
  scores += (size_t)sq_i * L * A.nh * sstride;
  const uint32_t p0 = pbase + blockIdx.y * kScKC;
  const uint32_t need_lo = window_lo(pos0 + t0, A.window), need_hi = pos0 + t0 + tn - 1;
  if (p0 > need_hi || p0 + kScKC <= need_lo) return;
  float* sq = sm;           // [R][hd + 16]
  float* sk = sm + R * rs;  // [kScKC][hd + 16]
  const int rw = A.nkv * hd, h4 = hd / 4;
  const int e = (int)threadIdx.x % h4, step = (int)blockDim.x / h4;
  const bool whole = (int)blockDim.x % h4 == 0;
  for (int i = threadIdx.x, row = (int)threadIdx.x / h4; i < R * h4; i += blockDim.x, row += step) {
    const int rr = whole ? row : i / h4, ee = whole ? e : i % h4, tt = rr / G, h = rr % G;
    const bool ok = tt < tn;
    cp16(sq + rr * rs + ee * 4, qn + (ok ? ((size_t)(t0 + tt) * A.nh + g * G + h) * hd + ee * 4 : 0), ok);
  }
  for (int i = threadIdx.x, pr = (int)threadIdx.x / h4; i < kScKC * h4; i += blockDim.x, pr += step) {
    const int rr = whole ? pr : i / h4, ee = whole ? e : i % h4;
    const uint32_t p = p0 + rr;
    const bool ok = p <= need_hi;
    cp16(sk + rr * rs + ee * 4, A.kcache + (ok ? (size_t)p * rw + g * hd + ee * 4 : 0), ok);
  }
  cp_commit();
  cp_wait<0>();
  __syncthreads();
  const int lane = threadIdx.x & 31, l = lane & 15, hh = lane >> 4;
  constexpr int KB = kScKC / 16, NWT = (R / 8) * KB;  // warp tiles of 8 rows x 16 keys
  for (int wt = (int)threadIdx.x >> 5; wt < NWT; wt += (int)blockDim.x >> 5) {
    const int r0 = (wt / KB) * 8, k0 = (wt % KB) * 16 + hh;  // keys k0 + 2k
    const float* qp = sq + r0 * rs + l;
    const float* kp = sk + k0 * rs + l;
    float2 acc[8][4];  // [row][key pair (2j, 2j + 1)], lane l
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[r][j] = make_float2(0.0f, 0.0f);
#pragma unroll 2
    for (int c = 0; c < hd / 16; ++c) {
      float qv[8], kv[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) qv[r] = qp[r * rs + 16 * c];
#pragma unroll
      for (int k = 0; k < 8; ++k) kv[k] = kp[2 * k * rs + 16 * c];
#pragma unroll
      for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          acc[r][j] = __ffma2_rn(make_float2(qv[r], qv[r]), make_float2(kv[2 * j], kv[2 * j + 1]), acc[r][j]);
    }
    float v[64];  // sum o = 8 row + key
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) v[8 * r + 2 * j] = acc[r][j].x, v[8 * r + 2 * j + 1] = acc[r][j].y;
    half_reduce16(v, l);
    const int row = r0 + (l >> 1), tt = row / G, h = row % G;  // sums 4l .. 4l + 3: row l / 2, keys 4 (l % 2) + i
    if (tt < tn) {
      const uint32_t pos = pos0 + t0 + tt, lo = window_lo(pos, A.window);
      float* out = scores + ((size_t)(t0 + tt) * A.nh + g * G + h) * sstride;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t p = p0 + k0 + 2 * (4 * (l & 1) + i);
        if (p >= lo && p <= pos) out[p - lo] = v[i];
      }
    }
  }
}

bool seq_gemm_supported(const MatView& w) {
  if (w.bits != 8 && w.bits != 4) return false;
  if (w.cols % 32) return false;
  if (!w.scale_f32 && (w.cols / 32) % 2) return false;  // f16 scales are staged in 4-byte pieces
  return true;
}

// Tile choice: estimated time = waves x time of one wave, with 2 resident CTAs per SM for 8 positions
// per thread and 3 for 4 (register-bound occupancy); a wave of 4-position tiles (48 positions per SM)
// takes about 0.78 of a wave of 8-position tiles (64 per SM), as measured on B200.
// Positions per thread (RN; a CTA takes 32 rows x 4 RN positions) for a projection of `rows` rows over
// T positions: the fewest estimated wave-times, a wave of RN = 8 (2 CTAs per SM) taking 8 units and a
// wave of RN = 4 or 6 (3 CTAs per SM) 1.55 units per position of RN (measured: the three shapes give
// the same throughput per SM when their last wave is full).
// With `concurrent` products running at once (a chunk's parts on their streams), the other parts
// fill the SMs a small grid leaves idle, so the most efficient tile per position (RN = 8) wins:
// measured 102.5k against 101.7k tokens/s for the cost model's choice at 4 parts of 128 positions.
static int gemm_rn(int rows, int T, int sms, int concurrent) {
  static const int forced = [] {  // tuning override: GEM_GEMM_RN=4, 6 or 8
    const char* e = std::getenv("GEM_GEMM_RN");
    return e ? std::atoi(e) : 0;
  }();
  if (forced == 4 || forced == 6 || forced == 8) return forced;
  if (concurrent > 1) return 8;
  const long long rt = (rows + kGemmBM - 1) / kGemmBM;
  auto cost = [&](int rn, int occ, double unit) {
    const long long ctas = (long long)((T + 4 * rn - 1) / (4 * rn)) * rt;
    return (double)((ctas + (long long)occ * sms - 1) / ((long long)occ * sms)) * unit * rn;
  };
  const double c8 = cost(8, 2, 1.0), c6 = cost(6, 3, 1.55), c4 = cost(4, 3, 1.55);
  if (c8 <= c6 && c8 <= c4) return 8;
  return c6 < c4 ? 6 : 4;
}

void launch_seq_gemm(const MatView& w, const int8_t* aq, const float* as, int T, float* y, int ldy, int sms,
                     cudaStream_t st, int concurrent) {
  const int rn = gemm_rn(w.rows, T, sms, concurrent);
#define F2(B, S, RNV)                                                                                            \
  do {                                                                                                          \
    using GT = GemmTile<B, S, RNV>;                                                                             \
    static bool init = false;                                                                                   \
    if (!init) {                                                                                                \
      cudaFuncSetAttribute(k_seq_gemm<B, S, RNV>, cudaFuncAttributeMaxDynamicSharedMemorySize, GT::SMEM);       \
      init = true;                                                                                              \
    }                                                                                                           \
    dim3 grid((T + GT::BN - 1) / GT::BN, (w.rows + kGemmBM - 1) / kGemmBM);                                    \
    launch_k(k_seq_gemm<B, S, RNV>, dim3(grid), dim3(kGemmThreads), GT::SMEM, st, w, aq, as, T, y, ldy);                          \
  } while (0)
#define F(B, S)                 \
  do {                          \
    if (rn == 8) F2(B, S, 8);     \
    else if (rn == 6) F2(B, S, 6); \
    else F2(B, S, 4);            \
  } while (0)
  GEM_DISPATCH_Q(w.bits, w.scale_f32, F);
#undef F
#undef F2
}

bool seq_head_f16_supported(const MatView& w) {
  return w.bits == 16 && w.cols > 0 && w.cols % 16 == 0 && (uintptr_t)w.q % 16 == 0 &&
         (w.rows + kH16Rows - 1) / kH16Rows <= 65535;
}

template <typename WT>
static void launch_dot16_gemm(const WT* w, const float* bias, int rows, int d, const float* x, int T, float* y, int ldy,
                              cudaStream_t st) {
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(k_seq_dot16_gemm<WT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kH16Smem);
    init = true;
  }
  const dim3 grid((T + kH16Pos - 1) / kH16Pos, (rows + kH16Rows - 1) / kH16Rows);  // position tiles fastest
  launch_k(k_seq_dot16_gemm<WT>, grid, dim3(kH16Threads), kH16Smem, st, w, bias, rows, d, x, T, y, ldy);
}

void launch_seq_head_f16(const MatView& w, const float* x, int T, float* y, int ldy, cudaStream_t st) {
  launch_dot16_gemm((const __half*)w.q, nullptr, w.rows, w.cols, x, T, y, ldy, st);
}

void launch_seq_attn(const AttnArgs& A, const float* qkv, int qkv_ld, int L, int nseq, uint32_t pos0, size_t kv_stride,
                     float* qn, float* scores, int sstride, int threads, float* part, int8_t* aq, float* as,
                     cudaStream_t st, cudaEvent_t kv_written) {
  const int G = A.nh / A.nkv, T = L * nseq;
  if (G < 1 || G > 8) return;  // rejected by the caller before any launch
  launch_k(k_seq_attn_prep, dim3(dim3(T, A.nkv)), dim3(256), (size_t)(G + 2) * A.hd * 4, st, A, qkv, qkv_ld, L, pos0, kv_stride, qn);
  if (kv_written) cudaEventRecord(kv_written, st);  // the chunk's K/V rows are in the cache
  const uint32_t pbase = window_lo(pos0, A.window);
  const int nchunk = (int)((pos0 + L - pbase + kScKC - 1) / kScKC);
  const int tps = (L + kAttnTQ - 1) / kAttnTQ;
  const dim3 sgrid(tps * nseq, nchunk, A.nkv), pgrid(tps * nseq, threads);
  const size_t ssm8 = ((size_t)kAttnTQ * G + kScKC) * (A.hd + 16) * 4;
  const size_t psm = ((size_t)kPvRows * A.hd + (size_t)kAttnTQ * G * kPvRows) * 4;
  const int pth = A.hd / 2;
#define F(GG)                                                                                                        \
  do {                                                                                                               \
    static bool init = false;                                                                                        \
    if (!init) {                                                                                                     \
      cudaFuncSetAttribute(k_seq_scores_tile8<GG>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);        \
      cudaFuncSetAttribute(k_seq_pv_tile<GG>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);             \
      cudaFuncSetAttribute(k_seq_pv_tile8<GG>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);            \
      init = true;                                                                                                   \
    }                                                                                                                \
    launch_k(k_seq_scores_tile8<GG>, dim3(sgrid), dim3(256), ssm8, st, A, qn, L, pos0, kv_stride, pbase, scores, sstride);          \
  } while (0)
  switch (G) {
    case 1: F(1); break;
    case 2: F(2); break;
    case 3: F(3); break;
    case 4: F(4); break;
    case 5: F(5); break;
    case 6: F(6); break;
    case 7: F(7); break;
    default: F(8); break;
  }
#undef F
  {
    static bool init = false;
    if (!init) {
      cudaFuncSetAttribute(k_seq_softmax, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      init = true;
    }
    const size_t es = (((size_t)sstride + 3) & ~(size_t)3) + 16;  // the kernel's row stride
    const int nw = (int)std::max<size_t>(1, std::min<size_t>(8, (size_t)(200 * 1024) / (es * 4)));
    launch_k(k_seq_softmax, dim3((T * A.nh + nw - 1) / nw), dim3(nw * 32), (size_t)nw * es * 4, st, A, T, L, pos0, scores, sstride);
  }
#define P(GG)                                                                                                    \
  do {                                                                                                           \
    if (A.hd == 256)                                                                                             \
      launch_k(k_seq_pv_tile8<GG>, dim3(pgrid), dim3(32 * GG), psm, st, A, L, pos0, kv_stride, scores, sstride,  \
               threads, part);                                                                                    \
    else                                                                                                         \
      launch_k(k_seq_pv_tile<GG>, dim3(pgrid), dim3(pth), psm, st, A, L, pos0, kv_stride, scores, sstride, threads, \
               part);                                                                                             \
  } while (0)
  switch (G) {
    case 1: P(1); break;
    case 2: P(2); break;
    case 3: P(3); break;
    case 4: P(4); break;
    case 5: P(5); break;
    case 6: P(6); break;
    case 7: P(7); break;
    default: P(8); break;
  }
#undef P
  launch_k(k_seq_pv_combine, dim3(dim3(T, A.nh)), dim3(A.hd), 0, st, A, part, threads, aq, as);
}

// Token ids and targets of a chunk: rows [seq][pos] read toks[seq * stride + c0 + pos] and the next id.
__global__ void k_seq_gather_tokens(const uint32_t* toks, size_t stride, int L, int c0, int T, uint32_t* tin,
                                    uint32_t* tgt) {
  pdl_wait();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const size_t i = (size_t)(t / L) * stride + c0 + t % L;
  tin[t] = toks[i];
  tgt[t] = toks[i + 1];
}

void launch_seq_gather_tokens(const uint32_t* toks, size_t stride, int L, int c0, int T, uint32_t* tin, uint32_t* tgt,
                              cudaStream_t st) {
  launch_k(k_seq_gather_tokens, dim3((T + 255) / 256), dim3(256), 0, st, toks, stride, L, c0, T, tin, tgt);
}

void launch_seq_glu_quant(const float* gu, int ff, int T, int silu, int8_t* aq, float* as, int sms, cudaStream_t st) {
  const long long tasks = (long long)T * (ff / 32);
  const int blocks = (int)std::min<long long>((tasks + 7) / 8, 1LL << 30);
  launch_k(k_seq_glu_quant, dim3(blocks), dim3(256), 0, st, gu, ff, T, silu, aq, as);
}

void launch_seq_class_logits(const float* A, const float* b, int k, const float* h, int d, int T, float* cl,
                             cudaStream_t st) {
  launch_dot16_gemm(A, b, k, d, h, T, cl, k, st);
}

void launch_seq_logit_reduce(const float* logits, int V, int T, const uint32_t* targets, const uint32_t* row_of,
                             const uint32_t* row_tok, float* lp, uint32_t* am, int* err, cudaStream_t st) {
  launch_k(k_seq_logit_reduce, dim3(T), dim3(1024), 0, st, logits, V, targets, row_of, row_tok, lp, am, err);
}

}  // namespace gem

namespace gem {
void launch_seq_logit_partials(const float* logits, int V, uint32_t row0, int T, const uint32_t* targets, uint32_t vocab,
                               const uint32_t* row_of, const uint32_t* row_tok, float* out, int* err, cudaStream_t st) {
  launch_k(k_seq_logit_partials, dim3(T), dim3(1024), 0, st, logits, V, row0, targets, vocab, row_of, row_tok, out, err);
}
void launch_seq_logit_combine(const float* parts, int nranks, int T, float* lp, uint32_t* am, cudaStream_t st) {
  launch_k(k_seq_logit_combine, dim3((T + 127) / 128), dim3(128), 0, st, parts, nranks, T, lp, am);
}
}  // namespace gem
