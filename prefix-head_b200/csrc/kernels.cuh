// Kernel argument structs and launchers shared by the host runtime (runtime.cpp) and the kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#ifdef __CUDACC__
#include "common.cuh"
#endif

namespace gem {

// Device error word: kernels that give up a bounded wait or meet an out-of-range caller id record a
// code here; the host reads and clears it after synchronising.
enum : int { ERR_NONE = 0, ERR_TIMEOUT = 1, ERR_RANGE = 2 };

// A weight matrix on the device (crates/gem/src/q8.rs:9-15, repacked): bits 8 = int8 plane
// [rows][cols]; bits 4 = GGUF Q4_0 nibble bytes [rows][cols/2]; bits 16 = f16 [rows][cols]. Scales
// (bits 8/4) are one per 32 weights, [rows][cols/32], f16 as stored in the GGUF or f32 after
// requantization (to_q8 / to_q4 produce f32 scales).
struct MatView {
  const void* q = nullptr;
  const void* s = nullptr;
  int rows = 0, cols = 0, bits = 8, scale_f32 = 0;
};

// A Q8_0 / Q4_0 matrix tiled for the tensor-core product (tc_gemm.cu): per (row tile of 128, 32-block)
// one 8704-byte chunk, the 128 x 32 weights as f16 in the MMA's K-major core-matrix order
// ([8-row group][8-column group][8][8]) followed by the 128 scales as f32; rows past the last are zero.
struct TcMat {
  const unsigned char* tiles = nullptr;
  int rows = 0, cols = 0;
};
bool tc_gemm_supported(const MatView& w);
size_t tc_tiled_bytes(const MatView& w);
// Builds the tiled copy of w into buf (tc_tiled_bytes), asynchronously on st.
void tc_tile(const MatView& w, void* buf, TcMat* out, cudaStream_t st);
// Y[t][r] (row stride ldy) = the exact row dot of W[r] and the quantized activation t (aq [T][cols],
// as [T][cols/32]), bit-identical to launch_seq_gemm; err receives ERR_TIMEOUT if a bounded wait
// gives up.
void launch_tc_gemm(const TcMat& W, const int8_t* aq, const float* as, int T, float* y, int ldy, int* err, int sms,
                    cudaStream_t st);

#ifdef __CUDACC__
// Mat::weight (q8.rs:112-126): the dequantized weight at row r, column j -- the bit-exact dequant
// definition (q * s in one fp32 rounding; nibble - 8 for Q4_0; the f16 value for F16).
template <int BITS, typename ST>
__device__ __forceinline__ float weight_at(const MatView& w, size_t r, int j) {  // q8.rs:112-126
  if constexpr (BITS == 16) {
    return __half2float(((const __half*)w.q)[r * w.cols + j]);
  } else if constexpr (BITS == 8) {
    float s = ld_scale((const ST*)w.s, (r * w.cols + j) / 32);
    return mul((float)((const int8_t*)w.q)[r * w.cols + j], s);
  } else {
    float s = ld_scale((const ST*)w.s, (r * w.cols + j) / 32);
    int blk = j / 32, k = j % 32;
    uint8_t byte = ((const uint8_t*)w.q)[r * w.cols / 2 + blk * 16 + (k % 16)];
    int nib = k < 16 ? (byte & 15) : (byte >> 4);
    return mul((float)(nib - 8), s);
  }
}
#endif

// Token, position, target and output slot of the step being run; written by k_begin_step (scoring
// loop) or by a host copy (single-token calls).
struct StepCur {
  uint32_t tok, pos, target, slot;
};

struct AttnArgs {
  const float* qkv;          // [nh*hd | nkv*hd | nkv*hd] raw projections
  const float* bqkv;         // biases in the same layout (qwen2) or null
  const float* q_norm;       // hd or null
  const float* k_norm;       // hd or null
  const float* rope_sin;     // [ctx][hd/2] for this layer's base
  const float* rope_cos;
  float* kcache;             // [ctx][nkv*hd]
  float* vcache;
  float* part;               // [nkv][nsplit][G][hd+2]
  float* att_out;            // nh*hd (optional, for tests)
  const StepCur* cur;
  int nh, nkv, hd, window, chunk, nsplit;
  float eps, qscale;
};

struct HeadArgs {
  MatView w;                 // output matrix (rows in token order, or class-permuted)
  const uint32_t* row_of;    // token -> row (null = identity)
  const uint32_t* row_tok;   // row -> token (null = identity)
  const int8_t* aq;          // [batch][d] quantized hidden states
  const float* as;           // [batch][d/32]
  const float* h;            // [batch][d] fp32 hidden states (F16 heads)
  const uint32_t* targets;   // [batch] or null (then cur->target)
  const StepCur* cur;
  float* part;               // [batch][parts] x float4
  float* tlogit;             // [batch]
  float* lp_out;             // indexed by batch item, or cur->slot
  uint32_t* am_out;
  int* err;                  // device error word
  int* cnt;                  // [batch] streamed-head CTAs done (zero between launches; the last CTA
                             // merges the partials), or null for the separate merge kernel
};

#ifdef __CUDACC__
// Log-sum-exp, argmax and log-prob of batch item bi from `nparts` per-CTA partials (max, sum of
// exp, best logit, its token), merged by the calling CTA in a fixed order (a thread per partial, then
// block_lse_best), so the result does not depend on which CTA runs it.
__device__ inline void head_merge(const HeadArgs& H, int bi, int nparts) {
  __shared__ float red_m[32], red_s[32], red_v[32];
  __shared__ uint32_t red_t[32];
  Lse L{-INFINITY, 0.0f};
  Best B{-INFINITY, 0xffffffffu};
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
    const float4 p = __ldcg((const float4*)H.part + (size_t)bi * nparts + i);
    L = lse_merge(L, Lse{p.x, p.y});
    B = best_merge(B, Best{p.z, __float_as_uint(p.w)});
  }
  block_lse_best(L, B, red_m, red_s, red_v, red_t);
  if (threadIdx.x == 0) {
    const float lse = L.m + logf(L.s);
    const uint32_t slot = H.targets ? (uint32_t)bi : H.cur->slot;
    if (H.lp_out) H.lp_out[slot] = __ldcg(H.tlogit + bi) - lse;
    if (H.am_out) H.am_out[slot] = B.tok;
  }
}
#endif

struct TwoLevelArgs {
  MatView w;                 // class-permuted output matrix: class c = rows [c*per, c*per + n_c)
  const float* A;            // [k][d] fp32
  const float* b;            // [k]
  const uint32_t* cls_of;    // token -> class
  const uint32_t* pos_of;    // token -> position inside its class
  const uint32_t* order;     // row -> token
  const int8_t* aq;
  const float* as;
  const float* h;
  const uint32_t* targets;
  const StepCur* cur;
  float* cl;                 // [batch][k]
  const float* cl_in;        // [batch][k] class logits already computed (k_tl_fused reads them), or null
  float* inner;              // [batch][per]
  float* lp_out;
  uint32_t* am_out;
  int* err;
  int k, per, class_ctas, vocab;
};

void launch_embed(const MatView& head, const uint32_t* row_of, const StepCur* cur, float scale, float* x, cudaStream_t st);
void launch_dequant_rows(const MatView& w, size_t r0, int nrows, float* out, cudaStream_t st);
void launch_residual_norm_quant(float* x, const float* delta, const float* w_post, const float* w_pre, float eps, int d,
                                int8_t* aq, float* as, float* xn_out, cudaStream_t st);
void launch_quantize(const float* x, int n, int8_t* aq, float* as, cudaStream_t st);
void launch_gemv(const MatView& w, const int8_t* aq, const float* as, const float* x, float* y, int sms, cudaStream_t st);
void launch_attn(const AttnArgs& A, int8_t* aq, float* as, cudaStream_t st);
void launch_glu_quant(const float* gu, int ff, int silu, int8_t* aq, float* as, float* gout, cudaStream_t st);
void launch_begin_step(const uint32_t* toks, uint32_t* step, uint32_t base_pos, uint32_t vocab, StepCur* cur, int* err,
                       cudaStream_t st);
void launch_end_step(uint32_t* step, cudaStream_t st);
int head_full_parts(int sms);
// Full head streamed through shared memory for Q8_0 output matrices with f16 scales: the matrix's GEMV
// copy ([16-row group][block][row][32 B] quants, [group][block][16] scales) and the launcher (batch items
// in blockIdx.y, partials merged as for launch_head_full_exact).
bool head_bulk_supported(const MatView& w);
size_t head_bulk_bytes(const MatView& w);
void launch_head_bulk_layout(const MatView& w, unsigned char* wq, __half* ws, cudaStream_t st);
void launch_head_full_bulk(const HeadArgs& H, const unsigned char* wq, const __half* ws, int batch, int sms, cudaStream_t st);
void launch_head_full(const HeadArgs& H, int batch, int sms, cudaStream_t st);
void launch_head_twolevel(const TwoLevelArgs& T, int batch, int sms, cudaStream_t st);
void launch_head_full_merge(const HeadArgs& H, int batch, int parts, cudaStream_t st);
void launch_tl_select(const TwoLevelArgs& T, int batch, uint32_t* top_of, cudaStream_t st);
void launch_tl_argmax(const TwoLevelArgs& T, int batch, const uint32_t* top_of, const float* top_inner, cudaStream_t st);

// Exact numerics (kernels_exact.cu): bit-identical to the reference's AVX-512 path.
void launch_gemv_exact(const MatView& w, const int8_t* aq, const float* as, const float* x, float* y, int sms,
                       cudaStream_t st);
void launch_residual_norm_quant_exact(float* x, const float* delta, const float* w_post, const float* w_pre, float eps,
                                      int d, int8_t* aq, float* as, float* xn_out, cudaStream_t st);
void launch_attn_exact(const AttnArgs& A, float* qn, float* scores, int sstride, int threads, int8_t* aq, float* as,
                       int sms, cudaStream_t st);
void launch_head_full_exact(const HeadArgs& H, int batch, int sms, cudaStream_t st);
void launch_tl_stage1_exact(const TwoLevelArgs& T, int batch, int class_ctas, int block_ctas, cudaStream_t st);
void launch_tl_top_exact(const TwoLevelArgs& T, int batch, const uint32_t* top_of, float* top_inner, cudaStream_t st);
// The exact two-level head in one launch: P = tl_parts(...) CTAs per hidden state (ceil(per / 32) when
// T.cl_in gives the class logits, [batch][k]), cnt[batch] zero between launches,
// part[batch][tl_part_floats(k, per)] floats of per-CTA partials; false (nothing launched) when its
// staging area does not fit in shared memory.
int tl_parts(int k, int per, int batch, int sms);
int tl_part_floats(int k, int per);
bool launch_tl_fused(const TwoLevelArgs& T, int batch, int sms, int* cnt, float* part, cudaStream_t st);

// Sequence-parallel scoring (seq.cu): every position of a chunk through one layer at a time, with the
// exact per-position arithmetic above. Activations are [T][n] row-major, scales [T][n/32].
// row_of (token -> row; null: token order) for an output matrix held in class order.
void launch_seq_embed(const MatView& E, const uint32_t* row_of, const uint32_t* toks, int T, int vocab, float scale,
                      float* x, int* err, cudaStream_t st);
void launch_seq_norm(float* x, const float* delta, const float* w_post, const float* w_pre, float eps, int d, int T,
                     int8_t* aq, float* as, float* xn_out, cudaStream_t st);
bool seq_gemm_supported(const MatView& w);
// `concurrent`: how many such products run at once on separate streams (tile choice).
void launch_seq_gemm(const MatView& w, const int8_t* aq, const float* as, int T, float* y, int ldy, int sms,
                     cudaStream_t st, int concurrent = 1);
// Full-head logits y[p][r] (p < T, row stride ldy) of an F16 output matrix against fp32 hidden states
// x [T][cols], each the exact dot16; needs cols a multiple of 16 and a 16-byte aligned matrix.
bool seq_head_f16_supported(const MatView& w);
void launch_seq_head_f16(const MatView& w, const float* x, int T, float* y, int ldy, cudaStream_t st);
// `kv_written` (optional) is recorded on `st` once the chunk's K/V rows are in the cache.
void launch_seq_attn(const AttnArgs& A, const float* qkv, int qkv_ld, int L, int nseq, uint32_t pos0, size_t kv_stride,
                     float* qn, float* scores, int sstride, int threads, float* part, int8_t* aq, float* as,
                     cudaStream_t st, cudaEvent_t kv_written = nullptr);
void launch_seq_logit_partials(const float* logits, int V, uint32_t row0, int T, const uint32_t* targets, uint32_t vocab,
                               const uint32_t* row_of, const uint32_t* row_tok, float* out, int* err, cudaStream_t st);
void launch_seq_logit_combine(const float* parts, int nranks, int T, float* lp, uint32_t* am, cudaStream_t st);
// Generation-side heads (decode.cu).
void launch_greedy_rank(const float* cl, int k, int top, float min_conf, int batch, uint32_t* sel, int* fallback,
                        cudaStream_t st);
void launch_greedy_rowlist(const uint32_t* sel, int top, int per, uint32_t total_rows, const uint32_t* always, int n_always,
                           int batch, uint32_t* rows, cudaStream_t st);
void launch_rows_exact(const MatView& w, const int8_t* aq, const float* as, const float* h, const uint32_t* rows, int nrows,
                       int batch, float* out, cudaStream_t st);
void launch_greedy_pick(const float* z, const uint32_t* rows, int top, int per, int n_always, const int* fallback,
                        const uint32_t* fb_row, const uint32_t* order, int batch, uint32_t* tok, cudaStream_t st);
void launch_sample_class(const float* cl, int k, float temp, unsigned long long* rng, uint32_t* cls, cudaStream_t st);
void launch_sample_member(const float* inner, int per, uint32_t total_rows, const uint32_t* cls, float temp,
                          unsigned long long* rng, const uint32_t* order, uint32_t* tok, cudaStream_t st);
void launch_seq_gather_tokens(const uint32_t* toks, size_t stride, int L, int c0, int T, uint32_t* tin, uint32_t* tgt,
                              cudaStream_t st);
void launch_seq_glu_quant(const float* gu, int ff, int T, int silu, int8_t* aq, float* as, int sms, cudaStream_t st);
void launch_seq_class_logits(const float* A, const float* b, int k, const float* h, int d, int T, float* cl,
                             cudaStream_t st);
void launch_seq_logit_reduce(const float* logits, int V, int T, const uint32_t* targets, const uint32_t* row_of,
                             const uint32_t* row_tok, float* lp, uint32_t* am, int* err, cudaStream_t st);
// Output-matrix rows gathered into another matrix of the same shape and format: dst row i = src row
// src_row[i] (the class-ordered head, permute_head, model.rs:242-249); y[i] = x[idx[i]].
void launch_gather_rows(const MatView& src, const uint32_t* src_row, const MatView& dst, cudaStream_t st);
void launch_gather_f32(const float* x, const uint32_t* idx, int n, float* y, cudaStream_t st);

#ifdef __CUDACC__
// Launches `k` with programmatic stream serialization (see pdl_wait); GEM_PDL=0 turns it off.
bool pdl_on();
template <typename... KArgs, typename... Args>
inline void launch_k(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  if (!pdl_on()) {
    k<<<grid, block, smem, st>>>(args...);
    return;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid, cfg.blockDim = block, cfg.dynamicSmemBytes = smem, cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at, cfg.numAttrs = 1;
  // a refused launch is retried as a plain one, which records its error for cudaGetLastError
  if (cudaLaunchKernelEx(&cfg, k, args...) != cudaSuccess) k<<<grid, block, smem, st>>>(args...);
}
#endif

}  // namespace gem
