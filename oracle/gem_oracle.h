/* TEST INFRASTRUCTURE ONLY — the oracle. A CPU restatement of the reference's per-token scoring path
 * (prefix-head crates/gem: q8.rs, model.rs, main.rs, gguf.rs, pool.rs; crates/nn/src/fast.rs exp/tanh).
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this library, and only as
 * the checker or the timed CPU baseline; the product library never links or calls it.
 *
 * Parity pins (what anchors this restatement to the reference):
 *   - Q8_0 / Q4_0 / F16 block layouts and the GGUF container: checked against the third-party gguf-py
 *     package (llama.cpp's own reader/writer, version 0.19.0) on seeded tensors.
 *   - exp_fast / tanh_fast / logsumexp: the reference's own accuracy tests (crates/nn/src/fast.rs:206-219)
 *     are re-run against this restatement.
 *   - The Gemma 3 forward as a whole: the reference ships no golden outputs for it (crates/gem has no
 *     tests; the data/retro golden files and the GGUF files are not in the repository), so the end-to-end
 *     forward is PARITY UNPINNED by reference goldens. It is cross-checked structurally against an
 *     independent Gemma 3 implementation (transformers' Gemma3 text model) on the same dequantized
 *     weights, within the noise of the reference's int8 activation quantization.
 *
 * All functions return 0 on success and a negative code on error (orc_last_error() has the message).
 */
#ifndef GEM_ORACLE_H
#define GEM_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_model orc_model;
typedef struct orc_mat orc_mat;

const char* orc_last_error(void);
/* "avx512", "avx2" or "scalar": what q8::detect() (q8.rs:395-408) picks on this CPU, honouring GEM_ISA. */
const char* orc_detect_isa(void);

/* Gemma::load (model.rs:154-233) + requantize(body_bits == 4, false) + requantize_head(head_bits)
 * (main.rs:205-210). isa = NULL picks orc_detect_isa(). threads = Pool size (pool.rs:35). */
orc_model* orc_open(const char* gguf_path, int ctx, int body_bits, int head_bits, int threads, const char* isa);
void orc_close(orc_model* m);
/* d, vocab, n_layers, ctx, bos (-1 when add_bos_token is false) */
int orc_info(const orc_model* m, int64_t* out5);
const char* orc_isa(const orc_model* m);

/* Gemma::forward (model.rs:286-430): writes the final-norm hidden state (d floats). */
int orc_forward(orc_model* m, uint32_t tok, uint32_t pos, float* h_out);
/* Full::run + Full::logprob (main.rs:30-37); argmax with lean.rs:36-38's rule (first maximum). */
int orc_full(orc_model* m, const float* h, uint32_t target, float* logprob, uint32_t* argmax, float* logits_out);
/* TwoLevel::load (main.rs:57-76) from prefix.order / prefix.A / prefix.b */
int orc_twolevel_load(orc_model* m, const char* prefix);
/* TwoLevel::logprob (main.rs:101-107). argmax = screening with the single most likely class
 * (lean.rs:46-76 with top = 1, no always-on rows, no fallback): the highest raw logit inside the
 * top class, returned as a token id. cl_out (k floats) / inner_out (per floats) are nullable. */
int orc_twolevel(orc_model* m, const float* h, uint32_t target, float* logprob, uint32_t* argmax,
                 float* cl_out, float* inner_t_out);
/* lean.rs:46-107 (Classes::next + next_token): greedy token by screening the `top` most likely classes
 * and the always-on rows (class-ordered row indices); below min_confidence, the full head's argmax
 * over the class-ordered rows (*fell_back = 1). */
int orc_greedy(orc_model* m, const float* h, int top, float min_confidence, const uint32_t* always, int n_always,
               uint32_t* tok, int* fell_back);
/* TwoLevel::sample (main.rs:109-141): class, then member, drawn at temperature temp with the
 * reference's xorshift64 generator (state updated in place). */
int orc_twolevel_sample(orc_model* m, const float* h, float temp, uint64_t* rng, uint32_t* tok);
/* gem bench's inner loop (main.rs:270-289): optional BOS forward, then for i < n: forward(toks[i],
 * i + off), head logprob of toks[i + 1]. head: 0 full, 1 two-level. body_s / head_s accumulate
 * wall time like tb / th. lp / am have n entries each (am nullable). */
int orc_score(orc_model* m, const uint32_t* toks, size_t n, int head, float* lp, uint32_t* am,
              double* body_s, double* head_s);

/* Kernel-level pieces, on matrices built from GGUF tensor bytes. kind: 8 Q8_0, 2 Q4_0, 1 F16. */
orc_mat* orc_mat_from_gguf(int kind, const uint8_t* raw, size_t rows, size_t cols);
void orc_mat_free(orc_mat* w);
/* to_q8 (q8.rs:129-145) or to_q4 (q8.rs:148-165); returns a new matrix */
orc_mat* orc_mat_requant(const orc_mat* w, int bits);
/* bits, rows, cols, bytes of the int8/nibble/f16 plane, number of scales */
int orc_mat_info(const orc_mat* w, int64_t* out5);
/* raw planes: q (row_bytes * rows) and s (rows * cols / 32 f32) */
int orc_mat_planes(const orc_mat* w, int8_t* q, float* s);
/* dequantized weights, Mat::row_f32 (q8.rs:167) for every row: rows * cols floats */
int orc_mat_dequant(const orc_mat* w, float* out);
/* Act::quantize(x) then matvec (q8.rs:439-461) over `threads` threads */
int orc_matvec(const orc_mat* w, const float* x, const char* isa, int threads, float* y);
/* Act::quantize (q8.rs:187-246): q (n int8), s (n / 32 floats) */
int orc_quantize(const float* x, size_t n, const char* isa, int8_t* q, float* s);
float orc_exp_fast(float x);
float orc_tanh_fast(float x);
float orc_lse(const float* v, size_t n);
float orc_f16(uint16_t h);

#ifdef __cplusplus
}
#endif
#endif
