/* gem-b200: a B200 (sm_100a) implementation of the per-token scoring path of prefix-head's `gem`
 * Gemma 3 runtime, behind a C ABI.
 *
 * The reference has no FFI layer: its boundary is gem's internal Rust API (crates/gem/src/model.rs,
 * q8.rs, main.rs). Each entry point below names the Rust function it stands in for, so a Rust host
 * can bind this header with an `extern "C"` block and keep its call sites.
 *
 * Conventions
 *   - Every function returns int: 0 (GEM_OK) or a negative gem_status; gem_last_error() returns a
 *     thread-local message for the last failure. Nothing panics, throws or aborts across the ABI.
 *   - A gem_model owns all of its device memory, one CUDA stream and its CUDA graphs. Host buffers are
 *     caller-owned and are filled before a call returns. A handle is not thread-safe (the reference's
 *     &mut self): use one handle per host thread and GPU.
 *   - Device-pointer variants (suffix _dev) take device buffers, enqueue on the model's stream and
 *     return without synchronising; gem_sync() waits for them.
 */
#ifndef GEM_B200_H
#define GEM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum gem_status {
  GEM_OK = 0,
  GEM_E_ARG = -1,      /* invalid argument (null pointer, bad size, unsupported option) */
  GEM_E_IO = -2,       /* file missing, unreadable or truncated */
  GEM_E_FORMAT = -3,   /* GGUF or class-file content the runtime does not support */
  GEM_E_CUDA = -4,     /* CUDA runtime error */
  GEM_E_NOMEM = -5,    /* device or host allocation failed */
  GEM_E_STATE = -6,    /* call out of order (e.g. a head before any forward) */
  GEM_E_RANGE = -7,    /* token id >= vocab, pos >= ctx, sequence index out of range */
  GEM_E_NCCL = -8,     /* collective setup or communication failed */
  GEM_E_TIMEOUT = -9,  /* a bounded device-side wait gave up; the kernel returned an error flag */
} gem_status;

typedef struct gem_model gem_model;

typedef struct gem_info {
  int64_t d, vocab, layers, n_heads, n_kv_heads, head_dim, ffn, ctx, window;
  int64_t bos;              /* -1 when tokenizer.ggml.add_bos_token is false */
  int64_t body_bits;        /* 8 or 4 (after requantization) */
  int64_t head_bits;        /* 8, 4 or 16 */
  int64_t classes, per;     /* two-level head: k classes of `per` rows (0 when not loaded) */
  int64_t max_seqs;         /* sequences with their own KV cache */
  int64_t body_bytes;       /* canonical (GGUF block size) bytes of the 7 projections x layers */
  int64_t head_bytes;       /* canonical bytes of the output matrix */
  int64_t device;
  int64_t kernels_per_token_full;      /* kernels one scoring step launches (-1 until first used) */
  int64_t kernels_per_token_twolevel;
} gem_info;

const char* gem_last_error(void);
int gem_version(void);

/* Gemma::load(&Gguf, ctx, tie = false) + requantize(body_bits == 4, false) + requantize_head(head_bits)
 * (crates/gem/src/model.rs:154, 268, 259; called as in crates/gem/src/main.rs:203-210). head_bits 0
 * keeps the file's type. max_seqs > 1 allocates independent KV caches for batched scoring. */
int gem_open(const char* gguf_path, int ctx, int body_bits, int head_bits, int device, int max_seqs,
             gem_model** out);
/* TwoLevel::load(&Gemma, prefix) (crates/gem/src/main.rs:57-76): reads prefix.order (u32 token ids),
 * prefix.A (f32 classes x d) and prefix.b (f32 classes), cuts the order into classes of
 * ceil(vocab / classes) tokens and gathers each class's rows of the output matrix into one
 * contiguous block on the device (main.rs:74). */
int gem_open_twolevel(gem_model* m, const char* prefix);
/* Drop (the reference frees on scope exit). */
void gem_close(gem_model* m);
int gem_get_info(const gem_model* m, gem_info* out);
/* Numerics of every later call.
 * GEM_NUMERICS_EXACT (the default, ref_threads 8): bit-identical hidden states and logits to the
 *   reference's AVX-512 path (q8.rs dot_avx512 / dot4_avx512 / dot16_avx512, model.rs dot512 and
 *   axpy512) run with a pool of ref_threads threads (gem bench --threads, main.rs:197); log-sum-exps
 *   differ only in summation order.
 * GEM_NUMERICS_FAST: tree reductions. The forward then differs from the reference by int8
 *   quantization flips, within the spread between the reference's own AVX2 and AVX-512 paths. */
enum { GEM_NUMERICS_EXACT = 0, GEM_NUMERICS_FAST = 1 };
int gem_set_numerics(gem_model* m, int mode, int ref_threads);
/* How gem_score / gem_score_dev run the scoring loop. With exact numerics every schedule gives the
 * same results (each position's arithmetic is that of the per-token forward); they differ in how
 * positions overlap. PARALLEL always computes with exact numerics.
 * GEM_SCHEDULE_SEQUENTIAL: one CUDA graph per token, each token finishing before the next starts.
 * GEM_SCHEDULE_PIPELINED (two-level head, exact numerics): one layer-pipelined kernel - each decoder
 *   layer and the head own a group of SMs and consecutive tokens flow through them as a wavefront.
 * GEM_SCHEDULE_PARALLEL: the tokens are known in advance, so all positions of a chunk (up to 1024)
 *   go through each layer together; the K/V rows of a chunk are written before its attention reads
 *   them. The projections become exact int8 matrix products that read each weight once per chunk.
 * GEM_SCHEDULE_AUTO (default): PARALLEL where the model supports it, else PIPELINED for the
 *   two-level head, else SEQUENTIAL. */
enum { GEM_SCHEDULE_AUTO = 0, GEM_SCHEDULE_SEQUENTIAL = 1, GEM_SCHEDULE_PIPELINED = 2, GEM_SCHEDULE_PARALLEL = 3 };
int gem_set_schedule(gem_model* m, int schedule);
/* The parallel schedule's body products (q/k/v, o, gate/up, down) on the 5th-generation tensor cores
 * (on != 0) or the CUDA cores (0, the default; GEM_TC=1 in the environment turns them on at gem_open).
 * Both compute the reference's row dot bit for bit (q8.rs:257-270): the tensor cores form each lane's
 * exact int8 pair sums (tcgen05.mma, f16 operands, f32 accumulators in tensor memory) and the CUDA
 * cores apply the reference's one fp32 FMA per lane and block. Turning them on builds a tiled f16 copy
 * of the body matrices (2.125 bytes per weight). No counterpart in the reference. */
int gem_set_tensor_cores(gem_model* m, int on);
/* Whether scoring with `head` (0 full, 1 two-level) runs pipelined; stages_ctas (nullable, 2 ints)
 * receives CTAs per layer stage and for the head stage. gem_last_error() then holds the reason. */
int gem_get_schedule(gem_model* m, int head, int* pipelined, int* stages_ctas);
/* The schedule (SEQUENTIAL, PIPELINED or PARALLEL) that scoring with `head` runs under the current
 * setting; gem_last_error() then names it, or why a faster one is not used. */
int gem_get_schedule_kind(gem_model* m, int head, int* kind);
/* Phase profile of pipelined scoring, gem's GEM_PROFILE (main.rs:312-317) on the device: while on,
 * CTA 0 of every stage timestamps its phases; gem_get_phase_profile returns mean microseconds per
 * token per phase, averaged over layer stages (16 phases: input wait, attn norm, q/k/v, barrier,
 * qk-norm + scores, barrier, softmax + P.V, barrier, combine + o, barrier, norms, gate/up, barrier,
 * down, barrier, hand-off) and for the head stage (6: input wait, final norm + class logits + target
 * block, barrier, class selection + top block, barrier, argmax). Turning it on clears the sums. */
int gem_set_profiling(gem_model* m, int on);
int gem_get_phase_profile(gem_model* m, double* layer_us, int n_layer, double* head_us, int n_head);
/* Profile of parallel scoring (while profiling is on): mean device microseconds per scoring call in
 * each of 10 launch groups, timed with events between them - embedding, norms, q/k/v product,
 * attention, o product, gate/up product, gate, down product, head, and the vocab-sharded head's
 * combine (the all-gather of the ranks' partial statistics and their merge; 0 unsharded). No
 * counterpart in the reference. */
int gem_get_parallel_profile(gem_model* m, double* us, int n);
/* Kernels launched by the last scoring call (gem_score / gem_score_dev). */
int gem_get_last_launches(gem_model* m, int64_t* n);
/* Failure-detection test hook for the pipelined schedule: layer stage `stage` (-1: none) computes but
 * never hands its residual on, so the next stage's wait, bounded by wait_ms, expires; the scoring call
 * then returns GEM_E_TIMEOUT and the model stays usable. wait_ms also bounds every device-side wait
 * afterwards (default 2000). */
int gem_test_withhold_stage(gem_model* m, int stage, int wait_ms);
/* Clears a sequence's KV cache (the reference rebuilds its cache per run; bench reuses it). */
int gem_reset(gem_model* m, int seq);
int gem_sync(gem_model* m);
/* The CUDA stream (cudaStream_t) every call of this model is enqueued on, so callers can order
 * their own work and time with events on it. */
int gem_get_stream(const gem_model* m, void** stream);

/* Gemma::forward(tok, pos) (model.rs:286-430) on sequence 0: runs one token, appends to the KV
 * cache, keeps the final-norm hidden state on the device for the head calls below and copies it to
 * h_out (d floats) when h_out is not NULL. */
int gem_forward(gem_model* m, uint32_t tok, uint32_t pos, float* h_out);
/* Full::run + Full::logprob(target) (main.rs:30-37) on the last forward's hidden state; argmax is the
 * first maximum of the logits (lean.rs:36-38). Either output may be NULL. */
int gem_full_logprob(gem_model* m, uint32_t target, float* logprob, uint32_t* argmax);
/* TwoLevel::logprob(target, h) (main.rs:101-107) on the last forward's hidden state. argmax: the
 * greedy token of screening with the single most likely class (lean.rs:46-76 with top = 1). */
int gem_twolevel_logprob(gem_model* m, uint32_t target, float* logprob, uint32_t* argmax);

/* gem bench / gem check's scoring loop (main.rs:270-289) on sequence 0: BOS forward when the model
 * has one, then for i < n: forward(toks[i], i + off), head logprob of toks[i + 1]. toks has n + 1
 * entries; logprob_out / argmax_out have n (argmax_out may be NULL). head: 0 full, 1 two-level.
 * Host buffers; the loop runs on the device under the schedule gem_set_schedule selects. Under the
 * parallel schedule a call repeated with the same n and head (and, for gem_score_dev, the same device
 * pointers) replays a CUDA graph of the previous identical call's launches from its third repetition;
 * the results are those of a direct call. */
int gem_score(gem_model* m, const uint32_t* toks, size_t n, int head, float* logprob_out,
              uint32_t* argmax_out);
/* Same loop on device buffers (toks_dev n + 1, outputs n), enqueued on the model's stream. */
int gem_score_dev(gem_model* m, const uint32_t* toks_dev, size_t n, int head, float* logprob_dev,
                  uint32_t* argmax_dev);
/* Batched scoring of nseq independent sequences (the bench loop run once per sequence): toks holds
 * nseq rows of len + 1 ids, logprob_out / argmax_out nseq rows of len. Each sequence starts at
 * position 0 (after the BOS forward) with its own KV slot; the parallel schedule scores up to
 * max_seqs (gem_open) sequences at once. No counterpart in the reference, which scores one text. */
int gem_score_batch(gem_model* m, const uint32_t* toks, size_t nseq, size_t len, int head, float* logprob_out,
                    uint32_t* argmax_out);
/* Same on device buffers, enqueued on the model's stream. */
int gem_score_batch_dev(gem_model* m, const uint32_t* toks_dev, size_t nseq, size_t len, int head,
                        float* logprob_dev, uint32_t* argmax_dev);

/* Generation (lean.rs, main.rs:109-141; gem complete / gem gen), on the last forward's hidden state.
 * gem_greedy: lean.rs Classes::next + next_token - the greedy token by screening the `top` most likely
 * classes and the always-on rows (class-ordered row indices), highest raw logit wins; when the most
 * likely class's probability is below min_confidence, the full head's argmax over the class-ordered
 * rows instead (*fell_back = 1). gem_twolevel_sample: TwoLevel::sample - a class, then a member, drawn
 * at `temperature` with the reference's xorshift64 generator (*rng_state is updated). */
int gem_greedy(gem_model* m, int top, float min_confidence, const uint32_t* always, int n_always, uint32_t* token,
               int* fell_back);
int gem_twolevel_sample(gem_model* m, float temperature, uint64_t* rng_state, uint32_t* token);
/* gem_greedy for `batch` hidden states on device buffers (always_dev, tok_dev, fallback_dev device). */
int gem_greedy_dev(gem_model* m, const float* h_dev, int batch, int top, float min_confidence, const uint32_t* always_dev,
                   int n_always, uint32_t* tok_dev, int* fallback_dev);
/* The completion loop (lean.rs:113-200 without the tokenizer): BOS, the prompt (all positions at once
 * under the parallel schedule), then up to max_new tokens, each chosen by `mode` from the hidden state
 * and fed back; a token in `stops` ends the loop and is not emitted. Writes the tokens to out and
 * their count to *n_out. */
enum { GEM_GEN_GREEDY_FULL = 0, GEM_GEN_GREEDY_SCREEN = 1, GEM_GEN_SAMPLE = 2 };
typedef struct gem_gen_opts {
  int mode;
  int top;               /* GREEDY_SCREEN: classes screened */
  float min_confidence;  /* GREEDY_SCREEN: fall back to the full head below this class probability */
  const uint32_t* always;
  int n_always;
  float temperature;     /* SAMPLE */
  uint64_t seed;         /* SAMPLE: xorshift64 state */
  const uint32_t* stops;
  int n_stops;
} gem_gen_opts;
int gem_generate(gem_model* m, const uint32_t* prompt, size_t n_prompt, size_t max_new, const gem_gen_opts* opts,
                 uint32_t* out, size_t* n_out);

/* Vocab-sharded full head across GPUs (one process and model handle per GPU, the body replicated):
 * gem_shard_init splits the output matrix's rows into nranks contiguous ranges of ceil(vocab/nranks)
 * and joins an NCCL communicator (id: 128 bytes from gem_nccl_unique_id on one rank, passed to all).
 * Full-head scoring then computes this rank's logits, per-position partial log-sum-exp / argmax /
 * target-logit statistics, all-gathers them over the ranks and merges them, so every rank returns the
 * unsharded log-probs and argmax (ties: lowest token id). Needs the parallel schedule. NCCL is loaded
 * at run time (libnccl.so.2). No counterpart in the reference, which has one CPU process. */
int gem_nccl_unique_id(void* id_out);
int gem_shard_init(gem_model* m, int nranks, int rank, const void* id);

/* Kernel-level entry points on caller-provided DEVICE buffers, enqueued on the model's stream.
 * They stand in for q8::matvec (q8.rs:439-461) with Act::quantize (q8.rs:187-246) fused in front,
 * Full::run/logprob (main.rs:30-37) and TwoLevel::logprob (main.rs:101-107), for a batch of hidden
 * states. */
/* y = layer matrix `which` of layer `layer` (0 q, 1 k, 2 v, 3 o, 4 gate, 5 up, 6 down; layer -1 = the
 * output matrix in token order) times x: x has cols floats, y rows floats. */
int gem_matvec_dev(gem_model* m, int layer, int which, const float* x_dev, float* y_dev);
/* Full head for `batch` hidden states h_dev[batch][d] with targets_dev[batch]. Enqueued on the model's
 * stream (gem_sync, or the stream from gem_get_stream, before reading the outputs); calls on one model
 * share its head scratch in stream order. */
int gem_head_full_dev(gem_model* m, const float* h_dev, const uint32_t* targets_dev, int batch,
                      float* logprob_dev, uint32_t* argmax_dev);
/* Two-level head for `batch` hidden states; enqueued like gem_head_full_dev. Exact numerics: one launch
 * below 24 hidden states; from 24 on (GEM_TL_PRODUCT_MIN sets the switch point) the class logits as one
 * product, then up to 128 states one launch for the blocks and argmax, above that four block kernels.
 * Every route gives the same results. */
int gem_head_twolevel_dev(gem_model* m, const float* h_dev, const uint32_t* targets_dev, int batch,
                          float* logprob_dev, uint32_t* argmax_dev);
/* gem_head_full_dev for callers that cannot allocate device memory when they call it (a process whose
 * memory belongs to another allocator or is planned up front, a loop that must not block in the
 * allocator). No counterpart in the reference, which runs on the CPU and allocates freely. Same
 * arguments and results as gem_head_full_dev; allocates nothing and does not synchronise (results
 * and range errors are visible after gem_sync). Its scratch is one static 1 MiB device array per GPU,
 * held until the process exits, so batch is limited (about 190 hidden states at d = 640; larger
 * batches return GEM_E_ARG). The first call on a device resolves that array's address: make it
 * before any stream capture. All calls on a device share the array: calls that overlap on the GPU
 * race. */
int gem_head_full_noalloc(gem_model* m, const float* h_dev, const uint32_t* targets_dev, int batch,
                          float* logprob_dev, uint32_t* argmax_dev);

#ifdef __cplusplus
}
#endif
#endif /* GEM_B200_H */
