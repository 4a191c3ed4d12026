// The C ABI of include/gem.h: model handle, load + upload, the per-token forward and heads as kernel
// sequences on one stream, and the scoring loop as a CUDA graph per token.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <string>
#include <vector>

#include "../../include/gem.h"
#include "host.hpp"
#include "internal.hpp"
#include "kernels.cuh"
#include "pipeline.cuh"

using namespace gem;

namespace {

// NCCL, loaded at run time (the library has no link-time dependency on it): inside a process that
// already uses NCCL (torch), dlopen returns that same library.
struct Nccl {
  void* h = nullptr;
  decltype(&ncclGetUniqueId) get_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  bool load() {
    if (h) return true;
    h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return false;
    get_id = (decltype(get_id))dlsym(h, "ncclGetUniqueId");
    init_rank = (decltype(init_rank))dlsym(h, "ncclCommInitRank");
    all_gather = (decltype(all_gather))dlsym(h, "ncclAllGather");
    destroy = (decltype(destroy))dlsym(h, "ncclCommDestroy");
    error_string = (decltype(error_string))dlsym(h, "ncclGetErrorString");
    return get_id && init_rank && all_gather && destroy && error_string;
  }
};
Nccl& nccl() {
  static Nccl n;
  return n;
}

thread_local std::string g_last_error;

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(e == cudaErrorMemoryAllocation ? GEM_E_NOMEM : GEM_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

template <typename T>
T* dev_alloc(size_t n) {
  void* p = nullptr;
  if (n == 0) n = 1;
  ck(cudaMalloc(&p, n * sizeof(T)), "cudaMalloc");
  return (T*)p;
}
template <typename T>
T* dev_upload(const std::vector<T>& v) {
  T* p = dev_alloc<T>(v.size());
  if (!v.empty()) ck(cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice), "upload");
  return p;
}

struct DevMat {
  MatView v;
  size_t bytes = 0;  // q plane + scale plane as stored
};

DevMat upload_mat(const HostMat& m, std::vector<void*>& owned) {
  DevMat d;
  d.v.rows = (int)m.rows;
  d.v.cols = (int)m.cols;
  d.v.bits = m.bits;
  d.v.scale_f32 = m.scale_f32() ? 1 : 0;
  void* q = dev_upload(m.q);
  owned.push_back(q);
  d.v.q = q;
  if (m.bits != 16) {
    void* s = m.scale_f32() ? (void*)dev_upload(m.s32) : (void*)dev_upload(m.s16);
    owned.push_back(s);
    d.v.s = s;
  }
  d.bytes = canonical_bytes(m);
  return d;
}

struct Layer {
  DevMat qkv, o, gu, down;
  float *attn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *post_attn = nullptr, *ffn_norm = nullptr,
        *post_ffw = nullptr, *bqkv = nullptr;
  bool swa = false;
  DevMat q_only, k_only, v_only, gate_only, up_only;  // views into qkv / gu for gem_matvec_dev
  TcMat tqkv, to, tgu, tdown;  // tiled copies for the tensor-core products (built by ensure_tc)
};

}  // namespace

struct gem_model {
  int device = 0, sms = 148;
  cudaStream_t st = nullptr;
  std::vector<void*> owned;
  // geometry (model.rs:32-69)
  int d = 0, vocab = 0, nl = 0, nh = 0, nkv = 0, hd = 0, ff = 0, window = 0, ctx = 0, max_seqs = 1;
  float eps = 0, embed_scale = 1, rope_base = 10000;
  bool silu = false, untied = false, gemma = true;
  int64_t bos = -1;
  int body_bits = 8, head_bits = 8;
  size_t body_bytes = 0;
  std::vector<Layer> layers;
  DevMat head, emb;  // emb used only when the file has a separate output matrix
  // permute_head (model.rs:242-249): once a two-level class file covers the vocabulary, head's rows
  // are in class order and row_of maps a token to its row (null: token order; row -> token is order)
  uint32_t* row_of = nullptr;
  std::vector<uint32_t> row_of_h;
  const uint32_t* row_tok() const { return row_of ? order : nullptr; }
  unsigned char* head_bulk_q = nullptr;  // the output matrix's GEMV copy for the streamed full head, built on first use
  __half* head_bulk_s = nullptr;
  float* out_norm = nullptr;
  float *rope_sin[2] = {nullptr, nullptr}, *rope_cos[2] = {nullptr, nullptr};
  float *kc = nullptr, *vc = nullptr;  // [seq][layer][ctx][nkv*hd]
  int chunk = 64, nsplit_swa = 1, nsplit_glob = 1;
  // activations
  float *x, *xn, *qkv, *att, *o, *gu, *g, *dn, *h, *part;
  int8_t *aq_d, *aq_att, *aq_ff, *haq;
  float *as_d, *as_att, *as_ff, *has;
  // step state and outputs
  StepCur* cur = nullptr;
  int* err = nullptr;  // device error word (kernels record out-of-range caller ids here)
  StepCur* cur_host = nullptr;  // pinned
  uint32_t *step = nullptr, *toks = nullptr, *am = nullptr;
  float* lp = nullptr;
  // heads
  int hbatch = 0;
  float *head_part = nullptr, *tlogit = nullptr, *cl = nullptr, *inner = nullptr;
  int* head_cnt = nullptr;  // the streamed full head's finished-CTA counters, one per batch item
  int* tl_cnt = nullptr;    // the fused two-level head's finished-CTA counters, one per batch item
  float* tl_part = nullptr;  // and its per-CTA partials
  int8_t* hb_q = nullptr;  // batched head calls: quantized hidden states [batch][d] and their scales
  float* hb_s = nullptr;
  // two-level (main.rs:40-51)
  bool two = false;
  int k = 0, per = 0;
  DevMat blocks;
  float *A = nullptr, *b = nullptr;
  uint32_t *cls_of = nullptr, *pos_of = nullptr, *order = nullptr;
  // numerics: exact = bit-identical to the reference's AVX-512 path with a pool of ref_threads
  bool exact = true;
  // the parallel schedule's body products on the tensor cores (tc_gemm.cu) instead of the CUDA cores;
  // GEM_TC=1 in the environment turns them on at gem_open
  bool tc = false, tc_ready = false;
  int ref_threads = 8;
  float *qn = nullptr, *scores = nullptr, *top_inner = nullptr;
  uint32_t* top_of = nullptr;
  // layer-pipelined scoring (pipeline.cu)
  int schedule = GEM_SCHEDULE_AUTO;
  bool pipe_ready = false;
  PipeArgs pipe{};
  size_t pipe_smem = 0;
  std::string pipe_why;  // why the pipeline is not used, for gem_get_schedule
  unsigned long long wait_ns = 2000000000ull;  // bound of every device-side wait
  int withhold_stage = -1;                     // failure-detection test hook
  unsigned long long* prof = nullptr;          // per-stage phase times of pipelined runs (nullable)
  // sequence-parallel scoring (seq.cu): buffers for up to seq_cap positions
  static constexpr int kSeqChunk = 1024;   // positions of one sequence per chunk
  static constexpr int kBatchRows = 4096;  // positions of all sequences per chunk (batched scoring)
  static constexpr int kHeadChunk = 256;   // positions per full-head logits pass
  int seq_cap = 0, seq_sstride = 0, logits_cap = 0, part_cap = 0;
  float* s_part = nullptr;  // P.V partials [T][nh][ref_threads][hd]
  uint32_t *s_tin = nullptr, *s_tgt = nullptr, *s_am = nullptr;  // chunk token ids, targets, argmax
  float* s_lp = nullptr;                                           // chunk log-probs
  float *s_x = nullptr, *s_y = nullptr, *s_gu = nullptr, *s_dn = nullptr, *s_h = nullptr, *s_qn = nullptr,
        *s_scores = nullptr, *s_logits = nullptr;
  int8_t *s_aq = nullptr, *s_haq = nullptr;
  float *s_as = nullptr, *s_has = nullptr;
  std::string seq_why;  // why the sequence-parallel schedule is not used
  // vocab-sharded full head (gem_shard_init): this rank's output-matrix rows and the communicator
  int shard_rank = 0, shard_n = 1, shard_row0 = 0, shard_rows = 0;
  ncclComm_t comm = nullptr;
  float *s_spart = nullptr, *s_sgath = nullptr;
  size_t spart_cap = 0;
  // per-category device time of parallel scoring (gem_set_profiling): events between launch groups
  enum { PAR_EMBED, PAR_NORM, PAR_QKV, PAR_ATTN, PAR_O, PAR_GU, PAR_GLU, PAR_DOWN, PAR_HEAD, PAR_COMBINE, PAR_CATS };
  bool par_prof = false;
  std::vector<cudaEvent_t> pev;
  std::vector<int> pcat;
  double par_us[PAR_CATS] = {};
  int64_t par_calls = 0;
  int64_t last_launches = 0;  // kernels the last scoring call launched
  // graphs
  cudaGraphExec_t score_graph[2] = {nullptr, nullptr};
  int64_t graph_kernels[2] = {-1, -1};
  void drop_graphs() {
    graph_kernels[0] = graph_kernels[1] = -1;
    for (auto& g : score_graph)
      if (g) {
        cudaGraphExecDestroy(g);
        g = nullptr;
      }
    drop_par_graph();
    par_seen = false;
  }
  // The parallel schedule of one sequence as a CUDA graph (score_parallel): the arguments it was
  // captured with, including the count of device allocations made before it (scratch that grows
  // moves, and the graph holds its addresses).
  struct ParKey {
    const uint32_t* toks;
    size_t stride, len;
    int which, parts;
    uint32_t base;
    float* lp;
    uint32_t* am;
    int64_t gen;
    bool operator==(const ParKey& o) const {
      return toks == o.toks && stride == o.stride && len == o.len && which == o.which && parts == o.parts &&
             base == o.base && lp == o.lp && am == o.am && gen == o.gen;
    }
  };
  cudaGraphExec_t par_graph = nullptr;
  ParKey par_key{};
  bool par_seen = false;  // par_key holds the arguments of the last direct call
  bool par_graph_failed = false;  // a capture failed on this model: launch directly from then on
  int64_t par_nk = 0;
  int64_t alloc_gen = 0;
  void drop_par_graph() {
    if (par_graph) {
      cudaGraphExecDestroy(par_graph);
      par_graph = nullptr;
    }
  }
  // GEM_PAR_GRAPH=0 launches every parallel-schedule call directly
  static bool par_graph_enabled() {
    static const bool on = [] {
      const char* e = std::getenv("GEM_PAR_GRAPH");
      return !(e && std::atoi(e) == 0);
    }();
    return on;
  }
  bool have_h = false;
  // generation-side heads (decode.cu): per-call scratch, grown on demand
  struct GenScratch {
    int8_t* q = nullptr;
    float *s = nullptr, *cl = nullptr, *z = nullptr, *logits = nullptr, *lp = nullptr;
    uint32_t *sel = nullptr, *rows = nullptr, *always = nullptr, *fb_row = nullptr, *tok = nullptr, *zeros = nullptr;
    int* fallback = nullptr;
    unsigned long long* rng = nullptr;
    size_t batch = 0, nrows = 0, nalways = 0, nlogits = 0;
  } gs;
  // host-buffer batched scoring: device copies of the ids and outputs
  uint32_t *btoks = nullptr, *bam = nullptr;
  float* blp = nullptr;
  size_t btoks_cap = 0, bout_cap = 0;
  void ensure_batch_io(size_t ntoks, size_t nout) {
    if (ntoks > btoks_cap) {
      btoks = alloc<uint32_t>(ntoks);
      btoks_cap = ntoks;
    }
    if (nout > bout_cap) {
      blp = alloc<float>(nout);
      bam = alloc<uint32_t>(nout);
      bout_cap = nout;
    }
  }

  // Split of a single sequence's chunk into parts on their own streams (score_parallel): part k
  // runs on split_st[k - 1] (part 0 on st), one layer behind part k - 1. split_ev[(k * nl) + l] marks
  // part k's layer-l attention (its K/V rows written); fork_ev / join_ev[k] bracket the chunk.
  static constexpr int kMaxParts = 8;
  cudaStream_t split_st[kMaxParts - 1] = {};
  std::vector<cudaEvent_t> split_ev, join_ev;
  cudaEvent_t fork_ev = nullptr;
  void ensure_split(int parts) {
    for (int k = 0; k < parts - 1; ++k)
      if (!split_st[k]) ck(cudaStreamCreateWithFlags(&split_st[k], cudaStreamNonBlocking), "stream");
    auto more = [](std::vector<cudaEvent_t>& v, size_t n) {
      while (v.size() < n) {
        cudaEvent_t e;
        ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
        v.push_back(e);
      }
    };
    more(split_ev, (size_t)(parts - 1) * nl);
    more(join_ev, (size_t)parts - 1);
    if (!fork_ev) ck(cudaEventCreateWithFlags(&fork_ev, cudaEventDisableTiming), "event");
  }
  // parts per single-sequence chunk (default 4): GEM_SPLIT=1 (or 0) runs one stream, 2..8 that many parts
  static int split_parts() {
    static const int n = [] {
      const char* e = std::getenv("GEM_SPLIT");
      const int v = e ? std::atoi(e) : 4;
      return std::max(1, std::min(kMaxParts, v));
    }();
    return n;
  }

  ~gem_model() {
    if (st) cudaStreamSynchronize(st);
    for (cudaStream_t x : split_st)
      if (x) cudaStreamSynchronize(x);
    for (cudaEvent_t e : pev) cudaEventDestroy(e);
    for (cudaEvent_t e : split_ev) cudaEventDestroy(e);
    for (cudaEvent_t e : join_ev) cudaEventDestroy(e);
    if (fork_ev) cudaEventDestroy(fork_ev);
    for (cudaStream_t x : split_st)
      if (x) cudaStreamDestroy(x);
    if (comm) nccl().destroy(comm);
    for (auto& g : score_graph)
      if (g) cudaGraphExecDestroy(g);
    if (par_graph) cudaGraphExecDestroy(par_graph);
    for (void* p : owned) cudaFree(p);
    if (cur_host) cudaFreeHost(cur_host);
    if (st) cudaStreamDestroy(st);
  }

  template <typename T>
  T* alloc(size_t n) {
    T* p = dev_alloc<T>(n);
    owned.push_back(p);
    ++alloc_gen;
    return p;
  }
  // Frees a buffer from alloc / upload (the graphs that used it must be dropped).
  void release(const void* p) {
    for (size_t i = 0; i < owned.size(); ++i)
      if (owned[i] == p) {
        cudaFree(owned[i]);
        owned.erase(owned.begin() + (long)i);
        ++alloc_gen;
        return;
      }
  }
  template <typename T>
  T* upload(const std::vector<T>& v) {
    T* p = dev_upload(v);
    owned.push_back(p);
    ++alloc_gen;
    return p;
  }
  float* upload_or_null(const std::vector<float>& v) { return v.empty() ? nullptr : upload(v); }

  void ensure_head_batch(int batch) {
    if (batch <= hbatch) return;
    int parts = head_full_parts(sms);
    head_part = alloc<float>((size_t)batch * parts * 4);
    tlogit = alloc<float>(batch);
    head_cnt = alloc<int>(batch);  // the streamed head's finished-CTA counters: zero between launches
    ck(cudaMemsetAsync(head_cnt, 0, (size_t)batch * sizeof(int), st), "head counters");
    tl_cnt = alloc<int>(batch);
    ck(cudaMemsetAsync(tl_cnt, 0, (size_t)batch * sizeof(int), st), "head counters");
    if (two) tl_part = alloc<float>((size_t)batch * tl_part_floats(k, per));
    hb_q = alloc<int8_t>((size_t)batch * d);
    hb_s = alloc<float>((size_t)batch * d / 32);
    if (two) {
      cl = alloc<float>((size_t)batch * k);
      inner = alloc<float>((size_t)batch * per);
      top_inner = alloc<float>((size_t)batch * per);
      top_of = alloc<uint32_t>(batch);
    }
    hbatch = batch;
  }

  // The tensor-core products' tiled copies of every layer's matrices (2.125 bytes per weight).
  void ensure_tc() {
    if (tc_ready) return;
    for (Layer& L : layers)
      for (auto [M, TM] : {std::pair<const DevMat*, TcMat*>{&L.qkv, &L.tqkv}, {&L.o, &L.to}, {&L.gu, &L.tgu}, {&L.down, &L.tdown}}) {
        if (!tc_gemm_supported(M->v)) throw Error(GEM_E_STATE, "tensor-core products need Q8_0/Q4_0 body weights");
        unsigned char* buf = alloc<unsigned char>(tc_tiled_bytes(M->v));
        tc_tile(M->v, buf, TM, st);
      }
    ck(cudaGetLastError(), "tile for the tensor cores");
    ck(cudaStreamSynchronize(st), "tile for the tensor cores");
    tc_ready = true;
  }
  // One of a layer's exact int8 products, Y[t][r] for the chunk's n positions: on the tensor cores
  // when they are on and the chunk fills a tile of positions, else on the CUDA cores. Both are
  // bit-identical.
  void product(const DevMat& M, const TcMat& TM, const int8_t* aq, const float* as, int n, float* y, int ldy,
               cudaStream_t s, int parts) {
    if (tc && tc_ready && n >= 16) launch_tc_gemm(TM, aq, as, n, y, ldy, err, sms, s);
    else launch_seq_gemm(M.v, aq, as, n, y, ldy, sms, s, parts);
  }

  AttnArgs attn_args(int l, int seq) const {
    const Layer& L = layers[l];
    AttnArgs A{};
    A.qkv = qkv;
    A.bqkv = L.bqkv;
    A.q_norm = L.q_norm;
    A.k_norm = L.k_norm;
    int tb = L.swa ? 0 : 1;
    A.rope_sin = rope_sin[tb];
    A.rope_cos = rope_cos[tb];
    size_t layer_elems = (size_t)ctx * nkv * hd;
    A.kcache = kc + ((size_t)seq * nl + l) * layer_elems;
    A.vcache = vc + ((size_t)seq * nl + l) * layer_elems;
    A.part = part;
    A.att_out = att;
    A.cur = cur;
    A.nh = nh, A.nkv = nkv, A.hd = hd;
    A.window = L.swa ? window : 0;
    A.chunk = chunk;
    A.nsplit = L.swa ? nsplit_swa : nsplit_glob;
    A.eps = eps;
    A.qscale = 1.0f / std::sqrt((float)hd);
    return A;
  }

  // Gemma::forward (model.rs:286-430) for the token in *cur, KV cache of `seq`; leaves the final-norm
  // hidden state in h and its quantization in (haq, has).
  void enqueue_body(int seq) {
    const DevMat& E = untied ? emb : head;
    launch_embed(E.v, untied ? nullptr : row_of, cur, embed_scale, x, st);
    // exact numerics with d <= 1152 in 32-blocks: the parallel schedule's norm kernel for one position
    // (one warp, the sequential sums fed by prefetched loads, quantization from registers), the same
    // arithmetic as the single-CTA per-token kernel
    const bool warp_norm = exact && d <= 1152 && d % 32 == 0;
    auto norm = [&](float* xx, const float* delta, const float* w_post, const float* w_pre, float e, int n, int8_t* aq,
                    float* as, float* xn_out, cudaStream_t s) {
      if (warp_norm) launch_seq_norm(xx, delta, w_post, w_pre, e, n, 1, aq, as, xn_out, s);
      else (exact ? launch_residual_norm_quant_exact : launch_residual_norm_quant)(xx, delta, w_post, w_pre, e, n, aq, as,
                                                                                   xn_out, s);
    };
    auto gemv = exact ? launch_gemv_exact : launch_gemv;
    for (int l = 0; l < nl; ++l) {
      const Layer& L = layers[l];
      const Layer* P = l > 0 ? &layers[l - 1] : nullptr;
      norm(x, P ? dn : nullptr, P ? P->post_ffw : nullptr, L.attn_norm, eps, d, aq_d, as_d, xn, st);
      gemv(L.qkv.v, aq_d, as_d, xn, qkv, sms, st);
      AttnArgs A = attn_args(l, seq);
      if (exact) launch_attn_exact(A, qn, scores, ctx, ref_threads, aq_att, as_att, sms, st);
      else launch_attn(A, aq_att, as_att, st);
      gemv(L.o.v, aq_att, as_att, att, o, sms, st);
      norm(x, o, L.post_attn, L.ffn_norm, eps, d, aq_d, as_d, xn, st);
      gemv(L.gu.v, aq_d, as_d, xn, gu, sms, st);
      launch_glu_quant(gu, ff, silu ? 1 : 0, aq_ff, as_ff, g, st);
      gemv(L.down.v, aq_ff, as_ff, g, dn, sms, st);
    }
    norm(x, dn, layers[nl - 1].post_ffw, out_norm, eps, d, haq, has, h, st);
  }

  HeadArgs head_args(const int8_t* qa, const float* sa, const float* hh, const uint32_t* targets, float* lpo, uint32_t* amo) {
    HeadArgs H{};
    H.w = head.v;
    H.row_of = row_of, H.row_tok = row_tok();
    H.aq = qa, H.as = sa, H.h = hh;
    H.targets = targets;
    H.cur = cur;
    H.part = head_part;
    H.tlogit = tlogit;
    H.lp_out = lpo;
    H.am_out = amo;
    H.err = err;
    return H;
  }
  TwoLevelArgs tl_args(const int8_t* qa, const float* sa, const float* hh, const uint32_t* targets, float* lpo, uint32_t* amo) {
    TwoLevelArgs T{};
    T.w = blocks.v;
    T.A = A, T.b = b, T.cls_of = cls_of, T.pos_of = pos_of, T.order = order;
    T.aq = qa, T.as = sa, T.h = hh;
    T.targets = targets;
    T.cur = cur;
    T.cl = cl, T.inner = inner;
    T.lp_out = lpo, T.am_out = amo;
    T.k = k, T.per = per, T.vocab = vocab;
    T.err = err;
    return T;
  }
  void run_head(int which, const int8_t* qa, const float* sa, const float* hh, const uint32_t* targets, int batch,
                float* lpo, uint32_t* amo) {
    ensure_head_batch(batch);
    if (which == 0) {
      HeadArgs H = head_args(qa, sa, hh, targets, lpo, amo);
      if (exact && head_bulk_q) {
        H.cnt = head_cnt;  // the last CTA merges; with qa null each CTA quantizes hh itself
        launch_head_full_bulk(H, head_bulk_q, head_bulk_s, batch, sms, st);
      } else if (exact) {
        launch_head_full_exact(H, batch, sms, st);
      } else {
        launch_head_full(H, batch, sms, st);
      }
      return;
    }
    TwoLevelArgs T = tl_args(qa, sa, hh, targets, lpo, amo);
    if (!exact) {
      launch_head_twolevel(T, batch, sms, st);
      return;
    }
    if (launch_tl_fused(T, batch, sms, tl_cnt, tl_part, st)) return;  // quantizes hh itself
    // a hidden size whose staging area does not fit in shared memory: four launches
    if (!qa) {
      launch_quantize(hh, batch * d, hb_q, hb_s, st);
      T.aq = hb_q, T.as = hb_s;
    }
    T.class_ctas = std::max(1, std::min(sms, (k + 15) / 16));  // one 16-class task per CTA where possible
    launch_tl_stage1_exact(T, batch, T.class_ctas, std::max(1, std::min(8, (per + 127) / 128)), st);
    launch_tl_select(T, batch, top_of, st);
    launch_tl_top_exact(T, batch, top_of, top_inner, st);
    launch_tl_argmax(T, batch, top_of, top_inner, st);
  }
  void enqueue_head(int which, float* lpo, uint32_t* amo) { run_head(which, haq, has, h, nullptr, 1, lpo, amo); }

  // Can a whole sequence go through each layer at once (seq.cu)?
  bool seq_supported() {
    seq_why.clear();
    const int G = nkv > 0 ? nh / nkv : 0;
    if (G < 1 || G > 8) seq_why = "more than 8 query heads per kv head";
    else if (hd % 32 || hd > 256 || d % 32 || d > 1152 || ff % 32)
      seq_why = "head_dim above 256, hidden size above 1152 or dimensions not in 32-blocks";
    for (const Layer& L : layers)
      for (const DevMat* w : {&L.qkv, &L.o, &L.gu, &L.down})
        if (seq_why.empty() && !seq_gemm_supported(w->v)) seq_why = "body weights not Q8_0/Q4_0 with even block counts";
    return seq_why.empty();
  }
  bool use_parallel() {
    if (schedule != GEM_SCHEDULE_AUTO && schedule != GEM_SCHEDULE_PARALLEL) return false;
    if (seq_supported()) return true;
    if (schedule == GEM_SCHEDULE_PARALLEL) throw Error(GEM_E_STATE, "sequence-parallel schedule unavailable: " + seq_why);
    return false;
  }

  void ensure_seq(int T) {
    if (T <= seq_cap) return;
    const size_t qkv_rows = (size_t)(nh + 2 * nkv) * hd;
    const size_t wide = std::max({(size_t)d, (size_t)nh * hd, (size_t)ff});
    s_x = alloc<float>((size_t)T * d);
    s_y = alloc<float>((size_t)T * std::max(qkv_rows, (size_t)d));
    s_gu = alloc<float>((size_t)T * 2 * ff);
    s_dn = alloc<float>((size_t)T * d);
    s_h = alloc<float>((size_t)T * d);
    s_qn = alloc<float>((size_t)T * nh * hd);
    seq_sstride = ctx;
    s_scores = alloc<float>((size_t)T * nh * seq_sstride);
    s_aq = alloc<int8_t>((size_t)T * wide);
    s_as = alloc<float>((size_t)T * wide / 32);
    s_haq = alloc<int8_t>((size_t)T * d);
    s_has = alloc<float>((size_t)T * d / 32);
    s_tin = alloc<uint32_t>(T);
    s_tgt = alloc<uint32_t>(T);
    s_am = alloc<uint32_t>(T);
    s_lp = alloc<float>(T);
    seq_cap = T;
  }

  // The exact two-level head over T hidden states (fp32 hh, quantized qa / sa) as the class logits'
  // tile product (every class row read once for all T) and the block kernels: target block, top
  // class, top block, argmax. Returns the kernels launched.
  // one_launch_tail: up to kTlGivenMax states, the blocks, log-sum-exps and argmax by k_tl_fused reading
  // the class logits (it quantizes hh itself) instead of the four block kernels; qa, sa may then be
  // null. Above that, ceil(per / 32) CTAs a state with a last-CTA block pass each lose to the block
  // kernels (256 states: 81 us against 69 us).
  static constexpr int kTlGivenMax = 128;
  int twolevel_product(const int8_t* qa, const float* sa, const float* hh, const uint32_t* targets, int T, float* lpo,
                       uint32_t* amo, bool one_launch_tail = false) {
    ensure_head_batch(T);
    launch_seq_class_logits(A, b, k, hh, d, T, cl, st);
    TwoLevelArgs TL = tl_args(qa, sa, hh, targets, lpo, amo);
    if (one_launch_tail && T <= kTlGivenMax) {
      TL.cl_in = cl;
      if (launch_tl_fused(TL, T, sms, tl_cnt, tl_part, st)) return 2;
      TL.cl_in = nullptr;
    }
    const bool quantize = !qa;  // the block kernels below need the quantized states
    if (quantize) {
      launch_quantize(hh, T * d, hb_q, hb_s, st);
      TL.aq = hb_q, TL.as = hb_s;
    }
    TL.class_ctas = 0;
    const int block_ctas = std::max(1, std::min(8, (per + 127) / 128));
    launch_tl_stage1_exact(TL, T, 0, block_ctas, st);
    launch_tl_select(TL, T, top_of, st);
    launch_tl_top_exact(TL, T, top_of, top_inner, st);
    launch_tl_argmax(TL, T, top_of, top_inner, st);
    return quantize ? 6 : 5;
  }
  int seq_head(int which, const uint32_t* targets, int T, float* lpo, uint32_t* amo) {
    // the block kernels at every T: a sequence's log-probs stay bit-identical whether it is scored alone
    // or in a batch (the one-launch tail merges the log-sum-exps in another order)
    if (which == 1) return twolevel_product(s_haq, s_has, s_h, targets, T, lpo, amo);
    if (comm) return seq_head_sharded(targets, T, lpo, amo);
    if (!full_head_gemm_supported()) {  // the per-position exact head kernels
      run_head(0, s_haq, s_has, s_h, targets, T, lpo, amo);
      return 2;
    }
    return full_head_gemm(s_haq, s_has, s_h, targets, T, lpo, amo);
  }
  // Whether the full head has a matrix-product path: Q8_0/Q4_0 output matrices against the quantized
  // hidden states, F16 ones against the fp32 hidden states.
  bool full_head_gemm_supported() const { return seq_gemm_supported(head.v) || seq_head_f16_supported(head.v); }
  // Full head for T hidden states (quantized q, s; fp32 h) as exact matrix products over chunks of
  // kHeadChunk positions (the output matrix read once per chunk), then log-sum-exp, argmax and the
  // target logit per position. Returns the kernels launched.
  int full_head_gemm(const int8_t* q, const float* s, const float* h, const uint32_t* targets, int T, float* lpo,
                     uint32_t* amo) {
    const int hc = std::min(T, kHeadChunk);
    if (hc > logits_cap) {
      s_logits = alloc<float>((size_t)hc * vocab);
      logits_cap = hc;
    }
    const bool f16 = !seq_gemm_supported(head.v);
    int launches = 0;
    for (int h0 = 0; h0 < T; h0 += hc) {
      const int n = std::min(hc, T - h0);
      if (f16)
        launch_seq_head_f16(head.v, h + (size_t)h0 * d, n, s_logits, vocab, st);
      else
        launch_seq_gemm(head.v, q + (size_t)h0 * d, s + (size_t)h0 * d / 32, n, s_logits, vocab, sms, st);
      launch_seq_logit_reduce(s_logits, vocab, n, targets + h0, row_of, row_tok(), lpo + h0, amo ? amo + h0 : nullptr,
                              err, st);
      launches += 2;
    }
    return launches;
  }

  // Scoring with every position of a chunk going through each layer together: tokens toks_d[0..n]
  // at positions base_pos.., log-probs of toks_d[i + 1] to lp_d[i].
  // Records an event after the launches of category `cat` when profiling is on.
  void par_mark(int cat) {
    if (!par_prof) return;
    const size_t i = pcat.size();
    if (i >= pev.size()) {
      cudaEvent_t e;
      ck(cudaEventCreate(&e), "event");
      pev.push_back(e);
    }
    ck(cudaEventRecord(pev[i], st), "event record");
    pcat.push_back(cat);
  }
  void par_collect() {
    if (!par_prof || pcat.empty()) return;
    ck(cudaStreamSynchronize(st), "stream sync");
    for (size_t i = 1; i < pcat.size(); ++i) {
      float ms = 0;
      ck(cudaEventElapsedTime(&ms, pev[i - 1], pev[i]), "event time");
      par_us[pcat[i]] += ms * 1e3;
    }
    pcat.clear();
    ++par_calls;
  }

  // The full head over this rank's rows [shard_row0, shard_row0 + shard_rows): logits, per-position
  // partial statistics, one all-gather of the partials over the ranks, and the merge (main.rs:30-37).
  int seq_head_sharded(const uint32_t* targets, int T, float* lpo, uint32_t* amo) {
    MatView w = head.v;
    const size_t rowbytes = (size_t)w.cols * w.bits / 8, sbytes = (size_t)(w.cols / 32) * (w.scale_f32 ? 4 : 2);
    w.q = (const unsigned char*)w.q + (size_t)shard_row0 * rowbytes;
    w.s = (const unsigned char*)w.s + (size_t)shard_row0 * sbytes;
    w.rows = shard_rows;
    const int hc = std::min(T, kHeadChunk);
    if (hc > logits_cap) {
      s_logits = alloc<float>((size_t)hc * vocab);  // sized for the whole vocabulary: reusable unsharded
      logits_cap = hc;
    }
    if ((size_t)T > spart_cap) {
      s_spart = alloc<float>((size_t)T * 5);
      s_sgath = alloc<float>((size_t)T * 5 * shard_n);
      spart_cap = T;
    }
    int launches = 0;
    for (int h0 = 0; h0 < T; h0 += hc) {
      const int n = std::min(hc, T - h0);
      launch_seq_gemm(w, s_haq + (size_t)h0 * d, s_has + (size_t)h0 * d / 32, n, s_logits, shard_rows, sms, st);
      launch_seq_logit_partials(s_logits, shard_rows, (uint32_t)shard_row0, n, targets + h0, (uint32_t)vocab, row_of,
                                row_tok(), s_spart + (size_t)h0 * 5, err, st);
      launches += 2;
    }
    par_mark(PAR_HEAD);  // this rank's rows: logits and partial statistics
    const ncclResult_t r = nccl().all_gather(s_spart, s_sgath, (size_t)T * 5, ncclFloat32, comm, st);
    if (r != ncclSuccess) throw Error(GEM_E_NCCL, std::string("ncclAllGather: ") + nccl().error_string(r));
    launch_seq_logit_combine(s_sgath, shard_n, T, lpo, amo, st);
    par_mark(PAR_COMBINE);  // the all-gather over the ranks and the merge
    return launches + 1;
  }

  // Scoring with every position of a chunk going through each layer together. toks_d holds nseq
  // sequences of len + 1 ids, `stride` ids apart; sequence s's log-probs of ids 1..len go to
  // lp_d[s * len ..] (argmax likewise). A chunk holds up to kBatchRows positions of whole sequences
  // (each in its own KV slot) or kSeqChunk positions of one long sequence.
  // One sequence's call repeated with the same arguments (the scoring loop of a benchmark or a
  // service: same buffers, new token ids) replays a CUDA graph of its ~900 launches: the first call
  // launches them directly, the second is captured and replayed, later ones replay. The graph reads
  // the token ids and writes the outputs through the same device pointers, so only their contents
  // may change between calls; profiling, batches and the vocab-sharded head launch directly.
  void score_parallel(const uint32_t* toks_d, size_t stride, int nseq, size_t len, int which, uint32_t base_pos,
                      float* lp_d, uint32_t* am_d) {
    if (nseq != 1 || par_prof || comm || par_graph_failed || !par_graph_enabled()) {
      drop_par_graph();
      par_seen = false;
      score_parallel_direct(toks_d, stride, nseq, len, which, base_pos, lp_d, am_d);
      return;
    }
    ParKey key{toks_d, stride, len, which, split_parts(), base_pos, lp_d, am_d, alloc_gen};
    if (par_graph && key == par_key) {
      ck(cudaGraphLaunch(par_graph, st), "graph launch");
      last_launches = par_nk;
      return;
    }
    const bool again = par_seen && key == par_key;
    drop_par_graph();
    par_seen = false;
    if (!again) {  // scratch grows here, if it does: the key takes the allocation count after the call
      score_parallel_direct(toks_d, stride, nseq, len, which, base_pos, lp_d, am_d);
      key.gen = alloc_gen;
      par_key = key;
      par_seen = true;
      return;
    }
    // A capture or instantiation that fails (the caller's thread already capturing, a driver without
    // the support) launches this call directly and turns the replay off for the model.
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    bool captured = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
    if (captured) {
      try {
        score_parallel_direct(toks_d, stride, nseq, len, which, base_pos, lp_d, am_d);
      } catch (...) {
        captured = false;
      }
      if (cudaStreamEndCapture(st, &g) != cudaSuccess) captured = false;
      if (captured && g && cudaGraphInstantiate(&ge, g, 0) != cudaSuccess) {
        ge = nullptr;
        captured = false;
      }
      if (g) cudaGraphDestroy(g);
    }
    if (!captured || !ge || alloc_gen != key.gen) {  // scratch that grew under capture: not expected either
      if (ge) cudaGraphExecDestroy(ge);
      cudaGetLastError();  // a failed capture call leaves no sticky error; clear the last-error slot
      par_graph_failed = true;
      score_parallel_direct(toks_d, stride, nseq, len, which, base_pos, lp_d, am_d);
      return;
    }
    par_graph = ge;
    par_key = key;
    par_seen = true;
    par_nk = last_launches;
    ck(cudaGraphLaunch(par_graph, st), "graph launch");
  }

  void score_parallel_direct(const uint32_t* toks_d, size_t stride, int nseq, size_t len, int which,
                             uint32_t base_pos, float* lp_d, uint32_t* am_d) {
    const int L = (int)std::min<size_t>(len, kSeqChunk);
    const int SC = std::max(1, std::min({nseq, max_seqs, kBatchRows / L}));
    const int cap = L * SC;
    ensure_seq(cap);
    if ((int64_t)cap * ref_threads > part_cap) {
      s_part = alloc<float>((size_t)cap * ref_threads * nh * hd);
      part_cap = cap * ref_threads;
    }
    const DevMat& E = untied ? emb : head;
    const int qkv_rows = (nh + 2 * nkv) * hd;
    const size_t kv_stride = (size_t)nl * ctx * nkv * hd;  // between the KV slots of two sequences
    int T = 0;
    int64_t nk = 0;
    pcat.clear();
    par_mark(-1);
    // positions start after a BOS forward in slot 0: the other slots get its K/V rows (position 0 is
    // never rewritten, so one copy serves every group of sequences)
    if (base_pos > 0)
      for (int s = 1; s < SC; ++s) copy_bos_kv(s);
    for (int s0 = 0; s0 < nseq; s0 += SC) {
      const int ns = std::min(SC, nseq - s0);
      for (size_t c0 = 0; c0 < len; c0 += L) {
        const int Lc = (int)std::min<size_t>(L, len - c0);
        T = Lc * ns;
        const uint32_t pos0 = base_pos + (uint32_t)c0;
        // One sequence's chunk runs as parts of at least 128 positions on their own streams, part k
        // behind part k - 1: its layer-l attention waits until part k - 1 has written its K/V rows of
        // layer l (after waiting for the parts before it); no part reads a later part's rows.
        // The parts' latency-bound kernels then overlap the other parts' matrix products. Each
        // position's arithmetic is the same. Buffers read and written at one width take row offsets;
        // those used at several widths (s_y, s_aq, s_as) take offsets of whole rows of their widest use.
        const int parts = (ns == 1 && !par_prof) ? std::max(1, std::min(split_parts(), Lc / 128)) : 1;
        const int Lp = (Lc + parts - 1) / parts;
        if (parts > 1) {
          ensure_split(parts);
          ck(cudaEventRecord(fork_ev, st), "fork");
          for (int k = 0; k < parts - 1; ++k) ck(cudaStreamWaitEvent(split_st[k], fork_ev, 0), "fork");
        }
        const size_t ywide = std::max((size_t)qkv_rows, (size_t)d);
        const size_t awide = std::max({(size_t)d, (size_t)nh * hd, (size_t)ff});
        struct Part {
          cudaStream_t s;
          int r0, n, L;
          float *x, *y, *gu, *dn, *qn, *sc, *part, *hx, *as, *has;
          int8_t *aq, *haq;
          uint32_t *tin, *tgt;
        };
        Part hv[kMaxParts];
        for (int k = 0; k < parts; ++k) {
          Part& q = hv[k];
          const size_t r0 = (size_t)k * Lp;
          q.s = k ? split_st[k - 1] : st, q.r0 = (int)r0;
          q.L = parts > 1 ? std::min(Lp, Lc - (int)r0) : Lc, q.n = parts > 1 ? q.L : T;
          q.x = s_x + r0 * d, q.dn = s_dn + r0 * d, q.gu = s_gu + r0 * 2 * ff, q.qn = s_qn + r0 * nh * hd;
          q.sc = s_scores + r0 * nh * seq_sstride, q.part = s_part + r0 * nh * ref_threads * hd;
          q.hx = s_h + r0 * d, q.haq = s_haq + r0 * d, q.has = s_has + r0 * (d / 32);
          q.tin = s_tin + r0, q.tgt = s_tgt + r0;
          q.y = s_y + r0 * ywide, q.aq = s_aq + r0 * awide, q.as = s_as + r0 * (awide / 32);
        }
        for (int k = 0; k < parts; ++k) {
          const Part& q = hv[k];
          launch_seq_gather_tokens(toks_d + (size_t)s0 * stride, stride, q.L, (int)c0 + q.r0, q.n, q.tin, q.tgt, q.s);
          launch_seq_embed(E.v, untied ? nullptr : row_of, q.tin, q.n, vocab, embed_scale, q.x, err, q.s);
        }
        par_mark(PAR_EMBED);
        for (int l = 0; l < nl; ++l) {
          const Layer& Ly = layers[l];
          const Layer* P = l > 0 ? &layers[l - 1] : nullptr;
          for (int k = 0; k < parts; ++k) {
            const Part& q = hv[k];
            launch_seq_norm(q.x, P ? q.dn : nullptr, P ? P->post_ffw : nullptr, Ly.attn_norm, eps, d, q.n, q.aq, q.as, nullptr,
                            q.s);
            par_mark(PAR_NORM);
            product(Ly.qkv, Ly.tqkv, q.aq, q.as, q.n, q.y, qkv_rows, q.s, parts);
            par_mark(PAR_QKV);
            if (k > 0) ck(cudaStreamWaitEvent(q.s, split_ev[(size_t)(k - 1) * nl + l], 0), "layer");
            launch_seq_attn(attn_args(l, 0), q.y, qkv_rows, q.L, ns, pos0 + (uint32_t)q.r0, kv_stride, q.qn, q.sc,
                            seq_sstride, ref_threads, q.part, q.aq, q.as, q.s,
                            k + 1 < parts ? split_ev[(size_t)k * nl + l] : nullptr);
            par_mark(PAR_ATTN);
            product(Ly.o, Ly.to, q.aq, q.as, q.n, q.y, d, q.s, parts);
            par_mark(PAR_O);
            launch_seq_norm(q.x, q.y, Ly.post_attn, Ly.ffn_norm, eps, d, q.n, q.aq, q.as, nullptr, q.s);
            par_mark(PAR_NORM);
            product(Ly.gu, Ly.tgu, q.aq, q.as, q.n, q.gu, 2 * ff, q.s, parts);
            par_mark(PAR_GU);
            launch_seq_glu_quant(q.gu, ff, q.n, silu ? 1 : 0, q.aq, q.as, sms, q.s);
            par_mark(PAR_GLU);
            product(Ly.down, Ly.tdown, q.aq, q.as, q.n, q.dn, d, q.s, parts);
            par_mark(PAR_DOWN);
            nk += 12;  // 2 norms, 4 matrix products, 5 attention kernels, the gate
          }
        }
        for (int k = 0; k < parts; ++k) {
          const Part& q = hv[k];
          launch_seq_norm(q.x, q.dn, layers[nl - 1].post_ffw, out_norm, eps, d, q.n, q.haq, q.has, q.hx, q.s);
        }
        for (int k = 1; k < parts; ++k) {  // the head reads every part's final hidden states
          ck(cudaEventRecord(join_ev[k - 1], split_st[k - 1]), "join");
          ck(cudaStreamWaitEvent(st, join_ev[k - 1], 0), "join");
        }
        par_mark(PAR_NORM);
        if (which < 0) continue;  // prefill only: no head
        nk += 4 + seq_head(which, s_tgt, T, s_lp, s_am);
        par_mark(PAR_HEAD);
        // rows [seq][Lc] of the chunk into [seq][len] of the caller's outputs
        ck(cudaMemcpy2DAsync(lp_d + (size_t)s0 * len + c0, len * 4, s_lp, (size_t)Lc * 4, (size_t)Lc * 4, ns,
                             cudaMemcpyDeviceToDevice, st), "lp");
        if (am_d)
          ck(cudaMemcpy2DAsync(am_d + (size_t)s0 * len + c0, len * 4, s_am, (size_t)Lc * 4, (size_t)Lc * 4, ns,
                               cudaMemcpyDeviceToDevice, st), "am");
      }
    }
    last_launches = nk;
    par_collect();
    // the last position's final hidden state, for later single-token head calls
    ck(cudaMemcpyAsync(h, s_h + (size_t)(T - 1) * d, (size_t)d * 4, cudaMemcpyDeviceToDevice, st), "h");
    ck(cudaMemcpyAsync(haq, s_haq + (size_t)(T - 1) * d, (size_t)d, cudaMemcpyDeviceToDevice, st), "haq");
    ck(cudaMemcpyAsync(has, s_has + (size_t)(T - 1) * (d / 32), (size_t)d / 32 * 4, cudaMemcpyDeviceToDevice, st), "has");
  }

  // The BOS position's K/V rows (position 0 of every layer) from KV slot 0 into slot `s`: every
  // sequence starts with the same BOS forward (main.rs:270-272).
  void copy_bos_kv(int s) {
    const size_t le = (size_t)ctx * nkv * hd, rw = (size_t)nkv * hd;
    for (float* c : {kc, vc})
      ck(cudaMemcpy2DAsync(c + (size_t)s * nl * le, le * 4, c, le * 4, rw * 4, nl, cudaMemcpyDeviceToDevice, st),
         "bos kv");
  }

  // lean.rs:46-107 for `batch` hidden states h_dev (device): greedy tokens by screening the `top` most
  // likely classes and n_always always-on rows (class-ordered row indices, device); with
  // min_conf > 0, items whose most likely class is below it take the full head's argmax over the
  // class-ordered rows. Asynchronous on the model's stream.
  void greedy(const float* h_dev, int batch, int top, float min_conf, const uint32_t* always_dev, int n_always,
              uint32_t* tok_dev, int* fallback_dev) {
    const int nrows = top * per + n_always;
    if ((size_t)batch > gs.batch) {
      gs.q = alloc<int8_t>((size_t)batch * d);
      gs.s = alloc<float>((size_t)batch * d / 32);
      gs.cl = alloc<float>((size_t)batch * k);
      gs.fallback = alloc<int>(batch);
      gs.fb_row = alloc<uint32_t>(batch);
      gs.tok = alloc<uint32_t>(batch);
      gs.lp = alloc<float>(batch);
      gs.zeros = alloc<uint32_t>(batch);
      ck(cudaMemsetAsync(gs.zeros, 0, (size_t)batch * 4, st), "memset");
      gs.batch = batch;
      gs.nrows = 0;
    }
    if ((size_t)batch * nrows > gs.nrows) {
      gs.sel = alloc<uint32_t>((size_t)batch * std::max(top, 1));
      gs.rows = alloc<uint32_t>((size_t)batch * nrows);
      gs.z = alloc<float>((size_t)batch * nrows);
      gs.nrows = (size_t)batch * nrows;
    }
    launch_quantize(h_dev, batch * d, gs.q, gs.s, st);
    launch_seq_class_logits(A, b, k, h_dev, d, batch, gs.cl, st);
    launch_greedy_rank(gs.cl, k, top, min_conf, batch, gs.sel, gs.fallback, st);
    launch_greedy_rowlist(gs.sel, top, per, (uint32_t)blocks.v.rows, always_dev, n_always, batch, gs.rows, st);
    launch_rows_exact(blocks.v, gs.q, gs.s, h_dev, gs.rows, nrows, batch, gs.z, st);
    const bool fb = min_conf > 0.0f;
    if (fb) {  // lean.rs:93-107: the full head over the class-ordered rows, argmax = first maximum
      if ((size_t)batch * vocab > gs.nlogits) {
        gs.logits = alloc<float>((size_t)batch * vocab);
        gs.nlogits = (size_t)batch * vocab;
      }
      if (!seq_gemm_supported(blocks.v)) throw Error(GEM_E_STATE, "the fallback needs a Q8_0/Q4_0 output matrix");
      launch_seq_gemm(blocks.v, gs.q, gs.s, batch, gs.logits, vocab, sms, st);
      launch_seq_logit_reduce(gs.logits, vocab, batch, gs.zeros, nullptr, nullptr, gs.lp, gs.fb_row, err, st);
    }
    launch_greedy_pick(gs.z, gs.rows, top, per, n_always, gs.fallback, fb ? gs.fb_row : nullptr, order, batch, tok_dev, st);
    if (fallback_dev) ck(cudaMemcpyAsync(fallback_dev, gs.fallback, (size_t)batch * 4, cudaMemcpyDeviceToDevice, st), "fb");
  }

  // TwoLevel::sample (main.rs:109-141) on the last forward's hidden state (h, haq, has).
  uint32_t sample(float temp, uint64_t* rng_host) {
    if (gs.batch < 1) greedy_scratch_min();
    if (!gs.rng) gs.rng = alloc<unsigned long long>(1);
    if (gs.nrows < (size_t)per) {
      gs.sel = alloc<uint32_t>(1);
      gs.rows = alloc<uint32_t>(per);
      gs.z = alloc<float>(per);
      gs.nrows = per;
    }
    ck(cudaMemcpyAsync(gs.rng, rng_host, 8, cudaMemcpyHostToDevice, st), "rng");
    launch_seq_class_logits(A, b, k, h, d, 1, gs.cl, st);
    launch_sample_class(gs.cl, k, temp, gs.rng, gs.sel, st);
    launch_greedy_rowlist(gs.sel, 1, per, (uint32_t)blocks.v.rows, nullptr, 0, 1, gs.rows, st);
    launch_rows_exact(blocks.v, haq, has, h, gs.rows, per, 1, gs.z, st);
    launch_sample_member(gs.z, per, (uint32_t)blocks.v.rows, gs.sel, temp, gs.rng, order, gs.tok, st);
    uint32_t t = 0;
    ck(cudaMemcpyAsync(&t, gs.tok, 4, cudaMemcpyDeviceToHost, st), "tok");
    ck(cudaMemcpyAsync(rng_host, gs.rng, 8, cudaMemcpyDeviceToHost, st), "rng");
    sync();
    return t;
  }
  void greedy_scratch_min() {
    gs.q = alloc<int8_t>(d);
    gs.s = alloc<float>(d / 32);
    gs.cl = alloc<float>(k);
    gs.fallback = alloc<int>(1);
    gs.fb_row = alloc<uint32_t>(1);
    gs.tok = alloc<uint32_t>(1);
    gs.lp = alloc<float>(1);
    gs.zeros = alloc<uint32_t>(1);
    ck(cudaMemsetAsync(gs.zeros, 0, 4, st), "memset");
    gs.batch = 1;
    gs.nrows = 0;
  }

  // Can the two-level scoring loop run as one layer-pipelined kernel on this model and GPU?
  bool pipeline_supported() {
    pipe_why.clear();
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device);
    if (!exact) pipe_why = "fast numerics";
    else if (!two) pipe_why = "no two-level head";
    else if (untied) pipe_why = "separate output matrix";
    else if (!coop) pipe_why = "no cooperative launch";
    else if (nh > 16 || nh + nkv > 15 || hd > 256) pipe_why = "head counts";
    else if (nl + 1 > sms) pipe_why = "more layers than SMs";
    else if (((nh + 2 * nkv) * hd) % 16 || d % 16 || ff % 32) pipe_why = "projection rows not in 16-row groups";
    return pipe_why.empty();
  }

  void setup_pipeline() {
    if (pipe_ready) return;
    PipeArgs& P = pipe;
    P = PipeArgs{};
    P.nl = nl, P.d = d, P.nh = nh, P.nkv = nkv, P.hd = hd, P.ff = ff, P.ctx = ctx, P.vocab = vocab;
    bool any_global = false;
    for (auto& L : layers) any_global |= !L.swa;
    P.max_npos = (any_global || window <= 0) ? ctx : std::min(window, ctx);
    P.eps = eps, P.qscale = 1.0f / std::sqrt((float)hd), P.embed_scale = embed_scale, P.silu = silu ? 1 : 0;
    P.layers_bits = layers[0].qkv.v.bits, P.layers_scale_f32 = layers[0].qkv.v.scale_f32;
    P.emb = head.v;
    P.emb_row = row_of;
    P.blocks = blocks.v;
    P.A = A, P.b = b, P.out_norm = out_norm, P.cls_of = cls_of, P.pos_of = pos_of, P.order = order;
    P.k = k, P.per = per;
    P.ref_threads = ref_threads;
    // CTAs per stage in proportion to the bytes each stage reads per token
    double layer_bytes = (double)body_bytes / nl + (double)P.max_npos / 2 * nkv * hd * 8;
    double head_bytes = (double)k * d * 4 + 2.0 * per * (blocks.bytes / std::max(1, blocks.v.rows));
    int G = std::max(1, (int)std::floor(sms / (nl + head_bytes / layer_bytes)));
    while (G > 1 && nl * G + 1 > sms) --G;
    P.G = G;
    P.GH = std::max(1, std::min(sms - nl * G, 32));
    std::vector<PipeLayer> pl(nl);
    size_t layer_elems = (size_t)ctx * nkv * hd;
    for (int l = 0; l < nl; ++l) {
      const Layer& L = layers[l];
      PipeLayer& q = pl[l];
      q.qkv = L.qkv.v, q.o = L.o.v, q.gu = L.gu.v, q.down = L.down.v;
      q.attn_norm = L.attn_norm, q.q_norm = L.q_norm, q.k_norm = L.k_norm, q.post_attn = L.post_attn;
      q.ffn_norm = L.ffn_norm, q.post_ffw = L.post_ffw, q.bqkv = L.bqkv;
      q.rope_sin = rope_sin[L.swa ? 0 : 1], q.rope_cos = rope_cos[L.swa ? 0 : 1];
      q.kcache = kc + (size_t)l * layer_elems;
      q.vcache = vc + (size_t)l * layer_elems;
      q.window = L.swa ? window : 0;
    }
    P.layers = upload(pl);
    P.ring = alloc<float>((size_t)(nl + 1) * PIPE_RING * d);
    P.ready = alloc<unsigned>((size_t)(nl + 1) * PIPE_RING);
    P.consumed = alloc<unsigned>((size_t)(nl + 1));
    P.bar = alloc<unsigned>((size_t)(nl + 1) * 32);
    P.scratch_stride = pipe_scratch_floats(nh, nkv, hd, d, ff, P.max_npos, ref_threads);
    P.scratch = alloc<float>(P.scratch_stride * nl);
    P.head_scratch = alloc<float>((size_t)k + 2 * per);
    P.err = err;
    P.checks = std::getenv("GEM_PIPELINE_CHECKS") ? 1 : 0;  // index self-checks (debugging aid)
    // weight ring: a slot holds one 16-row group of the widest projection (plus its scales)
    int max_stride = 0, max_sbytes = 0;
    for (const MatView* w : {&layers[0].qkv.v, &layers[0].o.v, &layers[0].gu.v, &layers[0].down.v}) {
      int rb = w->cols * w->bits / 8;
      max_stride = std::max(max_stride, rb + 32);
      max_sbytes = std::max(max_sbytes, w->bits == 16 ? 0 : (w->cols / 32) * (w->scale_f32 ? 4 : 2));
    }
    P.slot_scale_off = 16 * max_stride;
    P.slot_bytes = (16 * max_stride + 16 * max_sbytes + 127) / 128 * 128;
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    P.ring_slots = 0;
    for (int ns = 8; ns >= 2; --ns) {
      P.ring_slots = ns;
      if (pipe_smem_bytes(P) <= (size_t)optin) break;
      P.ring_slots = 0;
    }
    // The shared-memory weight ring measured slower than direct loads on the 270M workload (7.2k vs
    // 10.6k tokens/s): its refills arrive in bursts that slow the latency-bound phases around them.
    // It stays available for tuning (GEM_PIPE_RING_SLOTS=n) and is off by default.
    int want = 0;
    if (const char* e = std::getenv("GEM_PIPE_RING_SLOTS")) want = std::max(0, std::atoi(e));
    P.ring_slots = std::min(P.ring_slots, want);
    pipe_smem = std::max(pipe_smem_bytes(P), (size_t)120 * 1024);  // > half an SM: one CTA per SM
    pipe_ready = true;
  }

  // The scoring loop as one pipelined kernel on device buffers (toks: n + 1 ids).
  bool try_pipeline(const uint32_t* toks_d, size_t n, uint32_t base_pos, float* lp_d, uint32_t* am_d) {
    if (schedule == GEM_SCHEDULE_SEQUENTIAL || schedule == GEM_SCHEDULE_PARALLEL || !pipeline_supported()) return false;
    setup_pipeline();
    PipeArgs P = pipe;
    P.ref_threads = ref_threads;
    P.toks = toks_d, P.n = (int)n, P.base_pos = (int)base_pos, P.lp_out = lp_d, P.am_out = am_d, P.h_last = h;
    P.wait_ns = wait_ns;
    P.withhold_stage = withhold_stage;
    P.prof = prof;
    P.prof_from = 16;
    ck(cudaMemsetAsync(P.ready, 0, (size_t)(nl + 1) * PIPE_RING * sizeof(unsigned), st), "memset");
    ck(cudaMemsetAsync(P.consumed, 0, (size_t)(nl + 1) * sizeof(unsigned), st), "memset");
    ck(cudaMemsetAsync(P.bar, 0, (size_t)(nl + 1) * 32 * sizeof(unsigned), st), "memset");
    int rc = launch_pipe_score(P, pipe_smem, st);
    if (rc == -1) {
      pipe_why = "weight formats without a pipelined instantiation";
      return false;
    }
    if (rc != 0) throw Error(GEM_E_CUDA, std::string("pipelined launch: ") + cudaGetErrorString((cudaError_t)rc));
    launch_quantize(h, d, haq, has, st);  // the last token's hidden state, for later head calls
    return true;
  }

  void check_launch() { ck(cudaGetLastError(), "kernel launch"); }
  void sync() {
    ck(cudaStreamSynchronize(st), "stream sync");
    int e = 0;
    ck(cudaMemcpy(&e, err, sizeof(int), cudaMemcpyDeviceToHost), "error word");
    if (e != 0) {
      ck(cudaMemset(err, 0, sizeof(int)), "error word");
      if (e == ERR_RANGE) throw Error(GEM_E_RANGE, "a token or target id in device memory was >= vocab (replaced by 0)");
      throw Error(GEM_E_TIMEOUT, "a device-side wait gave up");
    }
  }
};

namespace {

}  // namespace

namespace gem {
bool model_head_view(const gem_model* m, ModelHeadView* out) {
  if (!m || !out) return false;
  out->w = m->head.v;
  out->row_of = m->row_of, out->row_tok = m->row_tok();
  out->exact = m->exact;
  out->st = m->st;
  out->sms = m->sms;
  out->device = m->device;
  out->d = m->d;
  out->err = m->err;
  return true;
}
void set_last_error(const std::string& msg) { g_last_error = msg; }
}  // namespace gem

namespace {

int fail_with(const std::exception& e) {
  g_last_error = e.what();
  if (auto* ge = dynamic_cast<const Error*>(&e)) return ge->code;
  return GEM_E_ARG;
}
#define API_BEGIN try {
#define API_END                        \
  }                                    \
  catch (const std::exception& e) {    \
    return fail_with(e);               \
  }                                    \
  return GEM_OK;

void rope_tables(gem_model* m, float base_model) {  // model.rs:228, 297-301
  float bases[2] = {10000.0f, base_model};
  int half = m->hd / 2;
  for (int t = 0; t < 2; ++t) {
    std::vector<float> inv(half), sn((size_t)m->ctx * half), cs((size_t)m->ctx * half);
    for (int i = 0; i < half; ++i) inv[i] = std::pow(bases[t], -2.0f * (float)i / (float)m->hd);
    for (int p = 0; p < m->ctx; ++p)
      for (int i = 0; i < half; ++i) {
        float a = (float)p * inv[i];
        sn[(size_t)p * half + i] = std::sin(a);
        cs[(size_t)p * half + i] = std::cos(a);
      }
    m->rope_sin[t] = m->upload(sn);
    m->rope_cos[t] = m->upload(cs);
  }
}

// Gemma::load's metadata (model.rs:154-170, 191, 207-209); host-only, so a bad file fails before
// any device work.
void read_meta(gem_model* m, const Gguf& g, int ctx) {
  std::string a = g.text("general.architecture");
  bool gemma = a == "gemma3";
  if (!gemma && a != "qwen2") throw Error(GEM_E_FORMAT, "unsupported architecture " + a);
  m->gemma = gemma;
  m->d = (int)g.u(a + ".embedding_length");
  m->nl = (int)g.u(a + ".block_count");
  m->nh = (int)g.u(a + ".attention.head_count");
  m->nkv = (int)g.u(a + ".attention.head_count_kv");
  m->hd = (int)g.u_or(a + ".attention.key_length", m->d / std::max(1, m->nh));
  m->ff = (int)g.u(a + ".feed_forward_length");
  m->eps = g.f(a + ".attention.layer_norm_rms_epsilon");
  m->window = (int)g.u_or(a + ".attention.sliding_window", 0);
  m->rope_base = g.f(a + ".rope.freq_base");
  m->bos = g.flag("tokenizer.ggml.add_bos_token") ? (int64_t)g.u("tokenizer.ggml.bos_token_id") : -1;
  m->embed_scale = gemma ? std::sqrt((float)m->d) : 1.0f;
  m->silu = !gemma;
  m->ctx = ctx;
  if (m->nl <= 0 || m->nh <= 0 || m->nkv <= 0 || m->nh % m->nkv) throw Error(GEM_E_FORMAT, "bad head counts");
  if (m->nh / m->nkv > 8) throw Error(GEM_E_FORMAT, "more than 8 query heads per kv head");
  if (m->hd % 32 || m->hd > 256 || m->d % 32 || m->ff % 32) throw Error(GEM_E_FORMAT, "unsupported dimensions");
  if (ctx <= 0) throw Error(GEM_E_ARG, "ctx must be positive");
  const char* need[] = {"output_norm.weight", "blk.0.attn_q.weight", "blk.0.ffn_down.weight"};
  for (const char* n : need) (void)g.info(n);
  if (!g.has("token_embd.weight") && !g.has("output.weight")) throw Error(GEM_E_FORMAT, "no output matrix");
}

void load_model(gem_model* m, const Gguf& g, int body_bits, int head_bits) {
  bool has_out = g.has("output.weight");
  bool gemma = m->gemma;
  float base = m->rope_base;
  // output matrix (head) and embedding
  HostMat head = load_mat(g, has_out ? "output.weight" : "token_embd.weight");
  if (has_out) {  // tie = false: the embedding is its own matrix (model.rs:155-157, 255-257)
    m->untied = true;
    HostMat e = load_mat(g, "token_embd.weight");
    m->emb = upload_mat(e, m->owned);
  }
  // requantize_head (model.rs:259-266); body_bits requantizes only the projections (main.rs:209)
  if (head_bits == 8) head = to_q8(head);
  else if (head_bits == 4) head = to_q4(head);
  else if (head_bits != 0) throw Error(GEM_E_ARG, "head_bits must be 0, 4 or 8");
  if (body_bits != 8 && body_bits != 4) throw Error(GEM_E_ARG, "body_bits must be 8 or 4");
  m->head = upload_mat(head, m->owned);
  if (head_bulk_supported(m->head.v)) {  // the streamed full head's copy, built once (never during a capture)
    const size_t ng = ((size_t)m->head.v.rows + 15) / 16, nb = m->head.v.cols / 32;
    m->head_bulk_q = m->alloc<unsigned char>(ng * nb * 512);
    m->head_bulk_s = m->alloc<__half>(ng * nb * 16);
    launch_head_bulk_layout(m->head.v, m->head_bulk_q, m->head_bulk_s, 0);
    ck(cudaStreamSynchronize(0), "head layout");  // done before any use on the model's (non-blocking) stream
  }
  m->vocab = (int)head.rows;
  m->head_bits = head.bits;
  if (head.cols != (size_t)m->d) throw Error(GEM_E_FORMAT, "output matrix width != embedding_length");

  m->layers.resize(m->nl);
  m->body_bytes = 0;
  for (int l = 0; l < m->nl; ++l) {
    auto p = [&](const char* s) { return "blk." + std::to_string(l) + "." + s; };
    HostMat mq = load_mat(g, p("attn_q.weight")), mk = load_mat(g, p("attn_k.weight")), mv = load_mat(g, p("attn_v.weight"));
    HostMat mo = load_mat(g, p("attn_output.weight"));
    HostMat mg = load_mat(g, p("ffn_gate.weight")), mu = load_mat(g, p("ffn_up.weight")), md = load_mat(g, p("ffn_down.weight"));
    if (body_bits == 4)  // requantize(body4) (model.rs:268-279)
      for (HostMat* x : {&mq, &mk, &mv, &mo, &mg, &mu, &md}) *x = to_q4(*x);
    if ((int)mq.rows != m->nh * m->hd || (int)mk.rows != m->nkv * m->hd || (int)mv.rows != m->nkv * m->hd ||
        (int)mo.rows != m->d || (int)mo.cols != m->nh * m->hd || (int)mg.rows != m->ff || (int)md.cols != m->ff)
      throw Error(GEM_E_FORMAT, "layer " + std::to_string(l) + ": projection shapes do not match the metadata");
    for (HostMat* x : {&mq, &mk, &mv, &mo, &mg, &mu, &md}) m->body_bytes += canonical_bytes(*x);
    // an odd number of f16 scales per row cannot be staged in 4-byte pieces: such planes are widened
    // to f32 (exact), which every kernel reads the same way
    for (HostMat* x : {&mq, &mk, &mv, &mo, &mg, &mu, &md})
      if (x->bits != 16 && !x->scale_f32() && (x->cols / 32) % 2) {
        x->s32.resize(x->s16.size());
        for (size_t i = 0; i < x->s16.size(); ++i) x->s32[i] = f16_value(x->s16[i]);
        x->s16.clear();
      }
    Layer& L = m->layers[l];
    L.qkv = upload_mat(concat_rows({&mq, &mk, &mv}), m->owned);
    L.o = upload_mat(mo, m->owned);
    L.gu = upload_mat(concat_rows({&mg, &mu}), m->owned);
    L.down = upload_mat(md, m->owned);
    L.attn_norm = m->upload_or_null(g.f32s(p("attn_norm.weight")));
    L.q_norm = m->upload_or_null(g.f32s_or_empty(p("attn_q_norm.weight")));
    L.k_norm = m->upload_or_null(g.f32s_or_empty(p("attn_k_norm.weight")));
    L.post_attn = m->upload_or_null(g.f32s_or_empty(p("post_attention_norm.weight")));
    L.ffn_norm = m->upload_or_null(g.f32s(p("ffn_norm.weight")));
    L.post_ffw = m->upload_or_null(g.f32s_or_empty(p("post_ffw_norm.weight")));
    std::vector<float> bq = g.f32s_or_empty(p("attn_q.bias")), bk = g.f32s_or_empty(p("attn_k.bias")), bv = g.f32s_or_empty(p("attn_v.bias"));
    if (!bq.empty() || !bk.empty() || !bv.empty()) {
      std::vector<float> all(mq.rows + mk.rows + mv.rows, 0.0f);
      std::copy(bq.begin(), bq.end(), all.begin());
      std::copy(bk.begin(), bk.end(), all.begin() + mq.rows);
      std::copy(bv.begin(), bv.end(), all.begin() + mq.rows + mk.rows);
      L.bqkv = m->upload(all);
    }
    L.swa = gemma && l % 6 < 5;  // model.rs:191
    auto sub = [](const DevMat& M, int r0, int rows) {
      DevMat v = M;
      size_t rb = (size_t)M.v.cols * M.v.bits / 8;
      v.v.q = (const uint8_t*)M.v.q + (size_t)r0 * rb;
      if (M.v.s) v.v.s = (const uint8_t*)M.v.s + (size_t)r0 * (M.v.cols / 32) * (M.v.scale_f32 ? 4 : 2);
      v.v.rows = rows;
      return v;
    };
    L.q_only = sub(L.qkv, 0, (int)mq.rows);
    L.k_only = sub(L.qkv, (int)mq.rows, (int)mk.rows);
    L.v_only = sub(L.qkv, (int)(mq.rows + mk.rows), (int)mv.rows);
    L.gate_only = sub(L.gu, 0, (int)mg.rows);
    L.up_only = sub(L.gu, (int)mg.rows, (int)mu.rows);
  }
  m->body_bits = m->layers[0].qkv.v.bits;
  std::vector<float> on = g.f32s("output_norm.weight");
  if ((int)on.size() != m->d) throw Error(GEM_E_FORMAT, "output_norm size");
  m->out_norm = m->upload(on);
  rope_tables(m, base);

  // KV caches and scratch
  size_t kv = (size_t)m->max_seqs * m->nl * m->ctx * m->nkv * m->hd;
  m->kc = m->alloc<float>(kv);
  m->vc = m->alloc<float>(kv);
  ck(cudaMemset(m->kc, 0, kv * 4), "memset");
  ck(cudaMemset(m->vc, 0, kv * 4), "memset");
  int max_npos_swa = m->window > 0 ? std::min(m->window, m->ctx) : m->ctx;
  m->chunk = 64;
  while ((m->ctx + m->chunk - 1) / m->chunk > 64) m->chunk *= 2;
  m->nsplit_swa = (max_npos_swa + m->chunk - 1) / m->chunk;
  m->nsplit_glob = (m->ctx + m->chunk - 1) / m->chunk;
  int G = m->nh / m->nkv;
  int qkv_rows = (m->nh + 2 * m->nkv) * m->hd;
  int wide = std::max({m->d, m->nh * m->hd, m->ff});
  m->x = m->alloc<float>(m->d);
  m->xn = m->alloc<float>(m->d);
  m->qkv = m->alloc<float>(qkv_rows);
  m->att = m->alloc<float>(m->nh * m->hd);
  m->o = m->alloc<float>(m->d);
  m->gu = m->alloc<float>(2 * (size_t)m->ff);
  m->g = m->alloc<float>(m->ff);
  m->dn = m->alloc<float>(m->d);
  m->h = m->alloc<float>(m->d);
  m->part = m->alloc<float>((size_t)m->nkv * m->nsplit_glob * G * (m->hd + 2));
  m->aq_d = m->alloc<int8_t>(wide);
  m->aq_att = m->alloc<int8_t>(wide);
  m->aq_ff = m->alloc<int8_t>(wide);
  m->haq = m->alloc<int8_t>(m->d);
  m->as_d = m->alloc<float>(wide / 32);
  m->as_att = m->alloc<float>(wide / 32);
  m->as_ff = m->alloc<float>(wide / 32);
  m->has = m->alloc<float>(m->d / 32);
  m->qn = m->alloc<float>((size_t)m->nh * m->hd);
  m->scores = m->alloc<float>((size_t)m->nh * m->ctx);
  m->cur = m->alloc<StepCur>(1);
  m->err = m->alloc<int>(1);
  ck(cudaMemset(m->err, 0, sizeof(int)), "memset");
  ck(cudaMallocHost(&m->cur_host, sizeof(StepCur)), "cudaMallocHost");
  m->step = m->alloc<uint32_t>(1);
  m->toks = m->alloc<uint32_t>((size_t)m->ctx + 1);
  m->lp = m->alloc<float>(m->ctx);
  m->am = m->alloc<uint32_t>(m->ctx);
  m->ensure_head_batch(1);
}

std::vector<uint8_t> read_all(const std::string& p) {
  std::ifstream f(p, std::ios::binary);
  if (!f) throw Error(GEM_E_IO, p + ": cannot open");
  return std::vector<uint8_t>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

}  // namespace

extern "C" {

const char* gem_last_error(void) { return g_last_error.c_str(); }
int gem_version(void) { return 1; }

int gem_open(const char* gguf_path, int ctx, int body_bits, int head_bits, int device, int max_seqs, gem_model** out) {
  API_BEGIN
  if (!gguf_path || !out) throw Error(GEM_E_ARG, "null argument");
  *out = nullptr;
  if (max_seqs < 1) throw Error(GEM_E_ARG, "max_seqs must be >= 1");
  if (body_bits != 8 && body_bits != 4) throw Error(GEM_E_ARG, "body_bits must be 8 or 4");
  if (head_bits != 0 && head_bits != 8 && head_bits != 4) throw Error(GEM_E_ARG, "head_bits must be 0, 4 or 8");
  auto m = std::make_unique<gem_model>();
  Gguf g(gguf_path);
  read_meta(m.get(), g, ctx);
  ck(cudaSetDevice(device), "cudaSetDevice");
  m->device = device;
  m->max_seqs = max_seqs;
  ck(cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, device), "device attribute");
  ck(cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking), "stream");
  load_model(m.get(), g, body_bits, head_bits);
  ck(cudaDeviceSynchronize(), "load");
  if (const char* e = std::getenv("GEM_TC"); e && std::atoi(e) == 1 && m->seq_supported()) {
    m->ensure_tc();
    m->tc = true;
  }
  *out = m.release();
  API_END
}

int gem_open_twolevel(gem_model* m, const char* prefix) {
  API_BEGIN
  if (!m || !prefix) throw Error(GEM_E_ARG, "null argument");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  std::string p(prefix);
  auto ob = read_all(p + ".order"), ab = read_all(p + ".A"), bb = read_all(p + ".b");
  if (ob.size() % 4 || ab.size() % 4 || bb.size() % 4) throw Error(GEM_E_FORMAT, "class files are not whole 32-bit words");
  std::vector<uint32_t> order(ob.size() / 4);
  std::memcpy(order.data(), ob.data(), ob.size());
  std::vector<float> A(ab.size() / 4), b(bb.size() / 4);
  std::memcpy(A.data(), ab.data(), ab.size());
  std::memcpy(b.data(), bb.data(), bb.size());
  // TwoLevel::load (main.rs:57-76)
  size_t k = b.size();
  if (k == 0) throw Error(GEM_E_FORMAT, ".b is empty");
  size_t per = (order.size() + k - 1) / k;
  size_t chunks = (order.size() + per - 1) / per;
  if (chunks != k) throw Error(GEM_E_FORMAT, ".order does not cut into as many classes as .b has entries");
  if (A.size() != k * (size_t)m->d) throw Error(GEM_E_FORMAT, ".A is not classes x d floats");
  std::vector<uint32_t> cls_of(m->vocab, 0), pos_of(m->vocab, 0);
  for (size_t i = 0; i < order.size(); ++i) {
    if (order[i] >= (uint32_t)m->vocab) throw Error(GEM_E_FORMAT, ".order holds a token id >= vocab");
    cls_of[order[i]] = (uint32_t)(i / per);
    pos_of[order[i]] = (uint32_t)(i % per);
  }
  // TwoLevel::load gathers the class blocks (main.rs:74); permute_head (model.rs:242-249, q8.rs:65-91)
  // then keeps the output matrix once, in class order. Here, when the class file covers every token
  // once, the rows are gathered on the device into class order (from the current order, if an earlier
  // class file permuted them) and the previous rows released: a second copy exists only during the
  // gather, and the class blocks are views into the one matrix. Otherwise the blocks are a copy.
  m->drop_graphs();
  const bool old_blocks_copy = m->two && m->blocks.v.q && m->blocks.v.q != m->head.v.q;
  const DevMat old_blocks = m->blocks;
  std::vector<uint32_t> src(order.size()), new_row_of(m->vocab, 0xffffffffu);
  bool perm = order.size() == (size_t)m->vocab;
  for (size_t i = 0; i < order.size(); ++i) {
    src[i] = m->row_of_h.empty() ? order[i] : m->row_of_h[order[i]];
    if (perm && new_row_of[order[i]] != 0xffffffffu) perm = false;  // a token in two classes
    if (perm) new_row_of[order[i]] = (uint32_t)i;
  }
  const MatView& hv = m->head.v;
  const size_t rb = (size_t)hv.cols * hv.bits / 8, sb = hv.bits == 16 ? 0 : (size_t)(hv.cols / 32) * (hv.scale_f32 ? 4 : 2);
  uint32_t* d_src = m->upload(src);
  DevMat gathered;
  gathered.v = hv;
  gathered.v.rows = (int)order.size();
  gathered.v.q = m->alloc<unsigned char>(order.size() * rb);
  gathered.v.s = sb ? m->alloc<unsigned char>(order.size() * sb) : nullptr;
  gathered.bytes = order.size() * (rb + sb);
  launch_gather_rows(hv, d_src, gathered.v, m->st);
  ck(cudaGetLastError(), "gather class blocks");
  ck(cudaStreamSynchronize(m->st), "gather class blocks");
  m->release(d_src);
  if (old_blocks_copy) {  // an earlier class file's blocks
    m->release(old_blocks.v.q);
    if (old_blocks.v.s) m->release(old_blocks.v.s);
  }
  if (perm) {
    m->release(m->head.v.q);
    if (m->head.v.s) m->release(m->head.v.s);
    if (m->row_of) m->release(m->row_of);
    m->head = gathered;
    m->row_of = m->upload(new_row_of);
    m->row_of_h = std::move(new_row_of);
    if (m->head_bulk_q) {  // the streamed full head's copy follows the rows' new order
      launch_head_bulk_layout(m->head.v, m->head_bulk_q, m->head_bulk_s, m->st);
      ck(cudaStreamSynchronize(m->st), "head layout");
    }
  }
  m->blocks = gathered;
  for (const void* p : {(const void*)m->A, (const void*)m->b, (const void*)m->cls_of, (const void*)m->pos_of,
                        (const void*)m->order})
    if (p) m->release(p);
  m->A = m->upload(A);
  m->b = m->upload(b);
  m->cls_of = m->upload(cls_of);
  m->pos_of = m->upload(pos_of);
  m->order = m->upload(order);
  m->k = (int)k;
  m->per = (int)per;
  m->two = true;
  m->pipe_ready = false;
  m->hbatch = 0;
  m->ensure_head_batch(1);
  m->drop_graphs();
  ck(cudaDeviceSynchronize(), "twolevel load");
  API_END
}

void gem_close(gem_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  delete m;
}

int gem_get_info(const gem_model* m, gem_info* o) {
  API_BEGIN
  if (!m || !o) throw Error(GEM_E_ARG, "null argument");
  o->d = m->d, o->vocab = m->vocab, o->layers = m->nl, o->n_heads = m->nh, o->n_kv_heads = m->nkv;
  o->head_dim = m->hd, o->ffn = m->ff, o->ctx = m->ctx, o->window = m->window, o->bos = m->bos;
  o->body_bits = m->body_bits, o->head_bits = m->head_bits, o->classes = m->two ? m->k : 0, o->per = m->two ? m->per : 0;
  o->max_seqs = m->max_seqs, o->body_bytes = (int64_t)m->body_bytes, o->head_bytes = (int64_t)m->head.bytes, o->device = m->device;
  o->kernels_per_token_full = m->graph_kernels[0];
  o->kernels_per_token_twolevel = m->graph_kernels[1];
  API_END
}

int gem_reset(gem_model* m, int seq) {
  API_BEGIN
  if (!m) throw Error(GEM_E_ARG, "null argument");
  if (seq < 0 || seq >= m->max_seqs) throw Error(GEM_E_RANGE, "sequence index out of range");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  size_t per_seq = (size_t)m->nl * m->ctx * m->nkv * m->hd;
  ck(cudaMemsetAsync(m->kc + (size_t)seq * per_seq, 0, per_seq * 4, m->st), "memset");
  ck(cudaMemsetAsync(m->vc + (size_t)seq * per_seq, 0, per_seq * 4, m->st), "memset");
  m->sync();
  API_END
}

int gem_set_numerics(gem_model* m, int mode, int ref_threads) {
  API_BEGIN
  if (!m) throw Error(GEM_E_ARG, "null argument");
  if (mode != GEM_NUMERICS_EXACT && mode != GEM_NUMERICS_FAST) throw Error(GEM_E_ARG, "unknown numerics mode");
  if (ref_threads < 1 || ref_threads > 1024) throw Error(GEM_E_ARG, "ref_threads must be in 1..1024");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  m->sync();
  m->exact = mode == GEM_NUMERICS_EXACT;
  if (m->ref_threads != ref_threads) m->pipe_ready = false;  // scratch is sized by the pool size
  m->ref_threads = ref_threads;
  m->drop_graphs();
  API_END
}

int gem_set_schedule(gem_model* m, int schedule) {
  API_BEGIN
  if (!m) throw Error(GEM_E_ARG, "null argument");
  if (schedule < GEM_SCHEDULE_AUTO || schedule > GEM_SCHEDULE_PARALLEL) throw Error(GEM_E_ARG, "unknown schedule");
  m->schedule = schedule;
  API_END
}

int gem_set_tensor_cores(gem_model* m, int on) {
  API_BEGIN
  if (!m) throw Error(GEM_E_ARG, "null argument");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  m->sync();
  if (on) m->ensure_tc();
  m->tc = on != 0;
  m->drop_graphs();  // a replayed graph holds the other products' launches
  API_END
}

int gem_get_schedule(gem_model* m, int head, int* pipelined, int* stages_ctas) {
  API_BEGIN
  if (!m) throw Error(GEM_E_ARG, "null argument");
  const bool parallel = (m->schedule == GEM_SCHEDULE_AUTO || m->schedule == GEM_SCHEDULE_PARALLEL) && m->seq_supported();
  bool ok = head == 1 && !parallel && (m->schedule == GEM_SCHEDULE_AUTO || m->schedule == GEM_SCHEDULE_PIPELINED) &&
            m->pipeline_supported();
  if (ok) m->setup_pipeline();
  if (parallel) m->pipe_why = "sequence-parallel schedule";
  if (pipelined) *pipelined = ok ? 1 : 0;
  if (stages_ctas) {
    stages_ctas[0] = ok ? m->pipe.G : 0;
    stages_ctas[1] = ok ? m->pipe.GH : 0;
  }
  if (!ok && m->pipe_why.empty()) m->pipe_why = head == 1 ? "sequential schedule requested" : "full head";
  g_last_error = ok ? std::string("pipelined") : m->pipe_why;
  API_END
}

int gem_get_schedule_kind(gem_model* m, int head, int* kind) {
  API_BEGIN
  if (!m || !kind) throw Error(GEM_E_ARG, "null argument");
  if (head != 0 && head != 1) throw Error(GEM_E_ARG, "head must be 0 (full) or 1 (two-level)");
  if ((m->schedule == GEM_SCHEDULE_AUTO || m->schedule == GEM_SCHEDULE_PARALLEL) && m->seq_supported()) {
    *kind = GEM_SCHEDULE_PARALLEL;
    g_last_error = "sequence-parallel";
  } else if (head == 1 && (m->schedule == GEM_SCHEDULE_AUTO || m->schedule == GEM_SCHEDULE_PIPELINED) &&
             m->pipeline_supported()) {
    *kind = GEM_SCHEDULE_PIPELINED;
    g_last_error = "pipelined";
  } else {
    *kind = GEM_SCHEDULE_SEQUENTIAL;
    g_last_error = !m->seq_why.empty() ? m->seq_why : m->pipe_why;
  }
  API_END
}

int gem_nccl_unique_id(void* id_out) {
  API_BEGIN
  if (!id_out) throw Error(GEM_E_ARG, "null argument");
  if (!nccl().load()) throw Error(GEM_E_STATE, std::string("libnccl.so.2 not loadable: ") + dlerror());
  ncclUniqueId id;
  const ncclResult_t r = nccl().get_id(&id);
  if (r != ncclSuccess) throw Error(GEM_E_NCCL, std::string("ncclGetUniqueId: ") + nccl().error_string(r));
  std::memcpy(id_out, &id, sizeof(id));
  API_END
}

int gem_shard_init(gem_model* m, int nranks, int rank, const void* id) {
  API_BEGIN
  if (!m || !id) throw Error(GEM_E_ARG, "null argument");
  if (nranks < 1 || rank < 0 || rank >= nranks) throw Error(GEM_E_RANGE, "rank out of range");
  if (m->comm) throw Error(GEM_E_STATE, "the head is already sharded");
  if (!nccl().load()) throw Error(GEM_E_STATE, std::string("libnccl.so.2 not loadable: ") + dlerror());
  if (m->head.v.bits == 16 || (!m->head.v.scale_f32 && (m->head.v.cols / 32) % 2))
    throw Error(GEM_E_STATE, "vocab sharding needs a Q8_0/Q4_0 output matrix");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  m->sync();
  const int per = (m->vocab + nranks - 1) / nranks;
  m->shard_row0 = std::min(m->vocab, rank * per);
  m->shard_rows = std::min(per, m->vocab - m->shard_row0);
  if (m->shard_rows <= 0) throw Error(GEM_E_RANGE, "more ranks than vocabulary rows");
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  const ncclResult_t r = nccl().init_rank(&c, nranks, uid, rank);
  if (r != ncclSuccess) throw Error(GEM_E_NCCL, std::string("ncclCommInitRank: ") + nccl().error_string(r));
  m->comm = c;
  m->shard_rank = rank, m->shard_n = nranks;
  API_END
}

int gem_set_profiling(gem_model* m, int on) {
  API_BEGIN
  if (!m) throw Error(GEM_E_ARG, "null argument");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  if (on && !m->prof) m->prof = m->alloc<unsigned long long>((size_t)(m->nl + 1) * PIPE_PHASES);
  if (on) ck(cudaMemsetAsync(m->prof, 0, (size_t)(m->nl + 1) * PIPE_PHASES * 8, m->st), "memset");
  if (!on) m->prof = nullptr;  // the buffer stays owned by the model
  m->par_prof = on != 0;
  for (double& v : m->par_us) v = 0;
  m->par_calls = 0;
  m->sync();
  API_END
}

int gem_get_parallel_profile(gem_model* m, double* us, int n) {
  API_BEGIN
  if (!m || !us) throw Error(GEM_E_ARG, "null argument");
  if (!m->par_prof) throw Error(GEM_E_STATE, "profiling is off");
  for (int i = 0; i < n && i < gem_model::PAR_CATS; ++i) us[i] = m->par_calls ? m->par_us[i] / (double)m->par_calls : 0.0;
  API_END
}

int gem_get_last_launches(gem_model* m, int64_t* n) {
  API_BEGIN
  if (!m || !n) throw Error(GEM_E_ARG, "null argument");
  *n = m->last_launches;
  API_END
}

int gem_get_phase_profile(gem_model* m, double* layer_us, int n_layer, double* head_us, int n_head) {
  API_BEGIN
  if (!m || !m->prof) throw Error(GEM_E_STATE, "profiling is off");
  m->sync();
  std::vector<unsigned long long> h((size_t)(m->nl + 1) * PIPE_PHASES);
  ck(cudaMemcpy(h.data(), m->prof, h.size() * 8, cudaMemcpyDeviceToHost), "profile");
  for (int i = 0; i < n_layer && i < PIPE_PHASES - 1; ++i) {
    double sum = 0, cnt = 0;
    for (int l = 0; l < m->nl; ++l) {
      sum += (double)h[(size_t)l * PIPE_PHASES + i];
      cnt += (double)h[(size_t)l * PIPE_PHASES + PIPE_PHASES - 1];
    }
    layer_us[i] = cnt > 0 ? sum / cnt / 1000.0 : 0.0;
  }
  const unsigned long long* hh = &h[(size_t)m->nl * PIPE_PHASES];
  for (int i = 0; i < n_head && i < PIPE_PHASES - 1; ++i)
    head_us[i] = hh[PIPE_PHASES - 1] ? (double)hh[i] / (double)hh[PIPE_PHASES - 1] / 1000.0 : 0.0;
  API_END
}

int gem_test_withhold_stage(gem_model* m, int stage, int wait_ms) {
  API_BEGIN
  if (!m) throw Error(GEM_E_ARG, "null argument");
  if (stage < -1 || stage >= m->nl) throw Error(GEM_E_RANGE, "stage out of range");
  if (wait_ms < 1 || wait_ms > 60000) throw Error(GEM_E_ARG, "wait_ms must be in 1..60000");
  m->withhold_stage = stage;
  m->wait_ns = (unsigned long long)wait_ms * 1000000ull;
  API_END
}

int gem_get_stream(const gem_model* m, void** stream) {
  API_BEGIN
  if (!m || !stream) throw Error(GEM_E_ARG, "null argument");
  *stream = (void*)m->st;
  API_END
}

int gem_sync(gem_model* m) {
  API_BEGIN
  if (!m) throw Error(GEM_E_ARG, "null argument");
  m->sync();
  API_END
}

int gem_forward(gem_model* m, uint32_t tok, uint32_t pos, float* h_out) {
  API_BEGIN
  if (!m) throw Error(GEM_E_ARG, "null argument");
  if (tok >= (uint32_t)m->vocab) throw Error(GEM_E_RANGE, "token id >= vocab");
  if (pos >= (uint32_t)m->ctx) throw Error(GEM_E_RANGE, "pos >= ctx");  // model.rs:287
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  m->sync();
  *m->cur_host = StepCur{tok, pos, 0, 0};
  ck(cudaMemcpyAsync(m->cur, m->cur_host, sizeof(StepCur), cudaMemcpyHostToDevice, m->st), "cur");
  m->enqueue_body(0);
  m->check_launch();
  if (h_out) ck(cudaMemcpyAsync(h_out, m->h, (size_t)m->d * 4, cudaMemcpyDeviceToHost, m->st), "h");
  m->sync();
  m->have_h = true;
  API_END
}

static int single_head(gem_model* m, int which, uint32_t target, float* logprob, uint32_t* argmax) {
  API_BEGIN
  if (!m) throw Error(GEM_E_ARG, "null argument");
  if (!m->have_h) throw Error(GEM_E_STATE, "no hidden state: call gem_forward first");
  if (which == 1 && !m->two) throw Error(GEM_E_STATE, "two-level head not loaded");
  if (target >= (uint32_t)m->vocab) throw Error(GEM_E_RANGE, "target id >= vocab");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  m->sync();
  StepCur c = *m->cur_host;
  *m->cur_host = StepCur{c.tok, c.pos, target, 0};
  ck(cudaMemcpyAsync(m->cur, m->cur_host, sizeof(StepCur), cudaMemcpyHostToDevice, m->st), "cur");
  m->enqueue_head(which, m->lp, m->am);
  m->check_launch();
  float lp;
  uint32_t am;
  ck(cudaMemcpyAsync(&lp, m->lp, 4, cudaMemcpyDeviceToHost, m->st), "lp");
  ck(cudaMemcpyAsync(&am, m->am, 4, cudaMemcpyDeviceToHost, m->st), "am");
  m->sync();
  if (logprob) *logprob = lp;
  if (argmax) *argmax = am;
  API_END
}

int gem_full_logprob(gem_model* m, uint32_t target, float* logprob, uint32_t* argmax) {
  return single_head(m, 0, target, logprob, argmax);
}
int gem_twolevel_logprob(gem_model* m, uint32_t target, float* logprob, uint32_t* argmax) {
  return single_head(m, 1, target, logprob, argmax);
}

static void run_score(gem_model* m, size_t n, int head) {
  if (head != 0 && head != 1) throw Error(GEM_E_ARG, "head must be 0 (full) or 1 (two-level)");
  if (head == 1 && !m->two) throw Error(GEM_E_STATE, "two-level head not loaded");
  size_t off = m->bos >= 0 ? 1 : 0;
  if (n + off > (size_t)m->ctx) throw Error(GEM_E_RANGE, "sequence longer than ctx");
  if (m->bos >= 0) {  // main.rs:270-272
    *m->cur_host = StepCur{(uint32_t)m->bos, 0, 0, 0};
    ck(cudaMemcpyAsync(m->cur, m->cur_host, sizeof(StepCur), cudaMemcpyHostToDevice, m->st), "cur");
    m->enqueue_body(0);
  }
  if (m->use_parallel()) {
    m->score_parallel(m->toks, n + 1, 1, n, head, (uint32_t)off, m->lp, m->am);
    m->have_h = true;
    return;
  }
  if (m->comm && head == 0) throw Error(GEM_E_STATE, "the vocab-sharded full head runs under the parallel schedule only");
  if (head == 1 && m->try_pipeline(m->toks, n, (uint32_t)off, m->lp, m->am)) {
    m->last_launches = 2;  // the pipelined kernel and the last hidden state's quantization
    m->have_h = true;
    return;
  }
  ck(cudaMemsetAsync(m->step, 0, 4, m->st), "step");
  if (!m->score_graph[head]) {
    cudaGraph_t g;
    ck(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal), "capture");
    try {
      launch_begin_step(m->toks, m->step, (uint32_t)off, (uint32_t)m->vocab, m->cur, m->err, m->st);
      m->enqueue_body(0);
      m->enqueue_head(head, m->lp, m->am);
      launch_end_step(m->step, m->st);
    } catch (...) {
      cudaStreamEndCapture(m->st, &g);
      throw;
    }
    ck(cudaStreamEndCapture(m->st, &g), "end capture");
    size_t nn = 0;
    ck(cudaGraphGetNodes(g, nullptr, &nn), "graph nodes");
    std::vector<cudaGraphNode_t> nodes(nn);
    ck(cudaGraphGetNodes(g, nodes.data(), &nn), "graph nodes");
    int64_t kernels = 0;
    for (auto nd : nodes) {
      cudaGraphNodeType t;
      ck(cudaGraphNodeGetType(nd, &t), "node type");
      kernels += t == cudaGraphNodeTypeKernel;
    }
    m->graph_kernels[head] = kernels;
    cudaGraphExec_t ge;
    cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    ck(e, "graph instantiate");
    m->score_graph[head] = ge;
  }
  for (size_t i = 0; i < n; ++i) ck(cudaGraphLaunch(m->score_graph[head], m->st), "graph launch");
  m->last_launches = m->graph_kernels[head] * (int64_t)n;
  m->have_h = true;
}

int gem_score(gem_model* m, const uint32_t* toks, size_t n, int head, float* logprob_out, uint32_t* argmax_out) {
  API_BEGIN
  if (!m || !toks || !logprob_out) throw Error(GEM_E_ARG, "null argument");
  if (n == 0) return GEM_OK;
  for (size_t i = 0; i <= n; ++i)
    if (toks[i] >= (uint32_t)m->vocab) throw Error(GEM_E_RANGE, "token id >= vocab");
  if (n + 1 > (size_t)m->ctx + 1) throw Error(GEM_E_RANGE, "sequence longer than ctx");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  ck(cudaMemcpyAsync(m->toks, toks, (n + 1) * 4, cudaMemcpyHostToDevice, m->st), "toks");
  run_score(m, n, head);
  ck(cudaMemcpyAsync(logprob_out, m->lp, n * 4, cudaMemcpyDeviceToHost, m->st), "lp");
  if (argmax_out) ck(cudaMemcpyAsync(argmax_out, m->am, n * 4, cudaMemcpyDeviceToHost, m->st), "am");
  m->sync();
  API_END
}

int gem_score_dev(gem_model* m, const uint32_t* toks_dev, size_t n, int head, float* logprob_dev, uint32_t* argmax_dev) {
  API_BEGIN
  if (!m || !toks_dev || !logprob_dev) throw Error(GEM_E_ARG, "null argument");
  if (n == 0) return GEM_OK;
  if (n > (size_t)m->ctx) throw Error(GEM_E_RANGE, "sequence longer than ctx");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  ck(cudaMemcpyAsync(m->toks, toks_dev, (n + 1) * 4, cudaMemcpyDeviceToDevice, m->st), "toks");
  run_score(m, n, head);
  ck(cudaMemcpyAsync(logprob_dev, m->lp, n * 4, cudaMemcpyDeviceToDevice, m->st), "lp");
  if (argmax_dev) ck(cudaMemcpyAsync(argmax_dev, m->am, n * 4, cudaMemcpyDeviceToDevice, m->st), "am");
  API_END
}

// Batched scoring: nseq independent sequences of len + 1 ids (device buffers).
static void run_score_batch(gem_model* m, const uint32_t* toks_d, size_t nseq, size_t len, int head, float* lp_d,
                            uint32_t* am_d) {
  if (head != 0 && head != 1) throw Error(GEM_E_ARG, "head must be 0 (full) or 1 (two-level)");
  if (head == 1 && !m->two) throw Error(GEM_E_STATE, "two-level head not loaded");
  const size_t off = m->bos >= 0 ? 1 : 0;
  if (len + off > (size_t)m->ctx) throw Error(GEM_E_RANGE, "sequence longer than ctx");
  if (nseq > (size_t)INT32_MAX) throw Error(GEM_E_RANGE, "too many sequences");
  if (m->use_parallel()) {
    if (m->bos >= 0) {  // main.rs:270-272, once: every sequence shares the BOS position's K/V rows
      *m->cur_host = StepCur{(uint32_t)m->bos, 0, 0, 0};
      ck(cudaMemcpyAsync(m->cur, m->cur_host, sizeof(StepCur), cudaMemcpyHostToDevice, m->st), "cur");
      m->enqueue_body(0);
    }
    m->score_parallel(toks_d, len + 1, (int)nseq, len, head, (uint32_t)off, lp_d, am_d);
    m->have_h = true;
    return;
  }
  for (size_t s = 0; s < nseq; ++s) {  // per-token schedules: one sequence after another in slot 0
    ck(cudaMemcpyAsync(m->toks, toks_d + s * (len + 1), (len + 1) * 4, cudaMemcpyDeviceToDevice, m->st), "toks");
    run_score(m, len, head);
    ck(cudaMemcpyAsync(lp_d + s * len, m->lp, len * 4, cudaMemcpyDeviceToDevice, m->st), "lp");
    if (am_d) ck(cudaMemcpyAsync(am_d + s * len, m->am, len * 4, cudaMemcpyDeviceToDevice, m->st), "am");
  }
}

int gem_score_batch(gem_model* m, const uint32_t* toks, size_t nseq, size_t len, int head, float* logprob_out,
                    uint32_t* argmax_out) {
  API_BEGIN
  if (!m || !toks || !logprob_out) throw Error(GEM_E_ARG, "null argument");
  if (nseq == 0 || len == 0) return GEM_OK;
  const size_t nt = nseq * (len + 1);
  for (size_t i = 0; i < nt; ++i)
    if (toks[i] >= (uint32_t)m->vocab) throw Error(GEM_E_RANGE, "token id >= vocab");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  m->ensure_batch_io(nt, nseq * len);
  ck(cudaMemcpyAsync(m->btoks, toks, nt * 4, cudaMemcpyHostToDevice, m->st), "toks");
  run_score_batch(m, m->btoks, nseq, len, head, m->blp, m->bam);
  ck(cudaMemcpyAsync(logprob_out, m->blp, nseq * len * 4, cudaMemcpyDeviceToHost, m->st), "lp");
  if (argmax_out) ck(cudaMemcpyAsync(argmax_out, m->bam, nseq * len * 4, cudaMemcpyDeviceToHost, m->st), "am");
  m->sync();
  API_END
}

int gem_score_batch_dev(gem_model* m, const uint32_t* toks_dev, size_t nseq, size_t len, int head, float* logprob_dev,
                        uint32_t* argmax_dev) {
  API_BEGIN
  if (!m || !toks_dev || !logprob_dev) throw Error(GEM_E_ARG, "null argument");
  if (nseq == 0 || len == 0) return GEM_OK;
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  run_score_batch(m, toks_dev, nseq, len, head, logprob_dev, argmax_dev);
  API_END
}

int gem_greedy_dev(gem_model* m, const float* h_dev, int batch, int top, float min_confidence, const uint32_t* always_dev,
                   int n_always, uint32_t* tok_dev, int* fallback_dev) {
  API_BEGIN
  if (!m || !h_dev || !tok_dev || batch <= 0) throw Error(GEM_E_ARG, "bad argument");
  if (!m->two) throw Error(GEM_E_STATE, "two-level head not loaded");
  if (top < 1 || top > m->k) throw Error(GEM_E_RANGE, "top must be in 1..classes");
  if (n_always < 0 || (n_always > 0 && !always_dev)) throw Error(GEM_E_ARG, "always-on rows");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  m->greedy(h_dev, batch, top, min_confidence, always_dev, n_always, tok_dev, fallback_dev);
  m->check_launch();
  API_END
}

int gem_greedy(gem_model* m, int top, float min_confidence, const uint32_t* always, int n_always, uint32_t* token,
               int* fell_back) {
  API_BEGIN
  if (!m || !token) throw Error(GEM_E_ARG, "null argument");
  if (!m->have_h) throw Error(GEM_E_STATE, "no hidden state: call gem_forward or gem_score first");
  if (!m->two) throw Error(GEM_E_STATE, "two-level head not loaded");
  if (top < 1 || top > m->k) throw Error(GEM_E_RANGE, "top must be in 1..classes");
  if (n_always < 0 || (n_always > 0 && !always)) throw Error(GEM_E_ARG, "always-on rows");
  for (int i = 0; i < n_always; ++i)
    if (always[i] >= (uint32_t)m->blocks.v.rows) throw Error(GEM_E_RANGE, "always-on row out of range");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  m->sync();
  if ((size_t)n_always > m->gs.nalways) {
    m->gs.always = m->alloc<uint32_t>(n_always);
    m->gs.nalways = n_always;
  }
  if (n_always) ck(cudaMemcpyAsync(m->gs.always, always, (size_t)n_always * 4, cudaMemcpyHostToDevice, m->st), "always");
  if (m->gs.batch < 1) m->greedy_scratch_min();
  m->greedy(m->h, 1, top, min_confidence, m->gs.always, n_always, m->gs.tok, m->gs.fallback);
  int fb = 0;
  ck(cudaMemcpyAsync(token, m->gs.tok, 4, cudaMemcpyDeviceToHost, m->st), "tok");
  ck(cudaMemcpyAsync(&fb, m->gs.fallback, 4, cudaMemcpyDeviceToHost, m->st), "fb");
  m->sync();
  if (fell_back) *fell_back = min_confidence > 0.0f ? fb : 0;
  API_END
}

int gem_twolevel_sample(gem_model* m, float temperature, uint64_t* rng_state, uint32_t* token) {
  API_BEGIN
  if (!m || !rng_state || !token) throw Error(GEM_E_ARG, "null argument");
  if (!m->have_h) throw Error(GEM_E_STATE, "no hidden state: call gem_forward or gem_score first");
  if (!m->two) throw Error(GEM_E_STATE, "two-level head not loaded");
  if (!(temperature > 0.0f)) throw Error(GEM_E_ARG, "temperature must be > 0");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  m->sync();
  *token = m->sample(temperature, rng_state);
  API_END
}

int gem_generate(gem_model* m, const uint32_t* prompt, size_t n_prompt, size_t max_new, const gem_gen_opts* o, uint32_t* out,
                 size_t* n_out) {
  API_BEGIN
  if (!m || !prompt || !o || !out || !n_out || n_prompt == 0) throw Error(GEM_E_ARG, "bad argument");
  if (o->mode < GEM_GEN_GREEDY_FULL || o->mode > GEM_GEN_SAMPLE) throw Error(GEM_E_ARG, "unknown mode");
  if (o->mode != GEM_GEN_GREEDY_FULL && !m->two) throw Error(GEM_E_STATE, "two-level head not loaded");
  for (size_t i = 0; i < n_prompt; ++i)
    if (prompt[i] >= (uint32_t)m->vocab) throw Error(GEM_E_RANGE, "token id >= vocab");
  const size_t off = m->bos >= 0 ? 1 : 0;
  if (off + n_prompt + max_new > (size_t)m->ctx) throw Error(GEM_E_RANGE, "prompt + max_new longer than ctx");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  m->sync();
  *n_out = 0;
  if (m->bos >= 0) {  // main.rs:270-272
    *m->cur_host = StepCur{(uint32_t)m->bos, 0, 0, 0};
    ck(cudaMemcpyAsync(m->cur, m->cur_host, sizeof(StepCur), cudaMemcpyHostToDevice, m->st), "cur");
    m->enqueue_body(0);
  }
  // the prompt: every position at once when the parallel schedule applies, else one forward per token
  if (m->use_parallel()) {
    std::vector<uint32_t> ids(prompt, prompt + n_prompt);
    ids.push_back(0);  // an unused target for the last position
    m->ensure_batch_io(ids.size(), 0);
    ck(cudaMemcpyAsync(m->btoks, ids.data(), ids.size() * 4, cudaMemcpyHostToDevice, m->st), "prompt");
    m->score_parallel(m->btoks, ids.size(), 1, n_prompt, -1, (uint32_t)off, nullptr, nullptr);
  } else {
    for (size_t i = 0; i < n_prompt; ++i) {
      m->sync();
      *m->cur_host = StepCur{prompt[i], (uint32_t)(off + i), 0, 0};
      ck(cudaMemcpyAsync(m->cur, m->cur_host, sizeof(StepCur), cudaMemcpyHostToDevice, m->st), "cur");
      m->enqueue_body(0);
    }
  }
  m->check_launch();
  m->sync();
  m->have_h = true;
  uint64_t rng = o->seed;
  std::vector<uint32_t> always(o->always, o->always + (o->always ? o->n_always : 0));
  size_t pos = off + n_prompt;
  for (size_t i = 0; i < max_new; ++i) {
    uint32_t t = 0;
    if (o->mode == GEM_GEN_GREEDY_FULL) {  // next_token without classes: argmax of the full head
      *m->cur_host = StepCur{0, (uint32_t)pos, 0, 0};
      ck(cudaMemcpyAsync(m->cur, m->cur_host, sizeof(StepCur), cudaMemcpyHostToDevice, m->st), "cur");
      m->enqueue_head(0, m->lp, m->am);
      ck(cudaMemcpyAsync(&t, m->am, 4, cudaMemcpyDeviceToHost, m->st), "am");
      m->sync();
    } else if (o->mode == GEM_GEN_GREEDY_SCREEN) {
      int fb = 0;
      const int rc = gem_greedy(m, o->top, o->min_confidence, always.data(), (int)always.size(), &t, &fb);
      if (rc != GEM_OK) return rc;
    } else {
      t = m->sample(o->temperature, &rng);
    }
    bool stop = false;
    for (int j = 0; j < o->n_stops; ++j) stop |= o->stops[j] == t;
    if (stop) break;  // lean.rs: a stop token ends the completion and is not emitted
    out[(*n_out)++] = t;
    if (i + 1 == max_new) break;
    *m->cur_host = StepCur{t, (uint32_t)pos, 0, 0};
    ck(cudaMemcpyAsync(m->cur, m->cur_host, sizeof(StepCur), cudaMemcpyHostToDevice, m->st), "cur");
    m->enqueue_body(0);
    m->check_launch();
    ++pos;
  }
  m->sync();
  API_END
}

int gem_matvec_dev(gem_model* m, int layer, int which, const float* x_dev, float* y_dev) {
  API_BEGIN
  if (!m || !x_dev || !y_dev) throw Error(GEM_E_ARG, "null argument");
  const DevMat* M = nullptr;
  if (layer == -1) M = &m->head;
  else if (layer >= 0 && layer < m->nl) {
    const Layer& L = m->layers[layer];
    const DevMat* all[7] = {&L.q_only, &L.k_only, &L.v_only, &L.o, &L.gate_only, &L.up_only, &L.down};
    if (which < 0 || which > 6) throw Error(GEM_E_ARG, "which must be 0..6");
    M = all[which];
  } else {
    throw Error(GEM_E_RANGE, "layer out of range");
  }
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  int cols = M->v.cols;
  int8_t* q = m->alloc<int8_t>(cols);
  float* s = m->alloc<float>(cols / 32);
  // the output matrix in class order: its rows' values back in token order, y[t] = row row_of[t]
  float* y_rows = layer == -1 && m->row_of ? m->alloc<float>(M->v.rows) : nullptr;
  launch_quantize(x_dev, cols, q, s, m->st);
  (m->exact ? launch_gemv_exact : launch_gemv)(M->v, q, s, x_dev, y_rows ? y_rows : y_dev, m->sms, m->st);
  if (y_rows) launch_gather_f32(y_rows, m->row_of, M->v.rows, y_dev, m->st);
  m->check_launch();
  m->sync();
  m->release(q);
  m->release(s);
  if (y_rows) m->release(y_rows);
  API_END
}

constexpr int kHeadGemmMin = 12;  // ~30 us per streamed state vs ~0.37 ms per 32-state product tile
// from this many hidden states on, the two-level head's class logits are one tile product (every class
// row read once) instead of the one-launch kernel's per-state passes (2048 classes: 37.7 against
// 43.1 us at 32 states, 33.8 against ~32 us at 16)
static int two_level_product_min() {
  static const int v = [] {
    const char* e = std::getenv("GEM_TL_PRODUCT_MIN");
    return e ? std::max(1, std::atoi(e)) : 24;
  }();
  return v;
}
static int batch_head(gem_model* m, int which, const float* h_dev, const uint32_t* targets_dev, int batch, float* lp_dev,
                      uint32_t* am_dev) {
  API_BEGIN
  if (!m || !h_dev || !targets_dev || batch <= 0) throw Error(GEM_E_ARG, "bad argument");
  if (which == 1 && !m->two) throw Error(GEM_E_STATE, "two-level head not loaded");
  ck(cudaSetDevice(m->device), "cudaSetDevice");
  m->ensure_head_batch(batch);  // the quantized hidden states live in the model's head scratch
  // from kHeadGemmMin hidden states on, the full head is cheaper as a matrix product (the output
  // matrix read once per 256 states) than as one streamed pass over it per state
  const bool product = which == 0 && m->exact && !m->comm && batch >= kHeadGemmMin && m->full_head_gemm_supported();
  const bool tl_product = which == 1 && m->exact && batch >= two_level_product_min();
  // the streamed full head and the one-launch two-level head quantize the hidden states in their CTAs
  const bool self_quant = (which == 0 && m->exact && m->head_bulk_q && !product) || (which == 1 && m->exact);
  if (!self_quant) launch_quantize(h_dev, batch * m->d, m->hb_q, m->hb_s, m->st);
  if (product)
    m->full_head_gemm(m->hb_q, m->hb_s, h_dev, targets_dev, batch, lp_dev, am_dev);
  else if (tl_product)
    m->twolevel_product(nullptr, nullptr, h_dev, targets_dev, batch, lp_dev, am_dev, true);
  else
    m->run_head(which, self_quant ? nullptr : m->hb_q, self_quant ? nullptr : m->hb_s, h_dev, targets_dev, batch,
                lp_dev, am_dev);
  m->check_launch();
  API_END
}

int gem_head_full_dev(gem_model* m, const float* h_dev, const uint32_t* targets_dev, int batch, float* lp_dev, uint32_t* am_dev) {
  return batch_head(m, 0, h_dev, targets_dev, batch, lp_dev, am_dev);
}
int gem_head_twolevel_dev(gem_model* m, const float* h_dev, const uint32_t* targets_dev, int batch, float* lp_dev,
                          uint32_t* am_dev) {
  return batch_head(m, 1, h_dev, targets_dev, batch, lp_dev, am_dev);
}

}  // extern "C"
