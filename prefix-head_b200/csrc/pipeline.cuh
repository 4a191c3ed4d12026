// Arguments of the layer-pipelined scoring kernel (pipeline.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include "kernels.cuh"

namespace gem {

constexpr int PIPE_RING = 4;     // residual slots between consecutive stages
constexpr int PIPE_PHASES = 24;  // profiled phases per stage

struct PipeLayer {
  MatView qkv, o, gu, down;
  const float *attn_norm, *q_norm, *k_norm, *post_attn, *ffn_norm, *post_ffw, *bqkv;
  const float *rope_sin, *rope_cos;  // [ctx][hd/2] for this layer's base
  float *kcache, *vcache;            // [ctx][nkv*hd] of the scored sequence
  int window;                        // 0 on global layers
};

struct PipeArgs {
  const PipeLayer* layers;  // device array [nl]
  int nl, d, nh, nkv, hd, ff, ctx, max_npos, vocab;
  float eps, qscale, embed_scale;
  int silu;
  int layers_bits, layers_scale_f32;
  MatView emb;              // embedding rows (the tied output matrix)
  const uint32_t* emb_row;  // token -> row of emb when it is held in class order (null: token order)
  // two-level head
  MatView blocks;
  const float *A, *b, *out_norm;
  const uint32_t *cls_of, *pos_of, *order;
  int k, per;
  // sequence
  const uint32_t* toks;  // n + 1 ids
  int n, base_pos;
  float* lp_out;
  uint32_t* am_out;
  float* h_last;  // final-norm hidden state of the last token (nullable)
  int ref_threads;
  // topology: G CTAs per layer, GH for the head
  int G, GH;
  // scratch (zeroed counters before every launch)
  float* ring;          // [nl + 1][PIPE_RING][d]
  unsigned* ready;      // [nl + 1][PIPE_RING]
  unsigned* consumed;   // [nl + 1]
  unsigned* bar;        // [nl + 1][32]
  float* scratch;       // [nl][scratch_stride]
  size_t scratch_stride;
  float* head_scratch;  // k + 2 * per
  int* err;
  int ring_slots, slot_bytes, slot_scale_off;  // weight ring geometry (layer stages)
  int checks;                                   // self-checks on (see check_ok)
  unsigned long long wait_ns;  // bound of every wait
  unsigned long long* prof;    // nullable: [nl + 1][PIPE_PHASES] summed phase times (ns), tokens >= prof_from
  int prof_from;
  int withhold_stage;          // test hook: this layer stage never hands its residual on (-1: none)
};

size_t pipe_scratch_floats(int nh, int nkv, int hd, int d, int ff, int max_npos, int ref_threads);
size_t pipe_smem_bytes(const PipeArgs& P);
// 0 on success; -1 when the model's weight formats have no instantiation; else a cudaError_t.
int launch_pipe_score(const PipeArgs& P, size_t smem, cudaStream_t st);

}  // namespace gem
