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

// Whether the kernel is stopping, decided once per CTA (every thread gets the same answer).
__device__ __forceinline__ bool cta_failed(int* err, int* s_flag) {
  __syncthreads();
  if (threadIdx.x == 0) *s_flag = ld_err(err) != 0;
  __syncthreads();
  return *s_flag != 0;
}

// Self-checks (PipeArgs::checks): an index outside its buffer records `site` in the error word and
// the access is skipped.
__device__ __forceinline__ bool check_ok(bool cond, int* err, int site) {
  if (!cond) atomicCAS(err, 0, 100 + site);
  return cond;
}

// L2 prefetch hint for [p, p + bytes) (cp.async.bulk.prefetch.L2); p 16-byte aligned.
__device__ __forceinline__ void prefetch_l2(const void* p, size_t bytes) {
  bytes &= ~(size_t)15;
  const char* c = (const char*)p;
  while (bytes > 0) {
    unsigned n = (unsigned)(bytes < 65536 ? bytes : 65536);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c), "r"(n) : "memory");
    c += n;
    bytes -= n;
  }
}
// Rust's `v.iter().map(|x| x * x).sum::<f32>()` with the squares computed by the whole CTA first: the
// remaining work is one thread's chain of n dependent additions, fed from registers.
__device__ __forceinline__ void squares(const float* v, int n, float* sq) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) sq[i] = mul(v[i], v[i]);
}
__device__ __forceinline__ float seq_sum(const float* sq, int n) {
  float s = 0.0f;
  int i = 0;
  for (; i + 16 <= n; i += 16) {
    float4 a = *(const float4*)(sq + i), b = *(const float4*)(sq + i + 4);
    float4 c = *(const float4*)(sq + i + 8), d = *(const float4*)(sq + i + 12);
    s = add(s, a.x); s = add(s, a.y); s = add(s, a.z); s = add(s, a.w);
    s = add(s, b.x); s = add(s, b.y); s = add(s, b.z); s = add(s, b.w);
    s = add(s, c.x); s = add(s, c.y); s = add(s, c.z); s = add(s, c.w);
    s = add(s, d.x); s = add(s, d.y); s = add(s, d.z); s = add(s, d.w);
  }
  for (; i < n; ++i) s = add(s, sq[i]);
  return s;
}
// r = 1 / sqrt(sum(v^2) / n + eps) with the reference's summation order; every thread gets r.
__device__ __forceinline__ float block_rms_r(const float* v, int n, float eps, float* sq, float* slot) {
  squares(v, n, sq);
  __syncthreads();
  if (threadIdx.x == 0) *slot = rms_r_exact(seq_sum(sq, n), n, eps);
  __syncthreads();
  return *slot;
}

// dot512 of `grp` query heads (smem, hd floats each) against one key row k, loaded once for all heads
// sharing it. k is in shared memory when k_smem (the current position's row), else in global memory
// written by other CTAs (L2 loads). Lane pair layout as dot512_pair.
template <int MAXG>
__device__ __forceinline__ void dot512_group(const float* q, const float* k, bool k_smem, int hd, int grp, int half,
                                             float* out) {
  float acc[MAXG][8];
#pragma unroll
  for (int h = 0; h < MAXG; ++h)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[h][i] = 0.0f;
  for (int c0 = 0; c0 < hd / 16; c0 += 4) {
    float4 kv[8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      int c = c0 + u < hd / 16 ? c0 + u : c0;
      const float4* src = (const float4*)(k + c * 16 + half * 8);
      if (k_smem) {
        kv[2 * u] = src[0];
        kv[2 * u + 1] = src[1];
      } else {
        kv[2 * u] = __ldcg(src);
        kv[2 * u + 1] = __ldcg(src + 1);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      int c = c0 + u;
      if (c >= hd / 16) break;
#pragma unroll
      for (int h = 0; h < MAXG; ++h) {
        if (h >= grp) break;
        const float4 a0 = *(const float4*)(q + h * hd + c * 16 + half * 8), a1 = *(const float4*)(q + h * hd + c * 16 + half * 8 + 4);
        const float4 b0 = kv[2 * u], b1 = kv[2 * u + 1];
        acc[h][0] = fmaf(a0.x, b0.x, acc[h][0]); acc[h][1] = fmaf(a0.y, b0.y, acc[h][1]);
        acc[h][2] = fmaf(a0.z, b0.z, acc[h][2]); acc[h][3] = fmaf(a0.w, b0.w, acc[h][3]);
        acc[h][4] = fmaf(a1.x, b1.x, acc[h][4]); acc[h][5] = fmaf(a1.y, b1.y, acc[h][5]);
        acc[h][6] = fmaf(a1.z, b1.z, acc[h][6]); acc[h][7] = fmaf(a1.w, b1.w, acc[h][7]);
      }
    }
  }
#pragma unroll
  for (int h = 0; h < MAXG; ++h) out[h] = h < grp ? reduce16_pair(acc[h]) : 0.0f;
}


// ------------------------------------------------------------------------------------------------
// Weight ring: a layer stage reads the same weight rows every token, in a fixed order (its q/k/v rows,
// o rows, gate rows, up rows, down rows). Those rows stream through NS shared-memory slots with 1D bulk
// copies (cp.async.bulk, completion on a per-slot mbarrier). A slot holds one tile of up to `gpt`
// 16-row groups of a segment; each group is consumed by one warp, and the last warp to finish a tile
// refills the slot with the tile NS places later in the sequence - which wraps into the next token's
// weights - so the ring keeps running ahead of the compute across phases. Rows are stored with a
// 32-byte pad so a warp's 16 rows fall in different banks.
// ------------------------------------------------------------------------------------------------
struct WSeg {
  MatView w;
  int r0, r1;     // rows of w this CTA reads
  int gpt;        // 16-row groups per tile
  int tile0;      // first tile of the segment within a token
  int ntiles;
  int row_bytes, row_stride, nb, sbytes;  // weight bytes per row, smem stride, 32-blocks, scale bytes per row
};
struct WRing {
  unsigned char* base;
  unsigned long long* full;  // NS mbarriers
  int* done;                 // NS: groups finished in the slot's current tile
  int* issued;               // NS: tile index loaded (or loading) into the slot, -1 = none
  int ns, slot_bytes, scale_off, nseg, tpt;
  long long total;           // tiles over the whole sequence
  int checks;
  int* err;
  WSeg seg[5];
};

__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(unsigned long long* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(unsigned long long* b, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Which segment / rows tile `i` (of the whole sequence) covers.
__device__ __forceinline__ const WSeg& ring_tile(const WRing& R, long long i, int& a, int& b) {
  int j = (int)(i % R.tpt), k = 0;
  while (k + 1 < R.nseg && j >= R.seg[k + 1].tile0) ++k;
  const WSeg& sg = R.seg[k];
  a = sg.r0 + (j - sg.tile0) * 16 * sg.gpt;
  b = min(sg.r1, a + 16 * sg.gpt);
  return sg;
}

// Issue tile i into its slot; called by a whole warp (lanes split the row copies).
__device__ void ring_issue(WRing& R, long long i) {
  if (i >= R.total) return;
  const int lane = threadIdx.x & 31, slot = (int)(i % R.ns);
  int a, b;
  const WSeg& sg = ring_tile(R, i, a, b);
  unsigned char* dst = R.base + (size_t)slot * R.slot_bytes;
  const unsigned bytes = (unsigned)((b - a) * (sg.row_bytes + sg.sbytes));
  if (R.checks) {
    bool ok = check_ok(a >= sg.r0 && b <= sg.r1 && a < b && b <= sg.w.rows, R.err, 1) &&
              check_ok((b - a) * sg.row_stride <= R.scale_off, R.err, 2) &&
              check_ok(R.scale_off + (b - a) * sg.sbytes <= R.slot_bytes, R.err, 3) &&
              check_ok(((size_t)a * sg.row_bytes) % 16 == 0 && sg.row_bytes % 16 == 0 && ((b - a) * sg.sbytes) % 16 == 0 &&
                           ((size_t)a * sg.sbytes) % 16 == 0, R.err, 4) &&
              check_ok(slot >= 0 && slot < R.ns, R.err, 5);
    if (!ok) return;
  }
  if (lane == 0) {
    R.issued[slot] = (int)i;
    R.done[slot] = 0;
    mbar_expect_tx(R.full + slot, bytes);
  }
  __syncwarp();
  for (int r = a + lane; r < b; r += 32)
    bulk_g2s(dst + (size_t)(r - a) * sg.row_stride, (const unsigned char*)sg.w.q + (size_t)r * sg.row_bytes,
             (unsigned)sg.row_bytes, R.full + slot);
  if (lane == 0 && sg.sbytes)
    bulk_g2s(dst + R.scale_off, (const unsigned char*)sg.w.s + (size_t)a * sg.sbytes, (unsigned)((b - a) * sg.sbytes),
             R.full + slot);
}

// Wait (bounded) until tile i has landed in its slot. A warp can reach a tile up to two ring laps ahead
// of its slot's content, and a parity wait cannot tell phase k from phase k + 2, so first wait until
// the slot has been issued with tile i itself (which implies the slot's previous tile, i - NS, has
// been consumed and its phase completed); only then is the parity of tile i unambiguous.
__device__ bool ring_wait(WRing& R, long long i, int* err, unsigned long long limit_ns) {
  const int slot = (int)(i % R.ns);
  unsigned long long* bar = R.full + slot;
  const unsigned parity = (unsigned)((i / R.ns) & 1);
  const volatile int* tag = R.issued + slot;
  if (*tag == (int)i && mbar_try(bar, parity)) return true;
  const unsigned long long t0 = now_ns();
  for (unsigned it = 0;; ++it) {
    if (*tag != (int)i) __nanosleep(64);
    else if (mbar_try(bar, parity)) return true;
    if ((it & 63) == 0) {
      if (ld_err(err) != 0) return false;
      if (now_ns() - t0 > limit_ns) {
        atomicCAS(err, 0, ERR_TIMEOUT);
        return false;
      }
    }
  }
}

// One row's exact dot (row_dot_exact) with the row's weights and scales in shared memory.
template <int BITS, typename ST>
__device__ __forceinline__ float row_dot_exact_smem(const unsigned char* q, const ST* srow, int nb, int half,
                                                    const int8_t* saq, const float* sas, const float* sx) {
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  if constexpr (BITS == 16) {
    const int4* row = (const int4*)q;
    for (int c = 0; c < nb * 2; ++c) {  // nb * 2 chunks of 16 halves
      int4 v = row[2 * c + half];
      const __half2* h2 = (const __half2*)&v;
      const float* xv = sx + c * 16 + half * 8;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float2 f = __half22float2(h2[k]);
        acc[2 * k] = fmaf(f.x, xv[2 * k], acc[2 * k]);
        acc[2 * k + 1] = fmaf(f.y, xv[2 * k + 1], acc[2 * k + 1]);
      }
    }
  } else {
    for (int b = 0; b < nb; ++b) {
      int4 wv;
      if constexpr (BITS == 8) {
        wv = ((const int4*)q)[2 * b + half];
      } else {
        int4 raw = ((const int4*)q)[b];
        const unsigned m = 0x0f0f0f0fu, e = 0x08080808u;
        int sh = half * 4;
        wv.x = (int)__vsub4(((unsigned)raw.x >> sh) & m, e);
        wv.y = (int)__vsub4(((unsigned)raw.y >> sh) & m, e);
        wv.z = (int)__vsub4(((unsigned)raw.z >> sh) & m, e);
        wv.w = (int)__vsub4(((unsigned)raw.w >> sh) & m, e);
      }
      block_fma(acc, wv, *(const int4*)(saq + b * 32 + half * 16), mul(ld_scale(srow, b), sas[b]));
    }
  }
  return reduce16_pair(acc);
}

// The rows of segments [s0, s1] for token t, from the ring: out(row, value). Returns false on abort.
template <int BITS, typename ST, typename F>
__device__ bool ring_rows(WRing& R, int t, int s0, int s1, const int8_t* saq, const float* sas, const float* sx,
                          int* err, unsigned long long limit_ns, F&& out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, half = lane & 1;
  // units: 16-row groups of the segments, in sequence order
  int units = 0;
  for (int k = s0; k <= s1; ++k) units += (R.seg[k].r1 - R.seg[k].r0 + 15) / 16;
  bool ok = true;
  for (int u = warp; u < units && ok; u += nw) {
    int k = s0, uu = u;
    while ((R.seg[k].r1 - R.seg[k].r0 + 15) / 16 <= uu) {
      uu -= (R.seg[k].r1 - R.seg[k].r0 + 15) / 16;
      ++k;
    }
    const WSeg& sg = R.seg[k];
    const long long tile = (long long)t * R.tpt + sg.tile0 + uu / sg.gpt;
    const int grp = uu % sg.gpt;
    ok = __all_sync(0xffffffffu, ring_wait(R, tile, err, limit_ns));  // one decision per warp
    if (!ok) break;
    const int slot = (int)(tile % R.ns);
    if (R.checks && !check_ok(grp < sg.gpt && tile < R.total && sg.tile0 + uu / sg.gpt < R.tpt, err, 6)) {
      ok = false;
      break;
    }
    const unsigned char* base = R.base + (size_t)slot * R.slot_bytes;
    const int row0 = sg.r0 + (uu / sg.gpt) * 16 * sg.gpt + grp * 16;
    const int rloc = grp * 16 + (lane >> 1);
    const int r = row0 + (lane >> 1);
    const bool valid = r < sg.r1;
    const int rl = valid ? rloc : grp * 16;
    float v = row_dot_exact_smem<BITS, ST>(base + (size_t)rl * sg.row_stride,
                                           (const ST*)(base + R.scale_off + (size_t)rl * sg.sbytes), sg.nb, half, saq,
                                           sas, sx);
    if (valid && half == 0) out(r, v);
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      fence_proxy_async();
      int tile_groups = min(sg.gpt, (sg.r1 - (sg.r0 + (uu / sg.gpt) * 16 * sg.gpt) + 15) / 16);
      __threadfence_block();
      last = atomicAdd(R.done + slot, 1) + 1 == tile_groups;
      __threadfence_block();
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) ring_issue(R, tile + R.ns);
  }
  return ok;
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
  float* sq;     // max(d, (nh + nkv) * hd): squares for the sequential sums
  int* ok;
  void* ring;    // WRing (layer stages)
  unsigned char* slots;
  unsigned long long* bars;
  int* ring_ints;  // done[NS], issued[NS]
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
  S.sq = (float*)take((size_t)max(P.d, (P.nh + P.nkv) * P.hd) * 4);
  S.ok = (int*)take(16);
  S.ring = take(sizeof(WRing));
  S.bars = (unsigned long long*)take((size_t)P.ring_slots * 8);
  S.ring_ints = (int*)take((size_t)P.ring_slots * 8);
  off = (off + 127) / 128 * 128;
  S.slots = base + off;
  return S;
}

// ------------------------------------------------------------------------------------------------
// A decoder layer stage.
// ------------------------------------------------------------------------------------------------
template <int BITS, typename ST, int BH, typename SH>
__device__ bool layer_tokens(const PipeArgs& P, int l, int c, const Smem& S, WRing& R) {
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

  unsigned long long ts[18];
  const bool prof = P.prof && c == 0 && tid == 0;
#define MARK(i) \
  if (prof) ts[i] = now_ns();
  for (int t = 0; t < P.n; ++t) {
    const uint32_t pos = P.base_pos + t;
    const int slot = t % PIPE_RING;
    MARK(0)
    if (tid == 0) {  // this token's first weights and KV rows, while the input is on its way
      const uint32_t lo0 = (L.window > 0 && pos + 1 > (uint32_t)L.window) ? pos + 1 - L.window : 0;
      const int np0 = (int)(pos + 1 - lo0);
      int2 pr = span(np0, 1);
      if (pr.y > pr.x) prefetch_l2(L.kcache + (size_t)(lo0 + pr.x) * rw, (size_t)(pr.y - pr.x) * rw * 4);
      const int per0 = (np0 + T - 1) / T;
      for (int tt = c; tt < T; tt += G) {
        int i0 = min(tt * per0, np0), i1 = min((tt + 1) * per0, np0);
        if (i1 > i0) prefetch_l2(L.vcache + (size_t)(lo0 + i0) * rw, (size_t)(i1 - i0) * rw * 4);
      }
    }
    // ---- input residual ----
    if (l == 0) {
      uint32_t tok = P.toks[t];
      if (tok >= (uint32_t)P.vocab) {
        if (tid == 0) atomicCAS(P.err, 0, ERR_RANGE);
        tok = 0;
      }
      const uint32_t erow = P.emb_row ? P.emb_row[tok] : tok;
      for (int j = tid; j < d; j += nt) S.x[j] = mul(emb_weight<BH, SH>(P.emb, erow, j), P.embed_scale);
    } else {
      if (tid == 0) *S.ok = wait_geq(P.ready + l * PIPE_RING + slot, (unsigned)t + 1, P.err, P.wait_ns);
      __syncthreads();
      if (!*S.ok) return false;
      const float* src = P.ring + ((size_t)l * PIPE_RING + slot) * d;
      for (int j = tid; j < d; j += nt) S.x[j] = ldcg(src + j);
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        atomicAdd(P.consumed + l, 1u);
      }
    }
    __syncthreads();
    MARK(1)
    // ---- attn_norm + quantize (model.rs:304-305) ----
    {
      const float r = block_rms_r(S.x, d, P.eps, S.sq, S.r);
      for (int j = tid; j < d; j += nt) S.xn[j] = mul(mul(S.x[j], r), nw[j]);
    }
    __syncthreads();
    quantize_smem(S.xn, d, S.aq, S.as);
    __syncthreads();
    MARK(2)
    // ---- q/k/v projections, this CTA's rows (model.rs:307-309) ----
    if (R.ns) ring_rows<BITS, ST>(R, t, 0, 0, S.aq, S.as, S.xn, P.err, P.wait_ns, [&](int r, float v) { qkv_g[r] = v; });
    else rows_exact<BITS, ST>(L.qkv, R.seg[0].r0, R.seg[0].r1, S.aq, S.as, S.xn, [&](int r, float v) { qkv_g[r] = v; });
    __syncthreads();
    if (cta_failed(P.err, S.ok)) return false;
    MARK(3)
    if (!stage_barrier(bar, epoch, G, P.err, S.ok, P.wait_ns)) return false;
    MARK(4)
    // ---- QK-norm, RoPE, q scale (model.rs:311-332), redundant in every CTA ----
    for (int j = tid; j < qkv_rows; j += nt) {
      float v = ldcg(qkv_g + j);
      if (L.bqkv) v = add(v, L.bqkv[j]);
      if (j < nh * hd) S.q[j] = v;
      else if (j < (nh + nkv) * hd) S.k[j - nh * hd] = v;
      else S.v[j - (nh + nkv) * hd] = v;
    }
    __syncthreads();
    for (int j = tid; j < (nh + nkv) * hd; j += nt) {  // S.q and S.k are adjacent heads of hd floats
      float v = j < nh * hd ? S.q[j] : S.k[j - nh * hd];
      S.sq[j] = mul(v, v);
    }
    __syncthreads();
    if (tid < nh + nkv) {
      const float* w = tid < nh ? L.q_norm : L.k_norm;
      S.r[1 + tid] = w ? rms_r_exact(seq_sum(S.sq + tid * hd, hd), hd, P.eps) : 1.0f;
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
    if (P.checks && !check_ok(pos < (uint32_t)P.ctx, P.err, 10)) return false;
    if (c == 0)  // KV append (model.rs:333-335)
      for (int j = tid; j < rw; j += nt) {
        L.kcache[(size_t)pos * rw + j] = S.k[j];
        L.vcache[(size_t)pos * rw + j] = S.v[j];
      }
    // ---- scores for this CTA's positions (model.rs:344-353); one key row serves its query group ----
    const uint32_t lo = (L.window > 0 && pos + 1 > (uint32_t)L.window) ? pos + 1 - L.window : 0;
    const int n_pos = (int)(pos + 1 - lo);
    if (P.checks && !check_ok(n_pos <= P.max_npos, P.err, 11)) return false;
    {
      int2 pr = span(n_pos, 1);
      const int lane = tid & 31, warp = tid >> 5, nw2 = nt >> 5, half = lane & 1;
      const int total = (pr.y - pr.x) * nkv;
      for (int base = warp * 16; base < total; base += nw2 * 16) {
        int u = base + (lane >> 1);
        bool okk = u < total;
        int uu = okk ? u : 0;
        int i = pr.x + uu / nkv, g = uu % nkv;
        const bool cur = lo + i == pos;
        const float* krow = cur ? S.k + g * hd : L.kcache + (size_t)(lo + i) * rw + g * hd;
        float sc[8];
        if (grp <= 4) dot512_group<4>(S.q + g * grp * hd, krow, cur, hd, grp, half, sc);
        else dot512_group<8>(S.q + g * grp * hd, krow, cur, hd, grp, half, sc);
        if (okk && half == 0) {
#pragma unroll
          for (int h = 0; h < 8; ++h)
            if (h < grp) sc_g[(size_t)(g * grp + h) * P.max_npos + i] = sc[h];
        }
      }
    }
    __syncthreads();
    MARK(5)
    if (!stage_barrier(bar, epoch, G, P.err, S.ok, P.wait_ns)) return false;
    MARK(6)
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
    // ---- P.V over the pool's position ranges (model.rs:362-376), this CTA's ranges. One thread per
    //      value column serves its query group; value loads are issued 8 positions ahead. ----
    {
      const int per = (n_pos + T - 1) / T;
      const int mine = (T - c + G - 1) / G;  // partitions c, c + G, ...
      const int lanes = nt / rw > 0 ? nt / rw : 1;
      for (int m0 = 0; m0 < mine; m0 += lanes) {
        const int m = m0 + tid / rw, col = tid % rw;
        const int tt = c + m * G;
        if (tid < lanes * rw && m < mine && tt < T) {
          const int i0 = min(tt * per, n_pos), i1 = min((tt + 1) * per, n_pos);
          const int g = col / hd, j = col % hd;
          float acc[8];
#pragma unroll
          for (int h = 0; h < 8; ++h) acc[h] = 0.0f;
          for (int i = i0; i < i1; i += 8) {
            float vv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              int ii = i + u;
              vv[u] = ii < i1 ? ((lo + ii == pos) ? S.v[col] : ldcg(L.vcache + (size_t)(lo + ii) * rw + col)) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              if (i + u >= i1) break;
#pragma unroll
              for (int h = 0; h < 8; ++h)
                if (h < grp) acc[h] = fmaf(S.p[(g * grp + h) * P.max_npos + i + u], vv[u], acc[h]);
            }
          }
#pragma unroll
          for (int h = 0; h < 8; ++h)
            if (h < grp) pv_g[(size_t)tt * nh * hd + (size_t)(g * grp + h) * hd + j] = acc[h];
        }
      }
    }
    __syncthreads();
    MARK(7)
    if (!stage_barrier(bar, epoch, G, P.err, S.ok, P.wait_ns)) return false;
    MARK(8)
    // ---- partials summed in thread order (model.rs:377-382), quantize (model.rs:384) ----
    for (int u = tid; u < nh * hd; u += nt) {
      float a = 0.0f;
      for (int t0 = 0; t0 < T; t0 += 8) {
        float part[8];
#pragma unroll
        for (int k2 = 0; k2 < 8; ++k2) part[k2] = t0 + k2 < T ? ldcg(pv_g + (size_t)(t0 + k2) * nh * hd + u) : 0.0f;
#pragma unroll
        for (int k2 = 0; k2 < 8; ++k2)
          if (t0 + k2 < T) a = add(a, part[k2]);
      }
      S.xn[u] = a;
    }
    __syncthreads();
    quantize_smem(S.xn, nh * hd, S.aq, S.as);
    __syncthreads();
    // ---- O projection, this CTA's rows (model.rs:386) ----
    if (R.ns) ring_rows<BITS, ST>(R, t, 1, 1, S.aq, S.as, S.xn, P.err, P.wait_ns, [&](int r, float v) { o_g[r] = v; });
    else rows_exact<BITS, ST>(L.o, R.seg[1].r0, R.seg[1].r1, S.aq, S.as, S.xn, [&](int r, float v) { o_g[r] = v; });
    __syncthreads();
    if (cta_failed(P.err, S.ok)) return false;
    MARK(9)
    if (!stage_barrier(bar, epoch, G, P.err, S.ok, P.wait_ns)) return false;
    MARK(10)
    // ---- post-attention norm, residual, ffn norm, quantize (model.rs:388-395) ----
    for (int j = tid; j < d; j += nt) S.xn[j] = ldcg(o_g + j);
    __syncthreads();
    {
      const float r = L.post_attn ? block_rms_r(S.xn, d, P.eps, S.sq, S.r) : 1.0f;
      for (int j = tid; j < d; j += nt) {
        float t2 = S.xn[j];
        if (L.post_attn) t2 = mul(t2, mul(r, L.post_attn[j]));
        S.x[j] = add(S.x[j], t2);
      }
      __syncthreads();
      const float r2 = block_rms_r(S.x, d, P.eps, S.sq, S.r + 1);
      for (int j = tid; j < d; j += nt) S.xn[j] = mul(mul(S.x[j], r2), L.ffn_norm[j]);
    }
    __syncthreads();
    quantize_smem(S.xn, d, S.aq, S.as);
    __syncthreads();
    MARK(11)
    // ---- gate/up for this CTA's FFN slice, GELU / SiLU, quantize (model.rs:397-417) ----
    {
      int2 fr = span(ff, 32);
      float* gbuf = S.p;  // reuse: 2 * slice floats
      const int n = fr.y - fr.x;
      auto put = [&](int r, float v) {
        if (r < ff) gbuf[r - fr.x] = v;
        else gbuf[n + r - ff - fr.x] = v;
      };
      if (R.ns) {
        ring_rows<BITS, ST>(R, t, 2, 3, S.aq, S.as, S.xn, P.err, P.wait_ns, put);
      } else {
        rows_exact<BITS, ST>(L.gu, fr.x, fr.y, S.aq, S.as, S.xn, put);
        rows_exact<BITS, ST>(L.gu, ff + fr.x, ff + fr.y, S.aq, S.as, S.xn, put);
      }
      __syncthreads();
      if (cta_failed(P.err, S.ok)) return false;
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
    __syncthreads();
    MARK(12)
    if (!stage_barrier(bar, epoch, G, P.err, S.ok, P.wait_ns)) return false;
    MARK(13)
    // ---- down projection, this CTA's rows (model.rs:419) ----
    for (int j = tid; j < ff / 16; j += nt) ((int4*)S.aq)[j] = __ldcg((const int4*)gq_g + j);
    for (int j = tid; j < ff / 32; j += nt) S.as[j] = ldcg(gs_g + j);
    __syncthreads();
    if (R.ns) ring_rows<BITS, ST>(R, t, 4, 4, S.aq, S.as, S.xn, P.err, P.wait_ns, [&](int r, float v) { dn_g[r] = v; });
    else rows_exact<BITS, ST>(L.down, R.seg[4].r0, R.seg[4].r1, S.aq, S.as, S.xn, [&](int r, float v) { dn_g[r] = v; });
    __syncthreads();
    if (cta_failed(P.err, S.ok)) return false;
    MARK(14)
    if (!stage_barrier(bar, epoch, G, P.err, S.ok, P.wait_ns)) return false;
    MARK(15)
    // ---- post-FFN norm and residual (model.rs:421-426); CTA 0 hands the residual on ----
    if (c == 0) {
      for (int j = tid; j < d; j += nt) S.xn[j] = ldcg(dn_g + j);
      __syncthreads();
      const float r = L.post_ffw ? block_rms_r(S.xn, d, P.eps, S.sq, S.r) : 1.0f;
      for (int j = tid; j < d; j += nt) {
        float t2 = S.xn[j];
        if (L.post_ffw) t2 = mul(t2, mul(r, L.post_ffw[j]));
        S.x[j] = add(S.x[j], t2);
      }
      if (l == P.withhold_stage) {  // test hook: nothing downstream will ever see this token
        __syncthreads();
        continue;
      }
      const int nxt = l + 1, gnext = nxt < P.nl ? G : P.GH;
      if (tid == 0) *S.ok = t < PIPE_RING ? 1 : wait_geq(P.consumed + nxt, (unsigned)(t - PIPE_RING + 1) * gnext, P.err, P.wait_ns);
      __syncthreads();
      if (!*S.ok) return false;
      float* dst = P.ring + ((size_t)nxt * PIPE_RING + slot) * d;
      for (int j = tid; j < d; j += nt) dst[j] = S.x[j];
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        st_release(P.ready + nxt * PIPE_RING + slot, (unsigned)t + 1);
      }
    }
    __syncthreads();
    MARK(16)
    if (prof && t >= P.prof_from) {
      unsigned long long* acc = P.prof + (size_t)l * PIPE_PHASES;
      for (int i = 0; i < 16; ++i) acc[i] += ts[i + 1] - ts[i];
      acc[PIPE_PHASES - 1] += 1;  // tokens counted
    }
  }
#undef MARK
  return true;
}

// ------------------------------------------------------------------------------------------------

// A decoder layer stage: sets up the weight ring, runs the tokens, then waits for every weight copy
// still in flight before the CTA exits (normally or on abort).
template <int BITS, typename ST, int BH, typename SH>
__device__ void layer_stage(const PipeArgs& P, int l, int c, const Smem& S) {
  const PipeLayer& L = P.layers[l];
  const int G = P.G, ff = P.ff, d = P.d, qkv_rows = (P.nh + 2 * P.nkv) * P.hd;
  WRing& R = *(WRing*)S.ring;
  auto span = [&](int total, int align) {
    int per = ((total + G - 1) / G + align - 1) / align * align;
    int a = min(total, c * per), b = min(total, a + per);
    return make_int2(a, b);
  };
  if (threadIdx.x == 0) {
    R.base = S.slots;
    R.full = S.bars;
    R.done = S.ring_ints;
    R.issued = S.ring_ints + P.ring_slots;
    R.ns = P.ring_slots;
    R.slot_bytes = P.slot_bytes;
    R.scale_off = P.slot_scale_off;
    R.checks = P.checks;
    R.err = P.err;
    int2 rq = span(qkv_rows, 16), ro = span(d, 16), fr = span(ff, 32);
    const MatView* ws[5] = {&L.qkv, &L.o, &L.gu, &L.gu, &L.down};
    const int2 rr[5] = {rq, ro, fr, make_int2(ff + fr.x, ff + fr.y), ro};
    int tile0 = 0;
    R.nseg = 5;
    for (int k = 0; k < 5; ++k) {
      WSeg& sg = R.seg[k];
      sg.w = *ws[k];
      sg.r0 = rr[k].x;
      sg.r1 = rr[k].y;
      sg.row_bytes = sg.w.cols * sg.w.bits / 8;
      sg.row_stride = sg.row_bytes + 32;  // 8-bank shift per row: a quarter warp's 4 rows x 2 halves hit 32 banks
      sg.nb = sg.w.cols / 32;
      sg.sbytes = sg.w.bits == 16 ? 0 : sg.nb * (sg.w.scale_f32 ? 4 : 2);
      int by_rows = R.scale_off / (16 * sg.row_stride);
      int by_scales = sg.sbytes ? (R.slot_bytes - R.scale_off) / (16 * sg.sbytes) : by_rows;
      sg.gpt = max(1, min(by_rows, by_scales));
      sg.tile0 = tile0;
      sg.ntiles = (sg.r1 - sg.r0 + 16 * sg.gpt - 1) / (16 * sg.gpt);
      tile0 += sg.ntiles;
    }
    R.tpt = tile0;
    R.total = R.ns ? (long long)P.n * R.tpt : 0;
    for (int k = 0; k < R.ns; ++k) {
      mbar_init(R.full + k, 1);
      R.done[k] = 0;
      R.issued[k] = -1;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x < 32)
    for (int k = 0; k < R.ns; ++k) ring_issue(R, k);
  __syncthreads();
  layer_tokens<BITS, ST, BH, SH>(P, l, c, S, R);
  __syncthreads();
  if (threadIdx.x == 0)  // copies still in flight must land before the CTA's shared memory goes away
    for (int k = 0; k < R.ns; ++k) {
      int i = R.issued[k];
      if (i < 0) continue;
      const unsigned long long t0 = now_ns();
      while (!mbar_try(R.full + k, (unsigned)((i / R.ns) & 1)) && now_ns() - t0 < 1000000000ull) {
      }
    }
  __syncthreads();
}

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
  unsigned long long ts[8];
  const bool prof = P.prof && c == 0 && tid == 0;
#define MARK(i) \
  if (prof) ts[i] = now_ns();
  for (int t = 0; t < P.n; ++t) {
    const int slot = t % PIPE_RING;
    MARK(0)
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
    MARK(1)
    // final norm (model.rs:428) and Act::quantize of h (main.rs:96)
    {
      const float r = block_rms_r(S.x, d, P.eps, S.sq, S.r);
      for (int j = tid; j < d; j += nt) S.xn[j] = mul(mul(S.x[j], r), P.out_norm[j]);
    }
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
    __syncthreads();
    MARK(2)
    if (!stage_barrier(bar, epoch, GH, P.err, S.ok, P.wait_ns)) return;
    MARK(3)
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
    __syncthreads();
    MARK(4)
    if (!stage_barrier(bar, epoch, GH, P.err, S.ok, P.wait_ns)) return;
    MARK(5)
    if (c == 0 && tid < 32) {
      Best B{-INFINITY, 0xffffffffu};
      for (int j = lane; j < tn; j += 32) B = best_merge(B, Best{ldcg(top_g + j), (uint32_t)j});
      for (int o = 16; o > 0; o >>= 1)
        B = best_merge(B, Best{__shfl_xor_sync(0xffffffffu, B.v, o), __shfl_xor_sync(0xffffffffu, B.tok, o)});
      if (lane == 0 && P.am_out) P.am_out[t] = P.order[tfirst + (B.tok < (uint32_t)tn ? B.tok : 0)];
    }
    __syncthreads();
    MARK(6)
    if (prof && t >= P.prof_from) {
      unsigned long long* acc = P.prof + (size_t)P.nl * PIPE_PHASES;
      for (int i = 0; i < 6; ++i) acc[i] += ts[i + 1] - ts[i];
      acc[PIPE_PHASES - 1] += 1;
    }
  }
#undef MARK
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

size_t pipe_smem_base_bytes(const PipeArgs& P);
size_t pipe_smem_bytes(const PipeArgs& P) {
  auto r16 = [](size_t b) { return (b + 15) / 16 * 16; };
  size_t wide = std::max(std::max(P.d, P.nh * P.hd), P.ff);
  size_t p = pipe_p_floats(P);
  size_t base = r16(P.d * 4) + r16(wide * 4) + r16(wide) + r16(wide / 32 * 4) + r16((size_t)P.nh * P.hd * 4) +
                2 * r16((size_t)P.nkv * P.hd * 4) + r16(p * 4) + r16(128) +
                r16((size_t)std::max(P.d, (P.nh + P.nkv) * P.hd) * 4) + 16 + r16(sizeof(WRing)) +
                r16((size_t)P.ring_slots * 8) + r16((size_t)P.ring_slots * 8);
  return (base + 127) / 128 * 128 + (size_t)P.ring_slots * P.slot_bytes;
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
