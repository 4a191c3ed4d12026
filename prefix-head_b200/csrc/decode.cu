// Generation-side heads: greedy screening (crates/gem/src/lean.rs:46-107) and two-level sampling
// (main.rs:109-141), for hidden states already on the device.
//
//   k_greedy_rank   class log-sum-exp, the confidence test and the `top` most likely classes
//   k_rows_exact    exact row logits (the reference's 16-lane dot) of the selected class blocks and the
//                   always-on rows, rows given as class-ordered indices
//   k_greedy_pick   highest raw logit over the selected classes (first maximum inside a class, strict
//                   `>` across classes, then across the always-on rows); the full head's argmax over
//                   the class-ordered rows when the confidence test failed
//   k_sample_*      TwoLevel::sample: xorshift64 uniform, draw at temperature (softmax weights, a
//                   sequential sum, a sequential scan), class then member
#include <algorithm>

#include "kernels.cuh"
#include "exact.cuh"

namespace gem {

namespace {

// Rust's f32::exp on Linux is libm's expf; exp in double rounded once to f32 is the correctly rounded
// value, which libm's expf returns except in rare near-halfway cases.
__device__ __forceinline__ float exp_ref(float x) { return (float)exp((double)x); }

}  // namespace

// One CTA per item: norm = log-sum-exp of the class logits; fallback = e^(cl_max - norm) < min_conf;
// sel[item][0..top) = the classes in descending logit order (ties: lower class first).
__global__ void k_greedy_rank(const float* cl, int k, int top, float min_conf, uint32_t* sel, int* fallback) {
  extern __shared__ unsigned char taken[];  // k flags
  __shared__ float rv[32];
  __shared__ uint32_t rc[32];
  __shared__ float rm[32], rs[32];
  const int item = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const float* z = cl + (size_t)item * k;
  for (int c = threadIdx.x; c < k; c += blockDim.x) taken[c] = 0;
  Lse L{-INFINITY, 0.0f};
  for (int c = threadIdx.x; c < k; c += blockDim.x) L = lse_add(L, z[c]);
  for (int o = 16; o > 0; o >>= 1)
    L = lse_merge(L, Lse{__shfl_xor_sync(0xffffffffu, L.m, o), __shfl_xor_sync(0xffffffffu, L.s, o)});
  if (lane == 0) rm[warp] = L.m, rs[warp] = L.s;
  __syncthreads();
  for (int i = 0; i < top; ++i) {
    Best B{-INFINITY, 0xffffffffu};
    for (int c = threadIdx.x; c < k; c += blockDim.x)
      if (!taken[c]) B = best_merge(B, Best{z[c], (uint32_t)c});
    for (int o = 16; o > 0; o >>= 1)
      B = best_merge(B, Best{__shfl_xor_sync(0xffffffffu, B.v, o), __shfl_xor_sync(0xffffffffu, B.tok, o)});
    if (lane == 0) rv[warp] = B.v, rc[warp] = B.tok;
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < nw; ++w) B = best_merge(B, Best{rv[w], rc[w]});
      const uint32_t c = B.tok < (uint32_t)k ? B.tok : 0;
      sel[(size_t)item * top + i] = c;
      taken[c] = 1;
      if (i == 0) {
        Lse T{rm[0], rs[0]};
        for (int w = 1; w < nw; ++w) T = lse_merge(T, Lse{rm[w], rs[w]});
        fallback[item] = exp_ref(B.v - (T.m + logf(T.s))) < min_conf ? 1 : 0;  // lean.rs:58-60
      }
    }
    __syncthreads();
  }
}

// Exact logits of `nrows` rows per item: rows[item][i] (a class-ordered row, or >= w.rows for none).
template <int BITS, typename ST>
__global__ void k_rows_exact(MatView w, const int8_t* aq, const float* as, const float* h, const uint32_t* rows, int nrows,
                             float* out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int item = blockIdx.y, d = w.cols;
  int8_t* saq = (int8_t*)smem_raw;
  float* sas = (float*)(smem_raw + d);
  float* sx = (float*)smem_raw;
  if (BITS == 16) {
    for (int j = threadIdx.x; j < d; j += blockDim.x) sx[j] = h[(size_t)item * d + j];
  } else {
    for (int j = threadIdx.x; j < d / 16; j += blockDim.x) ((int4*)saq)[j] = ((const int4*)(aq + (size_t)item * d))[j];
    for (int j = threadIdx.x; j < d / 32; j += blockDim.x) sas[j] = as[(size_t)item * (d / 32) + j];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, half = lane & 1;
  for (int base = (blockIdx.x * nw + warp) * 16; base < nrows; base += gridDim.x * nw * 16) {
    const int i = base + (lane >> 1);
    const uint32_t r = i < nrows ? rows[(size_t)item * nrows + i] : 0xffffffffu;
    const bool ok = r < (uint32_t)w.rows;
    const float z = row_dot_exact<BITS, ST>(w, ok ? r : 0, half, saq, sas, sx);
    if (i < nrows && half == 0) out[(size_t)item * nrows + i] = ok ? z : -INFINITY;
  }
}

// rows[item] = the selected classes' blocks (top x per rows, missing rows past a short last class
// marked >= nrows_total) followed by the always-on rows.
__global__ void k_greedy_rowlist(const uint32_t* sel, int top, int per, uint32_t total_rows, const uint32_t* always,
                                 int n_always, uint32_t* rows) {
  const int item = blockIdx.y, n = top * per + n_always;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    uint32_t r;
    if (i < top * per) {
      r = sel[(size_t)item * top + i / per] * (uint32_t)per + (uint32_t)(i % per);
      if (r >= total_rows) r = 0xffffffffu;
    } else {
      r = always[i - top * per];
    }
    rows[(size_t)item * n + i] = r;
  }
}

// lean.rs:61-76 and next_token (lean.rs:93-107). One thread per item: the scan order matters.
__global__ void k_greedy_pick(const float* z, const uint32_t* rows, int top, int per, int n_always, const int* fallback,
                              const uint32_t* fb_row, const uint32_t* order, int batch, uint32_t* tok) {
  const int item = blockIdx.x * blockDim.x + threadIdx.x;
  if (item >= batch) return;
  if (fallback && fb_row && fallback[item]) {
    tok[item] = order[fb_row[item]];
    return;
  }
  const int n = top * per + n_always;
  const float* zi = z + (size_t)item * n;
  const uint32_t* ri = rows + (size_t)item * n;
  float best = -INFINITY;
  uint32_t brow = ri[0];
  for (int c = 0; c < top; ++c) {
    int j = 0;  // argmax inside the class: first maximum
    for (int i = 1; i < per; ++i)
      if (zi[c * per + i] > zi[c * per + j]) j = i;
    if (zi[c * per + j] > best) best = zi[c * per + j], brow = ri[c * per + j];
  }
  for (int a = 0; a < n_always; ++a)
    if (zi[top * per + a] > best) best = zi[top * per + a], brow = ri[top * per + a];
  tok[item] = order[brow];
}

// ------------------------------------------------------------------------------------------------
// Sampling (main.rs:123-141)
// ------------------------------------------------------------------------------------------------
namespace {
__device__ __forceinline__ float uniform01(unsigned long long* rng) {
  unsigned long long x = *rng;
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  *rng = x;
  return div((float)(x >> 40), 16777216.0f);
}
// draw (main.rs:130-141) by one CTA: the weights e^((l - max) / temp) in parallel into shared memory,
// then one thread adds them in order, scales the uniform draw by the sum and scans.
__device__ int draw_block(const float* l, int n, float temp, unsigned long long* rng, float* w) {
  __shared__ float red[32];
  __shared__ int s_pick;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, l[i]);
  mx = block_max(mx, red);
  for (int i = threadIdx.x; i < n; i += blockDim.x) w[i] = exp_ref(div(sub(l[i], mx), temp));
  __syncthreads();
  if (threadIdx.x == 0) {
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) sum = add(sum, w[i]);
    float r = mul(uniform01(rng), sum);
    int pick = n - 1;
    for (int i = 0; i < n; ++i) {
      r = sub(r, w[i]);
      if (r <= 0.0f) {
        pick = i;
        break;
      }
    }
    s_pick = pick;
  }
  __syncthreads();
  return s_pick;
}
}  // namespace

__global__ void k_sample_class(const float* cl, int k, float temp, unsigned long long* rng, uint32_t* cls) {
  extern __shared__ float sw[];
  const int c = draw_block(cl, k, temp, rng, sw);
  if (threadIdx.x == 0) *cls = (uint32_t)c;
}
__global__ void k_sample_member(const float* inner, int per, uint32_t total_rows, const uint32_t* cls, float temp,
                                unsigned long long* rng, const uint32_t* order, uint32_t* tok) {
  extern __shared__ float sw[];
  const uint32_t first = *cls * (uint32_t)per;
  const int n = (int)min((uint32_t)per, total_rows - first);
  const int j = draw_block(inner, n, temp, rng, sw);
  if (threadIdx.x == 0) *tok = order[first + (uint32_t)j];
}

// ------------------------------------------------------------------------------------------------
void launch_greedy_rank(const float* cl, int k, int top, float min_conf, int batch, uint32_t* sel, int* fallback,
                        cudaStream_t st) {
  k_greedy_rank<<<batch, 256, (size_t)k, st>>>(cl, k, top, min_conf, sel, fallback);
}
void launch_greedy_rowlist(const uint32_t* sel, int top, int per, uint32_t total_rows, const uint32_t* always, int n_always,
                           int batch, uint32_t* rows, cudaStream_t st) {
  const int n = top * per + n_always;
  k_greedy_rowlist<<<dim3((n + 255) / 256, batch), 256, 0, st>>>(sel, top, per, total_rows, always, n_always, rows);
}
void launch_rows_exact(const MatView& w, const int8_t* aq, const float* as, const float* h, const uint32_t* rows, int nrows,
                       int batch, float* out, cudaStream_t st) {
  const int ctas = std::max(1, std::min(64, (nrows + 127) / 128));
  const size_t sm = w.bits == 16 ? (size_t)w.cols * 4 : (size_t)w.cols + (size_t)w.cols / 32 * 4;
#define F(B, S) k_rows_exact<B, S><<<dim3(ctas, batch), 256, sm, st>>>(w, aq, as, h, rows, nrows, out)
  if (w.bits == 16) F(16, __half);
  else if (w.bits == 8 && !w.scale_f32) F(8, __half);
  else if (w.bits == 8) F(8, float);
  else if (!w.scale_f32) F(4, __half);
  else F(4, float);
#undef F
}
void launch_greedy_pick(const float* z, const uint32_t* rows, int top, int per, int n_always, const int* fallback,
                        const uint32_t* fb_row, const uint32_t* order, int batch, uint32_t* tok, cudaStream_t st) {
  k_greedy_pick<<<(batch + 63) / 64, 64, 0, st>>>(z, rows, top, per, n_always, fallback, fb_row, order, batch, tok);
}
void launch_sample_class(const float* cl, int k, float temp, unsigned long long* rng, uint32_t* cls, cudaStream_t st) {
  k_sample_class<<<1, 256, (size_t)k * 4, st>>>(cl, k, temp, rng, cls);
}
void launch_sample_member(const float* inner, int per, uint32_t total_rows, const uint32_t* cls, float temp,
                          unsigned long long* rng, const uint32_t* order, uint32_t* tok, cudaStream_t st) {
  k_sample_member<<<1, 256, (size_t)per * 4, st>>>(inner, per, total_rows, cls, temp, rng, order, tok);
}

}  // namespace gem
