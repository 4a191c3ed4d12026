// Exact int8 matrix product on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// The reference's row dot (crates/gem/src/q8.rs:257-270, dot_avx512; dot4_avx512 for Q4_0) keeps 16
// fp32 lanes per row: for every 32-block b, lane i takes the exact integer pair sum
//     p_i = w[32b + 2i] * a[32b + 2i] + w[32b + 2i + 1] * a[32b + 2i + 1]       (madd_epi16)
// and rounds once: acc_i = fma(p_i, ws_b * as_b, acc_i); the 16 lanes are then added in
// _mm512_reduce_add_ps's halving order. Bit-identical results need every one of those roundings, so
// the per-block FMA cannot move into the tensor core's accumulator. What can move is the integer part:
// int8 and 4-bit values are exact in f16, a pair sum of two int8 products is exact in an f32
// accumulator whatever the order of its (zero) other terms, so one f16 MMA per half block yields the 8
// pair sums p_i of 8 lanes for every (row, position) at once, bit for bit.
//
// Layout of one MMA (M = 128 weight rows, N = 8 lanes x TP positions, K = 16 = half a block):
//   A[r][k]   = w[r][32b + 16h + k] as f16, K-major, from a copy of the matrix tiled at load time
//               (per row tile and block: [8-row group][K core matrix][8 rows][8 halves], 8 KiB, then
//               the 128 weight scales, so that one bulk copy brings both)
//   B[k][n]   = a[t][32b + 16h + k] if k is 2j or 2j + 1, else 0 (f16, K-major), where column
//               n = 32q + 4j + p holds lane j of position t = 4q + p (position group q)
//   D[r][n]   = p_(8h + j) of row r and position t, f32 in tensor memory
// B is zero except for one f16 pair per column. The zeros are written once per CTA; the converter
// warps write only the pairs of each block, 4-byte words laid out so that a warp's stores fall on
// distinct banks (two ways at most). The column order gives each epilogue warpgroup q the 32
// contiguous columns of its 4 positions in each half.
//
// Warp roles (TP = 4Q positions per tile; 1 + Q + 4Q warps, at most 4 per SM sub-partition): warp 0
// issues the MMAs (one thread; tcgen05.commit signals the stage and the accumulator buffer); warps
// 1..Q expand the int8 activations of one position group each and copy their scales into the stage,
// and lane 0 of warp 1 bulk-copies each block's weight tile and weight scales (mbarrier complete_tx);
// the rest are the epilogue: warp w of warpgroup q reads tensor-memory lanes 32 (w % 4) .. + 31 (its
// rows) for positions 4q..4q+3 and applies the reference's FMA per lane and block with the scale
// ws * as, from registers that hold the 16 lanes of its 4 positions. A stage is released when its MMAs
// have completed and every epilogue warp has read its scales. Tensor memory holds ND accumulator
// buffers (a block's two halves each), so the MMAs run up to ND - 1 blocks ahead of the epilogue: an
// MMA's issue-to-completion round trip is about 400 cycles on this GPU, longer than the epilogue's
// work on one block. At the end of a tile each thread reduces its lanes in the halving order and
// stores y[t][r]. The CTAs are persistent (one per SM, walking the tiles).
//
// The exactness argument leaves the CUDA cores exactly one FMA per lane, block, row and position (the
// reference's own arithmetic), half a packed FFMA2 instruction; the int8 pair products, their
// conversion to fp32 and the operand staging, which took three instructions per pair on the CUDA
// cores, run on the tensor cores and the copy engine. The bound is the FP32 FMA pipe.
//
// Every wait is bounded by the global timer: on expiry the waiter records ERR_TIMEOUT, raises a
// CTA-wide abort flag that every other waiter sees, the MMA thread waits (bounded) for the MMAs it
// issued, the copy thread for the copies it issued, and the tensor memory is freed before the CTA
// exits.
#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <cuda_fp16.h>

#include "kernels.cuh"

namespace gem {

namespace {

constexpr int kTcBM = 128;                          // weight rows per tile = tensor-memory lanes
constexpr int kTcA = kTcBM * 32 * 2;                // f16 weight tile of one 32-block: 8 KiB
constexpr int kTcChunk = kTcA + kTcBM * 4;          // tiled chunk: weight tile, then its 128 f32 scales
constexpr uint32_t kTcCols = 512;                   // tensor-memory allocation (a power of two)
constexpr unsigned long long kTcWaitNs = 1000000000ull;

// Q position groups of 4 (TP = 4Q positions per tile), S stages.
template <int Q, int S>
struct TcCfg {
  static constexpr int TP = 4 * Q;
  static constexpr int N = 8 * TP;                      // MMA N: 8 lanes x TP positions
  static constexpr int ND = (int)kTcCols / (2 * N);     // accumulator buffers of a block's two halves
  static constexpr int EpiWarps = 4 * Q;
  static constexpr int Epi0 = 1 + Q;                    // first epilogue warp
  // a warp of its own issues the bulk copies where that keeps at most 3 warps per SM sub-partition;
  // otherwise lane 0 of the first converter warp does
  static constexpr bool CopyWarp = Epi0 + EpiWarps + 1 <= 12;
  static constexpr int CopyW = Epi0 + EpiWarps;
  static constexpr int Threads = 32 * (Epi0 + EpiWarps + (CopyWarp ? 1 : 0));
  static constexpr int BHalf = TP * 256;                // expanded activations of one half block
  // a stage: the chunk as copied (weights at 0, scales at kTcA), the expanded activations, their scales
  static constexpr int BOff = kTcChunk;
  static constexpr int AsOff = BOff + 2 * BHalf;
  static constexpr int Stage = (AsOff + TP * 4 + 127) / 128 * 128;
  static constexpr int Bars = 3 * S + 2 * ND;           // full, bready, empty per stage; dfull, dempty per buffer
  static constexpr int Smem = S * Stage + Bars * 8 + 16;
  // instruction descriptor of kind::f16: D f32 (bit 4), A and B f16 and K-major (0), N >> 3, M >> 4
  static constexpr uint32_t Idesc = (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kTcBM >> 4) << 24);
  static_assert(ND >= 2, "double-buffered accumulators");
};

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
// try_wait with a suspend-time hint: a waiting thread sleeps until the phase completes (or the hint,
// 1 ms, elapses) instead of spinning, so waiting warps take no issue slots from the working ones.
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(su32(dst)),
               "l"(src), "r"(bytes), "r"(su32(bar))
               : "memory");
}

// Waits for the phase of parity `parity` of barrier b. Gives up when the CTA's abort flag is raised
// (if honor_abort) or after kTcWaitNs, raising the flag and recording ERR_TIMEOUT.
__device__ bool tc_wait(uint64_t* b, uint32_t parity, volatile int* abort, int* err, bool honor_abort = true) {
  if (mbar_try(b, parity)) return true;
  const unsigned long long t0 = gtimer();
  for (;;) {
    if (mbar_try(b, parity)) return true;
    if (honor_abort && *abort) return false;
    if (gtimer() - t0 > kTcWaitNs) {
      *abort = 1;
      if (err) atomicExch(err, ERR_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, no swizzle (K-major core matrices of 8 rows x 16 bytes): start
// address, leading byte offset (next core matrix along K), stride byte offset (next 8 rows), version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
// tcgen05.wait::ld, with the loaded registers as operands so no use of them moves above the wait.
__device__ __forceinline__ void tc_wait_ld(uint32_t (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
}

// Two int8 values packed in the low 16 bits of v as an f16 pair, the lower byte in the low half:
// x + 128 placed in the mantissa of 1024 (f16 bits 0x6400 | (x + 128)) is the exact f16 1152 + x, and
// subtracting 1152 is exact (integers below 2048).
__device__ __forceinline__ uint32_t pair16_f16(uint32_t v) {
  const uint32_t w = __byte_perm(v ^ 0x8080u, 0x64646464u, 0x5140);
  const __half2 h = __hsub2(*(const __half2*)&w, __half2half2(__ushort_as_half((unsigned short)0x6480u)));
  return *(const uint32_t*)&h;
}

// One CTA per SM walks its tiles (row tile major, so CTAs running together share weight tiles in L2);
// every role counts the CTA's blocks with the same running index j, which sets each barrier's stage,
// buffer and phase.
template <int Q, int S>
__global__ void __launch_bounds__(TcCfg<Q, S>::Threads, 1)
    k_tc_gemm(TcMat W, const int8_t* __restrict__ aq, const float* __restrict__ as, int T, float* __restrict__ y,
              int ldy, int* err) {
  using C = TcCfg<Q, S>;
  constexpr int ND = C::ND;
  extern __shared__ __align__(1024) unsigned char sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = W.cols / 32, ptiles = (T + C::TP - 1) / C::TP, ntiles = ((W.rows + kTcBM - 1) / kTcBM) * ptiles;
  const int mytiles = (int)blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = mytiles * nb;  // blocks this CTA processes
  uint64_t* bars = (uint64_t*)(sm + S * C::Stage);
  uint64_t* full = bars;            // weight tile and scales landed (copy engine)
  uint64_t* bready = full + S;      // expanded activations and their scales written (converter warps)
  uint64_t* empty = bready + S;     // the stage's MMAs finished and every epilogue warp read its scales
  uint64_t* dfull = empty + S;      // accumulator buffer d holds a block's pair sums
  uint64_t* dempty = dfull + ND;    // the epilogue has read buffer d
  uint32_t* tslot = (uint32_t*)(bars + C::Bars);
  volatile int* abort = (volatile int*)(tslot + 1);
  auto tile_of = [&](int i) { return (int)blockIdx.x + i * (int)gridDim.x; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(bready + s, Q);
      mbar_init(empty + s, 1 + C::EpiWarps);
    }
    for (int d = 0; d < ND; ++d) {
      mbar_init(dfull + d, 1);
      mbar_init(dempty + d, C::EpiWarps);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // the expanded activation tiles are zero except for the pairs each block writes: zero them once
  for (int i = threadIdx.x; i < S * (2 * C::BHalf / 16); i += C::Threads) {
    const int s = i / (2 * C::BHalf / 16), o = i % (2 * C::BHalf / 16);
    *(uint4*)(sm + s * C::Stage + C::BOff + o * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tslot)), "r"(kTcCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (C::CopyWarp && warp == C::CopyW) {
    // ---- copy engine: per block one 8704-byte chunk (weight tile and weight scales) ----
    if (lane == 0) {
      int j = 0;
      for (int i = 0; i < mytiles; ++i) {
        const size_t tb0 = (size_t)(tile_of(i) / ptiles) * nb;
        for (int b = 0; b < nb; ++b, ++j) {
          const int s = j % S;
          if (!tc_wait(empty + s, ((j / S) & 1) ^ 1, abort, err)) goto drained;
          mbar_expect_tx(full + s, kTcChunk);
          bulk_g2s(sm + s * C::Stage, W.tiles + (tb0 + b) * kTcChunk, kTcChunk, full + s);
        }
      }
    drained:
      // every copy issued lands before the CTA may exit
      for (int k = j > S ? j - S : 0; k < j; ++k) tc_wait(full + k % S, (k / S) & 1, abort, err, false);
    }
  } else if (warp == 0) {
    // ---- MMA issue: two MMAs per block into accumulator buffer j % ND ----
    if (lane == 0) {
      int j = 0;
      for (; j < total; ++j) {
        const int s = j % S, d = j % ND;
        const uint32_t ph = (j / S) & 1;
        if (!tc_wait(full + s, ph, abort, err) || !tc_wait(bready + s, ph, abort, err)) break;
        if (!tc_wait(dempty + d, ((j / ND) & 1) ^ 1, abort, err)) break;
        tc_fence_after();
        const uint32_t A = su32(sm + s * C::Stage), B = A + C::BOff;
#pragma unroll
        for (int h = 0; h < 2; ++h)
          tc_mma(tmem + (uint32_t)(d * 2 * C::N + h * C::N), sdesc(A + h * 256, 128, 512), sdesc(B + h * C::BHalf, 128, 256),
                 C::Idesc);
        tc_commit(empty + s);
        tc_commit(dfull + d);
      }
      // every MMA issued has completed before the tensor memory is freed (the last commit tracks them)
      if (j > 0) tc_wait(dfull + (j - 1) % ND, ((j - 1) / ND) & 1, abort, err, false);
    }
  } else if (warp <= Q) {
    // ---- activation expansion: converter warp q (each on its own SM sub-partition) writes, on lane
    // (jl, p), the pair of lane jl of position t = 4q + p for both halves: column n = 32q + 4 jl + p,
    // K core matrix jl / 4, row n % 8, word jl % 4; lane jl == 0 copies the position's scale. Its
    // loads run four blocks ahead. Lane 0 of the first converter warp also issues the stage's bulk
    // copy (weight tile and weight scales), which waits for the same release. ----
    pdl_wait();
    const int q = warp - 1, jl = lane >> 2, p = lane & 3;
    const bool copier = !C::CopyWarp && warp == 1 && lane == 0;
    const int wofs = C::BOff + q * 1024 + (jl >> 1) * 256 + (jl >> 2) * 128 + (4 * (jl & 1) + p) * 16 + (jl & 3) * 4;
    struct Cur {
      int i, b, t;  // tile ordinal, block, this lane's position (or -1 past the last tile)
      size_t tb0;   // first (row tile, block) index of the tile's weights
    };
    auto tile_start = [&](Cur& c) {
      if (c.i < mytiles) {
        const int tile = tile_of(c.i);
        c.t = (tile % ptiles) * C::TP + 4 * q + p;
        c.tb0 = (size_t)(tile / ptiles) * nb;
      } else {
        c.t = -1;
      }
    };
    auto advance = [&](Cur& c) {
      if (++c.b == nb) {
        c.b = 0;
        ++c.i;
        tile_start(c);
      }
    };
    // word jl of position p's block (the 8 lanes of a position read its 32 bytes) and, on lanes
    // jl == 0, the block's scale
    auto load = [&](const Cur& c, uint32_t& a, float& sv) {
      a = 0u;
      sv = 0.0f;
      if (c.t < 0 || c.t >= T) return;
      a = *(const uint32_t*)(aq + (size_t)c.t * W.cols + 32 * c.b + 4 * jl);
      if (jl == 0) sv = as[(size_t)c.t * nb + c.b];
    };
    // lane jl's pair of half h (bytes 16h + 2jl, + 1) sits in word 4h + jl / 2 of its position
    const int src0 = 4 * (jl >> 1) + p, src1 = 4 * (4 + (jl >> 1)) + p, sh = 16 * (jl & 1);
    Cur ld{0, 0, -1, 0}, cp{0, 0, -1, 0};
    tile_start(ld);
    tile_start(cp);
    uint32_t ra[4];
    float rs[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      load(ld, ra[k], rs[k]);
      advance(ld);
    }
    int issued = 0;  // blocks whose copies the copier issued
    bool go = true;
    for (int j0 = 0; go && j0 < total; j0 += 4) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = j0 + k;
        if (j >= total) {
          go = false;
          break;
        }
        const int s = j % S;
        if (!tc_wait(empty + s, ((j / S) & 1) ^ 1, abort, err)) {
          go = false;
          break;
        }
        unsigned char* dst = sm + s * C::Stage;
        if (copier) {
          mbar_expect_tx(full + s, kTcChunk);
          bulk_g2s(dst, W.tiles + (cp.tb0 + cp.b) * kTcChunk, kTcChunk, full + s);
          ++issued;
          advance(cp);
        }
        const uint32_t w0 = __shfl_sync(0xffffffffu, ra[k], src0), w1 = __shfl_sync(0xffffffffu, ra[k], src1);
        *(uint32_t*)(dst + wofs) = pair16_f16(w0 >> sh);
        *(uint32_t*)(dst + wofs + C::BHalf) = pair16_f16(w1 >> sh);
        if (jl == 0) ((float*)(dst + C::AsOff))[4 * q + p] = rs[k];
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(bready + s);
        load(ld, ra[k], rs[k]);
        advance(ld);
      }
    }
    if (copier)  // every copy issued lands before the CTA may exit
      for (int k = issued > S ? issued - S : 0; k < issued; ++k) tc_wait(full + k % S, (k / S) & 1, abort, err, false);
  } else if (warp < C::Epi0 + C::EpiWarps) {
    // ---- epilogue: the reference's FMA per lane and block, from tensor memory ----
    pdl_wait();
    const int q = (warp - C::Epi0) >> 2, quarter = warp & 3;
    const int rl = 32 * quarter + lane;
    const uint32_t trow = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(32 * q);
    int j = 0;
    bool go = true;
    for (int i = 0; go && i < mytiles; ++i) {
      const int tile = tile_of(i), rt = tile / ptiles, tq = (tile % ptiles) * C::TP + 4 * q;
      float2 acc[16][2];  // lane L of positions (0, 1) and (2, 3)
#pragma unroll
      for (int L = 0; L < 16; ++L) acc[L][0] = acc[L][1] = make_float2(0.0f, 0.0f);
      for (int b = 0; b < nb; ++b, ++j) {
        const int s = j % S, d = j % ND;
        const uint32_t ph = (j / S) & 1;
        if (!tc_wait(full + s, ph, abort, err) || !tc_wait(bready + s, ph, abort, err)) {
          go = false;
          break;
        }
        const unsigned char* stg = sm + s * C::Stage;
        const float wsr = ((const float*)(stg + kTcA))[rl];
        const float4 a4 = *(const float4*)(stg + C::AsOff + 16 * q);
        // ws_b * as_b (q8.rs:268), for positions (0, 1) and (2, 3)
        const float2 sc[2] = {make_float2(__fmul_rn(wsr, a4.x), __fmul_rn(wsr, a4.y)),
                              make_float2(__fmul_rn(wsr, a4.z), __fmul_rn(wsr, a4.w))};
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + s);
        if (!tc_wait(dfull + d, (j / ND) & 1, abort, err)) {
          go = false;
          break;
        }
        tc_fence_after();
        // chunk hc: half hc >> 1, this warpgroup's columns 16 (hc & 1) .. + 15 of that half; column m
        // is lane 8 (hc >> 1) + 4 (hc & 1) + m / 4 of position m % 4
        const uint32_t base = trow + (uint32_t)(d * 2 * C::N);
#pragma unroll
        for (int hc = 0; hc < 4; ++hc) {
          uint32_t v[16];
          tc_ld16(base + (uint32_t)((hc >> 1) * C::N + (hc & 1) * 16), v);
          tc_wait_ld(v);
          if (hc == 3) {  // buffer d is read: the MMAs of block j + ND may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(dempty + d);
          }
#pragma unroll
          for (int m = 0; m < 16; m += 2) {
            const int L = 8 * (hc >> 1) + 4 * (hc & 1) + (m >> 2), pp = (m & 3) >> 1;
            acc[L][pp] = __ffma2_rn(make_float2(__uint_as_float(v[m]), __uint_as_float(v[m + 1])), sc[pp], acc[L][pp]);
          }
        }
      }
      if (!go) break;
      // _mm512_reduce_add_ps: lanes i + 8 onto i, then 4, 2, 1 apart
      const int r = rt * kTcBM + rl;
#pragma unroll
      for (int pos = 0; pos < 4; ++pos) {
        float a[16];
#pragma unroll
        for (int L = 0; L < 16; ++L) a[L] = (pos & 1) ? acc[L][pos >> 1].y : acc[L][pos >> 1].x;
        float bs[8];
#pragma unroll
        for (int z = 0; z < 8; ++z) bs[z] = __fadd_rn(a[z], a[z + 8]);
        const float c0 = __fadd_rn(bs[0], bs[4]), c1 = __fadd_rn(bs[1], bs[5]), c2 = __fadd_rn(bs[2], bs[6]),
                    c3 = __fadd_rn(bs[3], bs[7]);
        const float val = __fadd_rn(__fadd_rn(c0, c2), __fadd_rn(c1, c3));
        if (tq + pos < T && r < W.rows) y[(size_t)(tq + pos) * ldy + r] = val;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols) : "memory");
  }
}

// The tiled f16 copy of a Q8_0 / Q4_0 matrix (exact: int8 and nibble - 8 are f16 integers) and its
// scales as f32, zero past the last row. One thread per (row tile, block, row).
template <int BITS, typename ST>
__global__ void k_tc_tile(MatView w, int row_tiles, unsigned char* out) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int nb = w.cols / 32;
  if (idx >= (size_t)row_tiles * nb * kTcBM) return;
  const int rl = (int)(idx % kTcBM);
  const size_t tb = idx / kTcBM;  // rt * nb + b
  const int b = (int)(tb % nb), rt = (int)(tb / nb);
  const int r = rt * kTcBM + rl;
  __half* dst = (__half*)(out + tb * kTcChunk) + (rl >> 3) * 256 + (rl & 7) * 8;
#pragma unroll 4
  for (int k = 0; k < 32; ++k) {
    int v = 0;
    if (r < w.rows) {
      if constexpr (BITS == 8) {
        v = ((const int8_t*)w.q)[(size_t)r * w.cols + 32 * b + k];
      } else {  // q8.rs:42-52: byte j holds weight j (low nibble) and j + 16 (high nibble), each + 8
        const uint8_t byte = ((const uint8_t*)w.q)[(size_t)r * (w.cols / 2) + 16 * b + (k & 15)];
        v = (int)(k < 16 ? (byte & 15) : (byte >> 4)) - 8;
      }
    }
    dst[(k >> 3) * 64 + (k & 7)] = __int2half_rn(v);
  }
  ((float*)(out + tb * kTcChunk + kTcA))[rl] = r < w.rows ? ld_scale((const ST*)w.s, (size_t)r * nb + b) : 0.0f;
}

}  // namespace

bool tc_gemm_supported(const MatView& w) {
  return (w.bits == 8 || w.bits == 4) && w.cols >= 32 && w.cols % 32 == 0 && w.rows > 0 &&
         (w.rows + kTcBM - 1) / kTcBM <= 65535;
}
static int tc_row_tiles(const MatView& w) { return (w.rows + kTcBM - 1) / kTcBM; }
size_t tc_tiled_bytes(const MatView& w) { return (size_t)tc_row_tiles(w) * (w.cols / 32) * kTcChunk; }

void tc_tile(const MatView& w, void* buf, TcMat* out, cudaStream_t st) {
  const int row_tiles = tc_row_tiles(w);
  unsigned char* o = (unsigned char*)buf;
  const size_t n = (size_t)row_tiles * (w.cols / 32) * kTcBM;
  const int threads = 256;
  const unsigned blocks = (unsigned)((n + threads - 1) / threads);
  if (w.bits == 8 && !w.scale_f32) k_tc_tile<8, __half><<<blocks, threads, 0, st>>>(w, row_tiles, o);
  else if (w.bits == 8) k_tc_tile<8, float><<<blocks, threads, 0, st>>>(w, row_tiles, o);
  else if (!w.scale_f32) k_tc_tile<4, __half><<<blocks, threads, 0, st>>>(w, row_tiles, o);
  else k_tc_tile<4, float><<<blocks, threads, 0, st>>>(w, row_tiles, o);
  out->tiles = o;
  out->rows = w.rows;
  out->cols = w.cols;
}

template <int Q, int S>
static void launch_tc_cfg(const TcMat& W, const int8_t* aq, const float* as, int T, float* y, int ldy, int* err, int sms,
                          cudaStream_t st) {
  using C = TcCfg<Q, S>;
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(k_tc_gemm<Q, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::Smem);
    init = true;
  }
  const int tiles = ((W.rows + kTcBM - 1) / kTcBM) * ((T + C::TP - 1) / C::TP);
  launch_k(k_tc_gemm<Q, S>, dim3(std::min(tiles, sms)), dim3(C::Threads), (size_t)C::Smem, st, W, aq, as, T, y, ldy, err);
}

// Tile shape: 12 positions per tile with two accumulator buffers (measured faster), or with
// GEM_TC_GROUPS=2 8 positions with four.
void launch_tc_gemm(const TcMat& W, const int8_t* aq, const float* as, int T, float* y, int ldy, int* err, int sms,
                    cudaStream_t st) {
  static const int groups = [] {
    const char* e = std::getenv("GEM_TC_GROUPS");
    return e && std::atoi(e) == 2 ? 2 : 3;
  }();
  if (groups == 3) launch_tc_cfg<3, 8>(W, aq, as, T, y, ldy, err, sms, st);
  else launch_tc_cfg<2, 8>(W, aq, as, T, y, ldy, err, sms, st);
}

}  // namespace gem
