// sampler.cu -- the guided (classifier-free guidance) argmax pass of the TTS
// step on the device: for every (codebook c, target frame t) row,
//
//   lp_c = log_softmax(cond row), lp_u = log_softmax(uncond row)
//   mix  = log_softmax(lp_c + g * (lp_c - lp_u))        (mix = lp_c if g == 0)
//   mix[mask_id] = -inf;  pred = first argmax;  score = max - c * layer_penalty
//
// as the reference's CPU loop computes it (cpp/src/model/tts.cpp:291-326 with
// log_softmax at :91-101), behind the accelerator hook LM::CudaSampleFn
// (cpp/src/model/lm.h:106-108), which the reference's CUDA runner serves with
// its guided_sample_kernel (cpp/src/backend/cuda/cuda_lm.cu:679-758).
//
// Layout: both logits planes are token-major [seq, C * V] fp32; the cond row
// of (c, t) is at token cond_seq - T + t, the uncond row at token t.
//
// One warp per row.  A row of V = 32 * kFull + kTail logits is read once
// from HBM into registers (lane l holds elements l, l + 32, ...: every load
// instruction is one coalesced 128-byte segment; rows need no alignment), and
// the three log-softmaxes, the mix and the argmax run on those registers with
// warp shuffles.  V is split at compile time (1025, the LM's audio
// vocabulary, is kFull = 32 plus one tail element), so only the tail is
// predicated; other V up to 2048 take a bounds-checked register kernel,
// longer rows a kernel that re-reads the row from global memory (L2).
//
// exp and log are the hardware's ex2.approx / lg2.approx on log2(e)-scaled
// arguments (relative error ~2^-22): the accurate library functions made the
// kernel instruction-bound at ~2900 instructions per row.  The sums are
// warp-tree ordered instead of the CPU's left-to-right order, so
// log-probabilities agree with the CPU loop to ~1e-6 and the argmax to within
// rounding ties.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "ovb_internal.h"
#include "ovb_ptx.cuh"

namespace ovb {
namespace {

constexpr int kSampleWarps = 8;  // rows per 256-thread block

// 4-byte global load with the evict-first hint, only when `pred` (else 0).
__device__ __forceinline__ float ld_cs_if(const float* p, bool pred) {
  float v = 0.f;
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q ld.global.cs.f32 %0, [%1];\n\t}"
      : "+f"(v)
      : "l"(p), "r"(static_cast<int>(pred))
      : "memory");
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// (value, index) of the first maximum: a larger value wins; equal values
// keep the smaller index.  NaN never wins (as `v > best` on the CPU).
__device__ __forceinline__ void warp_argmax(float& val, int& idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, val, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > val || (ov == val && oi < idx)) {
      val = ov;
      idx = oi;
    }
  }
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// exp(d) for d <= 0 and log(s) + m, through the base-2 hardware functions.
__device__ __forceinline__ float exp_le0(float d) { return ex2_approx(__fmul_rn(d, kLog2e)); }
__device__ __forceinline__ float lse_from(float s, float m) {
  return __fadd_rn(__fmul_rn(lg2_approx(s), kLn2), m);
}

// log-sum-exp of the lane-strided values x[k] (element lane + 32k): max, then
// the sum of exp(x - max), then log(sum) + max (tts.cpp:91-101).  Columns
// k < kFull are valid in every lane, column kFull in lanes < kTail.
template <int kFull, int kTail, int kPer>
__device__ __forceinline__ float row_lse(const float (&x)[kPer], int lane) {
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < kFull; ++k) m = fmaxf(m, x[k]);
  if (kTail > 0 && lane < kTail) m = fmaxf(m, x[kFull]);
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < kFull; ++k) s = __fadd_rn(s, exp_le0(__fsub_rn(x[k], m)));
  if (kTail > 0 && lane < kTail) s = __fadd_rn(s, exp_le0(__fsub_rn(x[kFull], m)));
  s = warp_sum(s);
  return lse_from(s, m);
}

// The same for a runtime V (columns valid while lane + 32k < n).
template <int kPer>
__device__ __forceinline__ float row_lse_n(const float (&x)[kPer], int lane, int n) {
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < kPer; ++k)
    if (lane + 32 * k < n) m = fmaxf(m, x[k]);
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k)
    if (lane + 32 * k < n) s = __fadd_rn(s, exp_le0(__fsub_rn(x[k], m)));
  s = warp_sum(s);
  return lse_from(s, m);
}

// Row (c, t) of warp `row` and its cond / uncond logits.
__device__ __forceinline__ void row_ptrs(int64_t row, const float* cond, int cond_seq,
                                         const float* uncond, int C, int V, int T, int* c,
                                         const float** lc, const float** lu) {
  *c = static_cast<int>(row / T);
  const int t = static_cast<int>(row - static_cast<int64_t>(*c) * T);
  const int64_t CV = static_cast<int64_t>(C) * V;
  *lc = cond + (static_cast<int64_t>(cond_seq) - T + t) * CV + static_cast<int64_t>(*c) * V;
  *lu = uncond + static_cast<int64_t>(t) * CV + static_cast<int64_t>(*c) * V;
}

// The mix, its log-softmax, the masked first argmax and the score, on the
// registers holding the row (xc: cond logits, xu: uncond logits).  valid(k)
// says whether column k exists in this lane.
template <int kPer, typename Valid, typename Lse>
__device__ __forceinline__ void finish_row(float (&xc)[kPer], const float (&xu)[kPer], float lse_c,
                                           float lse_u, float guidance, int mask_id, int lane,
                                           Valid valid, Lse lse, float* best_out, int* idx_out) {
  // mix (in xc): lp_c + g * (lp_c - lp_u); g == 0 keeps lp_c (the CPU path
  // skips the second log-softmax then).
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const float pc = __fsub_rn(xc[k], lse_c);
    const float pu = __fsub_rn(xu[k], lse_u);
    xc[k] = guidance != 0.f ? __fadd_rn(pc, __fmul_rn(guidance, __fsub_rn(pc, pu))) : pc;
  }
  const float lse2 = guidance != 0.f ? lse(xc) : 0.f;
  float best = -INFINITY;
  int best_j = 0;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int j = lane + 32 * k;
    if (valid(k) && j != mask_id) {
      const float v = __fsub_rn(xc[k], lse2);
      if (v > best) {
        best = v;
        best_j = j;
      }
    }
  }
  warp_argmax(best, best_j);
  *best_out = best;
  *idx_out = best_j;
}

// Row `row` of one pair's [C, T] output with V = 32 * kFull + kTail known
// at compile time (one warp).
template <int kFull, int kTail>
__device__ __forceinline__ void fixed_row(const float* __restrict__ cond, int cond_seq,
                                          const float* __restrict__ uncond, int C, int T,
                                          int64_t row, float guidance, float penalty, int mask_id,
                                          int32_t* __restrict__ pred, float* __restrict__ scores) {
  constexpr int kPer = kFull + (kTail > 0 ? 1 : 0);
  constexpr int V = 32 * kFull + kTail;
  const int lane = threadIdx.x & 31;
  int c;
  const float *lc, *lu;
  row_ptrs(row, cond, cond_seq, uncond, C, V, T, &c, &lc, &lu);
  // Both rows in one batch of loads, streamed once (evict-first).
  float xc[kPer], xu[kPer];
#pragma unroll
  for (int k = 0; k < kFull; ++k) {
    xc[k] = __ldcs(lc + lane + 32 * k);
    xu[k] = __ldcs(lu + lane + 32 * k);
  }
  if constexpr (kTail > 0) {
    xc[kFull] = ld_cs_if(lc + lane + 32 * kFull, lane < kTail);
    xu[kFull] = ld_cs_if(lu + lane + 32 * kFull, lane < kTail);
  }
  const float lse_c = row_lse<kFull, kTail>(xc, lane);
  const float lse_u = row_lse<kFull, kTail>(xu, lane);
  float best;
  int best_j;
  finish_row<kPer>(
      xc, xu, lse_c, lse_u, guidance, mask_id, lane,
      [&](int k) { return k < kFull || lane < kTail; },
      [&](const float (&x)[kPer]) { return row_lse<kFull, kTail>(x, lane); }, &best, &best_j);
  if (lane == 0) {
    pred[row] = best_j;
    scores[row] = __fsub_rn(best, __fmul_rn(static_cast<float>(c), penalty));
  }
}

template <int kFull, int kTail>
__global__ void __launch_bounds__(32 * kSampleWarps) guided_sample_fixed_kernel(
    const float* __restrict__ cond, int cond_seq, const float* __restrict__ uncond, int C, int T,
    float guidance, float penalty, int mask_id, int32_t* __restrict__ pred,
    float* __restrict__ scores) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kSampleWarps + (threadIdx.x >> 5);
  if (row >= static_cast<int64_t>(C) * T) return;  // whole warps only
  fixed_row<kFull, kTail>(cond, cond_seq, uncond, C, T, row, guidance, penalty, mask_id, pred,
                          scores);
}

// Several CFG pairs in one launch (the same rows as one launch per pair): the
// pairs' [C, T_p] outputs are concatenated, pair p's first at g.out0[p]; a
// warp finds its pair by scanning those offsets.
template <int kFull, int kTail>
__global__ void __launch_bounds__(32 * kSampleWarps) guided_sample_batch_kernel(
    const __grid_constant__ GuidedBatch g, int32_t* __restrict__ pred,
    float* __restrict__ scores) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kSampleWarps + (threadIdx.x >> 5);
  if (row >= g.out0[g.n]) return;  // whole warps only
  int p = 0;
  for (int i = 1; i < g.n; ++i)
    if (row >= g.out0[i]) p = i;
  fixed_row<kFull, kTail>(g.cond[p], g.cond_seq[p], g.uncond[p], g.C, g.T[p], row - g.out0[p],
                          g.guidance, g.penalty, g.mask_id, pred + g.out0[p], scores + g.out0[p]);
}

// Any V <= 32 * kPer, bounds-checked per column.
template <int kPer>
__global__ void __launch_bounds__(32 * kSampleWarps) guided_sample_reg_kernel(
    const float* __restrict__ cond, int cond_seq, const float* __restrict__ uncond, int C, int V,
    int T, float guidance, float penalty, int mask_id, int32_t* __restrict__ pred,
    float* __restrict__ scores) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kSampleWarps + (threadIdx.x >> 5);
  if (row >= static_cast<int64_t>(C) * T) return;
  int c;
  const float *lc, *lu;
  row_ptrs(row, cond, cond_seq, uncond, C, V, T, &c, &lc, &lu);
  float xc[kPer], xu[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int j = lane + 32 * k;
    xc[k] = ld_cs_if(lc + j, j < V);
    xu[k] = ld_cs_if(lu + j, j < V);
  }
  const float lse_c = row_lse_n<kPer>(xc, lane, V);
  const float lse_u = row_lse_n<kPer>(xu, lane, V);
  float best;
  int best_j;
  finish_row<kPer>(
      xc, xu, lse_c, lse_u, guidance, mask_id, lane, [&](int k) { return lane + 32 * k < V; },
      [&](const float (&x)[kPer]) { return row_lse_n<kPer>(x, lane, V); }, &best, &best_j);
  if (lane == 0) {
    pred[row] = best_j;
    scores[row] = __fsub_rn(best, __fmul_rn(static_cast<float>(c), penalty));
  }
}

// Any V: the same arithmetic with every pass re-reading the row.
__device__ __forceinline__ float row_lse_global(const float* x, int lane, int n) {
  float m = -INFINITY;
  for (int j = lane; j < n; j += 32) m = fmaxf(m, x[j]);
  m = warp_max(m);
  float s = 0.f;
  for (int j = lane; j < n; j += 32) s = __fadd_rn(s, exp_le0(__fsub_rn(x[j], m)));
  s = warp_sum(s);
  return lse_from(s, m);
}

__global__ void __launch_bounds__(32 * kSampleWarps) guided_sample_any_kernel(
    const float* __restrict__ cond, int cond_seq, const float* __restrict__ uncond, int C, int V,
    int T, float guidance, float penalty, int mask_id, int32_t* __restrict__ pred,
    float* __restrict__ scores) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kSampleWarps + (threadIdx.x >> 5);
  if (row >= static_cast<int64_t>(C) * T) return;
  const int c = static_cast<int>(row / T);
  const int t = static_cast<int>(row - static_cast<int64_t>(c) * T);
  const int64_t CV = static_cast<int64_t>(C) * V;
  const float* lc = cond + (static_cast<int64_t>(cond_seq) - T + t) * CV + static_cast<int64_t>(c) * V;
  const float* lu = uncond + static_cast<int64_t>(t) * CV + static_cast<int64_t>(c) * V;
  const float lse_c = row_lse_global(lc, lane, V);
  const float lse_u = row_lse_global(lu, lane, V);
  auto mix = [&](int j) {
    const float pc = __fsub_rn(lc[j], lse_c);
    if (guidance == 0.f) return pc;
    return __fadd_rn(pc, __fmul_rn(guidance, __fsub_rn(pc, __fsub_rn(lu[j], lse_u))));
  };
  float lse2 = 0.f;
  if (guidance != 0.f) {
    float m = -INFINITY;
    for (int j = lane; j < V; j += 32) m = fmaxf(m, mix(j));
    m = warp_max(m);
    float s = 0.f;
    for (int j = lane; j < V; j += 32) s = __fadd_rn(s, exp_le0(__fsub_rn(mix(j), m)));
    s = warp_sum(s);
    lse2 = lse_from(s, m);
  }
  float best = -INFINITY;
  int best_j = 0;
  for (int j = lane; j < V; j += 32) {
    if (j == mask_id) continue;
    const float v = guidance != 0.f ? __fsub_rn(mix(j), lse2) : mix(j);
    if (v > best) {
      best = v;
      best_j = j;
    }
  }
  warp_argmax(best, best_j);
  if (lane == 0) {
    pred[row] = best_j;
    scores[row] = __fsub_rn(best, __fmul_rn(static_cast<float>(c), penalty));
  }
}

}  // namespace

cudaError_t launch_guided_sample_batch(const GuidedBatch& g, int32_t* pred, float* scores,
                                       cudaStream_t s) {
  const int64_t rows = g.out0[g.n];
  if (rows <= 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>((rows + kSampleWarps - 1) / kSampleWarps));
  return launch_plain(guided_sample_batch_kernel<32, 1>, grid, dim3(32 * kSampleWarps), 0, s, g,
                      pred, scores);
}

cudaError_t launch_guided_sample(const float* cond, int cond_seq, const float* uncond, int C,
                                 int V, int T, float guidance, float penalty, int mask_id,
                                 int32_t* pred, float* scores, cudaStream_t s) {
  const int64_t rows = static_cast<int64_t>(C) * T;
  const dim3 grid(static_cast<unsigned>((rows + kSampleWarps - 1) / kSampleWarps));
  const dim3 block(32 * kSampleWarps);
  if (V == 1025)  // the LM's audio vocabulary (1024 codes + the mask token)
    return launch_plain(guided_sample_fixed_kernel<32, 1>, grid, block, 0, s, cond, cond_seq,
                        uncond, C, T, guidance, penalty, mask_id, pred, scores);
  if (V <= 32 * 33)
    return launch_plain(guided_sample_reg_kernel<33>, grid, block, 0, s, cond, cond_seq, uncond,
                        C, V, T, guidance, penalty, mask_id, pred, scores);
  if (V <= 32 * 64)
    return launch_plain(guided_sample_reg_kernel<64>, grid, block, 0, s, cond, cond_seq, uncond,
                        C, V, T, guidance, penalty, mask_id, pred, scores);
  return launch_plain(guided_sample_any_kernel, grid, block, 0, s, cond, cond_seq, uncond, C, V,
                      T, guidance, penalty, mask_id, pred, scores);
}

}  // namespace ovb
